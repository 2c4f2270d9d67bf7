"""KulaMamba: the Mamba-3 SSD layer, drop-in for ``mamba3.mamba3`` of the reference.

Same constructor, parameter names, shapes and default init as the reference
(mamba3/mamba3.py:48-123), so a ``state_dict`` moves between the two in either
direction and a seeded construction yields identical weights.  ``in_proj`` and
``out_proj`` stay cuBLAS GEMMs; everything between them runs in the sm_100a
kernels of ``libmamba3_b200`` (see ``ops.py``):

* ``forward`` / ``prefill`` -> ``mamba3_b200::layer_ssd`` (chunked parallel form)
* ``step``                  -> ``mamba3_b200::step_ssm`` (O(1) recurrent form)
* with gradients (training) -> the library's kernels forward and backward for the B / C
  preparation, the x-side MIMO weights, ``chunked_ssd`` and the gate; only the projection
  split and dt are torch ops.  There is no other path: where the kernels do not apply the
  call raises.

Deviation from the reference (documented): the ``angle`` entry of the inference
state is kept in fp32 whatever the model dtype (the reference accumulates it in
the model dtype, mamba3/mamba3.py:330, which drifts in bf16).
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib, ops
from .ssd import chunked_ssd


class ArgumentAssertionError(ValueError, AssertionError):
    """An argument the reference rejects with `assert` (mamba3/mamba3.py:77, 79, 85, 194): an
    AssertionError there, so callers that catch that catch this too; also a ValueError, as the
    other argument checks here are."""


class SequenceLengthError(ArgumentAssertionError):
    """An input with no tokens (the reference's message, mamba3/mamba3.py:194)."""


def _check_tokens(x):
    if x.dim() != 3:
        raise ValueError(f"expected (batch, seqlen, d_model), got {tuple(x.shape)}")
    if x.shape[1] <= 0:
        raise SequenceLengthError(f"Sequence length must be positive, got {x.shape[1]}")


class RMSNorm(nn.Module):
    """RMSNorm with the reference's semantics (mamba3/mamba3.py:19-35).  On CUDA without
    gradients (inference, decode) it is one kernel (``mamba3_b200::rmsnorm``); when autograd
    needs it (training) it runs as torch ops."""

    def __init__(self, d: int, eps: float = 1e-5, dim: int = -1):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(d))
        self.eps = eps
        self.dim = dim

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if (x.is_cuda and self.dim in (-1, x.ndim - 1) and x.dtype in (torch.float32, torch.bfloat16, torch.float16)
                and not (torch.is_grad_enabled() and (x.requires_grad or self.weight.requires_grad))):
            return ops.rmsnorm(x, self.weight, self.eps)
        inv = torch.rsqrt(x.float().pow(2).mean(self.dim, keepdim=True) + self.eps).to(x.dtype)
        shape = [1] * x.ndim
        shape[self.dim] = -1
        return x * inv * self.weight.view(*shape)


class _GateFn(torch.autograd.Function):
    """(y * silu(z * mimo_z) * mimo_down).sum(-1) (mamba3/mamba3.py:234-238) as one kernel each
    way (``mamba3_b200::gate_fwd`` / ``gate_bwd``): fp32 arithmetic inside, the parameter
    gradients summed over the rows in a fixed order."""

    @staticmethod
    def forward(ctx, y, z, mimo_z, mimo_down):
        ctx.save_for_backward(y, z, mimo_z, mimo_down)
        return ops.gate_fwd(y, z, mimo_z, mimo_down)

    @staticmethod
    def backward(ctx, dout):
        return ops.gate_bwd(*ctx.saved_tensors, dout.contiguous())


def _gate(y, z, mimo_z, mimo_down):
    """y (B,T,H,P,R), z (B,T,H*P) -> (B,T,H*P) through the gate kernels.  Parameters of another
    dtype than the activations (fp32 master weights under autocast) are cast to the activation
    dtype first; the cast is part of the autograd graph, so their gradients still arrive."""
    R = mimo_z.shape[-1]
    if not (y.is_cuda and R <= 4 and z.stride(-1) == 1 and y.dtype == z.dtype):
        raise _lib.M3bError("gate: CUDA activations of one dtype, mimo_rank <= 4 expected (no other path)")
    return _GateFn.apply(y.contiguous(), z, mimo_z.to(y.dtype), mimo_down.to(y.dtype))


class _BCFn(torch.autograd.Function):
    """RMSNorm + bias of B and C, their broadcast to the heads, the data-dependent rotation and the
    previous-token shift of B (mamba3/mamba3.py:203-232) as one kernel each way
    (``mamba3_b200::bc_fwd`` / ``bc_bwd``).  Returns (B_g, B_b, C), B_b empty without shift."""

    @staticmethod
    def forward(ctx, Bf, Cf, theta, dt, wB, bB, wC, bC, H, eps, shift):
        ctx.save_for_backward(Bf, Cf, theta, dt, wB, bB, wC, bC)
        ctx.cfg = (H, eps, shift)
        return ops.bc_fwd(Bf, Cf, theta, dt, wB, bB, wC, bC, H, eps, shift)

    @staticmethod
    def backward(ctx, dBg, dBb, dC):
        Bf, Cf, theta, dt, wB, bB, wC, bC = ctx.saved_tensors
        H, eps, shift = ctx.cfg
        shape = (*Bf.shape[:2], H, *bB.shape[1:])
        z = lambda g: torch.zeros(shape, dtype=Bf.dtype, device=Bf.device) if g is None else g.contiguous()  # noqa: E731
        g = ops.bc_bwd(Bf, Cf, theta, dt, wB, bB, wC, bC, z(dBg), z(dBb) if shift else None, z(dC), H, eps, shift)
        dBf, dCf, dth, ddt, dwB, dbB, dwC, dbC = g
        rot = theta is not None
        return dBf, dCf, dth if rot else None, ddt if rot else None, dwB, dbB, dwC, dbC, None, None, None


class _XFn(torch.autograd.Function):
    """x_raw = xf * mimo_x and, with the trapezoid, x_g = x_raw * lam and x_b = shifted x_raw *
    (1 - lam) exp(A dt) (mamba3/mamba3.py:218-230) as one kernel each way
    (``mamba3_b200::xprep_fwd`` / ``xprep_bwd``).  Returns (x_raw, x_g, x_b), the last two
    empty without the trapezoid."""

    @staticmethod
    def forward(ctx, xf, mimo_x, lam_raw, dt, A):
        ctx.save_for_backward(xf, mimo_x, lam_raw, dt, A)
        return ops.xprep_fwd(xf, mimo_x, lam_raw, dt, A)

    @staticmethod
    def backward(ctx, dxr, dxg, dxb):
        xf, mimo_x, lam_raw, dt, A = ctx.saved_tensors
        trap = lam_raw is not None
        shape = (*xf.shape[:2], *mimo_x.shape)
        z = lambda g: torch.zeros(shape, dtype=xf.dtype, device=xf.device) if g is None else g.contiguous()  # noqa: E731
        dxf, dmx, dlam, ddt, dA = ops.xprep_bwd(xf, mimo_x, lam_raw, dt, A, z(dxr), z(dxg) if trap else None,
                                                z(dxb) if trap else None)
        return (dxf, dmx, dlam, ddt, dA) if trap else (dxf, dmx, None, None, None)


class KulaMamba(nn.Module):
    """Mamba-3 layer: trapezoidal discretisation, data-dependent RoPE on B/C, MIMO rank R."""

    def __init__(
        self,
        d_model: int,
        d_state: int = 128,
        expand: int = 2,
        headdim: int = 64,
        ngroups: int | None = None,
        mimo_rank: int = 2,
        chunk_size: int = 64,
        bias: bool = False,
        dt_min: float = 0.001,
        dt_max: float = 0.1,
        use_trapezoidal: bool = True,
        use_complex_ssm: bool = True,
    ):
        super().__init__()
        self.d_model = d_model
        self.d_state = d_state
        self.expand = expand
        self.headdim = headdim
        self.mimo_rank = max(mimo_rank, 1)
        # chunk_size is accepted for API compatibility; the kernels pick their own
        # chunk length (128 / mimo_rank rounded up to a power of two), which changes
        # no result beyond fp32 rounding.
        self.chunk_size = chunk_size
        self.use_trapezoidal = use_trapezoidal
        self.use_complex_ssm = use_complex_ssm
        self.d_inner = expand * d_model
        if self.d_inner % headdim != 0:
            raise ArgumentAssertionError("expand * d_model must be a multiple of headdim")
        if d_state % 2 != 0:
            raise ArgumentAssertionError("d_state must be even (RoPE pairing)")
        self.nheads = self.d_inner // headdim
        self.ngroups = ngroups if ngroups is not None else 1
        if self.nheads % self.ngroups != 0:
            raise ArgumentAssertionError("nheads must be a multiple of ngroups")
        self.heads_per_group = self.nheads // self.ngroups
        H, P, N, R, G = self.nheads, headdim, d_state, self.mimo_rank, self.ngroups

        self._d_bc = G * N * R
        self._d_x = self.d_inner
        width = self.d_inner + self._d_x + 2 * self._d_bc + H
        width += H if use_trapezoidal else 0
        width += N // 2 if use_complex_ssm else 0
        self.in_proj = nn.Linear(d_model, width, bias=bias)

        self.A_log = nn.Parameter(torch.zeros(H))
        self.D = nn.Parameter(torch.ones(H))
        self.dt_bias = nn.Parameter(torch.zeros(H))
        self.B_norm = RMSNorm(N * R)
        self.C_norm = RMSNorm(N * R)
        self.B_bias = nn.Parameter(torch.ones(G, N, R))
        self.C_bias = nn.Parameter(torch.ones(G, N, R))
        self.mimo_x = nn.Parameter(torch.ones(H, P, R))
        self.mimo_z = nn.Parameter(torch.ones(H, P, R))
        self.mimo_down = nn.Parameter(torch.full((H, P, R), 1.0 / R))
        self.out_proj = nn.Linear(self.d_inner, d_model, bias=bias)
        self._init_weights(dt_min, dt_max)

    def _init_weights(self, dt_min: float, dt_max: float):
        """Default init of the reference (mamba3/mamba3.py:114-123), same RNG draws in the same order."""
        nn.init.kaiming_uniform_(self.in_proj.weight, a=math.sqrt(5))
        with torch.no_grad():
            u = torch.rand(self.nheads)
            dt = torch.exp(u * (math.log(dt_max) - math.log(dt_min)) + math.log(dt_min))
            # inverse softplus of dt
            self.dt_bias.copy_(dt + torch.log(-torch.expm1(-dt)))
            nn.init.uniform_(self.A_log, -4.0, -1.0)

    # -- plumbing ------------------------------------------------------------
    def _param_tensors(self):
        return (self.A_log, self.D, self.dt_bias, self.B_norm.weight, self.C_norm.weight, self.B_bias,
                self.C_bias, self.mimo_x, self.mimo_z, self.mimo_down)

    def _dims_tuple(self):
        d = self._dims()
        return (d["H"], d["P"], d["N"], d["R"], d["G"], d["trapezoidal"], d["complex_ssm"], d["norm_eps"])

    def _dims(self):
        return dict(H=self.nheads, P=self.headdim, N=self.d_state, R=self.mimo_rank, G=self.ngroups,
                    trapezoidal=self.use_trapezoidal, complex_ssm=self.use_complex_ssm,
                    norm_eps=float(self.B_norm.eps))

    def ssd_from_proj(self, proj, dt_scale=None, return_state=False, state=None, rms=None):
        """Everything between in_proj and out_proj: proj (B,T,d_in_proj) -> y (B,T,d_inner) [+ state].
        rms: the 1/rms rows that _project returns with this proj (optional)."""
        st = state or {}
        y, h, angle, prev_bx = ops.layer_ssd(proj, *self._param_tensors(), dt_scale, st.get("h"), st.get("angle"),
                                             st.get("prev_BX"), **self._dims(), return_state=return_state,
                                             rms=rms)
        if not return_state:
            return y
        return y, {"h": h, "angle": angle, "prev_BX": prev_bx}

    def _project(self, x):
        """(proj, rms): in_proj(x) and, where one kernel can give both, the layer's per-token 1/rms
        of B and C from the projection's epilogue (m3b_in_proj; then the layer forward skips its
        own pass over B and C).  That kernel takes bf16 CUDA inputs without gradients, 16-byte
        aligned rows and B / C columns on multiples of 16; otherwise in_proj is the nn.Linear
        (cuBLAS) and rms is None."""
        W, b = self.in_proj.weight, self.in_proj.bias
        if (x.is_cuda and x.dtype == torch.bfloat16 and W.dtype == torch.bfloat16
                and (b is None or b.dtype == torch.bfloat16) and not self._needs_grad(x)
                and x.shape[-1] % 8 == 0 and W.shape[0] % 8 == 0 and (2 * self.d_inner) % 16 == 0
                and (self.d_state * self.mimo_rank) % 16 == 0 and self._proj_segments() <= 128):
            d = self._dims()
            return ops.in_proj_rms(x, W, b, d["H"], d["P"], d["N"], d["R"], d["G"], d["norm_eps"])
        return self.in_proj(x), None

    def _proj_segments(self):
        """Column segments (of at most 256) m3b_in_proj cuts the projection row into."""
        NR, W = self.d_state * self.mimo_rank, self.in_proj.weight.shape[0]
        bc_end = 2 * self.d_inner + 2 * self.ngroups * NR
        return -(-2 * self.d_inner // 256) + 2 * self.ngroups * -(-NR // 256) + -(-(W - bc_end) // 256)

    def _needs_grad(self, x):
        return torch.is_grad_enabled() and (x.requires_grad or any(p.requires_grad for p in self.parameters()))

    def _ssd_train(self, proj, dt_scale, return_state):
        """Differentiable path between in_proj and out_proj (mamba3/mamba3.py:192-256): torch ops
        for the split and dt; library kernels (forward and backward) for the B/C norm + bias +
        rotation + shift (_BCFn), the x-side MIMO expansion and trapezoid weights (_XFn),
        chunked_ssd and the gate (_GateFn).  Parameters are cast to the activation dtype (so fp32
        master weights train under autocast); the returned angle state is fp32, as everywhere in
        this package.  -> y (B,T,d_inner) [, state]."""
        Bat, T, _ = proj.shape
        H, P, N, R, G = self.nheads, self.headdim, self.d_state, self.mimo_rank, self.ngroups
        sizes = [self.d_inner, self._d_x, self._d_bc, self._d_bc, H]
        sizes += [H] if self.use_trapezoidal else []
        sizes += [N // 2] if self.use_complex_ssm else []
        parts = list(torch.split(proj, sizes, dim=-1))
        z, xf, Bf, Cf, dt_raw = parts[:5]
        lam_raw = parts[5] if self.use_trapezoidal else None
        theta = parts[-1] if self.use_complex_ssm else None
        dt = F.softplus(dt_raw + self.dt_bias)
        if dt_scale is not None:
            dt = dt * dt_scale
        A = -torch.exp(self.A_log)
        ad = proj.dtype
        if not self._bc_kernel_ok(proj, dt):
            raise _lib.M3bError("training path: the B / C kernels take CUDA activations, H * d_state / 2 <= 2048 "
                                "and equal B / C norm eps (no other path)")
        B_r, B_b, C_r = _BCFn.apply(Bf, Cf, theta, dt, self.B_norm.weight.to(ad), self.B_bias.to(ad),
                                    self.C_norm.weight.to(ad), self.C_bias.to(ad), H, self.B_norm.eps,
                                    self.use_trapezoidal)
        cum = None
        if return_state and self.use_complex_ssm:
            cum = -(dt.float()[..., None] * theta.float()[..., None, :]).sum(1, keepdim=True)  # (B,1,H,N/2)
        if not self._x_kernel_ok(proj, dt, A):
            raise _lib.M3bError("training path: the x kernels take CUDA activations, headdim <= 256 and "
                                "mimo_rank <= 4 (no other path)")
        x_r, x_g, x_b = _XFn.apply(xf, self.mimo_x.to(ad), lam_raw, dt, A)
        if not self.use_trapezoidal:
            x_g, x_b, B_b = x_r, None, None
        out = chunked_ssd(x_g, x_b, B_r, B_b, C_r, dt, A, self.D, x_r, self.chunk_size,
                          return_final_state=return_state)
        y = _gate(out.y, z, self.mimo_z, self.mimo_down).reshape(Bat, T, self.d_inner)
        if not return_state:
            return y, None
        angle = cum[:, -1].float() if cum is not None else torch.zeros(Bat, H, N // 2, device=proj.device)
        prev_bx = torch.einsum("bhnr,bhpr->bhpn", B_r[:, T - 1], x_r[:, T - 1]).float()
        return y, {"h": out.h_final.float(), "angle": angle, "prev_BX": prev_bx}

    def _x_kernel_ok(self, proj, dt, A):
        """The x kernels apply: CUDA float activations, P <= 256, R <= 4 (parameters are cast to the
        activation dtype by the caller)."""
        fl = (torch.float32, torch.bfloat16, torch.float16)
        return (proj.is_cuda and proj.dtype in fl and dt.dtype in fl and A.dtype in fl and self.headdim <= 256
                and self.mimo_rank <= 4)

    def _bc_kernel_ok(self, proj, dt):
        """The B / C kernels apply: CUDA float activations, equal norm eps, H * N / 2 <= 2048 and the
        backward's rows in shared memory (parameters are cast to the activation dtype by the caller)."""
        H, N, R, G = self.nheads, self.d_state, self.mimo_rank, self.ngroups
        floats = 10 * G * N * R + 2 * H * N * R + 2 * N * R + 4 * G
        return (proj.is_cuda and proj.dtype in (torch.float32, torch.bfloat16, torch.float16)
                and dt.dtype in (torch.float32, torch.bfloat16, torch.float16)
                and self.B_norm.eps == self.C_norm.eps and H * (N // 2) <= 2048 and floats * 4 <= 200 * 1024)

    def _ssd(self, x, dt_scale, return_state, state=None):
        _check_tokens(x)
        proj, rms = self._project(x)
        st = state or {}
        if self._needs_grad(x):
            if st:
                raise NotImplementedError("prefill from a state with gradients enabled")
            y, out_st = self._ssd_train(proj, dt_scale, return_state)
            return self.out_proj(y), out_st
        if "prev_B" in st:  # compact state in, compact state out
            if dt_scale is not None:
                raise NotImplementedError("dt_scale with a compact state")
            y, out_st = ops.layer_state_compact(proj, self._param_tensors(), self._dims_tuple(), st)
            return self.out_proj(y), out_st
        y, h, angle, prev_bx = ops.layer_ssd(proj, *self._param_tensors(), dt_scale, st.get("h"), st.get("angle"),
                                             st.get("prev_BX"), **self._dims(), return_state=return_state,
                                             rms=rms)
        out = self.out_proj(y)
        if not return_state:
            return out, None
        return out, {"h": h, "angle": angle, "prev_BX": prev_bx}

    # -- reference API -------------------------------------------------------
    def forward(self, x, dt_scale=None):
        """(B, T, d_model) -> (B, T, d_model)   (mamba3/mamba3.py:260-262)."""
        return self._ssd(x, dt_scale, False)[0]

    def prefill(self, x, dt_scale=None, compact_state=False):
        """Forward plus the inference state after the last token (mamba3/mamba3.py:264-265).
        compact_state=True (extension) returns the compact state of allocate_inference_state."""
        if compact_state:
            if dt_scale is not None:
                raise NotImplementedError("dt_scale with a compact state")
            _check_tokens(x)
            y, st = ops.layer_state_compact(self.in_proj(x), self._param_tensors(), self._dims_tuple())
            return self.out_proj(y), st
        return self._ssd(x, dt_scale, True)

    def prefill_from(self, x, ssm_state, dt_scale=None):
        """Continue a prefill from an inference state (chunked prefill; no reference counterpart)."""
        return self._ssd(x, dt_scale, True, ssm_state)

    def forward_host(self, x_host, out=None, pieces=4, graph=False):
        """forward() of a batch held in pinned host memory, streamed through the GPU in `pieces`
        token ranges (no reference counterpart): the host->device copy of range i+1, the layer on
        range i and the device->host copy of range i-1 run on three streams and overlap, the
        state crossing range boundaries as in prefill_from.  Returns `out` (pinned host memory,
        allocated when None).  The caller's current stream is ordered after the last copy.

        graph=True captures the whole streamed forward for this (x_host, out) pair in a CUDA
        graph on first use and replays it afterwards: the same work without the per-range host
        overhead.  The graph keeps reading x_host and writing out, so it is only for callers that
        reuse the same pinned buffers (and the same weights) from call to call."""
        if x_host.is_cuda or x_host.dim() != 3 or not x_host.is_pinned():
            raise ValueError("forward_host expects a pinned host tensor (batch, seqlen, d_model)")
        dev = self.in_proj.weight.device
        B, T, D = x_host.shape
        if out is None:
            out = torch.empty(B, T, D, dtype=x_host.dtype, pin_memory=True)
        n = max(1, min(int(pieces), T))
        if not graph:
            self._forward_host_run(x_host, out, n, dev, [])
            return out
        cache = self.__dict__.get("_host_graphs")
        if cache is None:
            cache = {}
            object.__setattr__(self, "_host_graphs", cache)
        key = (x_host.data_ptr(), out.data_ptr(), tuple(x_host.shape), x_host.dtype, n, dev)
        if key not in cache:
            self._forward_host_run(x_host, out, n, dev, [])  # warm-up outside the capture
            torch.cuda.synchronize(dev)
            g = torch.cuda.CUDAGraph()
            s = torch.cuda.Stream(dev)
            s.wait_stream(torch.cuda.current_stream(dev))
            keep = []
            with torch.cuda.graph(g, stream=s):
                self._forward_host_run(x_host, out, n, dev, keep)
            torch.cuda.current_stream(dev).wait_stream(s)
            cache[key] = (g, keep)
        cache[key][0].replay()
        return out

    def _forward_host_run(self, x_host, out, n, dev, keep):
        from . import _lib

        B, T, D = x_host.shape
        capturing = torch.cuda.is_current_stream_capturing()
        edges = [T * i // n for i in range(n + 1)]
        span = max(edges[i + 1] - edges[i] for i in range(n))
        cmp = torch.cuda.current_stream(dev)
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        s_in.wait_stream(cmp)
        s_out.wait_stream(cmp)
        xb = [torch.empty(B, span, D, dtype=x_host.dtype, device=dev) for _ in range(2)]
        ev_in = [torch.cuda.Event() for _ in range(n)]
        ev_cmp = [torch.cuda.Event() for _ in range(n)]
        ev_out = [torch.cuda.Event() for _ in range(n)]
        state = None
        for i in range(n):
            t0, nt, k = edges[i], edges[i + 1] - edges[i], i % 2
            if i >= 2:
                s_in.wait_event(ev_cmp[i - 2])  # range i-2 has been read out of xb[k]
            _lib.copy_token_range(xb[k], 0, x_host, t0, nt, s_in)
            ev_in[i].record(s_in)
            cmp.wait_event(ev_in[i])
            y, state = self._ssd(xb[k][:, :nt], None, i + 1 < n, state)
            ev_cmp[i].record(cmp)
            s_out.wait_event(ev_cmp[i])
            _lib.copy_token_range(out, t0, y, 0, nt, s_out)
            if capturing:
                keep.append(y)  # held until the capture ends; the graph's pool keeps it after
            else:
                y.record_stream(s_out)  # its memory is not reused before this copy has run
            ev_out[i].record(s_out)
        cmp.wait_event(ev_out[n - 1])
        cmp.wait_stream(s_in)
        cmp.wait_stream(s_out)
        keep.extend(xb)

    def step(self, hidden_states, ssm_state, dt_scale=None):
        """One token: (B, d_model) or (B, 1, d_model) -> same shape, new state (mamba3/mamba3.py:267-322)."""
        squeeze = hidden_states.dim() == 2
        x_in = hidden_states if squeeze else hidden_states.squeeze(1)
        proj = self.in_proj(x_in)
        if "prev_B" in ssm_state:  # compact previous-token state (allocate_inference_state(compact=True))
            y, h, pb, px, angle = ops.step_ssm_compact(proj, *self._param_tensors(), ssm_state["h"],
                                                       ssm_state["prev_B"], ssm_state["prev_x"],
                                                       ssm_state["angle"], dt_scale, **self._dims())
            new_state = {"h": h, "angle": angle, "prev_B": pb, "prev_x": px}
        else:
            y, h, bx, angle = ops.step_ssm(proj, *self._param_tensors(), ssm_state["h"], ssm_state["prev_BX"],
                                           ssm_state["angle"], dt_scale, **self._dims())
            new_state = {"h": h, "angle": angle, "prev_BX": bx}
        out = self.out_proj(y)
        if not squeeze:
            out = out.unsqueeze(1)
        return out, new_state

    def allocate_inference_state(self, batch_size, dtype=None, device=None, compact=False):
        """Zero state {'h', 'angle', 'prev_BX'} (mamba3/mamba3.py:324-332); all fp32 (see module doc).
        compact=True (extension, opt-in) keeps the previous token as 'prev_B' (B,H,N,R) and
        'prev_x' (B,H,P,R) instead of 'prev_BX' (B,H,P,N): step() then moves half the state
        bytes per token; the outputs are the same."""
        device = device or self.in_proj.weight.device
        H, P, N = self.nheads, self.headdim, self.d_state
        f32 = dict(dtype=torch.float32, device=device)
        if compact:
            R = self.mimo_rank
            return {"h": torch.zeros(batch_size, H, P, N, **f32), "angle": torch.zeros(batch_size, H, N // 2, **f32),
                    "prev_B": torch.zeros(batch_size, H, N, R, **f32),
                    "prev_x": torch.zeros(batch_size, H, P, R, **f32)}
        return {"h": torch.zeros(batch_size, H, P, N, **f32), "angle": torch.zeros(batch_size, H, N // 2, **f32),
                "prev_BX": torch.zeros(batch_size, H, P, N, **f32)}
