"""torch.library custom ops over the C ABI.

Each op allocates its outputs with torch (the library itself never allocates)
and has a fake implementation so the modules trace under
``torch.compile(fullgraph=True)`` as single opaque nodes.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib
from .profiling import current_stage_events

# Which layer-forward algorithm m3b_layer_fwd runs: 0 automatic, 1 fused sequential,
# 2 chunk-parallel.  Both compute the same result; tests and benches pin one.
_LAYER_ALGO = 0


def set_layer_algo(algo: int) -> int:
    global _LAYER_ALGO
    prev, _LAYER_ALGO = _LAYER_ALGO, int(algo)
    return prev


def _prm(H, P, N, R, G, trap, cplx, eps, A_log, D, dt_bias, Bw, Cw, Bb, Cb, mx, mz, md):
    return _lib.layer_params(H, P, N, R, G, trap, cplx, eps, A_log, D, dt_bias, Bw, Cw, Bb, Cb, mx, mz, md)


# ---------------------------------------------------------------------------
# inter-chunk scan
# ---------------------------------------------------------------------------
@torch.library.custom_op("mamba3_b200::scan_fwd", mutates_args=())
def scan_fwd(decay: torch.Tensor, h_chunk: torch.Tensor, h_init: Optional[torch.Tensor]) -> torch.Tensor:
    hc = h_chunk if h_chunk.dtype in (torch.float32, torch.bfloat16) else h_chunk.float()
    hc = hc.contiguous()
    d = decay.float().contiguous()
    hi = None if h_init is None else h_init.float().contiguous()
    out = _lib.scan_fwd(d, hc, hi)
    return out if out.dtype == h_chunk.dtype else out.to(h_chunk.dtype)


@scan_fwd.register_fake
def _(decay, h_chunk, h_init):
    return torch.empty_like(h_chunk)


@torch.library.custom_op("mamba3_b200::scan_bwd", mutates_args=())
def scan_bwd(decay: torch.Tensor, h_states: torch.Tensor, grad_h: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor,
                                                                                          torch.Tensor]:
    """fp32 backward of the scan (mamba3/scan.py:102-140): (d_decay, d_chunk, d_h_init), all fp32;
    the caller drops d_h_init when the forward had no h_init and casts to its dtypes."""
    return _lib.scan_bwd(decay.float().contiguous(), h_states.float().contiguous(), grad_h.float().contiguous(),
                         True)


@scan_bwd.register_fake
def _(decay, h_states, grad_h):
    B, K, H, PN = h_states.shape
    f32 = dict(dtype=torch.float32, device=h_states.device)
    return torch.empty((B, K, H), **f32), torch.empty((B, K, H, PN), **f32), torch.empty((B, H, PN), **f32)


# ---------------------------------------------------------------------------
# layer forward / prefill (everything between in_proj and out_proj)
# ---------------------------------------------------------------------------
@torch.library.custom_op("mamba3_b200::layer_ssd", mutates_args=())
def layer_ssd(proj: torch.Tensor, A_log: torch.Tensor, D: torch.Tensor, dt_bias: torch.Tensor,
              B_norm_w: torch.Tensor, C_norm_w: torch.Tensor, B_bias: torch.Tensor, C_bias: torch.Tensor,
              mimo_x: torch.Tensor, mimo_z: torch.Tensor, mimo_down: torch.Tensor,
              dt_scale: Optional[torch.Tensor], h_init: Optional[torch.Tensor], angle_init: Optional[torch.Tensor],
              prev_bx_init: Optional[torch.Tensor],
              H: int, P: int, N: int, R: int, G: int, trapezoidal: bool, complex_ssm: bool, norm_eps: float,
              return_state: bool, rms: Optional[torch.Tensor] = None
              ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """rms: the (B*T, G, 2) 1/rms rows of in_proj_rms for this proj (optional)."""
    Bt, T, _ = proj.shape
    proj = proj.contiguous()
    dev = proj.device
    prm = _prm(H, P, N, R, G, trapezoidal, complex_ssm, norm_eps, A_log, D, dt_bias, B_norm_w, C_norm_w,
               B_bias, C_bias, mimo_x, mimo_z, mimo_down)
    y = torch.empty(Bt, T, H * P, dtype=proj.dtype, device=dev)
    f32 = dict(dtype=torch.float32, device=dev)
    if return_state:
        h_final = torch.empty(Bt, H, P, N, **f32)
        angle = torch.empty(Bt, H, N // 2, **f32)
        prev_bx = torch.empty(Bt, H, P, N, **f32)
    else:
        h_final = angle = prev_bx = None
    ds = None if dt_scale is None else dt_scale.to(proj.dtype).expand(Bt, T, H).contiguous()
    f = lambda t: None if t is None else t.float().contiguous()  # noqa: E731
    _lib.layer_fwd(prm, proj, y, dt_scale=ds, h_init=f(h_init), angle_init=f(angle_init),
                   prev_bx_init=f(prev_bx_init), h_final=h_final, angle_final=angle, prev_bx_final=prev_bx,
                   stage_events=current_stage_events(), algo=_LAYER_ALGO, rms_in=rms)
    if not return_state:
        e = torch.empty(0, **f32)
        return y, e, e.clone(), e.clone()
    return y, h_final, angle, prev_bx


@layer_ssd.register_fake
def _(proj, A_log, D, dt_bias, B_norm_w, C_norm_w, B_bias, C_bias, mimo_x, mimo_z, mimo_down, dt_scale, h_init,
      angle_init, prev_bx_init, H, P, N, R, G, trapezoidal, complex_ssm, norm_eps, return_state, rms=None):
    Bt, T, _ = proj.shape
    y = proj.new_empty(Bt, T, H * P)
    f32 = dict(dtype=torch.float32, device=proj.device)
    if return_state:
        return (y, torch.empty(Bt, H, P, N, **f32), torch.empty(Bt, H, N // 2, **f32),
                torch.empty(Bt, H, P, N, **f32))
    e = torch.empty(0, **f32)
    return y, e, e.clone(), e.clone()


# ---------------------------------------------------------------------------
# input projection with the layer's per-token 1/rms of B and C in its epilogue
# ---------------------------------------------------------------------------
@torch.library.custom_op("mamba3_b200::in_proj_rms", mutates_args=())
def in_proj_rms(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor], H: int, P: int, N: int,
                R: int, G: int, norm_eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """(proj, rms): proj = x weight^T (+ bias) in bf16 and the (rows, G, 2) fp32 1/rms of every
    token's B and C rows (m3b_in_proj); x (..., d_model) bf16."""
    prm = _lib.LayerParams()
    prm.H, prm.P, prm.N, prm.R, prm.G, prm.norm_eps = H, P, N, R, G, norm_eps
    return _lib.in_proj(x.contiguous(), weight.contiguous(), None if bias is None else bias.contiguous(), prm=prm)


@in_proj_rms.register_fake
def _(x, weight, bias, H, P, N, R, G, norm_eps):
    rows = x.numel() // x.shape[-1]
    return (x.new_empty(*x.shape[:-1], weight.shape[0]),
            torch.empty(rows, G, 2, dtype=torch.float32, device=x.device))


# ---------------------------------------------------------------------------
# chunked SSD on pre-processed tensors (the reference's chunked_ssd)
# ---------------------------------------------------------------------------
@torch.library.custom_op("mamba3_b200::chunked_ssd", mutates_args=())
def chunked_ssd(x_g: torch.Tensor, x_b: Optional[torch.Tensor], B_g: torch.Tensor, B_b: Optional[torch.Tensor],
                C: torch.Tensor, dt: torch.Tensor, A: torch.Tensor, D: torch.Tensor, x_raw: torch.Tensor,
                h_init: Optional[torch.Tensor], return_final_state: bool) -> tuple[torch.Tensor, torch.Tensor]:
    wd = x_g.dtype if x_g.dtype in (torch.float32, torch.bfloat16) else torch.float32
    c = lambda t: None if t is None else t.to(wd).contiguous()  # noqa: E731
    xg, xb, Bg, Bb, Cc, xr = map(c, (x_g, x_b, B_g, B_b, C, x_raw))
    Bt, T, H, P, R = xg.shape
    N = Bg.shape[3]
    y = torch.empty(Bt, T, H, P, R, dtype=wd, device=xg.device)
    hf = torch.empty(Bt, H, P, N, dtype=torch.float32, device=xg.device) if return_final_state else None
    A32 = A.float().contiguous()
    D32 = D.to(A32.dtype).contiguous()
    hi = None if h_init is None else h_init.float().contiguous()
    _lib.chunked_ssd(xg, xb, Bg, Bb, Cc, dt.float().contiguous(), A32, D32, xr, y, h_init=hi, h_final=hf)
    y = y if y.dtype == x_g.dtype else y.to(x_g.dtype)
    return y, (hf if hf is not None else torch.empty(0, dtype=torch.float32, device=xg.device))


@chunked_ssd.register_fake
def _(x_g, x_b, B_g, B_b, C, dt, A, D, x_raw, h_init, return_final_state):
    Bt, T, H, P, R = x_g.shape
    N = B_g.shape[3]
    hf = (torch.empty(Bt, H, P, N, dtype=torch.float32, device=x_g.device) if return_final_state
          else torch.empty(0, dtype=torch.float32, device=x_g.device))
    return torch.empty_like(x_g), hf


_NONE = lambda dev: torch.empty(0, dtype=torch.float32, device=dev)  # noqa: E731


@torch.library.custom_op("mamba3_b200::chunked_ssd_bwd", mutates_args=())
def chunked_ssd_bwd(x_g: torch.Tensor, x_b: Optional[torch.Tensor], B_g: torch.Tensor, B_b: Optional[torch.Tensor],
                    C: torch.Tensor, dt: torch.Tensor, A: torch.Tensor, D: torch.Tensor, x_raw: torch.Tensor,
                    h_init: Optional[torch.Tensor], dy: torch.Tensor,
                    dh_final: Optional[torch.Tensor]) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                                                               torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                                                               torch.Tensor, torch.Tensor]:
    """Gradients of chunked_ssd: (dx_g, dx_b, dB_g, dB_b, dC, ddt, dA, dD, dx_raw, dh_init), in the
    activation dtype (fp32 for ddt, dA, dD, dh_init); empty tensors stand for absent inputs."""
    wd = x_g.dtype if x_g.dtype in (torch.float32, torch.bfloat16) else torch.float32
    c = lambda t: None if t is None else t.to(wd).contiguous()  # noqa: E731
    f = lambda t: None if t is None else t.float().contiguous()  # noqa: E731
    A32 = A.float().contiguous()
    g = _lib.chunked_ssd_bwd(c(x_g), c(x_b), c(B_g), c(B_b), c(C), f(dt), A32, D.to(A32.dtype).contiguous(),
                             c(x_raw), c(dy), f(h_init), f(dh_final))
    dev = x_g.device
    o = lambda k: _NONE(dev) if g[k] is None else g[k]  # noqa: E731
    return (o("x_g"), o("x_b"), o("B_g"), o("B_b"), o("C"), o("dt"), o("A"), o("D"), o("x_raw"), o("h_init"))


@chunked_ssd_bwd.register_fake
def _(x_g, x_b, B_g, B_b, C, dt, A, D, x_raw, h_init, dy, dh_final):
    wd = x_g.dtype if x_g.dtype in (torch.float32, torch.bfloat16) else torch.float32
    dev = x_g.device
    e = lambda t, dtype=wd: _NONE(dev) if t is None else torch.empty(t.shape, dtype=dtype, device=dev)  # noqa: E731
    H = A.shape[0]
    return (e(x_g), e(x_b), e(B_g), e(B_b), e(C), e(dt, torch.float32), torch.empty(H, device=dev),
            torch.empty(H, device=dev), e(x_raw), e(h_init, torch.float32))


# ---------------------------------------------------------------------------
# RMSNorm of the blocks (mamba3/mamba3.py:19-35)
# ---------------------------------------------------------------------------
@torch.library.custom_op("mamba3_b200::rmsnorm", mutates_args=())
def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    return _lib.rmsnorm(x.contiguous(), weight.to(x.dtype), eps)


@rmsnorm.register_fake
def _(x, weight, eps):
    return torch.empty_like(x)


@torch.library.custom_op("mamba3_b200::swiglu_act", mutates_args=())
def swiglu_act(g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    return _lib.swiglu_act(g.contiguous(), u.contiguous())


@swiglu_act.register_fake
def _(g, u):
    return torch.empty_like(g)


@torch.library.custom_op("mamba3_b200::swiglu_rows", mutates_args=())
def swiglu_rows(gu: torch.Tensor) -> torch.Tensor:
    return _lib.swiglu_rows(gu.contiguous())


@swiglu_rows.register_fake
def _(gu):
    return gu.new_empty(*gu.shape[:-1], gu.shape[-1] // 2)


@torch.library.custom_op("mamba3_b200::add_rmsnorm", mutates_args=())
def add_rmsnorm(x: torch.Tensor, h: torch.Tensor, scale: float, weight: torch.Tensor,
                eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    return _lib.add_rmsnorm(x.contiguous(), h.contiguous(), scale, weight.to(x.dtype), eps)


@add_rmsnorm.register_fake
def _(x, h, scale, weight, eps):
    return torch.empty_like(x), torch.empty_like(x)


@torch.library.custom_op("mamba3_b200::scaled_add", mutates_args=())
def scaled_add(x: torch.Tensor, h: torch.Tensor, scale: float) -> torch.Tensor:
    return _lib.scaled_add(x.contiguous(), h.contiguous(), scale)


@scaled_add.register_fake
def _(x, h, scale):
    return torch.empty_like(x)


@torch.library.custom_op("mamba3_b200::gate_fwd", mutates_args=())
def gate_fwd(y: torch.Tensor, z: torch.Tensor, mimo_z: torch.Tensor, mimo_down: torch.Tensor) -> torch.Tensor:
    return _lib.gate_fwd(y, z, mimo_z, mimo_down)


@gate_fwd.register_fake
def _(y, z, mimo_z, mimo_down):
    return y.new_empty(*y.shape[:-3], y.shape[-3] * y.shape[-2])


@torch.library.custom_op("mamba3_b200::gate_bwd", mutates_args=())
def gate_bwd(y: torch.Tensor, z: torch.Tensor, mimo_z: torch.Tensor, mimo_down: torch.Tensor,
             dout: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    return _lib.gate_bwd(y, z, mimo_z, mimo_down, dout)


@gate_bwd.register_fake
def _(y, z, mimo_z, mimo_down, dout):
    return (torch.empty_like(y), y.new_empty(*y.shape[:-3], y.shape[-3] * y.shape[-2]),
            torch.empty_like(mimo_z), torch.empty_like(mimo_down))


@torch.library.custom_op("mamba3_b200::bc_fwd", mutates_args=())
def bc_fwd(Bf: torch.Tensor, Cf: torch.Tensor, theta: Optional[torch.Tensor], dt: torch.Tensor, wB: torch.Tensor,
           bB: torch.Tensor, wC: torch.Tensor, bC: torch.Tensor, H: int, eps: float,
           shift: bool) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    return _lib.bc_fwd(Bf, Cf, theta, dt, wB, bB, wC, bC, H, eps, shift)


@bc_fwd.register_fake
def _(Bf, Cf, theta, dt, wB, bB, wC, bC, H, eps, shift):
    G, N, R = bB.shape
    shape = (*Bf.shape[:2], H, N, R)
    return Bf.new_empty(shape), Bf.new_empty(shape if shift else (0,)), Bf.new_empty(shape)


@torch.library.custom_op("mamba3_b200::bc_bwd", mutates_args=())
def bc_bwd(Bf: torch.Tensor, Cf: torch.Tensor, theta: Optional[torch.Tensor], dt: torch.Tensor, wB: torch.Tensor,
           bB: torch.Tensor, wC: torch.Tensor, bC: torch.Tensor, dB_g: torch.Tensor, dB_b: Optional[torch.Tensor],
           dC: torch.Tensor, H: int, eps: float, shift: bool) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor,
                                                                     torch.Tensor, torch.Tensor, torch.Tensor,
                                                                     torch.Tensor, torch.Tensor]:
    return _lib.bc_bwd(Bf, Cf, theta, dt, wB, bB, wC, bC, dB_g, dB_b, dC, H, eps, shift)


@bc_bwd.register_fake
def _(Bf, Cf, theta, dt, wB, bB, wC, bC, dB_g, dB_b, dC, H, eps, shift):
    G, N, R = bB.shape
    rot = theta is not None
    return (Bf.new_empty(*Bf.shape[:2], G * N * R), Bf.new_empty(*Bf.shape[:2], G * N * R),
            Bf.new_empty((*Bf.shape[:2], N // 2) if rot else (0,)), dt.new_empty(dt.shape if rot else (0,)),
            torch.empty_like(wB), torch.empty_like(bB), torch.empty_like(wC), torch.empty_like(bC))


@torch.library.custom_op("mamba3_b200::xprep_fwd", mutates_args=())
def xprep_fwd(xf: torch.Tensor, mimo_x: torch.Tensor, lam_raw: Optional[torch.Tensor], dt: torch.Tensor,
              A: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    return _lib.xprep_fwd(xf, mimo_x, lam_raw, dt, A)


@xprep_fwd.register_fake
def _(xf, mimo_x, lam_raw, dt, A):
    shape = (*xf.shape[:2], *mimo_x.shape)
    other = shape if lam_raw is not None else (0,)
    return xf.new_empty(shape), xf.new_empty(other), xf.new_empty(other)


@torch.library.custom_op("mamba3_b200::xprep_bwd", mutates_args=())
def xprep_bwd(xf: torch.Tensor, mimo_x: torch.Tensor, lam_raw: Optional[torch.Tensor], dt: torch.Tensor,
              A: torch.Tensor, dx_raw: torch.Tensor, dx_g: Optional[torch.Tensor],
              dx_b: Optional[torch.Tensor]) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                                                     torch.Tensor]:
    return _lib.xprep_bwd(xf, mimo_x, lam_raw, dt, A, dx_raw, dx_g, dx_b)


@xprep_bwd.register_fake
def _(xf, mimo_x, lam_raw, dt, A, dx_raw, dx_g, dx_b):
    trap = lam_raw is not None
    return (xf.new_empty(*xf.shape[:2], mimo_x.shape[0] * mimo_x.shape[1]), torch.empty_like(mimo_x),
            xf.new_empty(dt.shape if trap else (0,)), dt.new_empty(dt.shape if trap else (0,)),
            A.new_empty(A.shape if trap else (0,)))


def kernel_ok(*ts) -> bool:
    """True when the element-wise block kernels apply: CUDA tensors of one float dtype and shape,
    and no autograd through them (training keeps the torch ops and their backward)."""
    t0 = ts[0]
    if not t0.is_cuda or t0.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        return False
    if any(t.shape != t0.shape or t.dtype != t0.dtype or t.device != t0.device for t in ts):
        return False
    return not (torch.is_grad_enabled() and any(t.requires_grad for t in ts))


# ---------------------------------------------------------------------------
# decode step (everything between in_proj and out_proj of KulaMamba.step)
# ---------------------------------------------------------------------------
@torch.library.custom_op("mamba3_b200::step_ssm", mutates_args=())
def step_ssm(proj: torch.Tensor, A_log: torch.Tensor, D: torch.Tensor, dt_bias: torch.Tensor,
             B_norm_w: torch.Tensor, C_norm_w: torch.Tensor, B_bias: torch.Tensor, C_bias: torch.Tensor,
             mimo_x: torch.Tensor, mimo_z: torch.Tensor, mimo_down: torch.Tensor,
             h: torch.Tensor, prev_bx: torch.Tensor, angle: torch.Tensor, dt_scale: Optional[torch.Tensor],
             H: int, P: int, N: int, R: int, G: int, trapezoidal: bool, complex_ssm: bool,
             norm_eps: float) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    Bt = proj.shape[0]
    proj = proj.contiguous()
    prm = _prm(H, P, N, R, G, trapezoidal, complex_ssm, norm_eps, A_log, D, dt_bias, B_norm_w, C_norm_w,
               B_bias, C_bias, mimo_x, mimo_z, mimo_down)
    h = h.float().contiguous()
    prev_bx = prev_bx.float().contiguous()
    angle = angle.contiguous()
    h_out = torch.empty_like(h)
    bx_out = torch.empty_like(prev_bx)
    angle_out = torch.empty(angle.shape, dtype=torch.float32, device=proj.device)
    y = torch.empty(Bt, H * P, dtype=proj.dtype, device=proj.device)
    ds = None if dt_scale is None else dt_scale.to(proj.dtype).reshape(Bt, -1).expand(Bt, H).contiguous()
    _lib.step(prm, proj, ds, h, prev_bx, angle, h_out, bx_out, angle_out, y)
    return y, h_out, bx_out, angle_out


@step_ssm.register_fake
def _(proj, A_log, D, dt_bias, B_norm_w, C_norm_w, B_bias, C_bias, mimo_x, mimo_z, mimo_down, h, prev_bx, angle,
      dt_scale, H, P, N, R, G, trapezoidal, complex_ssm, norm_eps):
    Bt = proj.shape[0]
    return (proj.new_empty(Bt, H * P), torch.empty_like(h, dtype=torch.float32),
            torch.empty_like(prev_bx, dtype=torch.float32), torch.empty(angle.shape, dtype=torch.float32,
                                                                        device=proj.device))


def step_ssm_(prm_tensors, dims, proj, h, prev_bx, angle, y, dt_scale=None, workspace=None):
    """In-place decode step for CUDA-graph loops: updates h, prev_bx, angle (fp32) and writes y.
    Returns the step workspace (pass it back in to reuse it)."""
    H, P, N, R, G, trap, cplx, eps = dims
    prm = _prm(H, P, N, R, G, trap, cplx, eps, *prm_tensors)
    return _lib.step(prm, proj, dt_scale, h, prev_bx, angle, h, prev_bx, angle, y, workspace=workspace)


# ---------------------------------------------------------------------------
# compact decode step: previous token as (B^ (N, R), x_r (P, R)) instead of prev_BX (P, N)
# ---------------------------------------------------------------------------
@torch.library.custom_op("mamba3_b200::step_ssm_compact", mutates_args=())
def step_ssm_compact(proj: torch.Tensor, A_log: torch.Tensor, D: torch.Tensor, dt_bias: torch.Tensor,
                     B_norm_w: torch.Tensor, C_norm_w: torch.Tensor, B_bias: torch.Tensor, C_bias: torch.Tensor,
                     mimo_x: torch.Tensor, mimo_z: torch.Tensor, mimo_down: torch.Tensor,
                     h: torch.Tensor, prev_b: torch.Tensor, prev_x: torch.Tensor, angle: torch.Tensor,
                     dt_scale: Optional[torch.Tensor], H: int, P: int, N: int, R: int, G: int, trapezoidal: bool,
                     complex_ssm: bool, norm_eps: float
                     ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    Bt = proj.shape[0]
    proj = proj.contiguous()
    prm = _prm(H, P, N, R, G, trapezoidal, complex_ssm, norm_eps, A_log, D, dt_bias, B_norm_w, C_norm_w,
               B_bias, C_bias, mimo_x, mimo_z, mimo_down)
    h = h.float().contiguous()
    prev_b = prev_b.float().contiguous()
    prev_x = prev_x.float().contiguous()
    angle = angle.contiguous()
    h_out = torch.empty_like(h)
    b_out = torch.empty_like(prev_b)
    x_out = torch.empty_like(prev_x)
    angle_out = torch.empty(angle.shape, dtype=torch.float32, device=proj.device)
    y = torch.empty(Bt, H * P, dtype=proj.dtype, device=proj.device)
    ds = None if dt_scale is None else dt_scale.to(proj.dtype).reshape(Bt, -1).expand(Bt, H).contiguous()
    _lib.step(prm, proj, ds, h, None, angle, h_out, None, angle_out, y, prev_b=prev_b, prev_x=prev_x,
              prev_b_out=b_out, prev_x_out=x_out)
    return y, h_out, b_out, x_out, angle_out


@step_ssm_compact.register_fake
def _(proj, A_log, D, dt_bias, B_norm_w, C_norm_w, B_bias, C_bias, mimo_x, mimo_z, mimo_down, h, prev_b, prev_x,
      angle, dt_scale, H, P, N, R, G, trapezoidal, complex_ssm, norm_eps):
    Bt = proj.shape[0]
    f = dict(dtype=torch.float32)
    return (proj.new_empty(Bt, H * P), torch.empty_like(h, **f), torch.empty_like(prev_b, **f),
            torch.empty_like(prev_x, **f), torch.empty(angle.shape, dtype=torch.float32, device=proj.device))


def step_ssm_compact_(prm_tensors, dims, proj, h, prev_b, prev_x, angle, y, dt_scale=None, workspace=None):
    """In-place compact decode step for CUDA-graph loops: updates h, prev_b, prev_x, angle.
    Returns the step workspace (pass it back in to reuse it)."""
    H, P, N, R, G, trap, cplx, eps = dims
    prm = _prm(H, P, N, R, G, trap, cplx, eps, *prm_tensors)
    return _lib.step(prm, proj, dt_scale, h, None, angle, h, None, angle, y, prev_b=prev_b, prev_x=prev_x,
                     prev_b_out=prev_b, prev_x_out=prev_x, workspace=workspace)


def layer_state_compact(proj, prm_tensors, dims, state=None):
    """Final state of the layer over proj's tokens in compact form: {'h', 'angle', 'prev_B',
    'prev_x'}; y is computed (and returned) as in the forward.  `state` (either form) is the
    state before the first token."""
    H, P, N, R, G, trap, cplx, eps = dims
    prm = _prm(H, P, N, R, G, trap, cplx, eps, *prm_tensors)
    proj = proj.contiguous()
    Bt, T, _ = proj.shape
    dev = proj.device
    f32 = dict(dtype=torch.float32, device=dev)
    y = torch.empty(Bt, T, H * P, dtype=proj.dtype, device=dev)
    out = {"h": torch.empty(Bt, H, P, N, **f32), "angle": torch.empty(Bt, H, N // 2, **f32),
           "prev_B": torch.empty(Bt, H, N, R, **f32), "prev_x": torch.empty(Bt, H, P, R, **f32)}
    st = state or {}
    pb = st.get("prev_BX")
    if pb is None and "prev_B" in st:
        pb = torch.einsum("bhnr,bhpr->bhpn", st["prev_B"].float(), st["prev_x"].float())
    f = lambda t: None if t is None else t.float().contiguous()  # noqa: E731
    _lib.layer_fwd(prm, proj, y, h_init=f(st.get("h")), angle_init=f(st.get("angle")), prev_bx_init=f(pb),
                   h_final=out["h"], angle_final=out["angle"], prev_b_final=out["prev_B"],
                   prev_x_final=out["prev_x"], stage_events=current_stage_events(), algo=_LAYER_ALGO)
    return y, out
