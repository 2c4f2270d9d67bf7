"""numpy restatement of the reference Mamba-3 layer -- TEST INFRASTRUCTURE ONLY.

Every function follows one piece of the reference (dorayaku/mamba3) and cites
it as ``file:line``.  The restatement keeps the reference's algorithm, including
its chunked "factored cumsum" formulation (``mamba3/ssd.py:44-58``) and the
per-token materialisation of the rank-contracted ``B x`` outer product
(``mamba3/ssd.py:187-205``), so that it reproduces the reference's numbers and
its cost profile when it is timed as the CPU baseline.

Arithmetic runs in ``dtype`` (float64 by default; float32 mirrors the
reference's fp32 CPU path).  Arrays use the reference's layouts:
activations (B, T, ...), states (B, H, P, N), angles (B, H, N/2).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

# ----------------------------------------------------------------------------
# elementwise helpers (torch semantics)
# ----------------------------------------------------------------------------


def softplus(x):
    """torch.nn.functional.softplus(beta=1, threshold=20) (mamba3/mamba3.py:200,278)."""
    x = np.asarray(x)
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))


def sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def silu(x):
    return x * sigmoid(x)


def rmsnorm(x, weight, eps=1e-5):
    """RMSNorm over the last dim (mamba3/mamba3.py:28-35)."""
    rms = 1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)
    return x * rms * weight


def apply_rope(t, cos, sin, N, R):
    """Pairwise rotation of (2i, 2i+1) along N, same for every rank (mamba3/mamba3.py:38-45).

    ``t``: (..., N, R); ``cos``/``sin``: (..., N/2) broadcast over the pair and rank axes.
    """
    lead = t.shape[:-2]
    rp = t.reshape(*lead, N // 2, 2, R)
    c = cos[..., None]
    s = sin[..., None]
    a = rp[..., 0, :]
    b = rp[..., 1, :]
    out = np.stack([a * c - b * s, a * s + b * c], axis=-2)
    return out.reshape(*lead, N, R)


# ----------------------------------------------------------------------------
# parameters
# ----------------------------------------------------------------------------


@dataclass
class LayerParams:
    """Parameters of one ``KulaMamba`` layer (names/shapes: mamba3/mamba3.py:95-111)."""

    d_model: int
    d_state: int
    expand: int
    headdim: int
    ngroups: int
    mimo_rank: int
    chunk_size: int
    use_trapezoidal: bool
    use_complex_ssm: bool
    in_proj_w: np.ndarray
    out_proj_w: np.ndarray
    A_log: np.ndarray
    D: np.ndarray
    dt_bias: np.ndarray
    B_norm_w: np.ndarray
    C_norm_w: np.ndarray
    B_bias: np.ndarray
    C_bias: np.ndarray
    mimo_x: np.ndarray
    mimo_z: np.ndarray
    mimo_down: np.ndarray
    in_proj_b: np.ndarray | None = None
    out_proj_b: np.ndarray | None = None
    extra: dict = field(default_factory=dict)

    @property
    def d_inner(self):
        return self.expand * self.d_model

    @property
    def nheads(self):
        return self.d_inner // self.headdim

    @classmethod
    def from_state_dict(cls, sd, *, d_model, d_state=128, expand=2, headdim=64, ngroups=None,
                        mimo_rank=2, chunk_size=64, use_trapezoidal=True, use_complex_ssm=True,
                        prefix="", dtype=np.float64):
        g = lambda k: np.asarray(sd[prefix + k], dtype=dtype)  # noqa: E731
        opt = lambda k: (np.asarray(sd[prefix + k], dtype=dtype)  # noqa: E731
                         if (prefix + k) in sd and sd[prefix + k] is not None else None)
        return cls(
            d_model=d_model, d_state=d_state, expand=expand, headdim=headdim,
            ngroups=ngroups if ngroups is not None else 1, mimo_rank=max(mimo_rank, 1),
            chunk_size=chunk_size, use_trapezoidal=use_trapezoidal, use_complex_ssm=use_complex_ssm,
            in_proj_w=g("in_proj.weight"), out_proj_w=g("out_proj.weight"),
            in_proj_b=opt("in_proj.bias"), out_proj_b=opt("out_proj.bias"),
            A_log=g("A_log"), D=g("D"), dt_bias=g("dt_bias"),
            B_norm_w=g("B_norm.weight"), C_norm_w=g("C_norm.weight"),
            B_bias=g("B_bias"), C_bias=g("C_bias"),
            mimo_x=g("mimo_x"), mimo_z=g("mimo_z"), mimo_down=g("mimo_down"),
        )


def _linear(x, w, b=None):
    y = x @ w.T
    if b is not None:
        y = y + b
    return y


def _split_proj(p: LayerParams, proj):
    """Split of the input projection (mamba3/mamba3.py:125-140, sizes :88-95)."""
    H, N, R, G = p.nheads, p.d_state, p.mimo_rank, p.ngroups
    d_bc = G * N * R
    sizes = [p.d_inner, p.d_inner, d_bc, d_bc, H]
    if p.use_trapezoidal:
        sizes.append(H)
    if p.use_complex_ssm:
        sizes.append(N // 2)
    offs = np.cumsum([0] + sizes)
    parts = [proj[..., offs[i]:offs[i + 1]] for i in range(len(sizes))]
    z, x, B, C, dt_raw = parts[:5]
    idx = 5
    lam_raw = theta = None
    if p.use_trapezoidal:
        lam_raw = parts[idx]
        idx += 1
    if p.use_complex_ssm:
        theta = parts[idx]
    return z, x, B, C, dt_raw, lam_raw, theta


def _expand_groups(p: LayerParams, t, axis):
    """repeat_interleave groups -> heads (mamba3/mamba3.py:142-145)."""
    hpg = p.nheads // p.ngroups
    return t if hpg == 1 else np.repeat(t, hpg, axis=axis)


def _process_BC_train(p: LayerParams, B_flat, C_flat, dt, theta):
    """B/C joint N*R RMSNorm, bias, group expansion, RoPE (mamba3/mamba3.py:147-168)."""
    Bat, T = dt.shape[:2]
    G, N, R = p.ngroups, p.d_state, p.mimo_rank
    B_r = rmsnorm(B_flat.reshape(Bat, T, G, N * R), p.B_norm_w).reshape(Bat, T, G, N, R) + p.B_bias
    C_r = rmsnorm(C_flat.reshape(Bat, T, G, N * R), p.C_norm_w).reshape(Bat, T, G, N, R) + p.C_bias
    B_r = _expand_groups(p, B_r, axis=2)
    C_r = _expand_groups(p, C_r, axis=2)
    cum_angles = None
    if p.use_complex_ssm and theta is not None:
        angle_inc = dt[..., :, None] * theta[..., None, :]           # (B,T,H,N/2)
        cum_angles = -np.cumsum(angle_inc, axis=1)
        c, s = np.cos(cum_angles), np.sin(cum_angles)
        B_r = apply_rope(B_r, c, s, N, R)
        C_r = apply_rope(C_r, c, s, N, R)
    return B_r, C_r, cum_angles


def _process_BC_step(p: LayerParams, B_flat, C_flat, dt, theta, angle_state):
    """Single-token version (mamba3/mamba3.py:170-190)."""
    Bat = B_flat.shape[0]
    G, N, R = p.ngroups, p.d_state, p.mimo_rank
    B_r = rmsnorm(B_flat.reshape(Bat, G, N * R), p.B_norm_w).reshape(Bat, G, N, R) + p.B_bias
    C_r = rmsnorm(C_flat.reshape(Bat, G, N * R), p.C_norm_w).reshape(Bat, G, N, R) + p.C_bias
    B_r = _expand_groups(p, B_r, axis=1)
    C_r = _expand_groups(p, C_r, axis=1)
    if p.use_complex_ssm and theta is not None:
        angle_inc = dt[..., :, None] * theta[..., None, :]
        angle_state = angle_state - angle_inc
        c, s = np.cos(angle_state), np.sin(angle_state)
        B_r = apply_rope(B_r, c, s, N, R)
        C_r = apply_rope(C_r, c, s, N, R)
    return B_r, C_r, angle_state


# ----------------------------------------------------------------------------
# inter-chunk scan and chunked SSD
# ----------------------------------------------------------------------------


def ssd_scan(decay, h_chunk, h_init=None):
    """Exclusive decay scan over chunks (mamba3/scan.py:34-44, mamba3/csrc/scan.cu:10-50).

    ``decay`` (B,K,H), ``h_chunk`` (B,K,H,PN), ``h_init`` (B,H,PN) or None ->
    ``h_states`` (B,K,H,PN) with h_states[0]=h_init, h_states[k+1]=decay[k]*h_states[k]+h_chunk[k].
    """
    B, K, H = decay.shape
    PN = h_chunk.shape[-1]
    h = np.zeros((B, H, PN), dtype=h_chunk.dtype) if h_init is None else np.array(h_init, dtype=h_chunk.dtype)
    out = np.empty((B, K, H, PN), dtype=h_chunk.dtype)
    out[:, 0] = h
    for k in range(K - 1):
        h = h * decay[:, k, :, None] + h_chunk[:, k]
        out[:, k + 1] = h
    return out


def ssd_scan_backward(decay, h_states, grad_h, has_h_init=False):
    """Gradients of ``ssd_scan`` (mamba3/scan.py:47-62, mamba3/csrc/scan.cu:52-126).

    The carry g starts at grad_h[:, K-1]; walking k = K-2 .. 0, chunk k's gradient is the
    carry g_{k+1}, the decay's is sum_j g_{k+1}[j] h_states[:, k, j], and the carry becomes
    grad_h[:, k] + decay[:, k] g_{k+1}.  The last chunk's gradients are zero; d_h_init is g_0.
    Returns (d_decay (B,K,H), d_chunk (B,K,H,PN), d_h_init (B,H,PN) or None).
    """
    B, K, H, PN = h_states.shape
    g = np.array(grad_h[:, K - 1], dtype=np.float64)
    d_decay = np.zeros((B, K, H))
    d_chunk = np.zeros((B, K, H, PN))
    for k in range(K - 2, -1, -1):
        d_chunk[:, k] = g
        d_decay[:, k] = (g * h_states[:, k]).sum(-1)
        g = grad_h[:, k] + decay[:, k, :, None] * g
    return d_decay, d_chunk, (g if has_h_init else None)


def chunked_ssd_backward(x_g, x_b, B_g, B_b, C, dt, A, D, x_raw, dy, h_init=None, dh_final=None):
    """Gradients of ``chunked_ssd`` (mamba3/ssd.py:118-244) -- what torch autograd returns
    through _IntraChunkFn.backward (mamba3/ssd.py:67-115), SSDScanFn.backward
    (mamba3/scan.py:102-140) and the surrounding torch ops -- for the loss
    <y, dy> + <h_final, dh_final>.

    The chunked forward is the token recurrence h_t = exp(A dt_t) h_{t-1} + dt_t Xt_t Bt_t^T
    (Xt = [x_g | x_b], Bt = [B_g | B_b]), y_t = h_t C_t + D x_raw_t, h_final = h_{T-1}; its
    gradients follow by the chain rule backwards in time with G_t = dL/dh_t.  Every state h_t
    is kept (small cases only), so the decay terms use <G_t, h_{t-1}> directly.
    Returns a dict: x_g, x_b, B_g, B_b, C, dt, A, D, x_raw, h_init (None where absent).
    """
    f = lambda a: None if a is None else np.asarray(a, dtype=np.float64)  # noqa: E731
    x_g, x_b, B_g, B_b, C, dt, A, D, x_raw, dy, h_init, dh_final = map(
        f, (x_g, x_b, B_g, B_b, C, dt, A, D, x_raw, dy, h_init, dh_final))
    Bat, T, H, P, R = x_g.shape
    N = B_g.shape[3]
    X2 = x_g if x_b is None else np.concatenate([x_g, x_b], axis=-1)   # (B,T,H,P,RI)
    B2 = B_g if B_b is None else np.concatenate([B_g, B_b], axis=-1)   # (B,T,H,N,RI)
    a = np.exp(A[None, None, :] * dt)                                  # (B,T,H)
    hs = np.empty((T + 1, Bat, H, P, N))                                # hs[t + 1] = h_t
    hs[0] = 0.0 if h_init is None else h_init
    for t in range(T):
        u = np.einsum("bhpj,bhnj->bhpn", X2[:, t], B2[:, t])
        hs[t + 1] = a[:, t, :, None, None] * hs[t] + dt[:, t, :, None, None] * u
    dX2 = np.zeros_like(X2)
    dB2 = np.zeros_like(B2)
    dC = np.einsum("tbhpn,bthpq->bthnq", hs[1:], dy)
    ddt = np.zeros_like(dt)
    dA = np.zeros(H)
    G = np.zeros((Bat, H, P, N)) if dh_final is None else dh_final.copy()
    a_next = np.ones((Bat, H))
    for t in range(T - 1, -1, -1):
        G = a_next[:, :, None, None] * G + np.einsum("bhpq,bhnq->bhpn", dy[:, t], C[:, t])
        dX2[:, t] = dt[:, t, :, None, None] * np.einsum("bhpn,bhnj->bhpj", G, B2[:, t])
        dB2[:, t] = dt[:, t, :, None, None] * np.einsum("bhpn,bhpj->bhnj", G, X2[:, t])
        u = np.einsum("bhpj,bhnj->bhpn", X2[:, t], B2[:, t])
        q = (G * hs[t]).sum(axis=(-2, -1))                             # <G_t, h_{t-1}>
        ddt[:, t] = (G * u).sum(axis=(-2, -1)) + A[None, :] * a[:, t] * q
        dA += (dt[:, t] * a[:, t] * q).sum(axis=0)
        a_next = a[:, t]
    out = dict(x_g=dX2[..., :R], x_b=None if x_b is None else dX2[..., R:], B_g=dB2[..., :R],
               B_b=None if B_b is None else dB2[..., R:], C=dC, dt=ddt, A=dA,
               D=(dy * x_raw).sum(axis=(0, 1, 3, 4)), x_raw=D[None, None, :, None, None] * dy,
               h_init=None if h_init is None else a_next[:, :, None, None] * G)
    return out


def chunked_ssd(x_g, x_b, B_g, B_b, C, dt, A, D, x_raw, chunk_size=64, h_init=None,
                return_final_state=False):
    """Chunked SSD forward (mamba3/ssd.py:118-244) with the factored intra-chunk cumsum
    of ``_IntraChunkFn.forward`` (mamba3/ssd.py:30-65).

    Shapes as in the reference: x_g/x_b/x_raw (B,T,H,P,R), B_g/B_b/C (B,T,H,N,R),
    dt (B,T,H), A/D (H,), h_init (B,H,P,N).  Returns (y (B,T,H,P,R), h_final or None).
    Processed one batch row and one chunk at a time to bound memory; the arithmetic is
    the reference's.
    """
    Bat, T, H, P, R = x_g.shape
    N = B_g.shape[3]
    CS = chunk_size
    has_beta = x_b is not None
    K = (T + CS - 1) // CS
    Tp = K * CS
    pad = Tp - T

    def padT(a):
        if a is None or pad == 0:
            return a
        w = [(0, 0)] * a.ndim
        w[1] = (0, pad)
        return np.pad(a, w)

    x_g, x_b, B_g, B_b, C, dt, x_raw = map(padT, (x_g, x_b, B_g, B_b, C, dt, x_raw))
    y = np.empty((Bat, Tp, H, P, R), dtype=x_g.dtype)
    h_final = np.empty((Bat, H, P, N), dtype=x_g.dtype) if return_final_state else None

    for b in range(Bat):
        # ssd.py:153-162 -- per-chunk inclusive cumsum of A*dt, chunk decay
        ld = (A[None, :] * dt[b]).reshape(K, CS, H)
        cum = np.cumsum(ld, axis=1).transpose(0, 2, 1)               # (K,H,CS)
        exp_cum = np.exp(cum)
        chunk_decay = exp_cum[:, :, -1]                               # (K,H)
        h_chunk = np.empty((K, H, P, N), dtype=x_g.dtype)
        y_intra = np.empty((K, H, R, CS, P), dtype=x_g.dtype)
        for k in range(K):
            sl = slice(k * CS, (k + 1) * CS)
            dtk = dt[b, sl].T                                         # (H,CS)
            xg = x_g[b, sl].transpose(1, 0, 2, 3)                     # (H,CS,P,R)
            Bg = B_g[b, sl].transpose(1, 0, 2, 3)                     # (H,CS,N,R)
            dtx = dtk[:, :, None, None] * xg                          # ssd.py:185
            if has_beta:                                              # ssd.py:187-198
                xb = x_b[b, sl].transpose(1, 0, 2, 3)
                Bb = B_b[b, sl].transpose(1, 0, 2, 3)
                dtx = np.concatenate([dtx, dtk[:, :, None, None] * xb], axis=-1)
                Bf = np.concatenate([Bg, Bb], axis=-1)
            else:                                                     # ssd.py:200-202
                Bf = Bg
            BX = np.matmul(dtx, Bf.transpose(0, 1, 3, 2))             # (H,CS,P,N), bmm of ssd.py:198
            # _IntraChunkFn.forward, ssd.py:44-58
            enc = np.exp(-cum[k])[:, :, None, None]
            ec = exp_cum[k][:, :, None, None]
            scaled = BX * enc
            mid = ec * np.cumsum(scaled, axis=1)
            Ck = C[b, sl].transpose(1, 0, 3, 2)                       # (H,CS,R,N)
            # bmm of ssd.py:49-56: per token (R x N) . (N x P)
            y_intra[k] = np.matmul(Ck, mid.transpose(0, 1, 3, 2)).transpose(0, 2, 1, 3)
            # ssd.py:207-208
            h_chunk[k] = chunk_decay[k][:, None, None] * scaled.sum(axis=1)
        # ssd.py:210-213 -- inter-chunk scan
        hi = None if h_init is None else h_init[b].reshape(1, H, P * N)
        h_states = ssd_scan(chunk_decay[None], h_chunk.reshape(1, K, H, P * N), hi)[0].reshape(K, H, P, N)
        for k in range(K):
            sl = slice(k * CS, (k + 1) * CS)
            Ck = C[b, sl].transpose(1, 3, 0, 2)                       # (H,R,CS,N)
            # ssd.py:215-222
            y_inter = np.matmul(Ck, h_states[k].transpose(0, 2, 1)[:, None]) * exp_cum[k][:, None, :, None]
            # ssd.py:224-233
            y_d = D[:, None, None, None] * x_raw[b, sl].transpose(1, 3, 0, 2)
            tot = y_intra[k] + y_inter + y_d                          # (H,R,CS,P)
            y[b, sl] = tot.transpose(2, 0, 3, 1)
        if return_final_state:                                        # ssd.py:235-242
            h_final[b] = chunk_decay[K - 1][:, None, None] * h_states[K - 1] + h_chunk[K - 1]
    return y[:, :T], h_final


# ----------------------------------------------------------------------------
# the layer
# ----------------------------------------------------------------------------


def layer_forward(p: LayerParams, x, dt_scale=None, return_state=False):
    """``KulaMamba._forward_impl`` (mamba3/mamba3.py:192-258). x: (B,T,d_model)."""
    Bat, T, _ = x.shape
    H, P, N, R = p.nheads, p.headdim, p.d_state, p.mimo_rank
    proj = _linear(x, p.in_proj_w, p.in_proj_b)                       # :197
    z, x_flat, B_flat, C_flat, dt_raw, lam_raw, theta = _split_proj(p, proj)
    dt = softplus(dt_raw + p.dt_bias)                                 # :200
    if dt_scale is not None:
        dt = dt * dt_scale
    A = -np.exp(p.A_log)                                              # :203
    dA = np.exp(A[None, None, :] * dt)
    B_proc, C_proc, cum_angles = _process_BC_train(p, B_flat, C_flat, dt, theta)
    x_r = x_flat.reshape(Bat, T, H, P, 1) * p.mimo_x[None, None]      # :210
    if p.use_trapezoidal:                                             # :212-224
        lam = sigmoid(lam_raw)
        scale_g = lam[..., None, None]
        scale_b = ((1.0 - lam) * dA)[..., None, None]
        x_gamma = x_r * scale_g
        x_prev = np.concatenate([np.zeros_like(x_r[:, :1]), x_r[:, :-1]], axis=1)
        B_prev = np.concatenate([np.zeros_like(B_proc[:, :1]), B_proc[:, :-1]], axis=1)
        x_beta = x_prev * scale_b
    else:
        x_gamma, x_beta, B_prev = x_r, None, None
    y_ssd, h_final = chunked_ssd(x_gamma, x_beta, B_proc, B_prev, C_proc, dt, A, p.D, x_r,
                                 p.chunk_size, return_final_state=return_state)
    z_r = z.reshape(Bat, T, H, P)[..., None] * p.mimo_z[None, None]  # :234-238
    y = (y_ssd * silu(z_r) * p.mimo_down[None, None]).sum(-1).reshape(Bat, T, p.d_inner)
    out = _linear(y, p.out_proj_w, p.out_proj_b)                      # :239
    state = None
    if return_state:                                                  # :241-256
        angle = cum_angles[:, T - 1] if cum_angles is not None else np.zeros((Bat, H, N // 2), x.dtype)
        prev_BX = np.einsum("bhnr,bhpr->bhpn", B_proc[:, T - 1], x_r[:, T - 1])
        state = {"h": h_final, "angle": angle, "prev_BX": prev_BX}
    return out, state


def layer_prefill(p: LayerParams, x, dt_scale=None):
    """``KulaMamba.prefill`` (mamba3/mamba3.py:264-265)."""
    return layer_forward(p, x, dt_scale, return_state=True)


def allocate_inference_state(p: LayerParams, batch_size, dtype=np.float64):
    """``KulaMamba.allocate_inference_state`` (mamba3/mamba3.py:324-332)."""
    H, P, N = p.nheads, p.headdim, p.d_state
    return {"h": np.zeros((batch_size, H, P, N), dtype),
            "angle": np.zeros((batch_size, H, N // 2), dtype),
            "prev_BX": np.zeros((batch_size, H, P, N), dtype)}


def layer_step(p: LayerParams, hidden, state, dt_scale=None):
    """``KulaMamba.step`` (mamba3/mamba3.py:267-322). hidden: (B,d_model) or (B,1,d_model)."""
    squeeze = hidden.ndim == 2
    xin = hidden if squeeze else hidden[:, 0]
    H, P, N, R = p.nheads, p.headdim, p.d_state, p.mimo_rank
    proj = _linear(xin, p.in_proj_w, p.in_proj_b)
    z, x_flat, B_flat, C_flat, dt_raw, lam_raw, theta = _split_proj(p, proj)
    dt = softplus(dt_raw + p.dt_bias)
    if dt_scale is not None:
        dt = dt * dt_scale
    A = -np.exp(p.A_log)
    dA = np.exp(A * dt)
    B_proc, C_proc, angle_state = _process_BC_step(p, B_flat, C_flat, dt, theta, state["angle"])
    x_r = x_flat.reshape(-1, H, P, 1) * p.mimo_x[None]
    if p.use_trapezoidal:
        lam = sigmoid(lam_raw)
        gamma = lam * dt
        beta = (1.0 - lam) * dt * dA
    else:
        gamma = dt
        beta = np.zeros_like(dt)
    curr_BX = np.einsum("bhnr,bhpr->bhpn", B_proc, x_r)               # :298
    h = (dA[:, :, None, None] * state["h"] + gamma[:, :, None, None] * curr_BX
         + beta[:, :, None, None] * state["prev_BX"])                 # :303-306
    y_pr = np.einsum("bhnr,bhpn->bhpr", C_proc, h) + p.D[None, :, None, None] * x_r  # :309-310
    z_r = z.reshape(-1, H, P)[..., None] * p.mimo_z[None]
    y = (y_pr * silu(z_r) * p.mimo_down[None]).sum(-1).reshape(-1, p.d_inner)
    out = _linear(y, p.out_proj_w, p.out_proj_b)
    if not squeeze:
        out = out[:, None]
    return out, {"h": h, "angle": angle_state, "prev_BX": curr_BX}


# ----------------------------------------------------------------------------
# blocks and the language model (harness around the layer)
# ----------------------------------------------------------------------------


def swiglu(x, w_gate, w_up, w_down):
    """``SwiGLU.forward`` (mamba3/block.py:25-26)."""
    return (silu(x @ w_gate.T) * (x @ w_up.T)) @ w_down.T


@dataclass
class BlockParams:
    """One ``KulaMambaBlock`` (mamba3/block.py:29-71)."""

    ssm: LayerParams
    ssm_norm_w: np.ndarray
    residual_scale: float
    norm_eps: float = 1e-5
    mlp_norm_w: np.ndarray | None = None
    w_gate: np.ndarray | None = None
    w_up: np.ndarray | None = None
    w_down: np.ndarray | None = None


def block_forward(bp: BlockParams, x):
    """``KulaMambaBlock.forward`` (mamba3/block.py:79-92), no checkpointing."""
    h = layer_forward(bp.ssm, rmsnorm(x, bp.ssm_norm_w, bp.norm_eps))[0]
    x = x + h * bp.residual_scale
    if bp.w_gate is not None:
        x = x + swiglu(rmsnorm(x, bp.mlp_norm_w, bp.norm_eps), bp.w_gate, bp.w_up, bp.w_down) * bp.residual_scale
    return x


def block_step(bp: BlockParams, x, state):
    """``KulaMambaBlock.step`` (mamba3/block.py:94-100)."""
    h, new_state = layer_step(bp.ssm, rmsnorm(x, bp.ssm_norm_w, bp.norm_eps), state)
    x = x + h * bp.residual_scale
    if bp.w_gate is not None:
        x = x + swiglu(rmsnorm(x, bp.mlp_norm_w, bp.norm_eps), bp.w_gate, bp.w_up, bp.w_down) * bp.residual_scale
    return x, new_state


def block_prefill(bp: BlockParams, x):
    """``KulaMambaBlock.prefill`` (mamba3/block.py:102-107)."""
    h, state = layer_prefill(bp.ssm, rmsnorm(x, bp.ssm_norm_w, bp.norm_eps))
    x = x + h * bp.residual_scale
    if bp.w_gate is not None:
        x = x + swiglu(rmsnorm(x, bp.mlp_norm_w, bp.norm_eps), bp.w_gate, bp.w_up, bp.w_down) * bp.residual_scale
    return x, state


def lm_forward(embedding, blocks, norm_w, lm_head_w, input_ids, norm_eps=1e-5):
    """``KulaMambaLM.forward`` logits (mamba3/block.py:178-185)."""
    x = embedding[input_ids]
    for bp in blocks:
        x = block_forward(bp, x)
    return rmsnorm(x, norm_w, norm_eps) @ lm_head_w.T


def lm_generate(embedding, blocks, norm_w, lm_head_w, input_ids, max_new_tokens, norm_eps=1e-5):
    """Greedy ``KulaMambaLM.generate`` with temperature=0 (mamba3/block.py:195-231)."""
    x = embedding[input_ids]
    states = []
    for bp in blocks:
        x, st = block_prefill(bp, x)
        states.append(st)
    logits = rmsnorm(x, norm_w, norm_eps)[:, -1] @ lm_head_w.T
    out = [input_ids]
    for _ in range(max_new_tokens):
        nxt = logits.argmax(-1)[:, None]
        out.append(nxt)
        x = embedding[nxt[:, 0]]
        for i, bp in enumerate(blocks):
            x, states[i] = block_step(bp, x, states[i])
        logits = rmsnorm(x, norm_w, norm_eps) @ lm_head_w.T
    return np.concatenate(out, axis=1)
