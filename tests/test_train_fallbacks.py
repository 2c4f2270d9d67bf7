"""Host-side pieces of the training path that run as torch ops: the B / C preparation and the gate
that KulaMamba falls back to when its kernels do not apply (mixed dtypes, e.g. fp32 parameters
with bf16 activations under autocast).  CPU, float64, against restatements of
mamba3/mamba3.py:203-238 written out here."""

import pytest
import torch
import torch.nn.functional as F


def _restated_bc(Bf, Cf, theta, dt, wB, bB, wC, bC, H, eps, trap):
    Bt, T, _ = Bf.shape
    G, N, R = bB.shape

    def norm(x, w, b):
        # the reference's RMSNorm takes the inverse RMS of x.float(), then casts it back
        x = x.reshape(Bt, T, G, N * R)
        inv = torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + eps).to(x.dtype)
        y = x * inv * w
        return (y.reshape(Bt, T, G, N, R) + b).repeat_interleave(H // G, dim=2)

    Br, Cr = norm(Bf, wB, bB), norm(Cf, wC, bC)
    cum = None
    if theta is not None:
        cum = torch.zeros(Bt, T, H, N // 2, dtype=Bf.dtype)
        run = torch.zeros(Bt, H, N // 2, dtype=Bf.dtype)
        for t in range(T):  # the angle as an explicit running sum
            run = run - dt[:, t, :, None] * theta[:, t, None, :]
            cum[:, t] = run
        c, s = torch.cos(cum)[..., None], torch.sin(cum)[..., None]
        out = []
        for x in (Br, Cr):
            a, b = x[..., 0::2, :], x[..., 1::2, :]
            y = torch.empty_like(x)
            y[..., 0::2, :] = a * c - b * s
            y[..., 1::2, :] = a * s + b * c
            out.append(y)
        Br, Cr = out
    Bb = None
    if trap:
        Bb = torch.zeros_like(Br)
        Bb[:, 1:] = Br[:, :-1]
    return Br, Bb, Cr, cum


@pytest.mark.parametrize("ngroups,complex_ssm,trap", [(1, True, True), (2, True, False), (1, False, True)])
def test_bc_torch_fallback_matches_restatement(ngroups, complex_ssm, trap):
    from mamba3_b200 import KulaMamba

    torch.manual_seed(ngroups * 10 + int(complex_ssm))
    m = KulaMamba(d_model=32, d_state=8, headdim=8, mimo_rank=2, ngroups=ngroups, use_complex_ssm=complex_ssm,
                  use_trapezoidal=trap).double()
    with torch.no_grad():
        for p in (m.B_norm.weight, m.C_norm.weight, m.B_bias, m.C_bias):
            p.add_(0.2 * torch.randn_like(p))
    Bt, T, H, N, R, G = 2, 9, m.nheads, m.d_state, m.mimo_rank, m.ngroups
    Bf = torch.randn(Bt, T, G * N * R, dtype=torch.float64)
    Cf = torch.randn(Bt, T, G * N * R, dtype=torch.float64)
    theta = torch.randn(Bt, T, N // 2, dtype=torch.float64) if complex_ssm else None
    dt = torch.rand(Bt, T, H, dtype=torch.float64) * 0.3
    got = m._bc_torch(Bf, Cf, theta, dt)
    want = _restated_bc(Bf, Cf, theta, dt, m.B_norm.weight, m.B_bias, m.C_norm.weight, m.C_bias, H,
                        m.B_norm.eps, trap)
    for g, w in zip(got, want):
        assert (g is None) == (w is None)
        if g is not None:
            torch.testing.assert_close(g, w, rtol=1e-12, atol=1e-12)


def test_gate_torch_fallback_matches_reference_expression():
    """On CPU tensors _gate takes the torch expression: (y * silu(z * mimo_z) * mimo_down).sum(-1)."""
    from mamba3_b200.mamba3 import _gate

    g = torch.Generator().manual_seed(3)
    Bt, T, H, P, R = 2, 5, 3, 4, 2
    y = torch.randn(Bt, T, H, P, R, generator=g, dtype=torch.float64)
    z = torch.randn(Bt, T, H * P, generator=g, dtype=torch.float64)
    mz = torch.randn(H, P, R, generator=g, dtype=torch.float64)
    md = torch.randn(H, P, R, generator=g, dtype=torch.float64)
    want = (y * F.silu(z.reshape(Bt, T, H, P, 1) * mz) * md).sum(-1).reshape(Bt, T, H * P)
    torch.testing.assert_close(_gate(y, z, mz, md), want, rtol=1e-12, atol=1e-12)
