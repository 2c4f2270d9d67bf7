"""The input projection with the layer's per-token prologue in its epilogue (m3b_in_proj).

proj = x W^T (+ bias) against the same product in fp32 rounded to bf16 (the kernel accumulates in
fp32 on the tensor cores in another order, so an element may land one bf16 step away), and the
1/rms of every group's B and C row against rsqrt(mean(v^2) + eps) of the kernel's own bf16 proj
row, which is what the layer forward's own pre-pass computes (mamba3/mamba3.py:200-204).
Shapes cover the layer configurations (d_model 768 / R 2, d_model 2048 / R 4 whose B and C rows
span two 256-column pieces, two groups), a row count that is not a multiple of the 128-row tile,
a d_model that is not a multiple of the 64-wide K step, and a bias.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _prm(H, P, N, R, G, eps=1e-5):
    from mamba3_b200 import _lib

    p = _lib.LayerParams()
    p.H, p.P, p.N, p.R, p.G, p.norm_eps = H, P, N, R, G, eps
    return p


def _ref_proj(x, W, b):
    y = x.float().reshape(-1, x.shape[-1]) @ W.float().t()
    if b is not None:
        y = y + b.float()
    return y


def _check_proj(proj, ref):
    got = proj.reshape(ref.shape).float()
    exact = got == ref.to(torch.bfloat16).float()
    # one bf16 step (2^-8 relative) at most; nearly every element exact
    err = ((got - ref).abs() / ref.abs().clamp_min(1e-3)).max().item()
    assert err < 8e-3, err
    assert exact.float().mean().item() > 0.97, exact.float().mean().item()


def _check_rms(proj, rms, H, P, N, R, G, eps=1e-5):
    rows = proj.shape[0] if proj.dim() == 2 else proj.shape[0] * proj.shape[1]
    p2 = proj.reshape(rows, -1).float()
    offB, NR = 2 * H * P, N * R
    for g in range(G):
        for k, off in enumerate((offB + g * NR, offB + (G + g) * NR)):
            v = p2[:, off:off + NR]
            ref = torch.rsqrt((v * v).mean(-1) + eps)
            rel = ((rms[:, g, k] - ref).abs() / ref).max().item()
            assert rel < 2e-6, (g, k, rel)


@pytest.mark.parametrize("rows,d_model,H,P,N,R,G,bias", [
    (1000, 768, 24, 64, 128, 2, 1, False),    # config 1 layer dims, a partial last row tile
    (4096, 768, 24, 64, 128, 2, 1, True),     # with a bias
    (700, 2048, 64, 64, 128, 4, 1, False),    # config 3: B / C rows of 512 in two pieces
    (300, 200, 4, 64, 128, 2, 2, False),      # two groups, d_model not a multiple of 64
    (64, 128, 4, 64, 128, 1, 1, False),       # one partial tile, rank 1
])
def test_in_proj_matches_fp32_product_and_rms(rows, d_model, H, P, N, R, G, bias):
    from mamba3_b200 import _lib

    g = torch.Generator().manual_seed(rows + d_model)
    d_proj = 2 * H * P + 2 * G * N * R + 2 * H + N // 2
    x = torch.randn(rows, d_model, generator=g).to(torch.bfloat16).cuda()
    W = (torch.randn(d_proj, d_model, generator=g) / d_model ** 0.5).to(torch.bfloat16).cuda()
    b = (0.1 * torch.randn(d_proj, generator=g)).to(torch.bfloat16).cuda() if bias else None
    proj, rms = _lib.in_proj(x, W, b, prm=_prm(H, P, N, R, G))
    torch.cuda.synchronize()
    _lib.check_device_errors()
    _check_proj(proj, _ref_proj(x, W, b))
    _check_rms(proj, rms, H, P, N, R, G)


def test_in_proj_without_rms_any_width():
    """No layer dimensions: a plain bf16 GEMM over any width that is a multiple of 8."""
    from mamba3_b200 import _lib

    g = torch.Generator().manual_seed(5)
    x = torch.randn(3, 77, 256, generator=g).to(torch.bfloat16).cuda()
    W = (torch.randn(520, 256, generator=g) / 16).to(torch.bfloat16).cuda()
    proj, rms = _lib.in_proj(x, W)
    torch.cuda.synchronize()
    assert rms is None and proj.shape == (3, 77, 520)
    _check_proj(proj, _ref_proj(x, W, None))


def test_in_proj_rejects_bad_strides_on_host():
    from mamba3_b200 import _lib

    x = torch.zeros(16, 100, dtype=torch.bfloat16, device="cuda")  # d_model not a multiple of 8
    W = torch.zeros(64, 100, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.M3bError, match="multiples of 8"):
        _lib.in_proj(x, W)


def test_layer_forward_with_fused_projection_equals_linear_path():
    """KulaMamba's inference forward takes the fused projection for bf16; the layer's output must
    match the path through nn.Linear and the layer's own pre-pass."""
    from mamba3_b200 import KulaMamba

    torch.manual_seed(0)
    m = KulaMamba(d_model=768, d_state=128, headdim=64, mimo_rank=2).cuda().to(torch.bfloat16).eval()
    x = torch.randn(4, 1000, 768, generator=torch.Generator().manual_seed(9)).to(torch.bfloat16).cuda()
    with torch.no_grad():
        proj, rms = m._project(x)
        assert rms is not None
        y_fused, st_fused = m.ssd_from_proj(proj, return_state=True, rms=rms)
        y_plain, st_plain = m.ssd_from_proj(proj, return_state=True)
        torch.cuda.synchronize()
        # same proj; the two 1/rms computations differ only in fp32 summation order
        d = (y_fused.float() - y_plain.float()).abs()
        assert (d.max() / y_plain.float().abs().max()).item() < 4e-3
        assert (d == 0).float().mean().item() > 0.99
        for k in st_plain:
            assert (st_fused[k] - st_plain[k]).abs().max().item() <= 1e-5 * st_plain[k].abs().max().item()
        lin = m.in_proj(x)
        y_lin = m.ssd_from_proj(lin)
        ref = y_lin.float()
        assert ((y_fused.float() - ref).abs().max() / ref.abs().max()).item() < 2e-2
        out = m(x)
        out_ref = m.out_proj(y_lin)
        assert ((out.float() - out_ref.float()).abs().max() / out_ref.float().abs().max()).item() < 2e-2
