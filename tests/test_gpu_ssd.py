"""chunked_ssd (pre-processed inputs, mamba3/ssd.py:118-244) on the GPU vs golden vectors and the oracle."""

import numpy as np
import pytest
import torch

import oracle
from goldens import SSD_CASES, load, max_rel
from helpers import to_np

pytestmark = pytest.mark.gpu

TOL = 2e-2  # bf16 tensor-core operands


def _t(d, k, dtype=torch.float32):
    return torch.from_numpy(d[k]).cuda().to(dtype) if k in d else None


@pytest.mark.parametrize("case", SSD_CASES)
def test_chunked_ssd_golden(case):
    from mamba3_b200 import chunked_ssd

    d = load(f"ssd_{case}")
    beta = bool(d["beta"])
    out = chunked_ssd(_t(d, "x_g"), _t(d, "x_b") if beta else None, _t(d, "B_g"), _t(d, "B_b") if beta else None,
                      _t(d, "C"), _t(d, "dt"), _t(d, "A"), _t(d, "D"), _t(d, "x_raw"), int(d["CS"]),
                      h_init=_t(d, "h_init"), return_final_state=True)
    assert out.y.dtype == torch.float32 and out.y.shape == d["y"].shape
    assert max_rel(to_np(out.y), d["y"]) < TOL
    assert max_rel(to_np(out.h_final), d["h_final"]) < TOL


@pytest.mark.parametrize("R,beta", [(1, True), (2, True), (2, False), (4, True)])
def test_chunked_ssd_bf16_vs_oracle(R, beta):
    from mamba3_b200 import chunked_ssd

    B, T, H, P, N = 2, 300, 3, 64, 128
    g = torch.Generator().manual_seed(7 + R)
    r = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
    x_g, x_b, x_raw = r(B, T, H, P, R), r(B, T, H, P, R), r(B, T, H, P, R)
    B_g, B_b, C = r(B, T, H, N, R), r(B, T, H, N, R), r(B, T, H, N, R)
    dt = torch.rand(B, T, H, generator=g) * 0.1 + 0.01
    A = -torch.exp(r(H).clamp(-4, -1))
    D = r(H)
    h_init = r(B, H, P, N)
    bf = lambda t: t.to(torch.bfloat16)  # noqa: E731
    ins = [bf(x_g), bf(x_b) if beta else None, bf(B_g), bf(B_b) if beta else None, bf(C)]
    out = chunked_ssd(*[None if t is None else t.cuda() for t in ins], dt.cuda(), A.cuda(), D.cuda(),
                      bf(x_raw).cuda(), 64, h_init=h_init.cuda(), return_final_state=True)
    n = lambda t: None if t is None else t.float().numpy().astype(np.float64)  # noqa: E731
    oy, oh = oracle.chunked_ssd(n(ins[0]), n(ins[1]), n(ins[2]), n(ins[3]), n(ins[4]), n(dt), n(A), n(D),
                                n(bf(x_raw)), 64, h_init=n(h_init), return_final_state=True)
    assert out.y.dtype == torch.bfloat16
    assert max_rel(to_np(out.y), oy) < TOL
    assert max_rel(to_np(out.h_final), oh) < TOL


def test_ssd_h_init_semantics():
    """h_init = zeros == None; a random h_init changes y (mamba3 tests :670-695)."""
    from mamba3_b200 import chunked_ssd

    B, T, H, P, R, N = 1, 16, 2, 4, 2, 8
    g = torch.Generator().manual_seed(670)
    r = lambda *s: torch.randn(*s, generator=g).cuda()  # noqa: E731
    x_g, x_b, B_g, B_b, C_t = r(B, T, H, P, R), r(B, T, H, P, R), r(B, T, H, N, R), r(B, T, H, N, R), r(B, T, H, N, R)
    dt = (torch.rand(B, T, H, generator=g) * 0.1 + 0.01).cuda()
    A = -torch.exp(torch.randn(H, generator=g).clamp(-4, -1)).cuda()
    D = torch.ones(H).cuda()
    x_raw = r(B, T, H, P, R)
    o0 = chunked_ssd(x_g, x_b, B_g, B_b, C_t, dt, A, D, x_raw, 8, return_final_state=True)
    o1 = chunked_ssd(x_g, x_b, B_g, B_b, C_t, dt, A, D, x_raw, 8, h_init=torch.zeros(B, H, P, N).cuda(),
                     return_final_state=True)
    assert (o0.y - o1.y).abs().max().item() < 1e-5
    o2 = chunked_ssd(x_g, x_b, B_g, B_b, C_t, dt, A, D, x_raw, 8, h_init=r(B, H, P, N), return_final_state=True)
    assert (o0.y - o2.y).abs().max().item() > 1e-3
