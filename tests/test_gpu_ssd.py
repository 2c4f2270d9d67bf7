"""chunked_ssd (pre-processed inputs, mamba3/ssd.py:118-244) on the GPU vs golden vectors and the oracle."""

import numpy as np
import pytest
import torch

import oracle
from goldens import SSD_BWD_CASES, SSD_CASES, load, max_rel
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


GRADS = ("x_g", "x_b", "B_g", "B_b", "C", "dt", "A", "D", "x_raw", "h_init")


@pytest.mark.parametrize("case", SSD_BWD_CASES)
def test_chunked_ssd_backward_golden(case):
    """Autograd through chunked_ssd (the backward kernel) == the reference's autograd gradients for
    <y, gy> + <h_final, ghf> (fp32; the backward computes in fp32, so 1e-4)."""
    from mamba3_b200 import chunked_ssd

    d = load(f"ssdbwd_{case}")
    beta = bool(d["beta"])
    final = "ghf" in d
    ins = {k: _t(d, k).requires_grad_(True) if k in d else None for k in GRADS}
    if not beta:
        ins["x_b"] = ins["B_b"] = None
    out = chunked_ssd(ins["x_g"], ins["x_b"], ins["B_g"], ins["B_b"], ins["C"], ins["dt"], ins["A"], ins["D"],
                      ins["x_raw"], int(d["CS"]), h_init=ins["h_init"], return_final_state=final)
    assert max_rel(to_np(out.y), d["y"]) < TOL
    loss = (out.y * _t(d, "gy")).sum()
    if final:
        loss = loss + (out.h_final * _t(d, "ghf")).sum()
    names = [k for k in GRADS if ins[k] is not None]
    grads = torch.autograd.grad(loss, [ins[k] for k in names])
    for k, gr in zip(names, grads):
        assert gr.dtype == ins[k].dtype and gr.shape == ins[k].shape, k
        assert max_rel(to_np(gr), d[f"d_{k}"]) < 1e-4, k


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("R,beta,T", [(2, True, 300), (1, False, 77), (4, True, 130)])
def test_chunked_ssd_backward_vs_oracle(dtype, R, beta, T):
    """The backward kernel through the C ABI at d_state 128 / headdim 64 against the fp64 oracle,
    with h_init and dh_final; bitwise identical on a second launch (no atomics)."""
    from mamba3_b200 import _lib

    B, H, P, N = 2, 3, 64, 128
    g = torch.Generator().manual_seed(31 + R + T)
    r = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
    x_g, x_b, x_raw, dy = r(B, T, H, P, R), r(B, T, H, P, R), r(B, T, H, P, R), r(B, T, H, P, R)
    B_g, B_b, C = r(B, T, H, N, R) * 0.3, r(B, T, H, N, R) * 0.3, r(B, T, H, N, R) * 0.3
    dt = torch.rand(B, T, H, generator=g) * 0.1 + 0.01
    A = -torch.exp(r(H).clamp(-4, -1))
    D = r(H)
    h_init, dhf = r(B, H, P, N), r(B, H, P, N)
    if not beta:
        x_b = B_b = None
    q = lambda t: None if t is None else t.to(dtype)  # noqa: E731
    x_g, x_b, B_g, B_b, C, x_raw, dy = map(q, (x_g, x_b, B_g, B_b, C, x_raw, dy))
    cu = lambda t: None if t is None else t.cuda().contiguous()  # noqa: E731
    args = [cu(t) for t in (x_g, x_b, B_g, B_b, C, dt, A, D, x_raw, dy, h_init, dhf)]
    got = _lib.chunked_ssd_bwd(*args)
    again = _lib.chunked_ssd_bwd(*args)
    for k in got:
        if got[k] is not None:
            assert torch.equal(got[k], again[k]), k
    npd = lambda t: None if t is None else t.double().numpy()  # noqa: E731
    exp = oracle.chunked_ssd_backward(*[npd(t) for t in (x_g, x_b, B_g, B_b, C, dt, A, D, x_raw, dy, h_init, dhf)])
    tol = 1e-4 if dtype == torch.float32 else 2e-2  # bf16 stores of the gradients
    for k, v in exp.items():
        if v is None:
            assert got[k] is None, k
            continue
        assert max_rel(to_np(got[k]), v) < (1e-4 if k in ("A", "D", "h_init", "dt") and dtype == torch.float32
                                            else tol), k


def test_chunked_ssd_backward_ragged_and_empty():
    """One token and zero tokens: gradients of the states and the head sums are still defined."""
    from mamba3_b200 import _lib

    g = torch.Generator().manual_seed(5)
    r = lambda *s: torch.randn(*s, generator=g).cuda()  # noqa: E731
    for T in (1, 0):
        B, H, P, N, R = 1, 2, 16, 32, 2
        x = [r(B, T, H, P, R), r(B, T, H, P, R), r(B, T, H, N, R), r(B, T, H, N, R), r(B, T, H, N, R)]
        dt = (torch.rand(B, T, H, generator=g) * 0.1 + 0.01).cuda()
        A, D = -torch.rand(H, generator=g).cuda() - 0.1, r(H)
        x_raw, dy, h_init, dhf = r(B, T, H, P, R), r(B, T, H, P, R), r(B, H, P, N), r(B, H, P, N)
        got = _lib.chunked_ssd_bwd(x[0], x[1], x[2], x[3], x[4], dt, A, D, x_raw, dy, h_init, dhf)
        npd = lambda t: t.double().cpu().numpy()  # noqa: E731
        exp = oracle.chunked_ssd_backward(*map(npd, (x[0], x[1], x[2], x[3], x[4], dt, A, D, x_raw, dy, h_init, dhf)))
        assert max_rel(to_np(got["h_init"]), exp["h_init"]) < 1e-5
        if T == 0:
            assert torch.equal(got["h_init"], dhf) and float(got["A"].abs().max()) == 0.0
        else:
            for k in ("x_g", "B_g", "C", "dt", "A", "D"):
                assert max_rel(to_np(got[k]), exp[k]) < 1e-4, k


@pytest.mark.parametrize("P,N,R,beta", [(96, 160, 2, True), (16, 256, 1, False)])
def test_chunked_ssd_backward_large_state_vs_oracle(P, N, R, beta):
    """State shapes past the register-tiled kernel (P > 64 or N > 128) take the shared-memory
    sweep kernel: same gradients."""
    from mamba3_b200 import _lib

    B, T, H = 1, 23, 2
    g = torch.Generator().manual_seed(P + N)
    r = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
    x_g, x_b, x_raw, dy = r(B, T, H, P, R), r(B, T, H, P, R), r(B, T, H, P, R), r(B, T, H, P, R)
    B_g, B_b, C = r(B, T, H, N, R) * 0.3, r(B, T, H, N, R) * 0.3, r(B, T, H, N, R) * 0.3
    dt = torch.rand(B, T, H, generator=g) * 0.1 + 0.01
    A, D = -torch.exp(r(H).clamp(-4, -1)), r(H)
    h_init, dhf = r(B, H, P, N), r(B, H, P, N)
    if not beta:
        x_b = B_b = None
    cu = lambda t: None if t is None else t.cuda().contiguous()  # noqa: E731
    got = _lib.chunked_ssd_bwd(*[cu(t) for t in (x_g, x_b, B_g, B_b, C, dt, A, D, x_raw, dy, h_init, dhf)])
    npd = lambda t: None if t is None else t.double().numpy()  # noqa: E731
    exp = oracle.chunked_ssd_backward(*[npd(t) for t in (x_g, x_b, B_g, B_b, C, dt, A, D, x_raw, dy, h_init, dhf)])
    for k, v in exp.items():
        if v is None:
            assert got[k] is None, k
        else:
            assert max_rel(to_np(got[k]), v) < 1e-4, k


@pytest.mark.parametrize("R,beta,T", [(2, True, 1000), (1, False, 200), (4, True, 161), (2, False, 64)])
def test_chunked_ssd_backward_tensor_cores_vs_token_sweeps(R, beta, T):
    """The tensor-core backward (chunk-level products, algo 0) against the token-sweep kernel
    (algo 1, fp32 CUDA cores, pinned to the oracle above) on the same bf16 inputs: every gradient
    within the bf16 tolerance, and bitwise identical on a second launch (no atomics)."""
    from mamba3_b200 import _lib

    B, H, P, N = 2, 3, 64, 128
    g = torch.Generator().manual_seed(7 * R + T)
    r = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
    x_g, x_b, x_raw, dy = r(B, T, H, P, R), r(B, T, H, P, R), r(B, T, H, P, R), r(B, T, H, P, R)
    B_g, B_b, C = r(B, T, H, N, R) * 0.3, r(B, T, H, N, R) * 0.3, r(B, T, H, N, R) * 0.3
    dt = torch.rand(B, T, H, generator=g) * 0.1 + 0.01
    A = -torch.exp(r(H).clamp(-4, 0))
    D = r(H)
    h_init, dhf = r(B, H, P, N), r(B, H, P, N)
    if not beta:
        x_b = B_b = None
    bf = lambda t: None if t is None else t.to(torch.bfloat16).cuda().contiguous()  # noqa: E731
    cu = lambda t: None if t is None else t.cuda().contiguous()  # noqa: E731
    args = [bf(x_g), bf(x_b), bf(B_g), bf(B_b), bf(C), cu(dt), cu(A), cu(D), bf(x_raw), bf(dy), cu(h_init), cu(dhf)]
    tc = _lib.chunked_ssd_bwd(*args, algo=0)
    again = _lib.chunked_ssd_bwd(*args, algo=0)
    sweep = _lib.chunked_ssd_bwd(*args, algo=1)
    for k in tc:
        if tc[k] is None:
            assert sweep[k] is None, k
            continue
        assert torch.equal(tc[k], again[k]), k
        err = max_rel(to_np(tc[k]), to_np(sweep[k]))
        assert err < 2e-2, (k, err)
