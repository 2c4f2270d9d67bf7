"""Kernel-level parity on the GPU: tensor-core self-test, inter-chunk scan, decode step.

Every call goes through the C ABI of libmamba3_b200 (ctypes) and is compared with
the CPU oracle or with golden vectors from the reference.
"""

import numpy as np
import pytest
import torch

import oracle
from goldens import LAYER_CASES, SCAN_BWD_CASES, SCAN_CASES, load, max_rel
from helpers import ours_layer_from_golden, to_np

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode", [0, 1, 2, 6])
def test_umma_selftest(mode):
    """bf16 operands: A K-major, A MN-major, B MN-major (shared memory), A in tensor memory."""
    from mamba3_b200 import _lib

    g = torch.Generator().manual_seed(100 + mode)
    A = torch.randn(128, 128, generator=g).to("cuda", torch.bfloat16)
    B = torch.randn(64, 128, generator=g).to("cuda", torch.bfloat16)
    D, err = _lib.selftest_umma(A, B, mode)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = A.float() @ B.float().T
    assert max_rel(to_np(D), to_np(ref)) < 1e-5


@pytest.mark.parametrize("mode", [3])
def test_umma_selftest_tf32(mode):
    """kind::tf32 with fp32 tiles, A and B K-major (the fp32 chunk kernels' layout): the product
    of the operands as tf32 (10 mantissa bits), accumulated in fp32."""
    from mamba3_b200 import _lib

    g = torch.Generator().manual_seed(200 + mode)
    A = torch.randn(128, 128, generator=g).cuda()
    B = torch.randn(64, 128, generator=g).cuda()
    D, err = _lib.selftest_umma(A, B, mode)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    exact = A.double() @ B.double().T
    # tf32 operands (2^-11 relative per element): well inside 1e-3, where bf16 operands are not
    assert max_rel(to_np(D), to_np(exact)) < 1e-3


@pytest.mark.parametrize("case", SCAN_CASES)
def test_scan_golden(case):
    from mamba3_b200 import ssd_scan

    d = load(f"scan_{case}")
    t = lambda k: torch.from_numpy(d[k]).cuda() if k in d else None  # noqa: E731
    hs = ssd_scan(t("decay"), t("h_chunk"), t("h_init"))
    assert hs.dtype == torch.float32
    assert max_rel(to_np(hs), d["h_states"]) < 1e-6


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", [(2, 5, 3, 16), (3, 64, 24, 8192), (1, 9, 2, 100)])
@pytest.mark.parametrize("with_init", [False, True])
def test_scan_vs_oracle(dtype, shape, with_init):
    from mamba3_b200 import _lib

    B, K, H, PN = shape
    g = torch.Generator().manual_seed(sum(shape))
    decay = torch.rand(B, K, H, generator=g)
    hc = torch.randn(B, K, H, PN, generator=g).to(dtype)
    hi = torch.randn(B, H, PN, generator=g) if with_init else None
    hf = torch.empty(B, H, PN, device="cuda")
    hs = _lib.scan_fwd(decay.cuda(), hc.cuda(), None if hi is None else hi.cuda(), h_final=hf)
    exp = oracle.ssd_scan(decay.double().numpy(), hc.double().numpy(), None if hi is None else hi.double().numpy())
    fin = exp[:, -1] * decay.double().numpy()[:, -1, :, None] + hc.double().numpy()[:, -1]
    tol = 1e-5 if dtype == torch.float32 else 1e-2  # bf16 output rounding
    assert max_rel(to_np(hs), exp) < tol
    assert max_rel(to_np(hf), fin) < 1e-5


@pytest.mark.parametrize("case", SCAN_BWD_CASES)
def test_scan_backward_golden(case):
    """ssd_scan's autograd gradients (reverse-scan kernel) == the reference's SSDScanFn.backward."""
    from mamba3_b200 import ssd_scan

    d = load(f"scanbwd_{case}")
    decay = torch.from_numpy(d["decay"]).cuda().requires_grad_(True)
    hc = torch.from_numpy(d["h_chunk"]).cuda().requires_grad_(True)
    hi = torch.from_numpy(d["h_init"]).cuda().requires_grad_(True) if "h_init" in d else None
    hs = ssd_scan(decay, hc, hi)
    assert max_rel(to_np(hs), d["h_states"]) < 1e-6
    ins = [decay, hc] + ([hi] if hi is not None else [])
    grads = torch.autograd.grad(hs, ins, torch.from_numpy(d["grad_h"]).cuda())
    assert max_rel(to_np(grads[0]), d["d_decay"]) < 1e-5
    assert max_rel(to_np(grads[1]), d["d_chunk"]) < 1e-6
    if hi is not None:
        assert max_rel(to_np(grads[2]), d["d_h_init"]) < 1e-6


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", [(2, 5, 3, 16), (3, 64, 24, 8192), (1, 9, 2, 100), (2, 2, 2, 8), (1, 33, 4, 24576),
                                   (8, 4, 48, 8192)])
def test_scan_backward_vs_oracle(dtype, shape):
    """The reverse-scan kernel through the C ABI against the oracle: vector paths (one block per
    state, several blocks per state with fixed-order partial sums), the scalar path (PN = 100),
    bf16 I/O; the result is bitwise the same on a second launch."""
    from mamba3_b200 import _lib

    B, K, H, PN = shape
    g = torch.Generator().manual_seed(7 + sum(shape))
    decay = torch.rand(B, K, H, generator=g)
    hs = torch.randn(B, K, H, PN, generator=g).to(dtype)
    gh = torch.randn(B, K, H, PN, generator=g).to(dtype)
    dd, dc, dhi = _lib.scan_bwd(decay.cuda(), hs.cuda(), gh.cuda(), True)
    dd2, dc2, dhi2 = _lib.scan_bwd(decay.cuda(), hs.cuda(), gh.cuda(), True)
    assert torch.equal(dd, dd2) and torch.equal(dc, dc2) and torch.equal(dhi, dhi2)
    ed, ec, ehi = oracle.ssd_scan_backward(decay.double().numpy(), hs.double().numpy(), gh.double().numpy(), True)
    tol = 1e-5 if dtype == torch.float32 else 1e-2  # bf16 d_chunk rounding
    assert dc.dtype == dtype
    assert max_rel(to_np(dc), ec) < tol
    assert max_rel(to_np(dd), ed) < 1e-4
    assert max_rel(to_np(dhi), ehi) < 1e-5


def test_scan_backward_bf16_autograd_matches_fp32():
    """bf16 h_chunk: the states are scanned and saved in fp32 (as the reference's CUDA path
    does), so the gradients equal the fp32 gradients up to the bf16 rounding of grad_h."""
    from mamba3_b200 import ssd_scan

    g = torch.Generator().manual_seed(3)
    decay = torch.rand(2, 12, 4, generator=g).cuda()
    hc = torch.randn(2, 12, 4, 64, 128, generator=g).cuda()
    gh = torch.randn(2, 12, 4, 64, 128, generator=g).cuda()
    out = {}
    for dt in (torch.float32, torch.bfloat16):
        d = decay.clone().requires_grad_(True)
        h = hc.to(dt).requires_grad_(True)
        hs = ssd_scan(d, h)
        assert hs.dtype == dt and hs.shape == hc.shape
        out[dt] = torch.autograd.grad(hs, [d, h], gh.to(dt))
    assert out[torch.bfloat16][1].dtype == torch.bfloat16
    assert max_rel(to_np(out[torch.bfloat16][0]), to_np(out[torch.float32][0])) < 2e-2
    assert max_rel(to_np(out[torch.bfloat16][1]), to_np(out[torch.float32][1])) < 2e-2


@pytest.mark.parametrize("case", LAYER_CASES)
def test_step_golden_fp32(case):
    """Decode steps from the reference's prefill state reproduce the reference's steps (fp32, 1e-4)."""
    d = load(f"layer_{case}")
    m = ours_layer_from_golden(d, torch.float32)
    T, n = int(d["T"]), int(d["n_steps"])
    x = torch.from_numpy(d["x"]).cuda()
    st = {"h": torch.from_numpy(d["pf_h"]).cuda(), "angle": torch.from_numpy(d["pf_angle"]).cuda(),
          "prev_BX": torch.from_numpy(d["pf_prev_BX"]).cuda()}
    ys = []
    with torch.no_grad():
        for t in range(T, T + n):
            y, st = m.step(x[:, t:t + 1], st)
            ys.append(y[:, 0])
    assert max_rel(to_np(torch.stack(ys, 1)), d["y_steps"]) < 1e-4
    assert max_rel(to_np(st["h"]), d["st_h"]) < 1e-4
    assert max_rel(to_np(st["prev_BX"]), d["st_prev_BX"]) < 1e-4
    assert max_rel(to_np(st["angle"]), d["st_angle"]) < 1e-4


@pytest.mark.parametrize("case", ["perturbed", "n128p64", "rank4"])
def test_step_bf16_vs_oracle(case):
    """bf16 model: step outputs vs the fp64 oracle on the same (bf16-rounded) weights, 2e-2."""
    from helpers import oracle_params

    d = load(f"layer_{case}")
    m = ours_layer_from_golden(d, torch.bfloat16)
    p = oracle_params(m)
    x = torch.from_numpy(d["x"]).cuda().to(torch.bfloat16)
    B = x.shape[0]
    st = m.allocate_inference_state(B)
    ost = oracle.allocate_inference_state(p, B)
    xs = to_np(x)
    for t in range(min(12, x.shape[1])):
        with torch.no_grad():
            y, st = m.step(x[:, t], st)
        oy, ost = oracle.layer_step(p, xs[:, t], ost)
        assert max_rel(to_np(y), oy) < 2e-2
    assert max_rel(to_np(st["h"]), ost["h"]) < 2e-2


@pytest.mark.parametrize("compact", [False, True], ids=["prev_bx", "compact"])
@pytest.mark.parametrize("R", [1, 2, 4])
def test_step_streaming_equals_single_kernel(R, compact):
    """d_state 128: the two-kernel streaming step (operand preparation + persistent state stream
    through a shared-memory ring) and the single kernel give the same state and output, in place
    and out of place, over more (batch, head) items than the persistent grid holds."""
    from mamba3_b200 import KulaMamba, _lib, ops

    torch.manual_seed(80 + R)
    m = KulaMamba(d_model=256, d_state=128, headdim=64, mimo_rank=R).cuda().to(torch.bfloat16).eval()
    B, H, P, N = 300, m.nheads, 64, 128
    g = torch.Generator().manual_seed(81)
    x = torch.randn(B, 256, generator=g).cuda().to(torch.bfloat16)
    with torch.no_grad():
        proj = m.in_proj(x)
    st = {"h": torch.randn(B, H, P, N, generator=g), "angle": torch.randn(B, H, N // 2, generator=g),
          "pb": torch.randn(B, H, N, R, generator=g), "px": torch.randn(B, H, P, R, generator=g),
          "pbx": torch.randn(B, H, P, N, generator=g)}
    st = {k: v.cuda() for k, v in st.items()}
    prm = ops._prm(H, P, N, R, 1, True, True, m.B_norm.eps, *m._param_tensors())
    outs = []
    for streaming in (False, True):
        s2 = {k: v.clone() for k, v in st.items()}
        y = torch.empty(B, H * P, dtype=torch.bfloat16, device="cuda")
        if compact:
            ws = _lib.step(prm, proj, None, s2["h"], None, s2["angle"], s2["h"], None, s2["angle"], y,
                           prev_b=s2["pb"], prev_x=s2["px"], prev_b_out=s2["pb"], prev_x_out=s2["px"],
                           streaming=streaming)
        else:
            ws = _lib.step(prm, proj, None, s2["h"], s2["pbx"], s2["angle"], s2["h"], s2["pbx"], s2["angle"], y,
                           streaming=streaming)
        assert (ws is not None) == streaming
        outs.append((y, s2))
    torch.cuda.synchronize()
    (y0, a0), (y1, a1) = outs
    assert max_rel(to_np(y1), to_np(y0)) < 1e-3  # y is bf16: a different fp32 summation order may flip a rounding
    for k in (("h", "angle", "pb", "px") if compact else ("h", "angle", "pbx")):
        assert max_rel(to_np(a1[k]), to_np(a0[k])) < 1e-5, k


def test_step_full_batch_state_layout():
    """cfg4 layer dims at batch 256: every (batch, head) state block is updated independently."""
    from mamba3_b200 import KulaMamba

    torch.manual_seed(4)
    m = KulaMamba(d_model=768, d_state=128, headdim=64, mimo_rank=2).cuda().to(torch.bfloat16).eval()
    B = 256
    g = torch.Generator().manual_seed(44)
    st = {"h": torch.randn(B, 24, 64, 128, generator=g).cuda(), "prev_BX": torch.randn(B, 24, 64, 128, generator=g).cuda(),
          "angle": torch.randn(B, 24, 64, generator=g).cuda()}
    x = torch.randn(B, 768, generator=g).cuda().to(torch.bfloat16)
    with torch.no_grad():
        y, st2 = m.step(x, st)
    # check three rows against the oracle on the same row alone
    from helpers import oracle_params

    p = oracle_params(m)
    for b in (0, 131, 255):
        ost = {k: to_np(v[b:b + 1]) for k, v in st.items()}
        oy, o2 = oracle.layer_step(p, to_np(x[b:b + 1]), ost)
        assert max_rel(to_np(y[b:b + 1]), oy) < 2e-2
        # bf16 projection output feeds the fp32 state update: bf16 I/O tolerance
        assert max_rel(to_np(st2["h"][b:b + 1]), o2["h"]) < 2e-2
        assert max_rel(to_np(st2["prev_BX"][b:b + 1]), o2["prev_BX"]) < 2e-2


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
@pytest.mark.parametrize("shape", [(4, 512, 768), (3, 5, 100), (2, 2048), (7, 64)])
def test_rmsnorm_kernel_matches_reference_formula(dtype, shape):
    """m3b_rmsnorm against the reference's torch formula (mamba3/mamba3.py:28-35): the same
    roundings, so bf16 / fp16 results agree to the last bit but for rare summation-order ties."""
    from mamba3_b200 import _lib

    g = torch.Generator().manual_seed(sum(shape))
    x = (torch.randn(*shape, generator=g) * 3).to("cuda", dtype)
    w = (torch.randn(shape[-1], generator=g) * 0.5 + 1).to("cuda", dtype)
    rms = torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-5).to(dtype)
    ref = x * rms * w
    y = _lib.rmsnorm(x, w, 1e-5)
    tol = 1e-6 if dtype == torch.float32 else 1e-2
    assert max_rel(to_np(y), to_np(ref)) < tol
    if dtype != torch.float32:
        assert (y == ref).float().mean().item() > 0.99
    x2 = x.clone()
    _lib.rmsnorm(x2, w, 1e-5, out=x2)  # in place
    assert torch.equal(x2, y)


def test_rmsnorm_module_uses_kernel_without_grad():
    """RMSNorm: the kernel under no_grad and the torch ops with autograd give the same values."""
    from mamba3_b200.mamba3 import RMSNorm

    norm = RMSNorm(768).cuda().to(torch.bfloat16)
    with torch.no_grad():
        norm.weight.copy_(torch.randn(768) * 0.3 + 1)
    x = torch.randn(8, 33, 768, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        y_k = norm(x)
    y_t = norm(x.requires_grad_(True))
    assert y_t.requires_grad
    assert max_rel(to_np(y_k), to_np(y_t)) < 1e-2


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
@pytest.mark.parametrize("n", [8 * 4096 * 2112, 1001])
def test_swiglu_and_residual_kernels_match_torch(dtype, n):
    """m3b_swiglu_act == F.silu(g) * u and m3b_scaled_add == x + h * s, rounded as torch stores
    them (vector path for n % 8 == 0, scalar path otherwise)."""
    import torch.nn.functional as F

    from mamba3_b200 import _lib

    g = torch.Generator().manual_seed(n % 97)
    a = (torch.randn(n, generator=g) * 3).to("cuda", dtype)
    b = torch.randn(n, generator=g).to("cuda", dtype)
    tol = 1e-6 if dtype == torch.float32 else 1e-2
    act = _lib.swiglu_act(a, b)
    ref = F.silu(a) * b
    assert max_rel(to_np(act), to_np(ref)) < tol
    res = _lib.scaled_add(a, b, 0.1443)
    ref2 = a + b * 0.1443
    assert max_rel(to_np(res), to_np(ref2)) < tol
    if dtype != torch.float32:
        assert (act == ref).float().mean().item() > 0.99
        assert (res == ref2).float().mean().item() > 0.99


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,d,f", [(256, 768, 2112), (3, 128, 384), (0, 768, 2112)])
def test_fused_block_steps_equal_unfused(dtype, rows, d, f):
    """The decoder's fused block steps give bit for bit what the separate kernels store:
    m3b_add_rmsnorm == m3b_scaled_add then m3b_rmsnorm (both outputs), and m3b_swiglu_rows on one
    [g | u] GEMM output == m3b_swiglu_act on its two halves."""
    from mamba3_b200 import _lib

    g = torch.Generator().manual_seed(rows + d)
    x = torch.randn(rows, d, generator=g).to("cuda", dtype)
    h = (torch.randn(rows, d, generator=g) * 4).to("cuda", dtype)
    w = (1 + 0.1 * torch.randn(d, generator=g)).to("cuda", dtype)
    x1, y1 = _lib.add_rmsnorm(x, h, 0.1443, w, 1e-5)
    x2 = _lib.scaled_add(x, h, 0.1443)
    y2 = _lib.rmsnorm(x2, w, 1e-5)
    assert torch.equal(x1, x2) and torch.equal(y1, y2)
    gu = (torch.randn(rows, 2 * f, generator=g) * 3).to("cuda", dtype)
    a1 = _lib.swiglu_rows(gu)
    a2 = _lib.swiglu_act(gu[:, :f].contiguous(), gu[:, f:].contiguous())
    assert a1.shape == (rows, f) and torch.equal(a1, a2)


@pytest.mark.parametrize("R,rows,dtype", [(1, 300, torch.float32), (2, 1000, torch.float32), (3, 129, torch.float32),
                                          (4, 257, torch.float32), (2, 1000, torch.bfloat16), (2, 0, torch.float32)])
def test_gate_kernels_match_torch_autograd(R, rows, dtype):
    """m3b_gate_fwd / m3b_gate_bwd (the gate and MIMO down-projection of mamba3/mamba3.py:234-238)
    against torch autograd of (y * silu(z * mimo_z) * mimo_down).sum(-1) in fp64, with z a
    strided column slice of a wider projection, as in the layer.  Tolerance (max abs error over
    max abs value): fp32 2e-5; bf16 2e-2 (inputs and outputs rounded to bf16)."""
    import torch.nn.functional as F

    from mamba3_b200 import _lib

    H, P, W = 3, 40, 3 * 40 + 17
    g = torch.Generator().manual_seed(R * 1000 + rows)
    y = torch.randn(rows, H, P, R, generator=g)
    proj = torch.randn(rows, W, generator=g) * 2
    mz = 1 + 0.3 * torch.randn(H, P, R, generator=g)
    md = torch.randn(H, P, R, generator=g) / R
    dout = torch.randn(rows, H * P, generator=g)
    dev = [t.to("cuda", dtype) for t in (y, proj, mz, md, dout)]
    yd, projd, mzd, mdd, doutd = dev
    out = _lib.gate_fwd(yd, projd[:, : H * P], mzd, mdd)
    dy, dz, dmz, dmd = _lib.gate_bwd(yd, projd[:, : H * P], mzd, mdd, doutd)
    ref_in = [t.to("cpu", torch.float64).clone().requires_grad_(True) for t in (yd, projd[:, : H * P], mzd, mdd)]
    yr, zr, mzr, mdr = ref_in
    ref = (yr * F.silu(zr.reshape(rows, H, P, 1) * mzr) * mdr).sum(-1).reshape(rows, H * P)
    ref.backward(doutd.to("cpu", torch.float64))
    tol = 2e-5 if dtype == torch.float32 else 2e-2
    if rows == 0:
        assert out.numel() == 0 and float(dmz.abs().sum()) == 0 and float(dmd.abs().sum()) == 0
        return
    assert max_rel(to_np(out), ref.detach().numpy()) < tol
    for got, want in ((dy, yr.grad), (dz, zr.grad), (dmz, mzr.grad), (dmd, mdr.grad)):
        assert got.shape == want.shape and got.dtype == dtype
        assert max_rel(to_np(got), want.numpy()) < tol


def _bc_reference(Bf, Cf, theta, dt, wB, bB, wC, bC, H, eps, shift):
    """B / C preparation of mamba3/mamba3.py:203-232 in torch ops (norm + bias, head broadcast,
    pairwise rotation by -cumsum(dt theta), previous-token shift)."""
    import torch.nn.functional as F

    Bt, T, _ = Bf.shape
    G, N, R = bB.shape

    def norm(x, w, b):
        x = x.reshape(Bt, T, G, N * R)
        y = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w
        return (y.reshape(Bt, T, G, N, R) + b).repeat_interleave(H // G, dim=2)

    Br, Cr = norm(Bf, wB, bB), norm(Cf, wC, bC)
    if theta is not None:
        cum = -(dt[..., None] * theta[..., None, :]).cumsum(dim=1)
        c, s = torch.cos(cum)[..., None], torch.sin(cum)[..., None]

        def rot(t):
            tp = t.reshape(Bt, T, H, N // 2, 2, R)
            a, b = tp[..., 0, :], tp[..., 1, :]
            return torch.stack([a * c - b * s, a * s + b * c], dim=-2).reshape(Bt, T, H, N, R)

        Br, Cr = rot(Br), rot(Cr)
    Bb = F.pad(Br[:, :-1], (0, 0, 0, 0, 0, 0, 1, 0)) if shift else None
    return Br, Bb, Cr


@pytest.mark.parametrize("G,H,R,T,rotate,shift,dtype", [
    (1, 4, 2, 150, True, True, torch.float32), (2, 4, 1, 150, True, True, torch.float32),
    (1, 3, 2, 64, False, True, torch.float32), (2, 2, 2, 70, True, False, torch.float32),
    (1, 2, 2, 1, True, True, torch.float32), (1, 2, 4, 100, True, True, torch.float32),
    (1, 2, 3, 100, True, True, torch.float32), (1, 4, 2, 150, True, True, torch.bfloat16),
    (1, 2, 4, 100, True, True, torch.bfloat16)])
def test_bc_kernels_match_torch_autograd(G, H, R, T, rotate, shift, dtype):
    """m3b_bc_fwd / m3b_bc_bwd against torch autograd of the reference's B / C preparation in
    fp64, with Bf, Cf and theta column slices of one wider projection (as in the layer) and
    ragged 64-token chunks.  Tolerance (max abs error over max abs value): fp32 1e-4 (fp32
    angles of up to ~40 rad), bf16 3e-2 (inputs and outputs rounded to bf16)."""
    from mamba3_b200 import _lib

    Bt, N, eps = 2, 16, 1e-5
    gnr, K = G * N * R, N // 2
    W = 2 * gnr + K + 5
    g = torch.Generator().manual_seed(G * 100 + H * 10 + T)
    proj = torch.randn(Bt, T, W, generator=g)
    dt = torch.rand(Bt, T, H, generator=g) * 0.3
    wB, wC = 1 + 0.2 * torch.randn(N * R, generator=g), 1 + 0.2 * torch.randn(N * R, generator=g)
    bB, bC = 1 + 0.2 * torch.randn(G, N, R, generator=g), 1 + 0.2 * torch.randn(G, N, R, generator=g)
    gouts = [torch.randn(Bt, T, H, N, R, generator=g) for _ in range(3)]
    dev = [t.to("cuda", dtype) for t in (proj, wB, bB, wC, bC, *gouts)]
    projd, wBd, bBd, wCd, bCd, gBd, gBbd, gCd = dev
    dtd = dt.to("cuda", dtype)
    sl = lambda p: (p[..., :gnr], p[..., gnr:2 * gnr], p[..., 2 * gnr:2 * gnr + K] if rotate else None)  # noqa: E731
    Bfd, Cfd, thd = sl(projd)
    Bg, Bb, Co = _lib.bc_fwd(Bfd, Cfd, thd, dtd, wBd, bBd, wCd, bCd, H, eps, shift)
    grads = _lib.bc_bwd(Bfd, Cfd, thd, dtd, wBd, bBd, wCd, bCd, gBd, gBbd if shift else None, gCd, H, eps, shift)

    f64 = lambda t: t.to("cpu", torch.float64).clone().requires_grad_(True)  # noqa: E731
    projr, dtr, wBr, bBr, wCr, bCr = (f64(t) for t in (projd, dtd, wBd, bBd, wCd, bCd))
    Bfr, Cfr, thr = sl(projr)
    rB, rBb, rC = _bc_reference(Bfr, Cfr, thr, dtr, wBr, bBr, wCr, bCr, H, eps, shift)
    loss = (rB * gBd.double().cpu()).sum() + (rC * gCd.double().cpu()).sum()
    if shift:
        loss = loss + (rBb * gBbd.double().cpu()).sum()
    loss.backward()
    tol = 1e-4 if dtype == torch.float32 else 3e-2
    assert max_rel(to_np(Bg), rB.detach().numpy()) < tol
    assert max_rel(to_np(Co), rC.detach().numpy()) < tol
    if shift:
        assert max_rel(to_np(Bb), rBb.detach().numpy()) < tol
    dBf, dCf, dth, ddt, dwB, dbB, dwC, dbC = grads
    pg = projr.grad
    want = [(dBf, pg[..., :gnr]), (dCf, pg[..., gnr:2 * gnr]), (dwB, wBr.grad), (dbB, bBr.grad),
            (dwC, wCr.grad), (dbC, bCr.grad)]
    if rotate:
        want += [(dth, pg[..., 2 * gnr:2 * gnr + K]), (ddt, dtr.grad)]
    for i, (got, ref) in enumerate(want):
        assert got.shape == ref.shape, i
        assert max_rel(to_np(got), ref.numpy()) < tol, i


@pytest.mark.parametrize("H,P,R,T,trap,dtype", [
    (4, 16, 2, 150, True, torch.float32), (3, 48, 1, 70, True, torch.float32), (2, 64, 4, 65, True, torch.float32),
    (4, 16, 3, 1, True, torch.float32), (4, 16, 2, 100, False, torch.float32), (4, 64, 2, 130, True, torch.bfloat16)])
def test_xprep_kernels_match_torch_autograd(H, P, R, T, trap, dtype):
    """m3b_xprep_fwd / m3b_xprep_bwd against torch autograd of the reference's x-side MIMO
    expansion and trapezoid weights (mamba3/mamba3.py:218-230) in fp64, with xf and lam_raw
    column slices of a wider projection; P = 48 leaves CTAs with part of a 256-channel block
    unused, and 64-row chunks cross sequence boundaries.  Tolerance (max abs error over max abs
    value): fp32 1e-5, bf16 2e-2."""
    import torch.nn.functional as F

    from mamba3_b200 import _lib

    Bt, C = 2, H * P
    W = C + H + 3
    g = torch.Generator().manual_seed(H * 1000 + P * 10 + T)
    proj = torch.randn(Bt, T, W, generator=g)
    dt = torch.rand(Bt, T, H, generator=g) * 0.3
    A = -torch.rand(H, generator=g) * 2
    mx = 1 + 0.3 * torch.randn(H, P, R, generator=g)
    gouts = [torch.randn(Bt, T, H, P, R, generator=g) for _ in range(3)]
    projd, dtd, Ad, mxd, g0, g1, g2 = (t.to("cuda", dtype) for t in (proj, dt, A, mx, *gouts))
    sl = lambda p: (p[..., :C], p[..., C:C + H] if trap else None)  # noqa: E731
    xfd, lrd = sl(projd)
    xr, xg, xb = _lib.xprep_fwd(xfd, mxd, lrd, dtd, Ad)
    dxf, dmx, dlam, ddt, dA = _lib.xprep_bwd(xfd, mxd, lrd, dtd, Ad, g0, g1 if trap else None,
                                             g2 if trap else None)

    f64 = lambda t: t.to("cpu", torch.float64).clone().requires_grad_(True)  # noqa: E731
    projr, dtr, Ar, mxr = (f64(t) for t in (projd, dtd, Ad, mxd))
    xfr, lrr = sl(projr)
    rr = xfr.reshape(Bt, T, H, P, 1) * mxr
    loss = (rr * g0.double().cpu()).sum()
    outs = [(xr, rr)]
    if trap:
        lam = torch.sigmoid(lrr)
        rg = rr * lam[..., None, None]
        rb = F.pad(rr[:, :-1], (0, 0, 0, 0, 0, 0, 1, 0)) * ((1 - lam) * torch.exp(Ar * dtr))[..., None, None]
        loss = loss + (rg * g1.double().cpu()).sum() + (rb * g2.double().cpu()).sum()
        outs += [(xg, rg), (xb, rb)]
    loss.backward()
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    for got, ref in outs:
        assert max_rel(to_np(got), ref.detach().numpy()) < tol
    want = [(dxf, projr.grad[..., :C]), (dmx, mxr.grad)]
    if trap:
        want += [(dlam, projr.grad[..., C:C + H]), (ddt, dtr.grad), (dA, Ar.grad)]
    for i, (got, ref) in enumerate(want):
        assert got.shape == ref.shape, i
        assert max_rel(to_np(got), ref.numpy()) < tol, i
