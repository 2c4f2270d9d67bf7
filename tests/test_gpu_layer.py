"""Layer-level parity of the chunked tensor-core forward / prefill on the GPU.

* fp32 models against the reference's golden outputs at 1e-3 (fp32 activations run the
  chunk-parallel kernels with tf32 tensor-core operands; the angle -- pure fp32
  arithmetic -- to 1e-4);
* bf16 models against the fp64 oracle on the same bf16-rounded weights (2e-2);
* properties at the benchmark sizes: causality (a prefix of the full-size output equals
  the oracle on that prefix), chaining (prefill of a split sequence == prefill of the
  whole), parallel == recurrent.
"""

import numpy as np
import pytest
import torch

import oracle
from goldens import LAYER_CASES, load, max_rel
from helpers import oracle_params, ours_layer_from_golden, to_np

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2
FP32_TOL = 1e-3


@pytest.fixture(params=[1, 2], ids=["fused", "chunked"], autouse=True)
def layer_algo(request):
    """Run every layer test on both layer-forward algorithms."""
    from mamba3_b200 import ops

    prev = ops.set_layer_algo(request.param)
    yield request.param
    ops.set_layer_algo(prev)


@pytest.mark.parametrize("case", LAYER_CASES)
def test_forward_prefill_golden_fp32(case):
    d = load(f"layer_{case}")
    m = ours_layer_from_golden(d, torch.float32)
    T = int(d["T"])
    x = torch.from_numpy(d["x"][:, :T]).cuda()
    with torch.no_grad():
        y = m(x)
        y2, st = m.prefill(x)
    assert max_rel(to_np(y), d["y"]) < FP32_TOL
    assert max_rel(to_np(y2), d["y"]) < FP32_TOL
    assert max_rel(to_np(st["h"]), d["pf_h"]) < FP32_TOL
    assert max_rel(to_np(st["angle"]), d["pf_angle"]) < 1e-4
    assert max_rel(to_np(st["prev_BX"]), d["pf_prev_BX"]) < 1e-4


@pytest.mark.parametrize("case", LAYER_CASES)
def test_forward_bf16_vs_oracle(case):
    d = load(f"layer_{case}")
    m = ours_layer_from_golden(d, torch.bfloat16)
    p = oracle_params(m)
    T = int(d["T"])
    x = torch.from_numpy(d["x"][:, :T]).cuda().to(torch.bfloat16)
    with torch.no_grad():
        y, st = m.prefill(x)
    oy, ost = oracle.layer_prefill(p, to_np(x))
    assert max_rel(to_np(y), oy) < BF16_TOL
    assert max_rel(to_np(st["h"]), ost["h"]) < BF16_TOL
    assert max_rel(to_np(st["prev_BX"]), ost["prev_BX"]) < BF16_TOL


@pytest.mark.parametrize("case", ["default", "perturbed", "rank1", "rank4", "euler", "real", "ngroups2"])
def test_parallel_equals_recurrent(case):
    """Forward (chunked, tensor cores) vs the step kernel token by token (fp32 model)."""
    d = load(f"layer_{case}")
    m = ours_layer_from_golden(d, torch.float32)
    x = torch.from_numpy(d["x"]).cuda()
    B, T = x.shape[:2]
    with torch.no_grad():
        y_par = m(x)
        st = m.allocate_inference_state(B)
        ys = []
        for t in range(T):
            yt, st = m.step(x[:, t:t + 1], st)
            ys.append(yt[:, 0])
    assert max_rel(to_np(torch.stack(ys, 1)), to_np(y_par)) < FP32_TOL


@pytest.mark.parametrize("R", [1, 2, 3, 4])
def test_parallel_equals_recurrent_n128(R):
    """d_state 128 (the step kernel's one-warp-per-state-row path for R = 1, 2, 4; the generic
    path for R = 3): forward vs token-by-token steps, fp32 model."""
    from mamba3_b200 import KulaMamba

    torch.manual_seed(12 + R)
    m = KulaMamba(d_model=128, d_state=128, headdim=64, mimo_rank=R).cuda().eval()
    x = torch.randn(2, 40, 128, generator=torch.Generator().manual_seed(R)).cuda()
    with torch.no_grad():
        y_par = m(x)
        st = m.allocate_inference_state(2)
        ys = []
        for t in range(x.shape[1]):
            yt, st = m.step(x[:, t:t + 1], st)
            ys.append(yt[:, 0])
    assert max_rel(to_np(torch.stack(ys, 1)), to_np(y_par)) < FP32_TOL


def test_chaining_prefill_from_state():
    """prefill(x[:, :T1]) then prefill_from(x[:, T1:]) == prefill(x) (sequence-split property)."""
    d = load("layer_n128p64")
    m = ours_layer_from_golden(d, torch.bfloat16)
    x = torch.from_numpy(d["x"]).cuda().to(torch.bfloat16)
    T1 = 70
    with torch.no_grad():
        y, st = m.prefill(x)
        y1, st1 = m.prefill(x[:, :T1])
        y2, st2 = m.prefill_from(x[:, T1:], st1)
    assert max_rel(to_np(torch.cat([y1, y2], 1)), to_np(y)) < BF16_TOL
    for k in ("h", "angle", "prev_BX"):
        assert max_rel(to_np(st2[k]), to_np(st[k])) < BF16_TOL


def test_extreme_decay_finite():
    """A_log = 0, dt_bias = 3 (mamba3 tests :410-423): segsum form stays finite."""
    from mamba3_b200 import KulaMamba

    torch.manual_seed(0)
    m = KulaMamba(d_model=64, d_state=16, headdim=16, mimo_rank=2, chunk_size=8).cuda().eval()
    with torch.no_grad():
        m.A_log.fill_(0.0)
        m.dt_bias.fill_(3.0)
        x = torch.randn(1, 300, 64, device="cuda")
        y = m(x)
    assert torch.isfinite(y).all() and y.abs().max() > 0
    p = oracle_params(m)
    oy, _ = oracle.layer_forward(p, to_np(x))
    assert max_rel(to_np(y), oy) < FP32_TOL


def test_mixed_decay_heads_n128():
    """Heads from weak to extreme decay in one layer (bf16, N = 128): chunks whose decay range is
    small and chunks whose range needs the per-element exponentials meet in one launch."""
    from mamba3_b200 import KulaMamba

    torch.manual_seed(4)
    m = KulaMamba(d_model=256, d_state=128, headdim=64, mimo_rank=2).cuda().eval()
    H = m.nheads
    with torch.no_grad():
        # A from -0.14 to -4, dt from ~0.0025 to ~0.7: chunk decay ranges from < 1 to ~180 (log2
        # units), on both sides of the point where the kernel switches to per-element exponentials,
        # and still within the float64 range of the oracle's exp(-cumsum) form
        m.A_log.copy_(torch.linspace(-2.0, 1.386, H))
        m.dt_bias.copy_(torch.linspace(-6.0, 0.0, H))
    m = m.to(torch.bfloat16)
    p = oracle_params(m)
    g = torch.Generator().manual_seed(5)
    x = torch.randn(2, 300, 256, generator=g).cuda().to(torch.bfloat16)
    with torch.no_grad():
        y, st = m.prefill(x)
    assert torch.isfinite(y).all()
    oy, ost = oracle.layer_prefill(p, to_np(x))
    assert max_rel(to_np(y), oy) < BF16_TOL
    assert max_rel(to_np(st["h"]), ost["h"]) < BF16_TOL


@pytest.mark.parametrize("graph", [False, True], ids=["eager", "graph"])
@pytest.mark.parametrize("pieces", [1, 3, 8])
def test_forward_host_streaming_equals_forward(pieces, graph):
    """forward_host (pinned host input streamed through the GPU in token ranges) == forward."""
    from mamba3_b200 import KulaMamba

    torch.manual_seed(6)
    m = KulaMamba(d_model=256, d_state=128, headdim=64, mimo_rank=2).cuda().to(torch.bfloat16).eval()
    g = torch.Generator().manual_seed(7)
    x = torch.randn(2, 333, 256, generator=g).to(torch.bfloat16).pin_memory()
    with torch.no_grad():
        ref = m(x.cuda())
        out = torch.empty_like(x).pin_memory()
        for _ in range(2 if graph else 1):  # a graph is captured on the first call, replayed after
            out.zero_()
            m.forward_host(x, out, pieces=pieces, graph=graph)
            torch.cuda.synchronize()
            assert max_rel(to_np(out), to_np(ref)) < BF16_TOL
        if graph:  # new input in the same buffer: the replay reads it
            x.copy_(torch.randn(x.shape, generator=g).to(torch.bfloat16))
            ref = m(x.cuda())
            m.forward_host(x, out, pieces=pieces, graph=True)
            torch.cuda.synchronize()
            assert max_rel(to_np(out), to_np(ref)) < BF16_TOL
    assert not out.is_cuda and out.is_pinned()


@pytest.mark.parametrize("B,T,seed", [(16, 4096, 1)])
def test_cfg1_full_size_prefix_parity(B, T, seed):
    """Config 1 at full size: rows 0 and B-1, first 256 tokens vs the oracle (causal prefix)."""
    from mamba3_b200 import KulaMamba

    torch.manual_seed(0)
    m = KulaMamba(d_model=768, d_state=128, headdim=64, mimo_rank=2, chunk_size=64).cuda().to(torch.bfloat16).eval()
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, T, 768, generator=g).cuda().to(torch.bfloat16)
    with torch.no_grad():
        y, st = m.prefill(x)
    assert torch.isfinite(y).all() and torch.isfinite(st["h"]).all()
    p = oracle_params(m)
    Tp = 256
    for b in (0, B - 1):
        oy, _ = oracle.layer_forward(p, to_np(x[b:b + 1, :Tp]))
        assert max_rel(to_np(y[b:b + 1, :Tp]), oy) < BF16_TOL


@pytest.mark.parametrize("T", [1, 2, 31, 63, 64, 65, 129])
@pytest.mark.parametrize("R", [1, 2, 4])
def test_ragged_lengths_n128(T, R):
    """Sequence lengths around the kernels' chunk length (128 / R tokens), down to one token,
    with d_state 128 (the TMA-staged fused path): prefill vs the oracle, bf16."""
    from mamba3_b200 import KulaMamba

    torch.manual_seed(40 + R)
    m = KulaMamba(d_model=128, d_state=128, headdim=64, mimo_rank=R).cuda().to(torch.bfloat16).eval()
    x = torch.randn(3, T, 128, generator=torch.Generator().manual_seed(T)).cuda().to(torch.bfloat16)
    with torch.no_grad():
        y, st = m.prefill(x)
    oy, ost = oracle.layer_prefill(oracle_params(m), to_np(x))
    assert max_rel(to_np(y), oy) < BF16_TOL
    assert max_rel(to_np(st["h"]), ost["h"]) < BF16_TOL
    assert max_rel(to_np(st["prev_BX"]), ost["prev_BX"]) < BF16_TOL


@pytest.mark.parametrize("d_model,R,B,T", [(768, 2, 8, 1000), (640, 2, 8, 500), (768, 4, 8, 256), (768, 1, 8, 1024)])
def test_fused_sequence_parts_equal_chunk_parallel(d_model, R, B, T, layer_algo):
    """With at least as many (batch, head) sequences as SMs the fused kernel cuts sequences into
    parts handed from CTA to CTA (state and angles through global memory): its outputs and final
    states equal the chunk-parallel algorithm's, which never cuts, and the state-only variant
    ends in the same state."""
    from mamba3_b200 import KulaMamba, ops, seqpar

    if layer_algo != 1:
        pytest.skip("runs both algorithms itself")
    torch.manual_seed(50 + R)
    m = KulaMamba(d_model=d_model, d_state=128, headdim=64, mimo_rank=R).cuda().to(torch.bfloat16).eval()
    x = torch.randn(B, T, d_model, generator=torch.Generator().manual_seed(T)).cuda().to(torch.bfloat16)
    with torch.no_grad():
        y1, st1 = m.prefill(x)
        so = seqpar.layer_state_only(m, m.in_proj(x))
        prev = ops.set_layer_algo(2)
        try:
            y2, st2 = m.prefill(x)
        finally:
            ops.set_layer_algo(prev)
    assert max_rel(to_np(y1), to_np(y2)) < BF16_TOL
    for k in ("h", "angle", "prev_BX"):
        assert max_rel(to_np(st1[k]), to_np(st2[k])) < (1e-4 if k == "angle" else BF16_TOL), k
        assert max_rel(to_np(so[k]), to_np(st2[k])) < (1e-4 if k == "angle" else BF16_TOL), k


def test_fused_sequence_parts_from_a_state(layer_algo):
    """Parts with an initial state: prefill_from over a range long enough to be cut into parts
    (8 x 24 sequences, 14 chunks) continues a prefill exactly as the whole prefill does."""
    from mamba3_b200 import KulaMamba

    if layer_algo != 1:
        pytest.skip("fused algorithm only")
    torch.manual_seed(61)
    m = KulaMamba(d_model=768, d_state=128, headdim=64, mimo_rank=2).cuda().to(torch.bfloat16).eval()
    x = torch.randn(8, 1000, 768, generator=torch.Generator().manual_seed(62)).cuda().to(torch.bfloat16)
    T1 = 104
    with torch.no_grad():
        y, st = m.prefill(x)
        y1, st1 = m.prefill(x[:, :T1])
        y2, st2 = m.prefill_from(x[:, T1:], st1)
    assert max_rel(to_np(torch.cat([y1, y2], 1)), to_np(y)) < BF16_TOL
    for k in ("h", "angle", "prev_BX"):
        assert max_rel(to_np(st2[k]), to_np(st[k])) < BF16_TOL, k


def test_dt_scale_matches_oracle():
    """dt_scale (mamba3/mamba3.py:200-202; reference test tests:160-166): forward and prefill with a
    per-token, per-head dt scale against the oracle, and it changes the output."""
    from mamba3_b200 import KulaMamba

    torch.manual_seed(71)
    m = KulaMamba(d_model=128, d_state=128, headdim=64, mimo_rank=2).cuda().to(torch.bfloat16).eval()
    g = torch.Generator().manual_seed(72)
    x = torch.randn(2, 150, 128, generator=g).cuda().to(torch.bfloat16)
    ds = (torch.rand(2, 150, m.nheads, generator=g) * 1.5 + 0.25).cuda().to(torch.bfloat16)
    with torch.no_grad():
        y0 = m(x)
        y = m(x, dt_scale=ds)
        y2, st = m.prefill(x, dt_scale=ds)
    oy, ost = oracle.layer_prefill(oracle_params(m), to_np(x), dt_scale=to_np(ds))
    assert max_rel(to_np(y), oy) < BF16_TOL
    assert max_rel(to_np(y2), oy) < BF16_TOL
    assert max_rel(to_np(st["h"]), ost["h"]) < BF16_TOL
    assert max_rel(to_np(y0), to_np(y)) > 1e-2


def test_long_sequence_forward_equals_steps():
    """Reference test tests:698-728 at its size (T = 512, small layer, fp32): forward vs 512 decode
    steps, at the reference's own 1e-3."""
    from mamba3_b200 import KulaMamba

    torch.manual_seed(73)
    m = KulaMamba(d_model=64, d_state=16, headdim=16, mimo_rank=2, chunk_size=8).cuda().eval()
    x = torch.randn(1, 512, 64, device="cuda")
    with torch.no_grad():
        y_par = m(x)
        st = m.allocate_inference_state(1)
        ys = []
        for t in range(512):
            yt, st = m.step(x[:, t:t + 1], st)
            ys.append(yt[:, 0])
    assert torch.isfinite(y_par).all()
    assert max_rel(to_np(torch.stack(ys, 1)), to_np(y_par)) < FP32_TOL


def test_mimo_ranks_interact():
    """Zeroing rank 1 of mimo_x changes the output (reference test tests:377-391)."""
    from mamba3_b200 import KulaMamba

    torch.manual_seed(74)
    m = KulaMamba(d_model=64, d_state=16, headdim=16, mimo_rank=2, chunk_size=8).cuda().eval()
    x = torch.randn(1, 16, 64, device="cuda")
    with torch.no_grad():
        y = m(x)
        m.mimo_x[:, :, 1] = 0.0
        y1 = m(x)
    assert (y - y1).abs().max().item() > 1e-5


@pytest.mark.parametrize("compact", [False, True], ids=["prev_bx", "compact"])
def test_dt_scale_steps_equal_forward(compact):
    """Decode steps with a per-token dt scale (mamba3/mamba3.py:279-280) reproduce the forward
    with the same scale (fp32 model)."""
    from mamba3_b200 import KulaMamba

    torch.manual_seed(75)
    m = KulaMamba(d_model=128, d_state=128, headdim=64, mimo_rank=2).cuda().eval()
    g = torch.Generator().manual_seed(76)
    x = torch.randn(2, 40, 128, generator=g).cuda()
    ds = (torch.rand(2, 40, m.nheads, generator=g) * 1.5 + 0.25).cuda()
    with torch.no_grad():
        y_par = m(x, dt_scale=ds)
        st = m.allocate_inference_state(2, compact=compact)
        ys = []
        for t in range(40):
            yt, st = m.step(x[:, t:t + 1], st, dt_scale=ds[:, t])
            ys.append(yt[:, 0])
    assert max_rel(to_np(torch.stack(ys, 1)), to_np(y_par)) < FP32_TOL
