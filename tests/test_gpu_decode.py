"""Decode: the CUDA-graph decoder against KulaMambaLM.generate, and step decode against the
parallel forward on the generated sequence (the reference's step == forward property,
mamba3 tests:294-314, at LM level)."""

import pytest
import torch

from goldens import max_rel
from helpers import to_np

pytestmark = pytest.mark.gpu


def _lm(dtype, seed=8, vocab=1000, n_layers=2):
    from mamba3_b200 import KulaMambaLM

    torch.manual_seed(seed)
    return KulaMambaLM(vocab_size=vocab, d_model=128, n_layers=n_layers, d_state=128, headdim=64,
                       mimo_rank=2).cuda().to(dtype).eval()


@pytest.mark.parametrize("compact", [True, False], ids=["compact", "prev_BX"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_graph_decoder_matches_generate(dtype, compact):
    from mamba3_b200.decode import GraphDecoder

    lm = _lm(dtype)
    g = torch.Generator().manual_seed(9)
    ids = torch.randint(0, 1000, (3, 20), generator=g).cuda()
    ref = lm.generate(ids, max_new_tokens=12, temperature=0.0)
    dec = GraphDecoder(lm, batch_size=3, max_new_tokens=12, compact=compact)
    out = dec.generate(ids, temperature=0.0)
    assert out.shape == ref.shape == (3, 32)
    assert torch.equal(out, ref)
    # a second generate reuses the captured graph from a fresh prefill
    assert torch.equal(dec.generate(ids, temperature=0.0), ref)


def test_graph_decoder_keeps_one_graph_per_sampling_rule():
    """One decoder: greedy, then sampled (temperature 1, top-2), then greedy again.  The sampling
    rule is part of the captured step, so the sampled call must replay a graph of its own: its
    tokens are each step's top-2 candidates (top-3 of the teacher-forced forward, one rank of
    slack for rounding), not all greedy; the greedy calls still equal generate's tokens."""
    from mamba3_b200.decode import GraphDecoder

    lm = _lm(torch.float32, seed=12)
    g = torch.Generator().manual_seed(13)
    ids = torch.randint(0, 1000, (3, 20), generator=g).cuda()
    ref = lm.generate(ids, max_new_tokens=12, temperature=0.0)
    dec = GraphDecoder(lm, batch_size=3, max_new_tokens=12)
    assert torch.equal(dec.generate(ids, temperature=0.0), ref)
    torch.manual_seed(14)
    smp = dec.generate(ids, temperature=1.0, top_k=2)
    assert smp.shape == ref.shape and torch.equal(smp[:, :20], ids)
    assert not torch.equal(smp, ref)  # 36 draws between two close candidates: not all greedy
    with torch.no_grad():
        logits = lm(smp)["logits"][:, 19:31]
    top3 = logits.topk(3, dim=-1).indices
    assert (top3 == smp[:, 20:32].unsqueeze(-1)).any(-1).all()
    assert torch.equal(dec.generate(ids, temperature=0.0), ref)
    assert len(dec.graphs) == 2


def test_step_logits_equal_parallel_forward():
    """Teacher-forced: logits of prefill + steps == logits of one forward over the sequence."""
    lm = _lm(torch.float32, seed=10)
    g = torch.Generator().manual_seed(11)
    ids = torch.randint(0, 1000, (2, 40), generator=g).cuda()
    with torch.no_grad():
        full = lm(ids)["logits"]
        x = lm.embedding(ids[:, :25])
        states = []
        for blk in lm.layers:
            x, st = blk.prefill(x)
            states.append(st)
        steps = [lm.lm_head(lm.norm(x))[:, -1]]
        for t in range(25, 40):
            x = lm.embedding(ids[:, t])
            for i, blk in enumerate(lm.layers):
                x, states[i] = blk.step(x, states[i])
            steps.append(lm.lm_head(lm.norm(x)))
    got = torch.stack(steps, 1)  # logits after tokens 24 .. 39
    assert max_rel(to_np(got), to_np(full[:, 24:40])) < 2e-2


@pytest.mark.parametrize("N,R", [(128, 1), (128, 2), (128, 4), (16, 2), (16, 3)])
def test_compact_state_steps_equal_prev_bx_steps(N, R):
    """Compact previous-token state (prev_B, prev_x): prefill gives factors whose product is
    prefill's prev_BX, and steps from either form give the same outputs and states."""
    from mamba3_b200 import KulaMamba

    torch.manual_seed(30 + R)
    m = KulaMamba(d_model=128, d_state=N, headdim=64 if N == 128 else 16, mimo_rank=R).cuda().eval()
    g = torch.Generator().manual_seed(31)
    x = torch.randn(2, 50, 128, generator=g).cuda()
    with torch.no_grad():
        y_a, st_a = m.prefill(x[:, :40])
        y_b, st_b = m.prefill(x[:, :40], compact_state=True)
        assert torch.equal(y_a, y_b)
        pbx = torch.einsum("bhnr,bhpr->bhpn", st_b["prev_B"], st_b["prev_x"])
        assert max_rel(to_np(pbx), to_np(st_a["prev_BX"])) < 1e-6
        for t in range(40, 50):
            ya, st_a = m.step(x[:, t], st_a)
            yb, st_b = m.step(x[:, t], st_b)
            assert max_rel(to_np(yb), to_np(ya)) < 1e-5
        assert max_rel(to_np(st_b["h"]), to_np(st_a["h"])) < 1e-5
        # a compact state also continues a prefill
        y_c, st_c = m.prefill_from(x[:, 40:], m.prefill(x[:, :40], compact_state=True)[1])
        y_d, st_d = m.prefill_from(x[:, 40:], m.prefill(x[:, :40])[1])
    assert max_rel(to_np(y_c), to_np(y_d)) < 1e-5
    assert "prev_B" in st_c and max_rel(to_np(st_c["h"]), to_np(st_d["h"])) < 1e-5


def test_compact_step_many_items_per_cta():
    """Config-4 shapes (batch 256 x 24 heads): the compact step from random factors equals the
    prev_BX step from their product, over three consecutive tokens."""
    from mamba3_b200 import KulaMamba

    torch.manual_seed(50)
    m = KulaMamba(d_model=768, d_state=128, headdim=64, mimo_rank=2).cuda().to(torch.bfloat16).eval()
    B = 256
    g = torch.Generator().manual_seed(51)
    full = m.allocate_inference_state(B)
    comp = m.allocate_inference_state(B, compact=True)
    for k in ("h", "angle"):
        full[k].copy_(torch.randn(full[k].shape, generator=g))
        comp[k].copy_(full[k])
    comp["prev_B"].copy_(torch.randn(comp["prev_B"].shape, generator=g))
    comp["prev_x"].copy_(torch.randn(comp["prev_x"].shape, generator=g))
    full["prev_BX"].copy_(torch.einsum("bhnr,bhpr->bhpn", comp["prev_B"], comp["prev_x"]))
    with torch.no_grad():
        for t in range(3):
            x = torch.randn(B, 768, generator=g).cuda().to(torch.bfloat16)
            ya, full = m.step(x, full)
            yb, comp = m.step(x, comp)
            assert max_rel(to_np(yb), to_np(ya)) < 1e-2, t
    assert max_rel(to_np(comp["h"]), to_np(full["h"])) < 1e-5
