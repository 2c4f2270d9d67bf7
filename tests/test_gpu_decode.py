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


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_graph_decoder_matches_generate(dtype):
    from mamba3_b200.decode import GraphDecoder

    lm = _lm(dtype)
    g = torch.Generator().manual_seed(9)
    ids = torch.randint(0, 1000, (3, 20), generator=g).cuda()
    ref = lm.generate(ids, max_new_tokens=12, temperature=0.0)
    dec = GraphDecoder(lm, batch_size=3, max_new_tokens=12)
    out = dec.generate(ids, temperature=0.0)
    assert out.shape == ref.shape == (3, 32)
    assert torch.equal(out, ref)
    # a second generate reuses the captured graph from a fresh prefill
    assert torch.equal(dec.generate(ids, temperature=0.0), ref)


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
