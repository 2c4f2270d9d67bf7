"""Parity at the BASELINE configurations' own sizes, against fixtures produced by running the
unmodified reference on the CPU (tests/golden/make_golden.py, config groups):

* config 0 -- fp32 layer, x (4, 1024, 768): the fp32 path (tf32 tensor-core operands) at 1e-3;
* config 1 -- bf16 layer, x (16, 4096, 768): rows 0, 7, 15 over all 4096 tokens and their final
  states, against the reference's fp32 path on the same bf16-rounded weights and inputs, 2e-2;
* config 2 -- the 24-layer LM on ids (64, 2048): final-norm hidden states every 32nd position and
  full logits at three positions of rows 0, 31, 63;
* config 3 -- the d_model 2048 / mimo_rank 4 layer over the first 16384 tokens of row 0 (the
  reference run segment by segment, chained through h_init), 2e-2;
* config 4 -- prefill (3 rows of the (256, 512) prompt) and 256 teacher-forced decode steps:
  final-norm hidden states every 8th step and logits at three steps; the greedy tokens.

For the 24-layer LM (configs 2 and 4) 2e-2 is below what any bf16 model reaches: the fixtures
also hold the reference's own deviation from its fp32 run when only its activations at module
boundaries are rounded to bf16 (the embedding, every norm output -- the GEMM operands --, every
sublayer output and the residual stream; all arithmetic fp32).  That floor is 1.7e-2 (config 4)
and 2.7e-2 to 7.1e-2 (config 2 rows); rounding the GEMM operands alone gives about 4e-2.  Those
tests allow max(2e-2, 2 x the floor of the same row).

The fixtures keep evenly spaced slices plus whole-tensor statistics (absmax, sum of squares),
which are compared at full size.  Tolerance: max|a - b| / max|b| (goldens.max_rel).
"""

import numpy as np
import pytest
import torch

from goldens import load, max_rel
from helpers import to_np

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-3
BF16_TOL = 2e-2

CFG_LAYER = dict(d_model=768, d_state=128, expand=2, headdim=64, mimo_rank=2, chunk_size=64)
CFG_LM = dict(vocab_size=32000, d_model=768, n_layers=24, d_state=128, headdim=64, mimo_rank=2,
              residual_scale="depth")
CFG3_LAYER = dict(d_model=2048, d_state=128, expand=2, headdim=64, mimo_rank=4, chunk_size=64)


def _stats_close(t, d, prefix, tol):
    """Whole-tensor absmax and root-mean-square against the reference's, relative."""
    t = t.detach().double()
    am, rms = float(t.abs().max()), float(torch.sqrt((t * t).sum() / t.numel()))
    ref_am = float(d[f"{prefix}.absmax"])
    ref_rms = float(np.sqrt(d[f"{prefix}.sumsq"] / d[f"{prefix}.numel"]))
    assert abs(am - ref_am) / ref_am < tol, (prefix, am, ref_am)
    assert abs(rms - ref_rms) / ref_rms < tol, (prefix, rms, ref_rms)


def _states_close(st, d, pre, heads, tol, angle_tol):
    assert max_rel(to_np(st["h"][:, heads]), d[f"{pre}st.h"]) < tol
    assert max_rel(to_np(st["prev_BX"][:, heads]), d[f"{pre}st.prev_BX"]) < tol
    assert max_rel(to_np(st["angle"]), d[f"{pre}st.angle"]) < angle_tol
    _stats_close(st["h"], d, f"{pre}st.h", tol)
    _stats_close(st["prev_BX"], d, f"{pre}st.prev_BX", tol)


def _layer(cfg, seed, dtype):
    from mamba3_b200 import KulaMamba

    torch.manual_seed(seed)
    return KulaMamba(**cfg).to("cuda", dtype).eval()


def test_config0_fp32_layer():
    d = load("cfg0_layer")
    m = _layer(CFG_LAYER, 0, torch.float32)
    x = torch.randn(4, 1024, 768, generator=torch.Generator().manual_seed(0)).cuda()
    with torch.no_grad():
        y, st = m.prefill(x)
        y_fwd = m(x)
    s = int(d["tok_stride"])
    err = max_rel(to_np(y[:, ::s]), d["y_tok"])
    print(f"config 0 fp32: y max rel err {err:.2e}")
    assert err < FP32_TOL
    assert max_rel(to_np(y_fwd[:, ::s]), d["y_tok"]) < FP32_TOL
    _stats_close(y, d, "y", FP32_TOL)
    _states_close(st, d, "", list(d["heads"]), FP32_TOL, 1e-4)


def test_config1_bf16_rows():
    d = load("cfg1_rows")
    m = _layer(CFG_LAYER, 0, torch.bfloat16)
    x = torch.randn(16, 4096, 768, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16).cuda()
    with torch.no_grad():
        y, st = m.prefill(x)  # the benchmark's whole batch; rows compared below
    s = int(d["tok_stride"])
    heads = list(d["heads"])
    for i, r in enumerate(d["rows"]):
        pre = f"r{i}."
        err = max_rel(to_np(y[r:r + 1, ::s]), d[pre + "y_tok"])
        print(f"config 1 row {r}: y max rel err {err:.2e}")
        assert err < BF16_TOL
        _stats_close(y[r:r + 1], d, pre + "y", BF16_TOL)
        st_r = {k: v[r:r + 1] for k, v in st.items()}
        _states_close(st_r, d, pre, heads, BF16_TOL, BF16_TOL)


def _lm():
    from mamba3_b200 import KulaMambaLM

    torch.manual_seed(2)
    return KulaMambaLM(**CFG_LM).to("cuda", torch.bfloat16).eval()


def test_config2_lm_rows():
    d = load("cfg2_lm")
    lm = _lm()
    ids = torch.randint(0, 32000, (64, 2048), generator=torch.Generator().manual_seed(2))
    rows = list(d["rows"])
    cap = {}
    hk = lm.norm.register_forward_hook(lambda mod, i, o: cap.__setitem__("h", o.detach()))
    with torch.no_grad():
        logits = lm(ids[rows].cuda())["logits"]
    hk.remove()
    s, pos = int(d["tok_stride"]), list(d["logit_pos"])
    for i in range(len(rows)):
        pre = f"r{i}."
        eh = max_rel(to_np(cap["h"][i:i + 1, ::s]), d[pre + "hid_tok"])
        el = max_rel(to_np(logits[i:i + 1, pos]), d[pre + "logits"])
        fh, fl = float(d["floor.hidden"][i]), float(d["floor.logits"][i])
        th, tl = max(BF16_TOL, 2 * fh), max(BF16_TOL, 2 * fl)
        print(f"config 2 row {rows[i]}: hidden max rel err {eh:.2e} (reference bf16 floor {fh:.2e}), "
              f"logits {el:.2e} (floor {fl:.2e})")
        assert eh < th and el < tl
        _stats_close(logits[i:i + 1].float(), d, pre + "logits", tl)


def test_config3_long_sequence_segment():
    d = load("cfg3_seg")
    m = _layer(CFG3_LAYER, 0, torch.bfloat16)
    T = int(d["T"])
    x = torch.randn(1, T, 2048, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16).cuda()
    with torch.no_grad():
        y, st = m.prefill(x)
    s = int(d["tok_stride"])
    err = max_rel(to_np(y[:, ::s]), d["y_tok"])
    print(f"config 3 (first {T} tokens of row 0): y max rel err {err:.2e}")
    assert err < BF16_TOL
    _stats_close(y, d, "y", BF16_TOL)
    _states_close(st, d, "", list(d["heads"]), BF16_TOL, BF16_TOL)


def test_config4_teacher_forced_decode():
    """Prefill then step with the reference's own greedy tokens fed back (teacher forcing), so
    every step's inputs are the reference's: hidden states and logits must agree.  Where the
    reference's top-2 logit margin is larger than our logit error, the argmax must agree too."""
    d = load("cfg4_decode")
    lm = _lm()
    prompt = torch.from_numpy(d["prompt"]).cuda()
    gen = torch.from_numpy(d["gen"]).cuda()
    n = gen.shape[1]
    hid, lgs = [], []
    with torch.no_grad():
        x = lm.embedding(prompt)
        states = []
        for blk in lm.layers:
            x, st = blk.prefill(x)
            states.append(st)
        h = lm.norm(x)[:, -1]
        hid.append(h)
        lgs.append(lm.lm_head(h))
        for i in range(1, n):
            x = lm.embedding(gen[:, i - 1])
            for j, blk in enumerate(lm.layers):
                x, states[j] = blk.step(x, states[j])
            h = lm.norm(x)
            hid.append(h)
            lgs.append(lm.lm_head(h))
    hid = torch.stack(hid, 1)
    lgs = torch.stack(lgs, 1).float()
    ss = int(d["step_stride"])
    eh = max_rel(to_np(hid[:, ::ss]), d["hid_step"])
    steps = list(d["logit_steps"])
    el = max_rel(to_np(lgs[:, steps]), d["logits"])
    fh, fl = float(d["floor.hidden"]), float(d["floor.logits"])
    print(f"config 4 teacher-forced: hidden max rel err {eh:.2e} (reference bf16 floor {fh:.2e}), "
          f"logits {el:.2e} (floor {fl:.2e})")
    assert eh < max(BF16_TOL, 2 * fh) and el < max(BF16_TOL, 2 * fl)
    # argmax agreement wherever the reference's margin exceeds twice our worst logit deviation
    dev = float(np.abs(to_np(lgs[:, steps]) - d["logits"]).max())
    margin = d["margin"]
    sure = margin > 2 * dev
    agree = (lgs.argmax(-1).cpu().numpy() == d["gen"])
    print(f"config 4: {int(sure.sum())} of {sure.size} steps with a clear margin, "
          f"argmax agreement there {float(agree[sure].mean()):.3f}, everywhere {float(agree.mean()):.3f}")
    assert agree[sure].all()


def test_config4_free_running_greedy_tokens():
    """The CUDA-graph decoder's own greedy tokens against the reference's: they agree up to the
    first step where the reference's top-2 margin is within bf16 noise (a near-tie, after which
    the two runs legitimately continue from different tokens)."""
    from mamba3_b200.decode import GraphDecoder

    d = load("cfg4_decode")
    lm = _lm()
    prompt = torch.from_numpy(d["prompt"]).cuda()
    n = d["gen"].shape[1]
    dec = GraphDecoder(lm, batch_size=prompt.shape[0], max_new_tokens=n)
    out = dec.generate(prompt, temperature=0.0)[:, prompt.shape[1]:].cpu().numpy()
    rate = float((out == d["gen"]).mean())
    print(f"config 4 free-running greedy: token match rate {rate:.3f}")
    for r in range(out.shape[0]):
        diff = np.nonzero(out[r] != d["gen"][r])[0]
        if diff.size:
            first = int(diff[0])
            assert d["margin"][r, first] < 0.05, (r, first, float(d["margin"][r, first]))
