"""The CPU oracle against golden vectors produced by the unmodified reference.

This pins the oracle: every GPU parity test compares the CUDA path with the
oracle, and this file shows the oracle reproduces the reference's own outputs.
"""

import numpy as np
import pytest

import oracle
from goldens import (LAYER_CASES, SCAN_BWD_CASES, SCAN_CASES, SSD_BWD_CASES, SSD_CASES, layer_cfg, load, max_rel,
                     state_dict)


@pytest.mark.parametrize("case", LAYER_CASES)
@pytest.mark.parametrize("dtype", [np.float64, np.float32])
def test_layer_forward_prefill_step(case, dtype):
    d = load(f"layer_{case}")
    cfg = layer_cfg(d)
    p = oracle.LayerParams.from_state_dict(state_dict(d), dtype=dtype, **cfg)
    T = int(d["T"])
    x = d["x"].astype(dtype)
    tol = 1e-5 if dtype == np.float64 else 1e-4
    y, st = oracle.layer_prefill(p, x[:, :T])
    assert max_rel(y, d["y"]) < tol
    assert max_rel(st["h"], d["pf_h"]) < tol
    assert max_rel(st["angle"], d["pf_angle"]) < tol
    assert max_rel(st["prev_BX"], d["pf_prev_BX"]) < tol
    ys = []
    for t in range(T, T + int(d["n_steps"])):
        yt, st = oracle.layer_step(p, x[:, t:t + 1], st)
        ys.append(yt[:, 0])
    assert max_rel(np.stack(ys, 1), d["y_steps"]) < tol
    assert max_rel(st["h"], d["st_h"]) < tol
    assert max_rel(st["prev_BX"], d["st_prev_BX"]) < tol
    assert max_rel(st["angle"], d["st_angle"]) < tol


@pytest.mark.parametrize("case", SSD_CASES)
def test_chunked_ssd(case):
    d = load(f"ssd_{case}")
    beta = bool(d["beta"])
    y, hf = oracle.chunked_ssd(d["x_g"].astype(np.float64), d["x_b"] if beta else None, d["B_g"],
                               d["B_b"] if beta else None, d["C"], d["dt"], d["A"], d["D"], d["x_raw"],
                               int(d["CS"]), h_init=d.get("h_init"), return_final_state=True)
    assert max_rel(y, d["y"]) < 1e-5
    assert max_rel(hf, d["h_final"]) < 1e-5


@pytest.mark.parametrize("case", SCAN_CASES)
def test_ssd_scan(case):
    d = load(f"scan_{case}")
    hs = oracle.ssd_scan(d["decay"].astype(np.float64), d["h_chunk"].astype(np.float64), d.get("h_init"))
    assert max_rel(hs, d["h_states"]) < 1e-6


@pytest.mark.parametrize("case", SSD_BWD_CASES)
def test_chunked_ssd_backward(case):
    """The oracle's chunked_ssd gradients == the reference's autograd gradients (fp32 CPU)."""
    d = load(f"ssdbwd_{case}")
    beta = bool(d["beta"])
    g = oracle.chunked_ssd_backward(d["x_g"], d["x_b"] if beta else None, d["B_g"], d["B_b"] if beta else None,
                                    d["C"], d["dt"], d["A"], d["D"], d["x_raw"], d["gy"], d.get("h_init"),
                                    d.get("ghf"))
    for k, v in g.items():
        if v is None:
            assert f"d_{k}" not in d
        else:
            assert max_rel(v, d[f"d_{k}"]) < 1e-5, k


@pytest.mark.parametrize("case", SCAN_BWD_CASES)
def test_ssd_scan_backward(case):
    """The oracle's scan gradients == the reference's autograd gradients (SSDScanFn.backward)."""
    d = load(f"scanbwd_{case}")
    hi = d.get("h_init")
    hs = oracle.ssd_scan(d["decay"].astype(np.float64), d["h_chunk"].astype(np.float64), hi)
    assert max_rel(hs, d["h_states"]) < 1e-6
    dd, dc, dhi = oracle.ssd_scan_backward(d["decay"].astype(np.float64), hs, d["grad_h"].astype(np.float64),
                                          has_h_init=hi is not None)
    assert max_rel(dd, d["d_decay"]) < 1e-5
    assert max_rel(dc, d["d_chunk"]) < 1e-6
    if hi is not None:
        assert max_rel(dhi, d["d_h_init"]) < 1e-6
    else:
        assert dhi is None


def test_lm_forward_and_greedy_generate():
    d = load("lm_small")
    cfg = {k[4:]: d[k].item() for k in d if k.startswith("cfg.")}
    sd = state_dict(d)
    blocks = _lm_blocks(sd, cfg)
    logits = oracle.lm_forward(sd["embedding.weight"].astype(np.float64), blocks, sd["norm.weight"],
                               sd["lm_head.weight"], d["ids"])
    assert max_rel(logits, d["logits"]) < 1e-5
    gen = oracle.lm_generate(sd["embedding.weight"].astype(np.float64), blocks, sd["norm.weight"],
                             sd["lm_head.weight"], d["ids"], int(d["gen"].shape[1] - d["ids"].shape[1]))
    assert (gen == d["gen"]).all()


def _lm_blocks(sd, cfg):
    import math

    from oracle.mamba3_oracle import BlockParams

    n = int(cfg["n_layers"])
    rs = 1.0 / math.sqrt(2 * n) if cfg.get("residual_scale") == "depth" else 1.0
    out = []
    for i in range(n):
        pre = f"layers.{i}."
        lp = oracle.LayerParams.from_state_dict(
            sd, prefix=pre + "ssm.", d_model=int(cfg["d_model"]), d_state=int(cfg["d_state"]),
            headdim=int(cfg["headdim"]), mimo_rank=int(cfg["mimo_rank"]), chunk_size=int(cfg["chunk_size"]))
        out.append(BlockParams(ssm=lp, ssm_norm_w=sd[pre + "ssm_norm.weight"], residual_scale=rs,
                               mlp_norm_w=sd.get(pre + "mlp_norm.weight"), w_gate=sd.get(pre + "mlp.w_gate.weight"),
                               w_up=sd.get(pre + "mlp.w_up.weight"), w_down=sd.get(pre + "mlp.w_down.weight")))
    return out
