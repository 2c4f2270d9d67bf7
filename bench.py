#!/usr/bin/env python
"""Benchmark of the Mamba-3 SSD hot path on B200.

Headline workload: KulaMamba layer forward in bf16 with fp32
accumulation, x (16, 4096, 768) ~ N(0,1) seed 1, weights = the seed-0 default init
cast to bf16 (d_state 128, headdim 64 -> 24 heads, mimo_rank 2).  One step = one
layer forward over the batch.  Weak scaling under torchrun: every rank runs the
full config-1 batch on its own GPU (batch sharding, no collective).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

`--impl reference` times the unmodified reference (pip-installed into baseline/_ref)
on the host CPU, all cores, on a bounded sample of the same workload (2 rows x 512
tokens per step); the GPU arm's cpu_baseline times the same sample.
Prints one JSON line on rank 0.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CFG1 = dict(batch=16, seqlen=4096, d_model=768, d_state=128, headdim=64, mimo_rank=2, chunk_size=64, expand=2)
METRIC = "KulaMamba layer forward tokens/s (config 1, bf16)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-steps", type=int, default=12, help="timed reference steps of the cpu_baseline")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=None, help="override config-1 batch (profiling captures)")
    ap.add_argument("--seqlen", type=int, default=None, help="override config-1 seqlen (profiling captures)")
    ap.add_argument("--algo", type=int, default=0, help="layer algorithm: 0 auto, 1 fused, 2 chunk-parallel")
    ap.add_argument("--no-decode", action="store_true", help="skip the config-4 decode measurement")
    ap.add_argument("--no-seqpar", action="store_true", help="skip the config-3 sequence-sharded measurement")
    ap.add_argument("--no-lm", action="store_true", help="skip the config-2 LM forward measurement")
    ap.add_argument("--no-scan", action="store_true", help="skip the scan forward / backward measurement")
    ap.add_argument("--no-train", action="store_true", help="skip the layer training-step measurement")
    ap.add_argument("--e2e-pieces", type=int, default=8,
                    help="token ranges forward_host streams the host batch in (copy/compute overlap)")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# CPU baseline and reference arm: the unmodified reference on the host cores
# ---------------------------------------------------------------------------
# One reference step is a bounded sample of the config-1 workload: REF_ROWS rows of REF_TOKENS
# tokens through the reference's own KulaMamba.forward (mamba3/mamba3.py:260) on the CPU, fp32
# (its CPU path; the bf16 cast of config 1 is a GPU-side choice).  The same sample serves the GPU
# arm's cpu_baseline and the --impl reference arm.
REF_ROWS, REF_TOKENS = 2, 512


def _reference_package():
    """The unmodified reference package (dorayaku/mamba3), pip-installed into baseline/_ref, or None."""
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "mamba3" / "__init__.py").exists():
        return None
    if str(ref) not in sys.path:
        sys.path.insert(0, str(ref))
    import mamba3

    return mamba3


def _cpu_model():
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def reference_cpu(steps: int, warmup: int, rows: int = REF_ROWS, tokens: int = REF_TOKENS):
    """Time `steps` reference steps (after `warmup` untimed ones) on all host cores.  Uses the
    reference itself from baseline/_ref; without it, the numpy restatement in oracle/ (kind
    "port")."""
    import torch

    cores = len(os.sched_getaffinity(0))
    M = _reference_package()
    x = torch.randn(rows, tokens, 768, generator=torch.Generator().manual_seed(1))
    if M is not None:
        torch.set_num_threads(cores)
        torch.manual_seed(0)
        layer = M.KulaMamba(d_model=768, d_state=128, expand=2, headdim=64, mimo_rank=2, chunk_size=64).eval()
        run = lambda: layer(x)  # noqa: E731
        kind, what = "reference", "the reference's KulaMamba.forward (baseline/_ref, torch CPU, fp32)"
    else:
        import numpy as np

        import oracle
        from mamba3_b200.mamba3 import KulaMamba

        torch.manual_seed(0)
        m = KulaMamba(d_model=768, d_state=128, headdim=64, mimo_rank=2, chunk_size=64)
        sd = {k: v.float().numpy() for k, v in m.state_dict().items()}
        p = oracle.LayerParams.from_state_dict(sd, d_model=768, d_state=128, headdim=64, mimo_rank=2,
                                               chunk_size=64, dtype=np.float32)
        xn = x.numpy()
        run = lambda: oracle.layer_forward(p, xn)  # noqa: E731
        kind, what = "port", "the numpy restatement of the reference in oracle/ (baseline/_ref absent), fp32"
    with torch.no_grad():
        for _ in range(max(1, warmup)):
            run()
        t0 = time.perf_counter()
        for _ in range(steps):
            run()
        dt = time.perf_counter() - t0
    return {"value": steps * rows * tokens / dt, "unit": "tokens/s", "cores": cores, "kind": kind,
            "sample": f"{rows} rows x {tokens} tokens of config 1 per step, {steps} timed steps after {warmup}; "
                      f"{what}; host CPU: {_cpu_model()}",
            "seconds": round(dt, 2), "ms_per_step": dt / steps * 1e3}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cb = reference_cpu(args.steps, args.warmup)
    v = cb["value"]
    line = {"metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": cb["ms_per_step"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": "config 1: KulaMamba layer forward (d_model 768, d_state 128, headdim 64, "
                                   "mimo_rank 2), x (16, 4096, 768) per GPU",
                       "sampled": cb["sample"]},
            "cpu_baseline": cb,
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def algorithmic_work(B, T, H=24, P=64, N=128, R=2, d_model=768, d_proj=3696):
    """Per-launch algorithmic FLOPs / bytes of each kernel of one layer forward (bf16 I/O).

    Tiles per (batch, chunk, head) with the kernels' chunk length L = 128 / R: rows (t,r) = 128,
    columns (s,q) = 128.  FLOPs count the tensor-core contractions; bytes count compulsory HBM
    traffic (each input read once, each output written once)."""
    L = 128 // R
    K = (T + L - 1) // L
    chunks = B * K * H
    tok = B * T
    # the reference's algorithmic work per (batch, 64-token chunk, head), dense chunk tiles:
    # C B~^T 2(CS R)(CS 2R)N + mask X~ 2(CS R)(CS 2R)P + state 2P(CS 2R)N + out 2(CS R)NP
    CS = 64
    ref_chunks = B * ((T + CS - 1) // CS) * H
    f_ref = ref_chunks * (2 * (CS * R) * (CS * 2 * R) * N + 2 * (CS * R) * (CS * 2 * R) * P
                          + 2 * P * (CS * 2 * R) * N + 2 * (CS * R) * N * P)
    f_state = chunks * 2 * N * 128 * P                 # S'^T (N x P) over K = 128
    f_out = chunks * (2 * 128 * 128 * N + 2 * 128 * P * 128 + 2 * 128 * P * N)  # S, P X, C H'
    st_bytes = chunks * P * N * 2                      # one bf16 state tensor
    tok_x = tok * H * P * 2                            # x (or z) columns of proj
    tok_bc = tok * 2 * N * R * 2                       # B and C columns (shared by the heads)
    tok_sc = tok * (2 * H + N // 2) * 2                # dt, lam, theta
    return {
        "ssd_fused": {"flops": f_ref, "bytes": 2 * tok_x + tok_bc + tok_sc + tok * H * P * 2},
        "chunk_out": {"flops": f_out, "bytes": 2 * tok_x + tok_bc + tok_sc + st_bytes + tok * H * P * 2},
        "chunk_state": {"flops": f_state, "bytes": tok_x + tok_bc + tok_sc + st_bytes},
        "scan": {"flops": 0, "bytes": 2 * st_bytes},
        "prep": {"flops": 0, "bytes": tok_bc + tok_sc + tok * 8 + B * K * H * (N // 2) * 4},
        "in_proj": {"flops": 2 * tok * d_model * d_proj, "bytes": tok * (d_model + d_proj) * 2},
        "out_proj": {"flops": 2 * tok * H * P * d_model, "bytes": tok * (H * P + d_model) * 2},
    }


def _peaks():
    if (ROOT / "MEASURED_PEAKS.json").exists():
        d = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        d["source"] = "measured (MEASURED_PEAKS.json)"
        return d
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def _flop_roofline(flops_per_token, tokens_per_s, issued_per_token=None):
    """Tensor-core roofline of a whole forward: algorithmic FLOPs (SURVEY convention) per second
    against the measured bf16 peak; beside it the FLOPs the kernels actually issue."""
    pk = _peaks()
    ach = flops_per_token * tokens_per_s / 1e12
    out = {"bound": "tensor", "achieved": ach, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
           "frac": ach / pk["bf16_tflops"], "flops_per_token": flops_per_token, "peak_source": pk["source"]}
    if issued_per_token is not None:
        iss = issued_per_token * tokens_per_s / 1e12
        out.update(issued_flops_per_token=issued_per_token, issued_tflops=iss, issued_frac=iss / pk["bf16_tflops"])
    return out


def run_decode(dev, world, rank, barrier):
    """Config 4: the 24-layer config-2 LM prefills (256 / world, 512) prompt tokens per rank and
    decodes greedily with the CUDA-graph decoder (compact previous-token state).  Also times the
    step kernel of one layer alone against its state bytes: compact (h read + write, the previous
    token's B^ and x_r read + write) and the reference's layout (h, prev_BX: 4 P N fp32 per
    (batch, head))."""
    import torch
    import torch.distributed as dist

    from mamba3_b200 import KulaMambaLM, ops
    from mamba3_b200.decode import GraphDecoder

    Bg, Tp, new = 256, 512, 256
    B = max(1, Bg // world)
    torch.manual_seed(2)
    lm = KulaMambaLM(vocab_size=32000, d_model=768, n_layers=24, d_state=128, headdim=64, mimo_rank=2,
                     residual_scale="depth").to(dev, torch.bfloat16).eval()
    g = torch.Generator().manual_seed(4)
    ids = torch.randint(0, 32000, (Bg, Tp), generator=g)[rank * B:(rank + 1) * B].to(dev)
    dec = GraphDecoder(lm, batch_size=B, max_new_tokens=new)

    def timed(fn):
        torch.cuda.synchronize()
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    with torch.no_grad():
        dec.prefill(ids)
        dec.decode(4)  # capture + warm-up
        ms_prefill = timed(lambda: dec.prefill(ids))
        steps = new - 1
        ms_dec = timed(lambda: dec.decode(steps))
        # the step kernel of layer 0 alone, in place on a state: the compact form the decoder
        # uses (h + the previous token's B^ and x_r) and the reference's prev_BX form
        ssm = lm.layers[0].ssm
        st = dec.states[0]
        full = ssm.allocate_inference_state(B, device=dev)
        proj = ssm.in_proj(torch.randn(B, 768, device=dev, dtype=torch.bfloat16))
        y = torch.empty(B, ssm.nheads * ssm.headdim, device=dev, dtype=torch.bfloat16)
        dims = GraphDecoder._dims(ssm)
        prm = ssm._param_tensors()
        ws = dec.step_ws
        run_c = lambda: ops.step_ssm_compact_(prm, dims, proj, st["h"], st["prev_B"], st["prev_x"], st["angle"], y,  # noqa: E731
                                              workspace=ws)
        run_f = lambda: ops.step_ssm_(prm, dims, proj, full["h"], full["prev_BX"], full["angle"], y,  # noqa: E731
                                      workspace=ws)
        for _ in range(3):
            run_c()
            run_f()
        reps = 50
        ms_k = timed(lambda: [run_c() for _ in range(reps)]) / reps
        ms_f = timed(lambda: [run_f() for _ in range(reps)]) / reps
    H, P, N, R = ssm.nheads, ssm.headdim, ssm.d_state, ssm.mimo_rank
    state_bytes = (2 * P * N + 2 * (N + P) * R) * 4 * B * H  # h read + write, B^ / x_r read + write
    full_bytes = 4 * P * N * 4 * B * H
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() \
        else {"hbm_gbs": 6650.0}
    gbs = state_bytes / (ms_k / 1e3) / 1e9
    gbs_f = full_bytes / (ms_f / 1e3) / 1e9
    # decode roofline (HBM): every token step moves each layer's state once and reads the weights
    # once; compact state = h read + write and the previous B^ / x_r, the convention of SURVEY
    # 8(d) = the reference's layout (h read + write, prev_BX read, BX write)
    w_bytes = sum(p.numel() * p.element_size() for p in lm.parameters())
    nl = len(lm.layers)
    per_tok_compact = nl * state_bytes + w_bytes
    per_tok_ref = nl * full_bytes + w_bytes
    t_tok = ms_dec / steps / 1e3
    pk = _peaks()
    roof = {"bound": "hbm", "achieved": per_tok_compact / t_tok / 1e9, "peak": pk["hbm_gbs"], "unit": "GB/s",
            "frac": per_tok_compact / t_tok / 1e9 / pk["hbm_gbs"], "bytes_per_token_step": per_tok_compact,
            "weights_bytes": w_bytes, "state_bytes_per_layer": state_bytes,
            "convention_bytes_per_token_step": per_tok_ref,
            "convention_ms_at_peak": per_tok_ref / (pk["hbm_gbs"] * 1e9) * 1e3,
            "compact_ms_at_peak": per_tok_compact / (pk["hbm_gbs"] * 1e9) * 1e3, "peak_source": pk["source"]}
    return {"workload": f"config 4: 24-layer LM, prompt ({Bg}, {Tp}) + {new} greedy tokens, batch {B} per GPU, "
                        "CUDA-graph decode (GraphDecoder)",
            "decode_tokens_per_s": world * B * steps / (ms_dec / 1e3), "ms_per_token": ms_dec / steps,
            "roofline": roof,
            "prefill_tokens_per_s": world * B * Tp / (ms_prefill / 1e3),
            "step_kernel": {"ms": ms_k, "state": "compact (h + previous B^, x_r)", "state_bytes": state_bytes,
                            "achieved_gbs": gbs, "peak_gbs": peaks["hbm_gbs"], "frac": gbs / peaks["hbm_gbs"],
                            "batch": B, "heads": H},
            "step_kernel_prev_bx": {"ms": ms_f, "state_bytes": full_bytes, "achieved_gbs": gbs_f,
                                    "frac": gbs_f / peaks["hbm_gbs"]}}


def run_scan(dev, world, rank, barrier):
    """The inter-chunk scan alone, forward and backward, on config-1 shaped states in fp32 (the
    dtype the reference's scan_forward / scan_backward run in): B 16 per GPU, K 64 chunks, H 24,
    PN 64 x 128.  Algorithmic bytes: forward h_chunk read + h_states write, backward h_states
    and grad_h read + d_chunk write (the (B, K, H) decays are negligible).  Each tensor is
    805 MB, larger than L2, so consecutive launches do not hit in L2."""
    import torch
    import torch.distributed as dist

    from mamba3_b200 import _lib

    B, K, H, PN = 16, 64, 24, 64 * 128
    g = torch.Generator(device=dev).manual_seed(5)
    decay = torch.rand(B, K, H, device=dev, generator=g)
    hc = torch.randn(B, K, H, PN, device=dev, generator=g)
    gh = torch.randn(B, K, H, PN, device=dev, generator=g)
    hs = torch.empty_like(hc)
    fwd = lambda: _lib.scan_fwd(decay, hc, None, h_states=hs)  # noqa: E731
    bwd = lambda: _lib.scan_bwd(decay, hs, gh, False)  # noqa: E731

    def timed(fn, reps=20):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / reps
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    ms_f, ms_b = timed(fwd), timed(bwd)
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() \
        else {"hbm_gbs": 6650.0}
    el = B * K * H * PN
    out = {"workload": f"inter-chunk scan, fp32 states ({B}, {K}, {H}, {PN}) per GPU"}
    for name, ms, nbytes in (("fwd", ms_f, 2 * 4 * el), ("bwd", ms_b, 3 * 4 * el)):
        gbs = nbytes / (ms / 1e3) / 1e9
        out[name] = {"ms": ms, "bytes": nbytes, "achieved_gbs": gbs, "frac": gbs / peaks["hbm_gbs"]}
    del hc, gh, hs
    torch.cuda.empty_cache()
    # chunked_ssd backward (m3b_chunked_ssd_bwd) on config-1 shaped rows: the gradients of one
    # layer's SSD core for 2 batch rows of 4096 tokens, 24 heads, P 64, N 128, R 2 (trapezoid)
    Bb, T, Hh, P, N, R = 2, 4096, 24, 64, 128, 2
    r = lambda *s: torch.randn(*s, device=dev, generator=g).to(torch.bfloat16)  # noqa: E731
    args = (r(Bb, T, Hh, P, R), r(Bb, T, Hh, P, R), r(Bb, T, Hh, N, R), r(Bb, T, Hh, N, R), r(Bb, T, Hh, N, R),
            torch.rand(Bb, T, Hh, device=dev, generator=g) * 0.1, -torch.rand(Hh, device=dev, generator=g) - 0.1,
            torch.randn(Hh, device=dev, generator=g), r(Bb, T, Hh, P, R), r(Bb, T, Hh, P, R))
    ms_s = timed(lambda: _lib.chunked_ssd_bwd(*args), reps=3)  # tensor-core path (algo 0)
    ms_w = timed(lambda: _lib.chunked_ssd_bwd(*args, algo=1), reps=1)  # the token sweeps, for comparison
    # token-recurrence multiply-adds per (token, head): h and G updates P N (RI + R), dC N R P,
    # dX P RI N, dB N RI P -- a fixed count, so that both paths are measured on the same scale
    ri = 2 * R
    flops = 2.0 * P * N * (3 * ri + 2 * R) * Bb * T * Hh
    out["ssd_bwd"] = {"workload": f"chunked_ssd backward, bf16 ({Bb}, {T}) x {Hh} heads, P {P}, N {N}, R {R}",
                      "ms": ms_s, "tokens_per_s": Bb * T / (ms_s / 1e3), "path": "tensor cores (chunk products)",
                      "recurrence_tflops": flops / (ms_s / 1e3) / 1e12,
                      "token_sweeps_ms": ms_w}
    return out


def run_train(dev, world, rank, barrier):
    """One training step of the config-1 layer (16 x 4096 tokens, d_model 768, bf16): forward through
    the differentiable path (torch ops around chunked_ssd) and backward (the chunked_ssd and scan
    backward kernels plus torch autograd for the rest), loss = sum of the output."""
    import torch
    import torch.distributed as dist

    from mamba3_b200 import KulaMamba

    torch.manual_seed(0)
    layer = KulaMamba(d_model=768, d_state=128, headdim=64, mimo_rank=2).to(dev, torch.bfloat16).train()
    g = torch.Generator(device=dev).manual_seed(6)
    x = torch.randn(16, 4096, 768, device=dev, generator=g).to(torch.bfloat16)

    def step():
        layer.zero_grad(set_to_none=True)
        layer(x).float().sum().backward()

    for _ in range(2):
        step()
    torch.cuda.synchronize()
    barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 3
    a.record()
    for _ in range(reps):
        step()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / reps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return {"workload": "config-1 layer training step (forward + backward), x (16, 4096, 768) bf16 per GPU",
            "ms_per_step": ms, "tokens_per_s": world * 16 * 4096 / (ms / 1e3)}


def run_lm(dev, world, rank, barrier):
    """Config 2: KulaMambaLM forward (vocab 32000, d_model 768, 24 layers, bf16, weights seed 2)
    on input_ids (64, 2048) U[0, 32000), batch-sharded: 64 / G rows per rank, no collective."""
    import torch
    import torch.distributed as dist

    from mamba3_b200 import KulaMambaLM

    Bg, T = 64, 2048
    B = max(1, Bg // world)
    torch.manual_seed(2)
    lm = KulaMambaLM(vocab_size=32000, d_model=768, n_layers=24, d_state=128, headdim=64, mimo_rank=2,
                     residual_scale="depth").to(dev, torch.bfloat16).eval()
    g = torch.Generator().manual_seed(2)
    ids = torch.randint(0, 32000, (Bg, T), generator=g)[rank * B:(rank + 1) * B].to(dev)
    with torch.no_grad():
        lm(ids)
        torch.cuda.synchronize()
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 3
        a.record()
        for _ in range(reps):
            lm(ids)
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / reps
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
    del lm
    torch.cuda.empty_cache()
    # per token: 24 x (projections 8.04 + SSD core 7.08 (convention) + SwiGLU MLP 9.73) + lm_head 49.2
    # MFLOP; the kernels issue 3.94 MFLOP of SSD tiles per token and layer (128 x 128 tiles per
    # 64-token chunk and head: S, P W, C H, H update)
    tps_gpu = B * T / (ms / 1e3)
    conv = 24 * (8.04e6 + 7.08e6 + 9.73e6) + 49.2e6
    issued = 24 * (8.04e6 + 10.49e6 * 24 / 64 + 9.73e6) + 49.2e6
    return {"workload": f"config 2: KulaMambaLM forward, 24 layers, vocab 32000, ids ({Bg}, {T}), "
                        f"{B} rows per GPU", "tokens_per_s": world * B * T / (ms / 1e3), "ms_per_step": ms,
            "scaling": "strong (global batch 64 split over the GPUs)",
            "roofline": _flop_roofline(conv, tps_gpu, issued)}


def run_seqpar(dev, world, rank, barrier):
    """Config 3: one d_model 2048 / 64-head / mimo_rank 4 layer over x (2, 131072, 2048),
    sequence-sharded: rank r holds tokens [r T/G, (r+1) T/G) of both rows and runs
    seqpar.prefill_sharded (local pass, one all_gather of shard summaries, exact second pass).
    On one GPU it is the plain prefill.  With G > 1 every rank also runs the unsharded prefill
    once (untimed) and compares its own output rows and, on the last rank, the final state: the
    line reports max |a - b| / max |b| over all ranks."""
    import torch
    import torch.distributed as dist

    from mamba3_b200 import KulaMamba, seqpar

    B, T, D = 2, 131072, 2048
    torch.manual_seed(0)
    layer = KulaMamba(d_model=D, d_state=128, headdim=64, mimo_rank=4).to(dev, torch.bfloat16).eval()
    Ts = T // world
    g = torch.Generator(device=dev).manual_seed(3)
    x_full = torch.randn(B, T, D, generator=g, device=dev).to(torch.bfloat16)
    x = x_full[:, rank * Ts:(rank + 1) * Ts].contiguous()

    def run():
        if world == 1:
            return layer.prefill(x)
        return seqpar.prefill_sharded(layer, x, return_state=True)

    with torch.no_grad():
        run()
        torch.cuda.synchronize()
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 3
        a.record()
        for _ in range(reps):
            run()
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / reps
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        parity = None
        if world > 1:
            y_sh, st_sh = run()
            y_ref, st_ref = layer.prefill(x_full)
            ref = y_ref[:, rank * Ts:(rank + 1) * Ts].float()
            last = rank == world - 1
            num = torch.stack([(y_sh.float() - ref).abs().max(),
                               (st_sh["h"] - st_ref["h"]).abs().max() if last else torch.zeros((), device=dev)])
            den = torch.stack([ref.abs().max(), st_ref["h"].abs().max() if last else torch.zeros((), device=dev)])
            dist.all_reduce(num, op=dist.ReduceOp.MAX)
            dist.all_reduce(den, op=dist.ReduceOp.MAX)
            parity = {"y_max_rel": float(num[0] / den[0]), "h_final_max_rel": float(num[1] / den[1]),
                      "against": "the unsharded prefill of the same input on each rank's GPU"}
            del y_ref, st_ref, y_sh, st_sh
    del x_full
    torch.cuda.empty_cache()
    # per token: projections 55.3 + SSD core 62.9 (convention) MFLOP; the kernels issue 21.0
    # MFLOP of SSD tiles per token (128 x 128 tiles per 32-token chunk and head, 64 heads)
    tps = B * T / (ms / 1e3)
    out = {"workload": f"config 3: layer d_model {D}, 64 heads, mimo_rank 4, x ({B}, {T}, {D}) bf16, "
                       f"sequence-sharded over {world} GPU(s), {Ts} tokens per GPU",
           "tokens_per_s": tps, "ms_per_step": ms, "scaling": "strong",
           "exchange": "one all_gather of (S, PB, Om, Lam, c0) per layer" if world > 1 else "none",
           "roofline": _flop_roofline(55.3e6 + 62.9e6, tps / world, 55.3e6 + 10.49e6 * 64 / 32)}
    if parity is not None:
        out["parity"] = parity
    return out


def profiled_traffic(kernel, B, T):
    """DRAM bytes (read + write) per launch of `kernel` from the committed ncu summary
    profiles/<kernel>_cfg1.txt (line 'dram_bytes_per_launch: N' measured at B0 x T0 tokens,
    scaled by tokens), or None."""
    f = ROOT / "profiles" / f"{kernel}_cfg1.txt"
    if not f.exists():
        return None
    vals = {}
    for ln in f.read_text().splitlines():
        if ":" in ln:
            k, _, v = ln.partition(":")
            vals[k.strip()] = v.strip()
    try:
        b = float(vals["dram_bytes_per_launch"])
        tok = float(vals.get("tokens", B * T))
    except (KeyError, ValueError):
        return None
    return b * (B * T) / tok


def bind_to_gpu_numa_node(index):
    """Restrict this process to the CPUs of the NUMA node its GPU hangs off (Linux sysfs), so the
    pinned host buffers it allocates land in that node's memory.  Returns the node, or None
    when the topology is not exposed (the process then keeps its CPUs)."""
    import torch

    try:
        pr = torch.cuda.get_device_properties(index)
        bus = f"{pr.pci_domain_id:04x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
        node = int(open(f"/sys/bus/pci/devices/{bus}/numa_node").read().strip())
        if node < 0:
            return None
        cpus = set()
        for part in open(f"/sys/devices/system/node/node{node}/cpulist").read().strip().split(","):
            lo, _, hi = part.partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
        cpus &= os.sched_getaffinity(0)
        if cpus:
            os.sched_setaffinity(0, cpus)
            return node
    except (OSError, ValueError, AttributeError):
        pass
    return None


def host_copy_gbs(dev, nbytes=1 << 28, reps=5):
    """Pinned host <-> device copy bandwidth of this rank (GB/s each way), CUDA events."""
    import torch

    h = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    d = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    out = {}
    for name, fn in (("h2d_gbs", lambda: d.copy_(h, non_blocking=True)),
                     ("d2h_gbs", lambda: h.copy_(d, non_blocking=True))):
        fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        out[name] = nbytes * reps / (a.elapsed_time(b) / 1e3) / 1e9
    # both directions at once (as forward_host runs them): bytes moved each way per second
    h2, d2 = torch.empty(nbytes, dtype=torch.uint8).pin_memory(), torch.empty(nbytes, dtype=torch.uint8, device=dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    cur = torch.cuda.current_stream(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record(cur)
    s_in.wait_stream(cur)
    s_out.wait_stream(cur)
    for _ in range(reps):
        with torch.cuda.stream(s_in):
            d.copy_(h, non_blocking=True)
        with torch.cuda.stream(s_out):
            h2.copy_(d2, non_blocking=True)
    cur.wait_stream(s_in)
    cur.wait_stream(s_out)
    b.record(cur)
    torch.cuda.synchronize()
    out["both_ways_gbs_each"] = nbytes * reps / (a.elapsed_time(b) / 1e3) / 1e9
    del h, d, h2, d2
    return out


def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    numa = bind_to_gpu_numa_node(local)  # before any pinned host buffer is allocated
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    from mamba3_b200 import KulaMamba, _lib
    from mamba3_b200.profiling import ClockSampler, stage_events

    c = dict(CFG1)
    if args.batch:
        c["batch"] = args.batch
    if args.seqlen:
        c["seqlen"] = args.seqlen
    B, T = c["batch"], c["seqlen"]
    from mamba3_b200 import ops as _ops

    _ops.set_layer_algo(args.algo)
    torch.manual_seed(0)
    layer = KulaMamba(d_model=c["d_model"], d_state=c["d_state"], headdim=c["headdim"], mimo_rank=c["mimo_rank"],
                      chunk_size=c["chunk_size"]).to(dev, torch.bfloat16).eval()
    g = torch.Generator().manual_seed(1 + rank)
    x_host = torch.randn(B, T, c["d_model"], generator=g).to(torch.bfloat16).pin_memory()
    x = x_host.to(dev)
    nst = len(_lib.LAYER_FWD_STAGES) + 1

    def mk():
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        return e

    ev = [[mk() for _ in range(nst + 2)] for _ in range(args.steps)]
    torch.cuda.synchronize()

    def step(i=None):
        if i is None:
            return layer(x)
        e = ev[i]
        e[0].record()
        proj, rms = layer._project(x)  # in_proj with the 1/rms of B and C from its epilogue
        with stage_events(e[1:1 + nst]):
            y = layer.ssd_from_proj(proj, rms=rms)
        out = layer.out_proj(y)
        e[-1].record()
        return out

    with torch.no_grad():
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clk:
            t0.record()
            for i in range(args.steps):
                step(i)
            t1.record()
            torch.cuda.synchronize()
        barrier()
        ms = t0.elapsed_time(t1) / args.steps
        if world > 1:
            tt = torch.tensor([ms], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            ms = float(tt.item())
        # per-kernel durations (ms), averaged over the timed steps
        names = ["in_proj", *_lib.LAYER_FWD_STAGES, "out_proj"]
        per = {n: 0.0 for n in names}
        for e in ev:
            marks = [e[0], *e[1:1 + nst], e[-1]]
            per["in_proj"] += e[0].elapsed_time(e[1])
            for j, n in enumerate(_lib.LAYER_FWD_STAGES):
                per[n] += e[1 + j].elapsed_time(e[2 + j])
            per["out_proj"] += e[nst].elapsed_time(e[-1])
            del marks
        per = {k: v / args.steps for k, v in per.items()}
        # the fused path leaves the angle / chunk-state / scan stages empty and times its single
        # kernel in the chunk_out slot
        fused = per["angle_prefix"] + per["chunk_state"] + per["scan"] < 0.02
        if fused:
            per["ssd_fused"] = per.pop("chunk_out")
            for k in ("angle_prefix", "chunk_state", "scan"):
                per.pop(k)
        # in_proj_kernel + ssd_fused (the projection's epilogue replaces prep) | in_proj_kernel,
        # prep, angle, state, scan, out
        launches_per_step = 2 if fused else 6
        if fused:
            per.pop("prep")

        # end to end through the public API: pinned host x -> layer -> pinned host y, streamed by
        # forward_host in token ranges so the copies in, the layer and the copies out overlap
        y_host = torch.empty(B, T, c["d_model"], dtype=torch.bfloat16).pin_memory()
        for _ in range(2):
            layer.forward_host(x_host, y_host, pieces=args.e2e_pieces, graph=True)
        torch.cuda.synchronize()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        ke = max(3, args.steps // 2)
        e0.record()
        for _ in range(ke):
            layer.forward_host(x_host, y_host, pieces=args.e2e_pieces, graph=True)
        e1.record()
        torch.cuda.synchronize()
        ms_e2e = e0.elapsed_time(e1) / ke
        if world > 1:
            tt = torch.tensor([ms_e2e], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            ms_e2e = float(tt.item())
        # every rank's host link, measured alone and then all ranks at once (contention)
        hc_alone = host_copy_gbs(dev) if rank == 0 else None
        barrier()
        hc = host_copy_gbs(dev)
        hcv = torch.tensor([hc["h2d_gbs"], hc["d2h_gbs"], hc["both_ways_gbs_each"]], device=dev)
        if world > 1:
            dist.all_reduce(hcv, op=dist.ReduceOp.MIN)

    decode = None if args.no_decode else run_decode(dev, world, rank, barrier)
    seqp = None if args.no_seqpar else run_seqpar(dev, world, rank, barrier)
    lmf = None if args.no_lm else run_lm(dev, world, rank, barrier)
    scan = None if args.no_scan else run_scan(dev, world, rank, barrier)
    train = None if args.no_train else run_train(dev, world, rank, barrier)

    if rank == 0:
        import math

        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() \
            else {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "fallback": True}
        work = algorithmic_work(B, T)
        ours = {k: v for k, v in per.items() if k not in ("in_proj", "out_proj", "last_bx")}
        dom = max(ours, key=ours.get)
        w = work.get(dom, {"flops": 0, "bytes": 0})
        t_s = per[dom] / 1e3
        t_tc = w["flops"] / (peaks["bf16_tflops"] * 1e12)
        t_hbm = w["bytes"] / (peaks["hbm_gbs"] * 1e9)
        if t_tc >= t_hbm:
            roof = {"bound": "tensor", "achieved": w["flops"] / t_s / 1e12, "peak": peaks["bf16_tflops"],
                    "unit": "TFLOP/s"}
        else:
            roof = {"bound": "hbm", "achieved": w["bytes"] / t_s / 1e9, "peak": peaks["hbm_gbs"], "unit": "GB/s"}
        roof["frac"] = roof["achieved"] / roof["peak"]
        roof["kernel"] = dom
        if dom == "ssd_fused":
            # what the kernel issues to the tensor cores: 128 x 128 tiles per (batch, 64-token
            # chunk, head) -- S = C^B^T (K = 128), P W, C^H'^T, the H update (K = 128, N = 64)
            chunks = B * ((T + 63) // 64) * 24
            issued = chunks * (2 * 128 * 128 * 128 + 3 * 2 * 128 * 64 * 128)
            roof["issued_tflops"] = issued / t_s / 1e12
            roof["issued_frac"] = roof["issued_tflops"] / peaks["bf16_tflops"]
        roof["traffic"] = profiled_traffic(dom, B, T)
        roof["peak_source"] = "measured (MEASURED_PEAKS.json)" if not peaks.get("fallback") else "fallback"
        kern = {}
        for k, v in per.items():
            wk = work.get(k)
            d = {"ms": round(v, 4)}
            if wk and v > 0:
                if wk["flops"]:
                    d["tflops"] = round(wk["flops"] / (v / 1e3) / 1e12, 1)
                d["gbs"] = round(wk["bytes"] / (v / 1e3) / 1e9, 1)
            kern[k] = d
        tokens = world * B * T
        line = {
            "metric": METRIC, "value": tokens / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "config 1: KulaMamba layer forward (d_model 768, d_state 128, headdim 64, "
                                   "mimo_rank 2), x (16, 4096, 768) per GPU", "global_batch": world * B,
                       "seq_len": T, "parallelism": f"batch-sharded x{world}, no collective",
                       "l2": "inputs larger than L2 (>1.5 GB touched per step)"},
            "roofline": roof,
            "kernels_ms": kern,
            "gpu_launches": launches_per_step * args.steps,
            "e2e": {"value": tokens / (ms_e2e / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": x_host.numel() * 2, "d2h_bytes_per_step": y_host.numel() * 2,
                    "ms_per_step": ms_e2e,
                    "api": f"KulaMamba.forward_host(pieces={args.e2e_pieces}, graph=True)",
                    "host_link": {"rank0_alone": hc_alone, "all_ranks_min_h2d_gbs": float(hcv[0]),
                                  "all_ranks_min_d2h_gbs": float(hcv[1]),
                                  "all_ranks_min_both_ways_gbs_each": float(hcv[2]), "numa_node_rank0": numa,
                                  # copies in and out run at once: the link's rate in that mode bounds a step
                                  "bound_ms_per_step": max(x_host.numel(), y_host.numel()) * 2 / (float(hcv[2]) * 1e9)
                                  * 1e3,
                                  "bound_ms_per_step_one_way_rates": max(x_host.numel() * 2 / (float(hcv[0]) * 1e9),
                                                                         y_host.numel() * 2 / (float(hcv[1]) * 1e9))
                                  * 1e3}},
            "clocks": clk.summary(),
        }
        if decode is not None:
            line["decode"] = decode
        if seqp is not None:
            line["seqpar"] = seqp
        if lmf is not None:
            line["lm_forward"] = lmf
        if scan is not None:
            line["scan"] = scan
        if train is not None:
            line["train_step"] = train
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = reference_cpu(args.cpu_steps, 2)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
