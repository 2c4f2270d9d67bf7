"""Generate golden vectors by running the unmodified reference (dorayaku/mamba3) on CPU.

Run in a container that has the reference checked out (it is not available on GPU boxes):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py [--ref /path/to/reference]

Writes ``tests/golden/*.npz``.  Inputs are drawn on CPU with
``torch.Generator().manual_seed(seed)`` in fp32; weights come from the reference's
own default init under ``torch.manual_seed(seed)``, optionally perturbed (so that
every parameter -- biases, MIMO factors, norm weights -- takes generic values).
Everything is computed by the reference's fp32 CPU path.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import sys
import time
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _np(t):
    return t.detach().cpu().numpy()


def _perturb(module, seed):
    g = torch.Generator().manual_seed(seed + 1000)
    with torch.no_grad():
        for name, p in module.named_parameters():
            if name.endswith("in_proj.weight") or name.endswith("out_proj.weight"):
                continue
            p.add_(0.25 * torch.randn(p.shape, generator=g))


def layer_case(M, name, seed, B, T, perturb, n_steps=4, **kw):
    torch.manual_seed(seed)
    layer = M.KulaMamba(**kw).eval()
    if perturb:
        _perturb(layer, seed)
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, T + n_steps, kw["d_model"], generator=g)
    with torch.no_grad():
        y = layer(x[:, :T])
        _, st = layer.prefill(x[:, :T])
        ys = []
        s = {k: v.clone() for k, v in st.items()}
        for t in range(T, T + n_steps):
            yt, s = layer.step(x[:, t:t + 1], s)
            ys.append(yt[:, 0])
        y_steps = torch.stack(ys, 1)
    out = {f"sd.{k}": _np(v) for k, v in layer.state_dict().items()}
    out.update(x=_np(x), y=_np(y), pf_h=_np(st["h"]), pf_angle=_np(st["angle"]), pf_prev_BX=_np(st["prev_BX"]),
               y_steps=_np(y_steps), st_h=_np(s["h"]), st_angle=_np(s["angle"]), st_prev_BX=_np(s["prev_BX"]),
               T=np.int64(T), n_steps=np.int64(n_steps), seed=np.int64(seed), perturb=np.int64(perturb))
    for k, v in kw.items():
        out[f"cfg.{k}"] = np.asarray(-1 if v is None else v)
    np.savez_compressed(HERE / f"layer_{name}.npz", **out)


def layer_grad_case(M, name, seed, B, T, perturb, **kw):
    """Parameter and input gradients of the reference layer for the loss <y, gy> (CPU fp32,
    train mode): what loss.backward() leaves in .grad (mamba3 tests:81-91 check only that
    they exist and are finite; these pin their values)."""
    torch.manual_seed(seed)
    layer = M.KulaMamba(**kw).train()
    if perturb:
        _perturb(layer, seed)
    g = torch.Generator().manual_seed(seed + 7)
    x = torch.randn(B, T, kw["d_model"], generator=g).requires_grad_(True)
    gy = torch.randn(B, T, kw["d_model"], generator=g)
    y = layer(x)
    (y * gy).sum().backward()
    out = {f"sd.{k}": _np(v) for k, v in layer.state_dict().items()}
    out.update({f"grad.{k}": _np(p.grad) for k, p in layer.named_parameters()})
    out.update(x=_np(x), gy=_np(gy), y=_np(y), grad_x=_np(x.grad), T=np.int64(T), seed=np.int64(seed))
    for k, v in kw.items():
        out[f"cfg.{k}"] = np.asarray(v)
    np.savez_compressed(HERE / f"grad_{name}.npz", **out)


def big_layer_case(M, name, seed, B, T):
    """BASELINE layer dims; weights are not stored (regenerated from ``seed``), only checksums."""
    kw = dict(d_model=768, d_state=128, expand=2, headdim=64, mimo_rank=2, chunk_size=64)
    torch.manual_seed(seed)
    layer = M.KulaMamba(**kw).eval()
    g = torch.Generator().manual_seed(seed + 1)
    x = torch.randn(B, T, 768, generator=g)
    with torch.no_grad():
        y, st = layer.prefill(x)
    sums = {f"wsum.{k}": np.float64(v.double().sum()) for k, v in layer.state_dict().items()}
    w = layer.in_proj.weight.detach().contiguous().numpy()
    np.savez_compressed(
        HERE / f"biglayer_{name}.npz", x=_np(x), y=_np(y), pf_h=_np(st["h"]), pf_angle=_np(st["angle"]),
        pf_prev_BX=_np(st["prev_BX"]), seed=np.int64(seed),
        in_proj_sha1=np.bytes_(hashlib.sha1(w.tobytes()).hexdigest().encode()), **sums)


def ssd_case(M, name, seed, B, T, H, P, R, N, CS, beta=True, with_h_init=True):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
    x_g, x_b = r(B, T, H, P, R), r(B, T, H, P, R)
    B_g, B_b, C = r(B, T, H, N, R), r(B, T, H, N, R), r(B, T, H, N, R)
    dt = torch.rand(B, T, H, generator=g) * 0.1 + 0.01
    A = -torch.exp(r(H).clamp(-4, -1))
    D = r(H)
    x_raw = r(B, T, H, P, R)
    h_init = r(B, H, P, N) if with_h_init else None
    out = M.chunked_ssd(x_g, x_b if beta else None, B_g, B_b if beta else None, C, dt, A, D, x_raw, CS,
                        h_init=h_init, return_final_state=True)
    d = dict(x_g=x_g, x_b=x_b, B_g=B_g, B_b=B_b, C=C, dt=dt, A=A, D=D, x_raw=x_raw, y=out.y, h_final=out.h_final)
    if h_init is not None:
        d["h_init"] = h_init
    d = {k: _np(v) for k, v in d.items()}
    np.savez_compressed(HERE / f"ssd_{name}.npz", CS=np.int64(CS), beta=np.int64(beta), **d)


def ssd_bwd_case(M, name, seed, B, T, H, P, R, N, CS, beta=True, with_h_init=True, with_final=True):
    """Gradients of the reference's chunked_ssd through torch autograd (CPU fp32) for the loss
    <y, gy> + <h_final, ghf>: every input that takes a gradient, seeded inputs as ssd_case."""
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
    ins = dict(x_g=r(B, T, H, P, R), x_b=r(B, T, H, P, R), B_g=r(B, T, H, N, R), B_b=r(B, T, H, N, R),
               C=r(B, T, H, N, R), dt=torch.rand(B, T, H, generator=g) * 0.1 + 0.01,
               A=-torch.exp(r(H).clamp(-4, -1)), D=r(H), x_raw=r(B, T, H, P, R))
    ins["h_init"] = r(B, H, P, N) if with_h_init else None
    if not beta:
        ins["x_b"] = ins["B_b"] = None
    gy = r(B, T, H, P, R)
    ghf = r(B, H, P, N) if with_final else None
    leaves = {k: v.clone().requires_grad_(True) for k, v in ins.items() if v is not None}
    args = {k: leaves.get(k) for k in ins}
    out = M.chunked_ssd(args["x_g"], args["x_b"], args["B_g"], args["B_b"], args["C"], args["dt"], args["A"],
                        args["D"], args["x_raw"], CS, h_init=args["h_init"], return_final_state=with_final)
    loss = (out.y * gy).sum() + ((out.h_final * ghf).sum() if with_final else 0.0)
    names = list(leaves)
    grads = torch.autograd.grad(loss, [leaves[k] for k in names])
    d = {k: _np(v) for k, v in ins.items() if v is not None}
    d.update({f"d_{k}": _np(gr) for k, gr in zip(names, grads)})
    d.update(gy=_np(gy), y=_np(out.y))
    if with_final:
        d.update(ghf=_np(ghf), h_final=_np(out.h_final))
    np.savez_compressed(HERE / f"ssdbwd_{name}.npz", CS=np.int64(CS), beta=np.int64(beta), **d)


def scan_case(M, name, seed, B, K, H, PN, with_h_init):
    g = torch.Generator().manual_seed(seed)
    decay = torch.rand(B, K, H, generator=g) * 0.9
    h_chunk = torch.randn(B, K, H, PN, generator=g)
    h_init = torch.randn(B, H, PN, generator=g) if with_h_init else None
    hs = M.ssd_scan(decay, h_chunk, h_init)
    d = dict(decay=_np(decay), h_chunk=_np(h_chunk), h_states=_np(hs))
    if with_h_init:
        d["h_init"] = _np(h_init)
    np.savez_compressed(HERE / f"scan_{name}.npz", **d)


def scan_bwd_case(M, name, seed, B, K, H, PN, with_h_init):
    """Gradients of the reference's ssd_scan through its autograd Function (SSDScanFn.backward,
    mamba3/scan.py:102-140; on CPU its torch loop mamba3/scan.py:47-62)."""
    g = torch.Generator().manual_seed(seed)
    decay = (torch.rand(B, K, H, generator=g) * 0.9).requires_grad_(True)
    h_chunk = torch.randn(B, K, H, PN, generator=g).requires_grad_(True)
    h_init = torch.randn(B, H, PN, generator=g).requires_grad_(True) if with_h_init else None
    grad_h = torch.randn(B, K, H, PN, generator=g)
    hs = M.ssd_scan(decay, h_chunk, h_init)
    ins = [decay, h_chunk] + ([h_init] if with_h_init else [])
    grads = torch.autograd.grad(hs, ins, grad_h)
    d = dict(decay=_np(decay), h_chunk=_np(h_chunk), grad_h=_np(grad_h), h_states=_np(hs), d_decay=_np(grads[0]),
             d_chunk=_np(grads[1]))
    if with_h_init:
        d.update(h_init=_np(h_init), d_h_init=_np(grads[2]))
    np.savez_compressed(HERE / f"scanbwd_{name}.npz", **d)


def lm_case(M, name, seed, B, T, n_new, **kw):
    torch.manual_seed(seed)
    lm = M.KulaMambaLM(**kw).eval()
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, kw["vocab_size"], (B, T), generator=g)
    with torch.no_grad():
        logits = lm(ids)["logits"]
        gen = lm.generate(ids, max_new_tokens=n_new, temperature=0.0)
    out = {f"sd.{k}": _np(v) for k, v in lm.state_dict().items()}
    out.update(ids=_np(ids), logits=_np(logits), gen=_np(gen), seed=np.int64(seed))
    for k, v in kw.items():
        out[f"cfg.{k}"] = np.asarray(v)
    np.savez_compressed(HERE / f"lm_{name}.npz", **out)


# ---------------------------------------------------------------------------
# BASELINE configs 0-4 at their own sizes.  The full outputs are too large to commit,
# so each fixture keeps evenly spaced token (or step) slices, a few heads of the states,
# and whole-tensor statistics (absmax, sum of squares) that a test compares at full size.
# ---------------------------------------------------------------------------
CFG_LAYER = dict(d_model=768, d_state=128, expand=2, headdim=64, mimo_rank=2, chunk_size=64)
CFG_LM = dict(vocab_size=32000, d_model=768, n_layers=24, d_state=128, headdim=64, mimo_rank=2,
              residual_scale="depth")
CFG3_LAYER = dict(d_model=2048, d_state=128, expand=2, headdim=64, mimo_rank=4, chunk_size=64)


def _bf16_round_(module):
    """Round every parameter to bf16 in place (values stay fp32): the weights a bf16 model holds."""
    with torch.no_grad():
        for p in module.parameters():
            p.copy_(p.to(torch.bfloat16).float())


def _stats(prefix, t):
    t = t.detach().double()
    return {f"{prefix}.absmax": np.float64(t.abs().max()), f"{prefix}.sumsq": np.float64((t * t).sum()),
            f"{prefix}.sum": np.float64(t.sum()), f"{prefix}.numel": np.int64(t.numel())}


def _state_slices(st, heads):
    return {"h": _np(st["h"][:, heads]), "angle": _np(st["angle"].float()),
            "prev_BX": _np(st["prev_BX"][:, heads]), **_stats("h", st["h"]), **_stats("prev_BX", st["prev_BX"])}


def cfg0_case(M):
    """Config 0: fp32 layer forward + prefill state, x (4, 1024, 768) ~ N(0,1) (CPU generator seed 0),
    weights = the reference's default init under torch.manual_seed(0)."""
    torch.manual_seed(0)
    layer = M.KulaMamba(**CFG_LAYER).eval()
    x = torch.randn(4, 1024, 768, generator=torch.Generator().manual_seed(0))
    with torch.no_grad():
        y, st = layer.prefill(x)
    heads = [0, 11, 23]
    out = {"y_tok": _np(y[:, ::16]), "tok_stride": np.int64(16), "heads": np.asarray(heads), **_stats("y", y)}
    out.update({f"st.{k}": v for k, v in _state_slices(st, heads).items()})
    np.savez_compressed(HERE / "cfg0_layer.npz", **out)


def cfg1_case(M, rows=(0, 7, 15)):
    """Config 1 rows: the config-0 weights rounded to bf16, x (16, 4096, 768) ~ N(0,1) (CPU generator
    seed 1) rounded to bf16; the reference's fp32 path on those values, one row at a time."""
    torch.manual_seed(0)
    layer = M.KulaMamba(**CFG_LAYER).eval()
    _bf16_round_(layer)
    x = torch.randn(16, 4096, 768, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16).float()
    heads = [0, 12, 23]
    out = {"rows": np.asarray(rows), "tok_stride": np.int64(32), "heads": np.asarray(heads)}
    for i, r in enumerate(rows):
        with torch.no_grad():
            y, st = layer.prefill(x[r:r + 1])
        out[f"r{i}.y_tok"] = _np(y[:, ::32])
        out.update({f"r{i}.{k}": v for k, v in _stats("y", y).items()})
        out.update({f"r{i}.st.{k}": v for k, v in _state_slices(st, heads).items()})
    np.savez_compressed(HERE / "cfg1_rows.npz", **out)


def _lm_bf16(M, seed=2):
    torch.manual_seed(seed)
    lm = M.KulaMambaLM(**CFG_LM).eval()
    _bf16_round_(lm)
    return lm


def cfg2_case(M, rows=(0, 31, 63)):
    """Config 2 rows: the 24-layer LM under torch.manual_seed(2) with bf16-rounded weights, input_ids
    (64, 2048) uniform in [0, 32000) (CPU generator seed 2); final-norm hidden states every 32nd
    position and full logits at three positions (mamba3/block.py:178-193)."""
    lm = _lm_bf16(M)
    ids = torch.randint(0, 32000, (64, 2048), generator=torch.Generator().manual_seed(2))
    cap = {}
    hk = lm.norm.register_forward_hook(lambda m, i, o: cap.__setitem__("h", o.detach()))
    pos = [0, 1023, 2047]
    out = {"rows": np.asarray(rows), "tok_stride": np.int64(32), "logit_pos": np.asarray(pos)}
    for i, r in enumerate(rows):
        with torch.no_grad():
            logits = lm(ids[r:r + 1])["logits"]
        out[f"r{i}.hid_tok"] = _np(cap["h"][:, ::32])
        out[f"r{i}.logits"] = _np(logits[:, pos])
        out.update({f"r{i}.{k}": v for k, v in _stats("logits", logits).items()})
        out[f"r{i}.argmax"] = _np(logits.argmax(-1))
    hk.remove()
    np.savez_compressed(HERE / "cfg2_lm.npz", **out)


def segmented_prefill(M, layer, x, seg):
    """The reference's layer prefill over x (B, T, d) computed segment by segment, each segment a
    call of the reference's chunked_ssd continuing from the previous one's state (h_init,
    mamba3/ssd.py:118-131).  The projection, norms, rotation (with the angle carried across
    segments), MIMO, trapezoid (with the previous token carried) and gate are the reference's own
    modules and formulas (mamba3/mamba3.py:192-256).  Needed where the reference cannot hold the
    whole sequence (config 3: its per-token P x N products would take hundreds of GB)."""
    from mamba3 import mamba3 as MM

    Bat, T, _ = x.shape
    H, P, N, R, G = layer.nheads, layer.headdim, layer.d_state, layer.mimo_rank, layer.ngroups
    h = None
    ang = torch.zeros(Bat, 1, H, N // 2)
    x_last = B_last = None
    ys = []
    for t0 in range(0, T, seg):
        xs = x[:, t0:t0 + seg]
        Ts = xs.shape[1]
        proj = layer.in_proj(xs)
        z, x_flat, B_flat, C_flat, dt_raw, lam_raw, theta_raw = layer._split_proj(proj)
        dt = F_softplus(dt_raw + layer.dt_bias)
        A = -torch.exp(layer.A_log)
        dA = torch.exp(A[None, None, :] * dt)
        B_r = layer.B_norm(B_flat.reshape(Bat, Ts, G, N * R)).reshape(Bat, Ts, G, N, R) + layer.B_bias[None, None]
        C_r = layer.C_norm(C_flat.reshape(Bat, Ts, G, N * R)).reshape(Bat, Ts, G, N, R) + layer.C_bias[None, None]
        B_r, C_r = layer._expand_groups(B_r), layer._expand_groups(C_r)
        cum = ang - (dt.unsqueeze(-1) * theta_raw.unsqueeze(-2)).cumsum(dim=1)
        c, s = torch.cos(cum).unsqueeze(-1).unsqueeze(-1), torch.sin(cum).unsqueeze(-1).unsqueeze(-1)
        B_r, C_r = MM._apply_rope(B_r, c, s, N, R), MM._apply_rope(C_r, c, s, N, R)
        ang = cum[:, -1:]
        x_r = x_flat.reshape(Bat, Ts, H, P, 1) * layer.mimo_x[None, None]
        lam = torch.sigmoid(lam_raw)
        x_gamma = x_r * lam.unsqueeze(-1).unsqueeze(-1)
        prev_x = torch.zeros_like(x_r[:, :1]) if x_last is None else x_last
        prev_B = torch.zeros_like(B_r[:, :1]) if B_last is None else B_last
        x_beta = torch.cat([prev_x, x_r[:, :-1]], 1) * ((1.0 - lam) * dA).unsqueeze(-1).unsqueeze(-1)
        B_prev = torch.cat([prev_B, B_r[:, :-1]], 1)
        o = M.chunked_ssd(x_gamma, x_beta, B_r, B_prev, C_r, dt, A, layer.D, x_r, layer.chunk_size, h_init=h,
                          return_final_state=True)
        h = o.h_final
        z_r = z.reshape(Bat, Ts, H, P).unsqueeze(-1) * layer.mimo_z[None, None]
        y = (o.y * F_silu(z_r) * layer.mimo_down[None, None]).sum(-1).reshape(Bat, Ts, layer.d_inner)
        ys.append(layer.out_proj(y))
        x_last, B_last = x_r[:, -1:], B_r[:, -1:]
    prev_BX = torch.einsum("bhnr,bhpr->bhpn", B_last[:, 0], x_last[:, 0])
    return torch.cat(ys, 1), {"h": h.float(), "angle": ang[:, 0], "prev_BX": prev_BX.float()}


def F_softplus(t):
    return torch.nn.functional.softplus(t)


def F_silu(t):
    return torch.nn.functional.silu(t)


def cfg3_case(M, T=16384, seg=1024):
    """Config 3, row 0 of x (2, 131072, 2048), first T tokens: the layer (d_model 2048, 64 heads,
    mimo_rank 4) under torch.manual_seed(0) with bf16-rounded weights; x ~ N(0,1) drawn as
    (1, T, 2048) from the CPU generator seed 3 and rounded to bf16; the segmented reference."""
    # the segmented form first reproduces the reference's own prefill on a small layer
    torch.manual_seed(5)
    small = M.KulaMamba(d_model=64, d_state=16, headdim=16, mimo_rank=4, chunk_size=8).eval()
    xs = torch.randn(2, 45, 64, generator=torch.Generator().manual_seed(5))
    with torch.no_grad():
        y0, s0 = small.prefill(xs)
        y1, s1 = segmented_prefill(M, small, xs, 16)
    for a, b in ((y0, y1), (s0["h"], s1["h"]), (s0["angle"], s1["angle"]), (s0["prev_BX"], s1["prev_BX"])):
        assert float((a - b).abs().max() / b.abs().max()) < 1e-5
    torch.manual_seed(0)
    layer = M.KulaMamba(**CFG3_LAYER).eval()
    _bf16_round_(layer)
    x = torch.randn(1, T, 2048, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16).float()
    with torch.no_grad():
        y, st = segmented_prefill(M, layer, x, seg)
    heads = [0, 31, 63]
    out = {"T": np.int64(T), "tok_stride": np.int64(128), "heads": np.asarray(heads), "y_tok": _np(y[:, ::128]),
           **_stats("y", y)}
    out.update({f"st.{k}": v for k, v in _state_slices(st, heads).items()})
    np.savez_compressed(HERE / "cfg3_seg.npz", **out)


def cfg4_case(M, rows=(0, 127, 255), new=256):
    """Config 4 rows: the config-2 LM (bf16-rounded weights) prefills prompts (256, 512) uniform in
    [0, 32000) (CPU generator seed 4) and generates `new` tokens greedily with the reference's own
    generate loop (mamba3/block.py:195-231).  Kept: the generated tokens, the final-norm hidden
    state of every 8th decode step, full logits at three steps, and each step's top-2 logit margin
    (a bf16 run may legitimately pick the other token where the margin is tiny)."""
    lm = _lm_bf16(M)
    ids = torch.randint(0, 32000, (256, 512), generator=torch.Generator().manual_seed(4))[list(rows)]
    hid, lg = [], []

    def hook(m, i, o):
        hid.append(o.detach()[:, -1] if o.dim() == 3 else o.detach())

    hk = lm.norm.register_forward_hook(hook)
    hk2 = lm.lm_head.register_forward_hook(lambda m, i, o: lg.append(o.detach()))
    with torch.no_grad():
        gen = lm.generate(ids, max_new_tokens=new, temperature=0.0)
    hk.remove()
    hk2.remove()
    # hid[i] / lg[i]: after the prefill (i = 0) and after each decode step; logits lg[i] choose token i
    logits = torch.stack(lg[:new], 1)  # (rows, new, vocab)
    top2 = logits.topk(2, dim=-1).values
    steps = [0, 127, 255]
    hid_all = torch.stack(hid[:new], 1)
    out = {"rows": np.asarray(rows), "prompt": _np(ids), "gen": _np(gen[:, 512:]), "step_stride": np.int64(8),
           "hid_step": _np(hid_all[:, ::8]), "logit_steps": np.asarray(steps), "logits": _np(logits[:, steps]),
           "margin": _np(top2[..., 0] - top2[..., 1])}
    np.savez_compressed(HERE / "cfg4_decode.npz", **out)


def _bf16_points(x):
    return x.to(torch.bfloat16).float()


def _lm_forward_bf16_points(lm, ids):
    """The reference LM's forward (mamba3/block.py:79-92,178-193) with every activation rounded to
    bf16 where a bf16 model holds it between modules: the embedding, each norm's output (the
    GEMM operands), each sublayer's output and the residual stream after each add.  Everything
    else stays fp32, so this is a lower bound of what any bf16 implementation deviates by."""
    x = _bf16_points(lm.embedding(ids))
    for blk in lm.layers:
        h = _bf16_points(blk.ssm(_bf16_points(blk.ssm_norm(x))))
        x = _bf16_points(x + h * blk.residual_scale)
        g = _bf16_points(blk.mlp(_bf16_points(blk.mlp_norm(x))))
        x = _bf16_points(x + g * blk.residual_scale)
    hid = _bf16_points(lm.norm(x))
    return hid, lm.lm_head(hid)


def cfg2_floor(M, rows=(0, 31, 63)):
    """Adds to cfg2_lm.npz how far the reference itself moves when its activations are bf16 at the
    module boundaries (same rows, slices and metric as the test): the floor of a bf16 LM."""
    d = dict(np.load(HERE / "cfg2_lm.npz"))
    lm = _lm_bf16(M)
    ids = torch.randint(0, 32000, (64, 2048), generator=torch.Generator().manual_seed(2))
    s, pos = int(d["tok_stride"]), list(d["logit_pos"])
    fh, fl = [], []
    for i, r in enumerate(rows):
        with torch.no_grad():
            hid, logits = _lm_forward_bf16_points(lm, ids[r:r + 1])
        ref_h, ref_l = d[f"r{i}.hid_tok"], d[f"r{i}.logits"]
        fh.append(float(np.abs(_np(hid[:, ::s]) - ref_h).max() / np.abs(ref_h).max()))
        fl.append(float(np.abs(_np(logits[:, pos]) - ref_l).max() / np.abs(ref_l).max()))
    d["floor.hidden"] = np.asarray(fh)
    d["floor.logits"] = np.asarray(fl)
    print("cfg2 bf16 floor: hidden", fh, "logits", fl)
    np.savez_compressed(HERE / "cfg2_lm.npz", **d)


def cfg4_floor(M):
    """Adds to cfg4_decode.npz the same floor for the teacher-forced decode: the reference's
    prefill and steps (mamba3/block.py:94-107) with bf16 activations at the module boundaries,
    fed the reference's own greedy tokens."""
    d = dict(np.load(HERE / "cfg4_decode.npz"))
    lm = _lm_bf16(M)
    prompt = torch.from_numpy(d["prompt"])
    gen = torch.from_numpy(d["gen"])
    n = gen.shape[1]
    hid, lgs = [], []
    with torch.no_grad():
        x = _bf16_points(lm.embedding(prompt))
        states = []
        for blk in lm.layers:
            h, st = blk.ssm.prefill(_bf16_points(blk.ssm_norm(x)))
            x = _bf16_points(x + _bf16_points(h) * blk.residual_scale)
            x = _bf16_points(x + _bf16_points(blk.mlp(_bf16_points(blk.mlp_norm(x)))) * blk.residual_scale)
            states.append(st)
        hh = _bf16_points(lm.norm(x)[:, -1])
        hid.append(hh)
        lgs.append(lm.lm_head(hh))
        for i in range(1, n):
            x = _bf16_points(lm.embedding(gen[:, i - 1]))
            for j, blk in enumerate(lm.layers):
                h, states[j] = blk.ssm.step(_bf16_points(blk.ssm_norm(x)), states[j])
                x = _bf16_points(x + _bf16_points(h) * blk.residual_scale)
                x = _bf16_points(x + _bf16_points(blk.mlp(_bf16_points(blk.mlp_norm(x)))) * blk.residual_scale)
            hh = _bf16_points(lm.norm(x))
            hid.append(hh)
            lgs.append(lm.lm_head(hh))
    hid = torch.stack(hid, 1)
    lgs = torch.stack(lgs, 1)
    ss, steps = int(d["step_stride"]), list(d["logit_steps"])
    fh = float(np.abs(_np(hid[:, ::ss]) - d["hid_step"]).max() / np.abs(d["hid_step"]).max())
    fl = float(np.abs(_np(lgs[:, steps]) - d["logits"]).max() / np.abs(d["logits"]).max())
    d["floor.hidden"] = np.float64(fh)
    d["floor.logits"] = np.float64(fl)
    print("cfg4 bf16 floor: hidden", fh, "logits", fl)
    np.savez_compressed(HERE / "cfg4_decode.npz", **d)


def config_groups(M, only=""):
    for name, fn in (("cfg0", cfg0_case), ("cfg1", cfg1_case), ("cfg2", cfg2_case), ("cfg3", cfg3_case),
                     ("cfg4", cfg4_case)):
        if only in ("configs", name):
            t0 = time.time()
            fn(M)
            print(f"{name}: {time.time() - t0:.1f} s", flush=True)
    for name, fn in (("cfg2", cfg2_floor), ("cfg4", cfg4_floor)):
        if only in ("configs", name, name + "floor"):
            t0 = time.time()
            fn(M)
            print(f"{name} floor: {time.time() - t0:.1f} s", flush=True)


def grad_groups(M):
    small = dict(d_model=64, d_state=16, headdim=16, mimo_rank=2, expand=2, chunk_size=8)
    layer_grad_case(M, "default", 61, 2, 21, True, **small)
    layer_grad_case(M, "rank1_ngroups2", 62, 1, 17, True, **{**small, "mimo_rank": 1, "ngroups": 2})
    layer_grad_case(M, "alloff", 63, 2, 12, True, **{**small, "use_trapezoidal": False, "use_complex_ssm": False})


def ssd_bwd_groups(M):
    ssd_bwd_case(M, "trap", 51, 2, 19, 2, 8, 2, 16, 8)
    ssd_bwd_case(M, "euler", 52, 1, 16, 3, 4, 1, 8, 4, beta=False, with_h_init=False, with_final=False)
    ssd_bwd_case(M, "rank4", 53, 1, 13, 2, 16, 4, 16, 8, with_final=False)
    ssd_bwd_case(M, "single", 54, 2, 1, 1, 4, 2, 8, 8)


def scan_bwd_groups(M):
    scan_bwd_case(M, "hinit", 33, 2, 5, 3, 16, True)
    scan_bwd_case(M, "zero", 34, 1, 9, 2, 24, False)
    scan_bwd_case(M, "k1", 35, 2, 1, 2, 8, True)
    scan_bwd_case(M, "odd", 36, 1, 6, 3, 13, True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("MAMBA3_REFERENCE", "/root/reference"))
    ap.add_argument("--only", default="", help="write only the fixture groups with this name prefix (e.g. scanbwd)")
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    import mamba3 as M  # the unmodified reference package

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    if args.only == "scanbwd":
        scan_bwd_groups(M)
        return
    if args.only == "ssdbwd":
        ssd_bwd_groups(M)
        return
    if args.only == "grad":
        grad_groups(M)
        return
    if args.only in ("cfg2floor", "cfg4floor"):
        config_groups(M, args.only)
        return
    if args.only == "configs" or args.only.startswith("cfg"):
        config_groups(M, args.only)
        return
    small = dict(d_model=64, d_state=16, headdim=16, mimo_rank=2, expand=2, chunk_size=8)
    layer_case(M, "default", 11, 2, 24, False, **small)
    layer_case(M, "perturbed", 12, 2, 37, True, **small)
    layer_case(M, "rank1", 13, 1, 20, True, **{**small, "mimo_rank": 1})
    layer_case(M, "rank4", 14, 1, 40, True, **{**small, "mimo_rank": 4})
    layer_case(M, "euler", 15, 1, 19, True, **{**small, "use_trapezoidal": False})
    layer_case(M, "real", 16, 1, 21, True, **{**small, "use_complex_ssm": False})
    layer_case(M, "alloff", 17, 1, 16, True, **{**small, "use_trapezoidal": False,
                                                 "use_complex_ssm": False, "mimo_rank": 1})
    layer_case(M, "ngroups2", 18, 2, 30, True, **{**small, "ngroups": 2})
    layer_case(M, "single", 19, 2, 1, True, **small)
    layer_case(M, "n128p64", 20, 1, 150, True, d_model=128, d_state=128, headdim=64, mimo_rank=2,
               expand=2, chunk_size=64)
    big_layer_case(M, "cfg0dims", 0, 1, 96)
    ssd_case(M, "trap", 21, 2, 16, 2, 4, 2, 8, 8)
    ssd_case(M, "euler", 22, 1, 21, 3, 8, 1, 16, 8, beta=False, with_h_init=False)
    ssd_case(M, "rank4", 23, 1, 40, 2, 16, 4, 16, 16)
    scan_case(M, "hinit", 31, 2, 4, 3, 8, True)
    scan_case(M, "zero", 32, 2, 7, 2, 24, False)
    scan_bwd_groups(M)
    ssd_bwd_groups(M)
    grad_groups(M)
    lm_case(M, "small", 41, 2, 12, 6, vocab_size=256, d_model=64, n_layers=2, d_state=16, headdim=16,
            mimo_rank=2, chunk_size=8, use_mlp=True, residual_scale="depth")
    total = sum(p.stat().st_size for p in HERE.glob("*.npz"))
    print(f"wrote {len(list(HERE.glob('*.npz')))} fixtures, {total / 1e6:.2f} MB")


if __name__ == "__main__":
    main()
