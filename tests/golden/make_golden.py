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
