"""Sequence-parallel prefill of one KulaMamba layer over the ranks of a process group.

Rank r of G holds tokens [r T/G, (r+1) T/G) of every batch row (the long-sequence
configuration).  For fixed inputs, the layer's state after a shard is an affine function of
the state before it.  With a = angle, h = state, pb = prev_BX at the shard's first token:

    h'  = e^Lam (h + c0 pb) + Rot(a) S        S, PB, Om: the shard's final h, prev_BX and
    a'  = a + Om                              angle from a zero state; Lam = sum of A dt over
    pb' = Rot(a) PB                           the shard; c0 = (1 - lam) dt of its first token

Rot(a) turns the (2i, 2i+1) columns of the (P, N) state by the angle pair a_i, the frame
in which a shard's rotated B terms live when its prefix angle is a (RoPE angles add, and
rotating both sides of a dot product leaves it unchanged, so the shard's own outputs do not
depend on a).  So:

1. every rank runs the layer on its shard from the zero state and keeps (S, PB, Om, Lam, c0);
2. one all_gather exchanges the tuples (2 P N + N/2 + 2 floats per (batch, head)) into one
   (world, summary) buffer;
3. rank r folds the tuples of ranks 0 .. r-1 into its exact initial state (one kernel,
   m3b_seqpar_fold; `fold` below is the same algebra in torch ops);
4. rank r runs the layer on its shard again from that state (prefill_from).

The exchange is the only collective.  Step 1 asks only for the state (no C^, no intra-chunk
products, no y), which costs a fraction of a full pass; the exchange is tiny.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def rotate_pairs(s: torch.Tensor, ang: torch.Tensor) -> torch.Tensor:
    """Rot(ang) on the (2i, 2i+1) columns of s (..., P, N) with ang (..., N/2):
    (s0, s1) -> (s0 cos - s1 sin, s0 sin + s1 cos), the rotation the layer applies to B."""
    c = torch.cos(ang).unsqueeze(-2)
    sn = torch.sin(ang).unsqueeze(-2)
    s0, s1 = s[..., 0::2], s[..., 1::2]
    return torch.stack((s0 * c - s1 * sn, s0 * sn + s1 * c), dim=-1).flatten(-2)


def shard_scalars(proj: torch.Tensor, A_log, dt_bias, H: int, P: int, N: int, R: int, G: int, trapezoidal: bool):
    """Lam = sum_t A dt_t over the shard (B, H) and c0 = (1 - lam_0) dt_0 (B, H) from the
    projection of the shard's tokens (layout of mamba3/mamba3.py:125-140)."""
    off_dt = 2 * H * P + 2 * G * N * R
    dt = F.softplus(proj[..., off_dt:off_dt + H].float() + dt_bias.float())
    A = -torch.exp(A_log.float())
    lam_sum = (dt * A).sum(dim=1)
    if trapezoidal:
        lam0 = torch.sigmoid(proj[:, 0, off_dt + H:off_dt + 2 * H].float())
        c0 = (1.0 - lam0) * dt[:, 0]
    else:
        c0 = torch.zeros_like(lam_sum)
    return lam_sum, c0


def advance(state: dict, aff: dict) -> dict:
    """The state after a shard with affine summary `aff`, given the state before it."""
    h, a, pb = state["h"], state["angle"], state["prev_BX"]
    e = torch.exp(aff["Lam"]).unsqueeze(-1).unsqueeze(-1)
    c0 = aff["c0"].unsqueeze(-1).unsqueeze(-1)
    return {"h": e * (h + c0 * pb) + rotate_pairs(aff["S"], a),
            "angle": a + aff["Om"],
            "prev_BX": rotate_pairs(aff["PB"], a)}


def zero_state(like: dict) -> dict:
    return {"h": torch.zeros_like(like["S"]), "angle": torch.zeros_like(like["Om"]),
            "prev_BX": torch.zeros_like(like["PB"])}


def fold(affs: list, upto: int) -> dict:
    """Initial state of shard `upto` from the summaries of shards 0 .. upto-1, in a fixed number
    of batched tensor operations whatever `upto` is.  Unrolling advance() from the zero state:
    the angle before shard g is a_g = sum_{j<g} Om_j, shard g's incoming prev_BX is
    pb_g = Rot(a_{g-1}) PB_{g-1} (zero for g = 0), and
        h = sum_{g<upto} exp(sum_{g<j<upto} Lam_j) (e^Lam_g c0_g pb_g + Rot(a_g) S_g)."""
    if upto <= 0:
        return zero_state(affs[0])
    st = {k: torch.stack([a[k] for a in affs[:upto]]) for k in _KEYS}  # leading dim: shard g
    om_c = torch.cumsum(st["Om"], 0)
    a_g = om_c - st["Om"]                                   # angle before shard g
    rs = rotate_pairs(st["S"], a_g)
    rpb = rotate_pairs(st["PB"], a_g)                       # shard g's final prev_BX, global frame
    pb_in = torch.cat([torch.zeros_like(rpb[:1]), rpb[:-1]])
    lam = st["Lam"]
    after = lam.sum(0, keepdim=True) - torch.cumsum(lam, 0)  # sum_{g<j<upto} Lam_j
    w = lambda t: t.unsqueeze(-1).unsqueeze(-1)  # noqa: E731  (B,H) -> (B,H,1,1)
    h = (w(torch.exp(after)) * (w(torch.exp(lam) * st["c0"]) * pb_in + rs)).sum(0)
    return {"h": h, "angle": om_c[-1], "prev_BX": rpb[-1]}


_KEYS = ("S", "PB", "Om", "Lam", "c0")


def pack(aff: dict) -> torch.Tensor:
    return torch.cat([aff[k].float().reshape(-1) for k in _KEYS])


def unpack(buf: torch.Tensor, like: dict) -> dict:
    out, o = {}, 0
    for k in _KEYS:
        n = like[k].numel()
        out[k] = buf[o:o + n].view(like[k].shape)
        o += n
    return out


def _gather_flat(aff: dict, group=None) -> torch.Tensor:
    """all_gather of every rank's packed summary into one (world, n) buffer.  A first all_gather
    of the summaries' shapes makes every rank raise ValueError, instead of exchanging garbage,
    when the ranks do not hold the same problem (batch rows, heads, headdim, d_state)."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    mine = pack(aff)
    shape = torch.tensor([d for k in _KEYS for d in (*aff[k].shape, -1)], dtype=torch.int64, device=mine.device)
    head = torch.zeros(64, dtype=torch.int64, device=mine.device)
    head[:min(64, shape.numel())] = shape[:64]
    heads = torch.empty(world * 64, dtype=torch.int64, device=mine.device)
    dist.all_gather_into_tensor(heads, head, group=group)
    heads = heads.view(world, 64)
    if not bool((heads == heads[:1]).all()):
        raise ValueError("seqpar.exchange: ranks hold summaries of different shapes "
                         f"({[h[h != 0].tolist()[:8] for h in heads]})")
    out = torch.empty(world * mine.numel(), dtype=mine.dtype, device=mine.device)
    dist.all_gather_into_tensor(out, mine, group=group)
    return out.view(world, mine.numel())


def exchange(aff: dict, group=None) -> list:
    """Every rank's summary, as a list of dicts (rank order)."""
    flat = _gather_flat(aff, group)
    return [unpack(flat[g], aff) for g in range(flat.shape[0])]


def fold_device(flat: torch.Tensor, upto: int, like: dict) -> dict:
    """fold() of the gathered (world, n) summaries in one kernel (m3b_seqpar_fold)."""
    from . import _lib

    Bt, H, P, N = like["S"].shape
    dev = flat.device
    st = {"h": torch.empty(Bt, H, P, N, dtype=torch.float32, device=dev),
          "angle": torch.empty(Bt, H, N // 2, dtype=torch.float32, device=dev),
          "prev_BX": torch.empty(Bt, H, P, N, dtype=torch.float32, device=dev)}
    _lib.seqpar_fold(flat, upto, Bt, H, P, N, st["h"], st["angle"], st["prev_BX"])
    return st


def layer_state_only(layer, proj: torch.Tensor, rms=None) -> dict:
    """The layer's state after `proj`'s tokens from the zero state, without the outputs: the
    kernels skip C, the intra-chunk products and y where they can (m3b_layer_fwd state_only).
    rms: the 1/rms rows the projection's epilogue gave with proj (optional)."""
    from . import _lib, ops

    d = layer._dims()
    H, P, N = d["H"], d["P"], d["N"]
    prm = ops._prm(H, P, N, d["R"], d["G"], d["trapezoidal"], d["complex_ssm"], d["norm_eps"],
                   *layer._param_tensors())
    proj = proj.contiguous()
    Bt, T, _ = proj.shape
    dev = proj.device
    y = torch.empty(Bt, T, H * P, dtype=proj.dtype, device=dev)  # required buffer; may stay unwritten
    f32 = dict(dtype=torch.float32, device=dev)
    st = {"h": torch.empty(Bt, H, P, N, **f32), "angle": torch.empty(Bt, H, N // 2, **f32),
          "prev_BX": torch.empty(Bt, H, P, N, **f32)}
    _lib.layer_fwd(prm, proj, y, h_final=st["h"], angle_final=st["angle"], prev_bx_final=st["prev_BX"],
                   algo=ops._LAYER_ALGO, state_only=True, rms_in=rms)
    return st


def layer_summary(layer, proj: torch.Tensor, rms=None) -> dict:
    """Step 1 on this rank's shard: the layer from the zero state, kept as an affine summary."""
    st = layer_state_only(layer, proj, rms)
    d = layer._dims()
    lam_sum, c0 = shard_scalars(proj, layer.A_log, layer.dt_bias, d["H"], d["P"], d["N"], d["R"], d["G"],
                                d["trapezoidal"])
    return {"S": st["h"], "PB": st["prev_BX"], "Om": st["angle"], "Lam": lam_sum, "c0": c0}


@torch.no_grad()
def prefill_sharded(layer, x_shard: torch.Tensor, group=None, return_state: bool = False):
    """KulaMamba.prefill of a sequence split over the ranks of `group` (rank r holds the r-th
    contiguous token range of every row): returns this rank's output rows (and the state after
    its shard, which on the last rank is the state after the whole sequence)."""
    import torch.distributed as dist

    rank = dist.get_rank(group)
    proj, rms = layer._project(x_shard)
    aff = layer_summary(layer, proj, rms)
    flat = _gather_flat(aff, group)
    st = fold_device(flat, rank, aff) if rank > 0 else None
    y, st_out = layer.ssd_from_proj(proj, return_state=True, state=st, rms=rms)
    out = layer.out_proj(y)
    return (out, st_out) if return_state else out
