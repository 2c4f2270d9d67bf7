"""Sequence-parallel prefill (mamba3_b200.seqpar): the cross-shard state algebra against the
oracle on CPU, the exchange over a 2-rank gloo group, and the whole scheme on one GPU.

The oracle (fp64 restatement of the reference) plays the layer on CPU: a shard's summary is
its prefill from the zero state; folding the summaries of the shards before a boundary must
give the state the oracle reaches by prefilling the whole prefix."""

import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import oracle
from goldens import max_rel
from helpers import oracle_params


def _setup(seed=0, R=2, trapezoidal=True, complex_ssm=True):
    from mamba3_b200 import KulaMamba

    torch.manual_seed(seed)
    m = KulaMamba(d_model=64, d_state=16, headdim=16, mimo_rank=R, use_trapezoidal=trapezoidal,
                  use_complex_ssm=complex_ssm)
    p = oracle_params(m)
    x = torch.randn(2, 90, 64, generator=torch.Generator().manual_seed(seed + 1), dtype=torch.float64).numpy()
    return m, p, x


def _summary(m, p, x_shard):
    """Oracle shard summary: prefill from zero + Lam, c0 from the shard's projection."""
    from mamba3_b200 import seqpar

    _, st = oracle.layer_prefill(p, x_shard)
    proj = torch.from_numpy(oracle.mamba3_oracle._linear(x_shard, p.in_proj_w, p.in_proj_b))
    d = m._dims()
    lam_sum, c0 = seqpar.shard_scalars(proj.double(), torch.from_numpy(p.A_log), torch.from_numpy(p.dt_bias),
                                       d["H"], d["P"], d["N"], d["R"], d["G"], d["trapezoidal"])
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).double()  # noqa: E731
    return {"S": t(st["h"]), "PB": t(st["prev_BX"]), "Om": t(st["angle"]), "Lam": lam_sum.double(),
            "c0": c0.double()}


def _shards(T, n):
    e = [T * i // n for i in range(n + 1)]
    return list(zip(e[:-1], e[1:]))


@pytest.mark.parametrize("variant", [dict(), dict(R=1), dict(trapezoidal=False), dict(complex_ssm=False)])
def test_fold_reaches_the_prefix_state(variant):
    from mamba3_b200 import seqpar

    m, p, x = _setup(**variant)
    cuts = _shards(x.shape[1], 3)
    affs = [_summary(m, p, x[:, a:b]) for a, b in cuts]
    for g in range(1, len(cuts)):
        st = seqpar.fold(affs, g)
        _, ref = oracle.layer_prefill(p, x[:, :cuts[g][0]])
        for k in ("h", "angle", "prev_BX"):
            assert max_rel(st[k].numpy(), ref[k]) < 1e-6, (g, k)  # Lam, c0 are formed in fp32


@pytest.mark.gpu
@pytest.mark.parametrize("world", [1, 3, 8])
def test_fold_kernel_matches_fold(world):
    """m3b_seqpar_fold over a gathered (world, n) buffer against fold() in float64 on the CPU
    (fold itself is pinned to the oracle's prefix states above), for every rank's upto."""
    from mamba3_b200 import seqpar

    g = torch.Generator().manual_seed(world)
    B, H, P, N = 2, 5, 16, 32
    affs = [{"S": torch.randn(B, H, P, N, generator=g), "PB": torch.randn(B, H, P, N, generator=g),
             "Om": 3 * torch.randn(B, H, N // 2, generator=g), "Lam": -torch.rand(B, H, generator=g) * 4,
             "c0": torch.rand(B, H, generator=g)} for _ in range(world)]
    flat = torch.stack([seqpar.pack(a) for a in affs]).cuda()
    for upto in range(world + 1):
        st = seqpar.fold_device(flat, upto, {k: v.cuda() for k, v in affs[0].items()})
        ref = seqpar.fold([{k: v.double() for k, v in a.items()} for a in affs], upto)
        for k in ("h", "angle", "prev_BX"):
            err = float((st[k].cpu().double() - ref[k]).abs().max() / max(float(ref[k].abs().max()), 1e-30))
            assert err < 1e-5 if upto > 0 else float(st[k].abs().max()) == 0.0, (upto, k, err)


def test_rotate_pairs_composes_angles():
    from mamba3_b200 import seqpar

    g = torch.Generator().manual_seed(3)
    s = torch.randn(2, 3, 4, 8, generator=g, dtype=torch.float64)
    a1 = torch.randn(2, 3, 4, generator=g, dtype=torch.float64)
    a2 = torch.randn(2, 3, 4, generator=g, dtype=torch.float64)
    both = seqpar.rotate_pairs(seqpar.rotate_pairs(s, a1), a2)
    assert torch.allclose(both, seqpar.rotate_pairs(s, a1 + a2), atol=1e-12)


def _gloo_worker(rank, world, port, out_q):
    import torch.distributed as dist

    from mamba3_b200 import seqpar

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        m, p, x = _setup(seed=5)
        a, b = _shards(x.shape[1], world)[rank]
        aff = {k: v.float() for k, v in _summary(m, p, x[:, a:b]).items()}
        affs = seqpar.exchange(aff)
        st = seqpar.fold(affs, rank)
        if rank > 0:
            _, ref = oracle.layer_prefill(p, x[:, :a])
            err = max(max_rel(st[k].double().numpy(), ref[k]) for k in ("h", "angle", "prev_BX"))
        else:
            err = float(max(st[k].abs().max() for k in st))  # rank 0 starts from zero
        out_q.put((rank, err))
    finally:
        dist.destroy_process_group()


def test_exchange_over_gloo_world2():
    """Two CPU ranks: all_gather of the fp32 summaries, fold, compare with the oracle."""
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gloo_worker, args=(r, 2, port, q)) for r in range(2)]
    for pr in procs:
        pr.start()
    res = dict(q.get(timeout=240) for _ in procs)
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    assert res[0] == 0.0
    assert res[1] < 1e-5  # fp32 exchange


def _free_port():
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_fault_worker(rank, world, port, scenario, out_q):
    """Failure scenarios of the exchange on CPU ranks (no GPU): 'mismatch' -- rank 1 holds a
    different problem (one batch row instead of two); 'departed' -- rank 1 leaves the group
    between steps, before the exchange, and rank 0's exchange must end with an error within the
    process group's timeout instead of waiting for good."""
    from datetime import timedelta

    import torch.distributed as dist

    from mamba3_b200 import seqpar

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    try:
        m, p, x = _setup(seed=5)
        a, b = _shards(x.shape[1], world)[rank]
        if scenario == "mismatch" and rank == 1:
            x = x[:1]
        if scenario == "departed" and rank == 1:
            out_q.put((rank, "left"))
            return  # leaves between steps: no collective in flight
        aff = {k: v.float() for k, v in _summary(m, p, x[:, a:b]).items()}
        try:
            seqpar.exchange(aff)
            out_q.put((rank, "no error"))
        except ValueError as e:
            out_q.put((rank, f"ValueError: {e}"))
        except Exception as e:  # noqa: BLE001  (gloo raises RuntimeError / DistBackendError)
            out_q.put((rank, f"{type(e).__name__}"))
    finally:
        if not (scenario == "departed" and rank == 1):
            dist.destroy_process_group()


@pytest.mark.parametrize("scenario", ["mismatch", "departed"])
def test_exchange_failures_over_gloo(scenario):
    import time

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_fault_worker, args=(r, 2, port, scenario, q)) for r in range(2)]
    t0 = time.time()
    for pr in procs:
        pr.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for pr in procs:
        pr.join(timeout=60)
    assert time.time() - t0 < 100
    if scenario == "mismatch":
        assert res[0].startswith("ValueError") and res[1].startswith("ValueError"), res
        assert "different shapes" in res[0]
    else:
        assert res[1] == "left"
        assert res[0] != "no error", res  # the remaining rank's exchange failed instead of hanging


@pytest.mark.gpu
@pytest.mark.parametrize("shards", [2, 4])
def test_sharded_prefill_on_one_gpu(shards):
    """The scheme with the CUDA layer, shards run one after another in one process."""
    from mamba3_b200 import KulaMamba, seqpar

    torch.manual_seed(14)
    m = KulaMamba(d_model=256, d_state=128, headdim=64, mimo_rank=2).cuda().to(torch.bfloat16).eval()
    x = torch.randn(2, 400, 256, generator=torch.Generator().manual_seed(15)).cuda().to(torch.bfloat16)
    with torch.no_grad():
        y_ref, st_ref = m.prefill(x)
        cuts = _shards(x.shape[1], shards)
        projs = [m.in_proj(x[:, a:b]) for a, b in cuts]
        affs = [seqpar.layer_summary(m, pr) for pr in projs]
        ys, st = [], None
        for g, pr in enumerate(projs):
            st_in = seqpar.fold(affs, g) if g > 0 else None
            y, st = m.ssd_from_proj(pr, return_state=True, state=st_in)
            ys.append(m.out_proj(y))
    assert max_rel(torch.cat(ys, 1).float().cpu().numpy(), y_ref.float().cpu().numpy()) < 2e-2
    for k in ("h", "angle", "prev_BX"):
        assert max_rel(st[k].float().cpu().numpy(), st_ref[k].float().cpu().numpy()) < 2e-2


@pytest.mark.gpu
@pytest.mark.parametrize("R,dtype", [(1, torch.bfloat16), (2, torch.bfloat16), (4, torch.bfloat16),
                                     (2, torch.float32)])
def test_state_only_pass_matches_prefill_state(R, dtype):
    """The state-only first pass (skips C^, the intra-chunk products and y on the TMA path;
    fp32 rows take the full path) gives prefill's state."""
    from mamba3_b200 import KulaMamba, seqpar

    torch.manual_seed(20 + R)
    m = KulaMamba(d_model=128, d_state=128, headdim=64, mimo_rank=R).cuda().to(dtype).eval()
    x = torch.randn(2, 300, 128, generator=torch.Generator().manual_seed(R)).cuda().to(dtype)
    with torch.no_grad():
        _, ref = m.prefill(x)
        st = seqpar.layer_state_only(m, m.in_proj(x))
    for k in ("h", "angle", "prev_BX"):
        assert max_rel(st[k].cpu().numpy(), ref[k].cpu().numpy()) < 1e-5, k
