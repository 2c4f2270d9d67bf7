"""The chunked formulation of the chunked_ssd backward, checked on the CPU against the oracle's
token recurrence (oracle.chunked_ssd_backward, which follows the reference's autograd through
mamba3/ssd.py:67-115 and mamba3/scan.py:102-140).

The library's backward kernel walks the tokens one at a time.  A tensor-core version needs the
gradients as per-chunk matrix products, with chunks independent once two P x N matrices per
chunk boundary are known:
  * h_in[k], the state entering chunk k (the forward's chunk scan);
  * Gx[k] = a_{t1} G_{t1}, dL/dh arriving from beyond chunk k (a reverse chunk scan:
    Gx[k-1] = Gamma(end, in) Gx[k] + sum_t Gamma(t, in) dy_t C_t^T, Gx[K-1] = dh_final).
Inside a chunk, with Gamma(t, s) the decay product over (s, t], the score tiles
M[t,q,s,j] = C_t[:,q] . Bt_s[:,j] (the forward's own) and W[t,q,s,j] = dy_t[:,q] . Xt_s[:,j]
give dXt, dBt and dC as masked products, and ddt / dA follow from per-token scalars through the
same suffix recurrence the kernel uses.  This test pins that algebra in float64.
"""

import numpy as np
import pytest

import oracle


def _chunked_backward(X2, B2, C, dt, A, dy, h_init, dhf, L, q=lambda a: a):
    """One (batch row, head): X2 (T,P,RI), B2 (T,N,RI), C (T,N,R), dt (T,), dy (T,P,R),
    h_init / dhf (P,N) -> dX2, dB2, dC, ddt, dA, dh_init by chunk-level products.  ``q`` rounds
    every matrix-product operand as a tensor-core kernel would stage it (identity: exact)."""
    T = dt.shape[0]
    K = (T + L - 1) // L
    la = A * dt
    spans = [(k * L, min(T, (k + 1) * L)) for k in range(K)]
    cums = [np.cumsum(la[t0:t1]) for t0, t1 in spans]
    # forward chunk scan: the state entering each chunk
    h_in = [h_init]
    for (t0, t1), c in zip(spans, cums):
        w = np.exp(c[-1] - c) * dt[t0:t1]
        h_in.append(np.exp(c[-1]) * h_in[-1] + np.einsum("spj,snj->pn", q(w[:, None, None] * X2[t0:t1]),
                                                          q(B2[t0:t1])))
    h_final = h_in[-1]
    # reverse chunk scan: dL/dh arriving at each chunk's end from the chunks after it
    Gx = [None] * K
    Gx[K - 1] = dhf
    dh_init = None
    for k in range(K - 1, -1, -1):
        (t0, t1), c = spans[k], cums[k]
        g_in = np.exp(c[-1]) * Gx[k] + np.einsum("tpq,tnq->pn", q(np.exp(c)[:, None, None] * dy[t0:t1]),
                                                  q(C[t0:t1]))
        if k > 0:
            Gx[k - 1] = g_in
        else:
            dh_init = g_in
    dX2, dB2, dC = np.zeros_like(X2), np.zeros_like(B2), np.zeros_like(C)
    for k, ((t0, t1), c) in enumerate(zip(spans, cums)):
        n = t1 - t0
        X, Bm, Cm, d, g = X2[t0:t1], B2[t0:t1], C[t0:t1], dt[t0:t1], dy[t0:t1]
        gam = np.where(np.arange(n)[:, None] >= np.arange(n)[None, :], np.exp(c[:, None] - c[None, :]), 0.0)
        gm = gam * d[None, :]                                   # Gamma(t, s) dt_s, t >= s
        X, Bm, Cm, g = q(X), q(Bm), q(Cm), q(g)
        M = np.einsum("tnq,snj->tqsj", Cm, Bm)
        W = np.einsum("tpq,spj->tqsj", g, X)
        Mg, Wg = q(M * gm[:, None, :, None]), q(W * gm[:, None, :, None])  # masked tiles, restaged
        tail = np.exp(c[-1] - c) * d                            # Gamma(end, s) dt_s
        dX2[t0:t1] = tail[:, None, None] * np.einsum("pn,snj->spj", q(Gx[k]), Bm) + np.einsum(
            "tpq,tqsj->spj", g, Mg)
        dB2[t0:t1] = tail[:, None, None] * np.einsum("pn,spj->snj", q(Gx[k]), X) + np.einsum(
            "tnq,tqsj->snj", Cm, Wg)
        dC[t0:t1] = np.exp(c)[:, None, None] * np.einsum("pn,tpq->tnq", q(h_in[k]), g) + np.einsum(
            "snj,tqsj->tnq", Bm, Wg)
    # per-token scalars and the suffix recurrence m_t = m_{t+1} + e_t - dt_t fr_t
    fr = np.einsum("tpj,tpj->t", X2, dX2) / dt
    e = np.einsum("tnq,tnq->t", C, dC)
    m = float((dhf * h_final).sum())
    ddt, dA = np.zeros(T), 0.0
    for t in range(T - 1, -1, -1):
        m = m + e[t] - dt[t] * fr[t]
        ddt[t] = fr[t] + A * m
        dA += dt[t] * m
    return dX2, dB2, dC, ddt, dA, dh_init


@pytest.mark.parametrize("T,L,beta", [(37, 8, True), (64, 16, True), (5, 8, False), (33, 1, True)])
def test_chunked_backward_equals_token_recurrence(T, L, beta):
    """Chunk-level products (ragged last chunk, a single partial chunk, chunks of one token)
    give the oracle's gradients to float64 rounding (1e-10 relative)."""
    rng = np.random.default_rng(T * 100 + L)
    Bt, H, P, N, R = 2, 2, 6, 8, 2
    x_g = rng.standard_normal((Bt, T, H, P, R))
    x_b = rng.standard_normal((Bt, T, H, P, R)) if beta else None
    B_g = rng.standard_normal((Bt, T, H, N, R))
    B_b = rng.standard_normal((Bt, T, H, N, R)) if beta else None
    C = rng.standard_normal((Bt, T, H, N, R))
    dt = rng.uniform(0.01, 0.3, (Bt, T, H))
    A = -rng.uniform(0.5, 3.0, H)
    D = rng.standard_normal(H)
    x_raw = rng.standard_normal((Bt, T, H, P, R))
    dy = rng.standard_normal((Bt, T, H, P, R))
    h_init = rng.standard_normal((Bt, H, P, N))
    dhf = rng.standard_normal((Bt, H, P, N))
    ref = oracle.chunked_ssd_backward(x_g, x_b, B_g, B_b, C, dt, A, D, x_raw, dy, h_init, dhf)
    X2 = x_g if x_b is None else np.concatenate([x_g, x_b], axis=-1)
    B2 = B_g if B_b is None else np.concatenate([B_g, B_b], axis=-1)
    dA_sum = np.zeros(H)
    for b in range(Bt):
        for h in range(H):
            dX2, dB2, dC, ddt, dA, dh0 = _chunked_backward(
                X2[b, :, h], B2[b, :, h], C[b, :, h], dt[b, :, h], A[h], dy[b, :, h], h_init[b, h], dhf[b, h], L)
            dA_sum[h] += dA
            rel = lambda a, r: np.abs(a - r).max() / max(np.abs(r).max(), 1e-30)  # noqa: E731
            assert rel(dX2[..., :R], ref["x_g"][b, :, h]) < 1e-10
            assert rel(dB2[..., :R], ref["B_g"][b, :, h]) < 1e-10
            if beta:
                assert rel(dX2[..., R:], ref["x_b"][b, :, h]) < 1e-10
                assert rel(dB2[..., R:], ref["B_b"][b, :, h]) < 1e-10
            assert rel(dC, ref["C"][b, :, h]) < 1e-10
            assert rel(ddt, ref["dt"][b, :, h]) < 1e-10
            assert rel(dh0, ref["h_init"][b, h]) < 1e-10
    assert np.abs(dA_sum - ref["A"]).max() / np.abs(ref["A"]).max() < 1e-10


def test_chunked_backward_with_bf16_operands_stays_within_training_tolerance():
    """The same algebra with every matrix-product operand rounded to bf16, at the config-1 head
    shape (P 64, N 128, R 2, trapezoid, 64-token chunks, 256 tokens).  dX, dB and dC stay within
    1e-2 of the float64 oracle, and ddt within the training tests' 3e-2.  ddt is the sensitive
    output: its suffix sums accumulate the per-token errors."""
    import torch

    def bf(a):
        return torch.from_numpy(np.ascontiguousarray(a)).to(torch.bfloat16).double().numpy()

    rng = np.random.default_rng(0)
    T, H, P, N, R, L = 256, 2, 64, 128, 2, 64
    x_g = rng.standard_normal((1, T, H, P, R))
    x_b = rng.standard_normal((1, T, H, P, R)) * 0.5
    B_g = rng.standard_normal((1, T, H, N, R)) * 0.3
    B_b = rng.standard_normal((1, T, H, N, R)) * 0.3
    C = rng.standard_normal((1, T, H, N, R)) * 0.3
    dt = rng.uniform(0.001, 0.1, (1, T, H))
    A = -rng.uniform(1, 16, H)
    dy = rng.standard_normal((1, T, H, P, R))
    ref = oracle.chunked_ssd_backward(x_g, x_b, B_g, B_b, C, dt, A, np.ones(H), x_g, dy)
    X2, B2 = np.concatenate([x_g, x_b], -1), np.concatenate([B_g, B_b], -1)
    rel = lambda a, r: np.abs(a - r).max() / np.abs(r).max()  # noqa: E731
    zero = np.zeros((P, N))
    for h in range(H):
        dX2, dB2, dC, ddt, _, _ = _chunked_backward(X2[0, :, h], B2[0, :, h], C[0, :, h], dt[0, :, h], A[h],
                                                    dy[0, :, h], zero, zero, L, q=bf)
        assert rel(dX2[..., :R], ref["x_g"][0, :, h]) < 1e-2
        assert rel(dB2[..., :R], ref["B_g"][0, :, h]) < 1e-2
        assert rel(dX2[..., R:], ref["x_b"][0, :, h]) < 1e-2  # the trapezoid halves feed the x / B
        assert rel(dB2[..., R:], ref["B_b"][0, :, h]) < 1e-2  # preparation backwards
        assert rel(dC, ref["C"][0, :, h]) < 1e-2
        assert rel(ddt, ref["dt"][0, :, h]) < 3e-2
