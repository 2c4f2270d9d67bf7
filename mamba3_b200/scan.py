"""Inter-chunk SSD scan, drop-in for ``mamba3.scan`` of the reference.

``ssd_scan(chunk_decay, h_chunk, h_init=None)`` returns the exclusive states
h[0] = h_init, h[k+1] = decay[k] * h[k] + h_chunk[k] (mamba3/scan.py:1-4,
:388-389), computed with an fp32 carry by the sm_100a scan kernel and returned
in ``h_chunk.dtype``.  Unlike the reference (mamba3/scan.py:15-31, :69-71) there
is no silent torch fallback: non-CUDA inputs raise.
"""

from __future__ import annotations

import torch

from . import ops


def _flat(chunk_decay, h_chunk, h_init):
    """(B,K,H,...) -> (B,K,H,PN) and (B,H,...) -> (B,H,PN), as mamba3/scan.py:72-79 does."""
    B, K, H = chunk_decay.shape
    hc = h_chunk.reshape(B, K, H, -1)
    hi = None if h_init is None else h_init.reshape(B, H, -1)
    return hc, hi


class SSDScanFn(torch.autograd.Function):
    """Autograd entry point with the reference's name (mamba3/scan.py:65-140).

    Forward: the scan in fp32 (the states are saved in fp32, as the reference's CUDA path
    saves them) and returned in ``h_chunk.dtype``.  Backward: the reverse-scan kernel
    (``mamba3_b200::scan_bwd``); gradients in the dtypes mamba3/scan.py:136-140 returns.
    """

    @staticmethod
    def forward(ctx, chunk_decay, h_chunk, h_init=None):
        hc, hi = _flat(chunk_decay, h_chunk, h_init)
        h_states = ops.scan_fwd(chunk_decay, hc.float(), hi)
        ctx.save_for_backward(chunk_decay, h_states)
        ctx.has_h_init = h_init is not None
        ctx.shapes = (h_chunk.shape, None if h_init is None else h_init.shape)
        return h_states.reshape(h_chunk.shape).to(h_chunk.dtype)

    @staticmethod
    def backward(ctx, grad_h):
        chunk_decay, h_states = ctx.saved_tensors
        shape, init_shape = ctx.shapes
        d_decay, d_chunk, d_h_init = ops.scan_bwd(chunk_decay, h_states, grad_h.reshape(h_states.shape))
        return (d_decay.to(chunk_decay.dtype), d_chunk.reshape(shape).to(grad_h.dtype),
                d_h_init.reshape(init_shape).to(grad_h.dtype) if ctx.has_h_init else None)


def ssd_scan(chunk_decay, h_chunk, h_init=None):
    """h_states[:,0] = h_init (or 0), h_states[:,k+1] = decay[:,k] h_states[:,k] + h_chunk[:,k]
    (mamba3/scan.py:143-144); differentiable through SSDScanFn when an input requires grad."""
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in (chunk_decay, h_chunk, h_init)):
        return SSDScanFn.apply(chunk_decay, h_chunk, h_init)
    hc, hi = _flat(chunk_decay, h_chunk, h_init)
    return ops.scan_fwd(chunk_decay, hc, hi).reshape(h_chunk.shape)
