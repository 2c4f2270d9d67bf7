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


class SSDScanFn(torch.autograd.Function):
    """Autograd entry point with the reference's name (mamba3/scan.py:65-100)."""

    @staticmethod
    def forward(ctx, chunk_decay, h_chunk, h_init=None):
        return ops.scan_fwd(chunk_decay, h_chunk, h_init)

    @staticmethod
    def backward(ctx, grad_h):
        raise NotImplementedError("mamba3_b200: the scan backward kernel is not built yet (forward/inference only)")


def ssd_scan(chunk_decay, h_chunk, h_init=None):
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in (chunk_decay, h_chunk, h_init)):
        return SSDScanFn.apply(chunk_decay, h_chunk, h_init)
    return ops.scan_fwd(chunk_decay, h_chunk, h_init)
