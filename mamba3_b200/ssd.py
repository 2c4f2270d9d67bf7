"""Chunked SSD entry point, drop-in for ``mamba3.ssd`` of the reference.

``chunked_ssd`` takes the reference's pre-processed tensors
(mamba3/ssd.py:118-131) and returns ``SSDOutput(y, h_final)``.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops


@dataclass
class SSDOutput:
    """(mamba3/ssd.py:22-25)"""

    y: torch.Tensor
    h_final: torch.Tensor | None = None


class ChunkedSSDFn(torch.autograd.Function):
    """Autograd for chunked_ssd: the forward kernels, and the backward kernel
    (``mamba3_b200::chunked_ssd_bwd``) for the gradients the reference gets from autograd
    through _IntraChunkFn (mamba3/ssd.py:27-115), SSDScanFn (mamba3/scan.py:65-140) and the
    torch ops of mamba3/ssd.py:118-244.  Gradients come back in each input's dtype."""

    @staticmethod
    def forward(ctx, x_g, x_b, B_g, B_b, C, dt, A, D, x_raw, h_init, return_final_state):
        y, hf = ops.chunked_ssd(x_g, x_b, B_g, B_b, C, dt, A, D, x_raw, h_init, return_final_state)
        ctx.save_for_backward(x_g, x_b, B_g, B_b, C, dt, A, D, x_raw, h_init)
        ctx.final = return_final_state
        return y, hf

    @staticmethod
    def backward(ctx, dy, dhf):
        ins = ctx.saved_tensors
        dhf = dhf if ctx.final and dhf is not None and dhf.numel() > 0 else None
        g = ops.chunked_ssd_bwd(*ins, dy, dhf)
        out = [None if t is None or not need else gi.to(t.dtype)
               for t, gi, need in zip(ins, g, ctx.needs_input_grad)]
        return (*out, None)


def chunked_ssd(x_g, x_b, B_g, B_b, C, dt, A, D, x_raw, chunk_size=64, h_init=None, return_final_state=False):
    """Chunked SSD on pre-processed inputs (mamba3/ssd.py:118-244); differentiable through
    ChunkedSSDFn when an input requires grad.

    x_g, x_b, x_raw: (B,T,H,P,R); B_g, B_b, C: (B,T,H,N,R); dt: (B,T,H); A, D: (H,);
    h_init: (B,H,P,N) or None.  ``x_b``/``B_b`` None selects the Euler form.  ``chunk_size``
    is accepted for API compatibility; the kernels use their own chunk length, which does
    not change the result beyond fp32 rounding.  Returns SSDOutput(y in x_g.dtype, h_final fp32).
    """
    ins = (x_g, x_b, B_g, B_b, C, dt, A, D, x_raw, h_init)
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in ins):
        y, hf = ChunkedSSDFn.apply(*ins, return_final_state)
    else:
        y, hf = ops.chunked_ssd(*ins, return_final_state)
    return SSDOutput(y=y, h_final=hf if return_final_state else None)
