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


def chunked_ssd(x_g, x_b, B_g, B_b, C, dt, A, D, x_raw, chunk_size=64, h_init=None, return_final_state=False):
    """Chunked SSD forward on pre-processed inputs (mamba3/ssd.py:118-244).

    x_g, x_b, x_raw: (B,T,H,P,R); B_g, B_b, C: (B,T,H,N,R); dt: (B,T,H); A, D: (H,);
    h_init: (B,H,P,N) or None.  ``x_b``/``B_b`` None selects the Euler form.  ``chunk_size``
    is accepted for API compatibility; the kernels use their own chunk length, which does
    not change the result beyond fp32 rounding.  Returns SSDOutput(y in x_g.dtype, h_final fp32).
    """
    y, hf = ops.chunked_ssd(x_g, x_b, B_g, B_b, C, dt, A, D, x_raw, h_init, return_final_state)
    return SSDOutput(y=y, h_final=hf if return_final_state else None)
