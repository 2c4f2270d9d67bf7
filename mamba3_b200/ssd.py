"""Chunked SSD entry point, drop-in for ``mamba3.ssd`` of the reference.

``chunked_ssd`` takes the reference's pre-processed tensors
(mamba3/ssd.py:118-131) and returns ``SSDOutput(y, h_final)``.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class SSDOutput:
    """(mamba3/ssd.py:22-25)"""

    y: torch.Tensor
    h_final: torch.Tensor | None = None


def chunked_ssd(x_g, x_b, B_g, B_b, C, dt, A, D, x_raw, chunk_size=64, h_init=None, return_final_state=False):
    raise NotImplementedError("mamba3_b200.chunked_ssd: general (pre-processed input) kernel not built yet")
