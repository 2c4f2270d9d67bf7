"""Shared test helpers: build the product modules from golden fixtures, run the oracle."""

from __future__ import annotations

import numpy as np
import torch

import oracle
from goldens import layer_cfg, state_dict


def has_gpu():
    return torch.cuda.is_available()


def ours_layer_from_golden(d, dtype=torch.float32, device="cuda"):
    from mamba3_b200 import KulaMamba

    cfg = layer_cfg(d)
    m = KulaMamba(**cfg)
    sd = {k: torch.from_numpy(v.copy()) for k, v in state_dict(d).items()}
    m.load_state_dict(sd)
    return m.to(device=device, dtype=dtype).eval()


def oracle_params(module, dtype=np.float64):
    """Oracle parameters from a product KulaMamba (weights as stored, so bf16 rounding is included)."""
    sd = {k: v.detach().float().cpu().numpy() for k, v in module.state_dict().items()}
    return oracle.LayerParams.from_state_dict(
        sd, d_model=module.d_model, d_state=module.d_state, expand=module.expand, headdim=module.headdim,
        ngroups=module.ngroups, mimo_rank=module.mimo_rank, chunk_size=module.chunk_size,
        use_trapezoidal=module.use_trapezoidal, use_complex_ssm=module.use_complex_ssm, dtype=dtype)


def to_np(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


def seeded_normal(shape, seed, dtype=torch.float32, device="cuda"):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g).to(device=device, dtype=dtype)
