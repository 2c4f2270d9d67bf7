"""Loading of the committed golden fixtures (``tests/golden/*.npz``) for tests."""

from __future__ import annotations

from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"

LAYER_CASES = ["default", "perturbed", "rank1", "rank4", "euler", "real", "alloff", "ngroups2", "single",
               "n128p64"]
SSD_CASES = ["trap", "euler", "rank4"]
SCAN_CASES = ["hinit", "zero"]
SCAN_BWD_CASES = ["hinit", "zero", "k1", "odd"]
SSD_BWD_CASES = ["trap", "euler", "rank4", "single"]


def load(name):
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


def layer_cfg(d):
    cfg = {k[4:]: d[k].item() for k in d if k.startswith("cfg.")}
    if cfg.get("ngroups", None) == -1:
        cfg["ngroups"] = None
    for k in ("use_trapezoidal", "use_complex_ssm"):
        if k in cfg:
            cfg[k] = bool(cfg[k])
    return cfg


def state_dict(d, prefix="sd."):
    return {k[len(prefix):]: d[k] for k in d if k.startswith(prefix)}


def max_rel(a, b):
    """max|a-b| / max|b| -- the parity metric used throughout the tests."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.abs(b).max()
    return float(np.abs(a - b).max() / (den if den > 0 else 1.0))
