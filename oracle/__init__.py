"""CPU oracle for the Mamba-3 SSD hot path -- TEST INFRASTRUCTURE ONLY.

This package restates the reference algorithm (dorayaku/mamba3) in numpy so the
CUDA product path can be checked against it.  It is a checker, never a
fallback: only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
``cpu_baseline`` / ``--impl reference`` legs may import it.  The package
``mamba3_b200`` never imports anything from here.

Parity is pinned: ``tests/test_oracle_golden.py`` checks every function here
against golden vectors produced by running the unmodified reference
(``tests/golden/make_golden.py``).
"""

from .mamba3_oracle import (  # noqa: F401
    LayerParams,
    allocate_inference_state,
    apply_rope,
    block_forward,
    block_prefill,
    block_step,
    chunked_ssd,
    chunked_ssd_backward,
    layer_forward,
    layer_prefill,
    layer_step,
    lm_forward,
    lm_generate,
    rmsnorm,
    softplus,
    ssd_scan,
    ssd_scan_backward,
    swiglu,
)
