"""CPU-only checks of the boundary and the host logic (no kernel launches)."""

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest
import torch

from goldens import LAYER_CASES, layer_cfg, load, state_dict

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        names |= set(re.findall(r"M3B_API\s+[\w\s\*]+?\b(m3b_\w+)\s*\(", h.read_text()))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    from mamba3_b200 import _lib

    names = declared_symbols()
    assert len(names) >= 8
    h = ctypes.CDLL(str(_lib.LIB_PATH))
    for n in names:
        assert hasattr(h, n), n
    assert set(names) == set(_lib.SIGNATURES), "ctypes binding must cover exactly the header"
    L = _lib.lib()
    assert L.m3b_abi_version() == 8
    assert L.m3b_strerror(0) == b"ok"


def test_library_rejects_bad_args_without_gpu():
    """Argument validation runs on the host and reports status codes, never aborts."""
    from mamba3_b200 import _lib

    L = _lib.lib()
    a = _lib.ScanArgs()
    assert L.m3b_scan_fwd(ctypes.byref(a), None) == 1  # M3B_ERR_INVALID_ARG: null pointers
    assert b"null" in L.m3b_last_error()
    s = _lib.StepArgs()
    assert L.m3b_step(ctypes.byref(s), None) == 1
    f = _lib.LayerFwdArgs()
    assert L.m3b_layer_fwd_workspace(ctypes.byref(f)) == 0
    assert L.m3b_layer_fwd(ctypes.byref(f), None, 0, None) == 1
    sb = _lib.ScanBwdArgs()
    assert L.m3b_scan_bwd_workspace(ctypes.byref(sb)) == 0
    assert L.m3b_scan_bwd(ctypes.byref(sb), None, 0, None) == 1
    assert b"null" in L.m3b_last_error()


def test_training_entry_points_reject_bad_arguments_without_a_gpu():
    """The training-path entry points (gate, B / C preparation, x-side weights) validate their
    arguments on the host and report an error code and message before touching the device:
    null structs and pointers, odd N, oversized P, ranks past the kernels' limit."""
    import ctypes

    from mamba3_b200 import _lib

    L = _lib.lib()
    assert L.m3b_gate_fwd(None, None) == 1
    g = _lib.GateArgs(10, 0, 8, 2, 0)  # rows, z_stride, channels, R, dtype; no pointers
    assert L.m3b_gate_fwd(ctypes.byref(g), None) == 1 and b"null" in L.m3b_last_error()
    assert L.m3b_gate_bwd(ctypes.byref(g), None, 0, None) == 1
    assert L.m3b_gate_bwd_workspace(ctypes.byref(g)) == 1 * 8 * 2 * 2 * 4  # one 128-row chunk of partials
    assert L.m3b_bc_fwd(None, None, 0, None) == 1
    bc = _lib.BcArgs(1, 0, 4, 1, 15, 2, 1, 1, 0, 0, 1e-5)  # N = 15: odd
    assert L.m3b_bc_fwd_workspace(ctypes.byref(bc)) == 0
    assert L.m3b_bc_fwd(ctypes.byref(bc), None, 0, None) == 1 and b"even" in L.m3b_last_error()
    bc = _lib.BcArgs(1, 4, 4, 1, 16, 2, 1, 1, 0, 0, 1e-5)  # tokens but no pointers
    assert L.m3b_bc_bwd(ctypes.byref(bc), None, 0, None) == 1 and b"null" in L.m3b_last_error()
    bc = _lib.BcArgs(1, 4, 64, 1, 128, 2, 1, 1, 0, 0, 1e-5)  # H * N / 2 = 4096 > 2048
    assert L.m3b_bc_fwd(ctypes.byref(bc), None, 0, None) == 2  # M3B_ERR_UNSUPPORTED
    assert L.m3b_xprep_fwd(None, None) == 1
    xp = _lib.XprepArgs(1, 4, 2, 300, 2, 1, 0, 0, 0)  # P = 300 > 256
    assert L.m3b_xprep_fwd(ctypes.byref(xp), None) == 2 and b"P <= 256" in L.m3b_last_error()
    xp = _lib.XprepArgs(1, 4, 2, 64, 5, 1, 0, 0, 0)  # R = 5 > 4
    assert L.m3b_xprep_bwd_workspace(ctypes.byref(xp)) == 0
    assert L.m3b_xprep_bwd(ctypes.byref(xp), None, 0, None) == 2


@pytest.mark.parametrize("case", ["default", "rank1", "ngroups2", "euler", "real"])
def test_seeded_init_matches_reference(case):
    """Same constructor, names, shapes and RNG draws as the reference: identical weights under a seed."""
    from mamba3_b200 import KulaMamba

    d = load(f"layer_{case}")
    if int(d["perturb"]):
        pytest.skip("perturbed fixture")
    torch.manual_seed(int(d["seed"]))
    m = KulaMamba(**layer_cfg(d))
    ref = state_dict(d)
    sd = m.state_dict()
    assert set(sd) == set(ref)
    for k, v in sd.items():
        np.testing.assert_array_equal(v.numpy(), ref[k], err_msg=k)


def test_seeded_init_matches_reference_big():
    """Config-0 dims: weight checksums of the reference's seed-0 init."""
    import hashlib

    from mamba3_b200 import KulaMamba

    d = load("biglayer_cfg0dims")
    torch.manual_seed(int(d["seed"]))
    m = KulaMamba(d_model=768, d_state=128, expand=2, headdim=64, mimo_rank=2, chunk_size=64)
    for k, v in m.state_dict().items():
        assert abs(float(v.double().sum()) - float(d[f"wsum.{k}"])) < 1e-9 * max(1.0, abs(float(d[f"wsum.{k}"])))
    w = m.in_proj.weight.detach().contiguous().numpy()
    assert hashlib.sha1(w.tobytes()).hexdigest().encode() == bytes(d["in_proj_sha1"])


def test_lm_structure_matches_reference():
    from mamba3_b200 import KulaMambaLM

    d = load("lm_small")
    cfg = {k[4:]: d[k].item() for k in d if k.startswith("cfg.")}
    torch.manual_seed(int(d["seed"]))
    lm = KulaMambaLM(**cfg)
    ref = state_dict(d)
    sd = lm.state_dict()
    assert set(sd) == set(ref)
    for k, v in sd.items():
        np.testing.assert_array_equal(v.numpy(), ref[k], err_msg=k)


def test_cpu_tensors_raise_no_fallback():
    from mamba3_b200 import KulaMamba, ssd_scan
    from mamba3_b200._lib import M3bError

    m = KulaMamba(d_model=64, d_state=16, headdim=16, chunk_size=8)
    with pytest.raises(M3bError):
        m(torch.randn(1, 8, 64))
    with pytest.raises(M3bError):
        m.step(torch.randn(1, 64), m.allocate_inference_state(1))
    with pytest.raises(M3bError):
        ssd_scan(torch.rand(1, 2, 1), torch.randn(1, 2, 1, 4))


def test_empty_sequence_raises_like_the_reference():
    """T = 0: the reference asserts T > 0 (mamba3/mamba3.py:194); the same message, an
    AssertionError (and a ValueError), before anything touches a device."""
    from mamba3_b200 import KulaMamba

    m = KulaMamba(d_model=64, d_state=16, headdim=16, chunk_size=8)
    x = torch.zeros(2, 0, 64)
    for call in (lambda: m(x), lambda: m.prefill(x), lambda: m.prefill(x, compact_state=True)):
        with pytest.raises(AssertionError, match="Sequence length must be positive, got 0"):
            call()
        with pytest.raises(ValueError):
            call()


@pytest.mark.parametrize("kw", [dict(d_model=60, headdim=16), dict(d_state=15), dict(ngroups=3)],
                         ids=["headdim", "odd_d_state", "ngroups"])
def test_constructor_rejects_what_the_reference_asserts(kw):
    """The reference rejects these with `assert` (mamba3/mamba3.py:77, 79, 85): an AssertionError
    here too (and a ValueError)."""
    from mamba3_b200 import KulaMamba

    args = dict(d_model=64, d_state=16, headdim=16, chunk_size=8)
    args.update(kw)
    with pytest.raises(AssertionError):
        KulaMamba(**args)
    with pytest.raises(ValueError):
        KulaMamba(**args)


def test_state_shapes_and_dtypes():
    from mamba3_b200 import KulaMamba

    m = KulaMamba(d_model=64, d_state=16, headdim=16, chunk_size=8)
    st = m.allocate_inference_state(2, dtype=torch.bfloat16, device="cpu")
    assert st["h"].shape == (2, 8, 16, 16) and st["prev_BX"].shape == (2, 8, 16, 16)
    assert st["angle"].shape == (2, 8, 8)
    assert all(v.dtype == torch.float32 for v in st.values())


def test_compact_state_shapes():
    """allocate_inference_state(compact=True): the previous token as (N, R) and (P, R) factors."""
    from mamba3_b200 import KulaMamba

    m = KulaMamba(d_model=64, d_state=16, headdim=16, mimo_rank=2, chunk_size=8)
    st = m.allocate_inference_state(2, device="cpu", compact=True)
    assert set(st) == {"h", "angle", "prev_B", "prev_x"}
    assert st["prev_B"].shape == (2, 8, 16, 2) and st["prev_x"].shape == (2, 8, 16, 2)
    assert all(v.dtype == torch.float32 for v in st.values())


# The reference's public signatures (parameter names and defaults, in order), as its sources
# declare them; the drop-in API takes every one of them the same way and may only add keyword
# parameters with defaults after them.
REFERENCE_SIGNATURES = {
    # mamba3/mamba3.py:50
    "KulaMamba.__init__": [("d_model", None), ("d_state", 128), ("expand", 2), ("headdim", 64), ("ngroups", None),
                           ("mimo_rank", 2), ("chunk_size", 64), ("bias", False), ("dt_min", 0.001),
                           ("dt_max", 0.1), ("use_trapezoidal", True), ("use_complex_ssm", True)],
    # mamba3/mamba3.py:260, 264, 267, 324
    "KulaMamba.forward": [("x", None), ("dt_scale", None)],
    "KulaMamba.prefill": [("x", None), ("dt_scale", None)],
    "KulaMamba.step": [("hidden_states", None), ("ssm_state", None), ("dt_scale", None)],
    "KulaMamba.allocate_inference_state": [("batch_size", None), ("dtype", None), ("device", None)],
    # mamba3/block.py:31
    "KulaMambaBlock.__init__": [("d_model", None), ("d_state", 128), ("expand", 2), ("headdim", 64),
                                ("ngroups", None), ("mimo_rank", 2), ("chunk_size", 64), ("use_mlp", True),
                                ("mlp_expand", 2.667), ("norm_eps", 1e-05), ("bias", False), ("residual_scale", 1.0),
                                ("gradient_checkpointing", False), ("use_trapezoidal", True),
                                ("use_complex_ssm", True)],
    # mamba3/block.py:112, 178, 196
    "KulaMambaLM.__init__": [("vocab_size", None), ("d_model", 768), ("n_layers", 12), ("d_state", 128),
                             ("expand", 2), ("headdim", 64), ("ngroups", None), ("mimo_rank", 2), ("chunk_size", 64),
                             ("use_mlp", True), ("tie_weights", True), ("norm_eps", 1e-05), ("bias", False),
                             ("residual_scale", "depth"), ("gradient_checkpointing", False),
                             ("use_trapezoidal", True), ("use_complex_ssm", True)],
    "KulaMambaLM.forward": [("input_ids", None), ("labels", None)],
    "KulaMambaLM.generate": [("input_ids", None), ("max_new_tokens", 100), ("temperature", 1.0), ("top_k", None)],
    # mamba3/ssd.py:118, mamba3/scan.py:144
    "chunked_ssd": [("x_g", None), ("x_b", None), ("B_g", None), ("B_b", None), ("C", None), ("dt", None),
                    ("A", None), ("D", None), ("x_raw", None), ("chunk_size", 64), ("h_init", None),
                    ("return_final_state", False)],
    "ssd_scan": [("chunk_decay", None), ("h_chunk", None), ("h_init", None)],
}


@pytest.mark.parametrize("name", sorted(REFERENCE_SIGNATURES))
def test_public_signatures_match_the_reference(name):
    import inspect

    import mamba3_b200

    obj = mamba3_b200
    for part in name.split("."):
        obj = getattr(obj, part)
    params = [p for p in inspect.signature(obj).parameters.values() if p.name != "self"]
    want = REFERENCE_SIGNATURES[name]
    got = [(p.name, None if p.default is inspect.Parameter.empty else p.default) for p in params[:len(want)]]
    assert got == want
    for p in params[len(want):]:  # extensions: keyword parameters with defaults only
        assert p.default is not inspect.Parameter.empty, p.name
