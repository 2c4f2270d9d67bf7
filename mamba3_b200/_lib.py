"""ctypes binding of ``libmamba3_b200.so`` (the C ABI in ``include/mamba3_b200.h``).

This module only marshals torch tensors into the C structs and calls the
library on the tensors' device and current stream.  There is no fallback: if
the library is missing or a tensor is not on a CUDA device the call raises.
"""

from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

import torch

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libmamba3_b200.so"

F32, BF16, F16 = 0, 1, 2
_DT = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}

_lock = threading.Lock()
_lib = None


class M3bError(RuntimeError):
    """A failed call into libmamba3_b200 (status code + detail message)."""


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DT[dt]
    except KeyError:
        raise M3bError(f"unsupported dtype {dt}") from None


class ScanArgs(C.Structure):
    _fields_ = [("decay", C.c_void_p), ("h_chunk", C.c_void_p), ("h_init", C.c_void_p), ("h_states", C.c_void_p),
                ("h_final", C.c_void_p), ("B", C.c_int64), ("K", C.c_int64), ("H", C.c_int64), ("PN", C.c_int64),
                ("dtype", C.c_int32)]


class ScanBwdArgs(C.Structure):
    _fields_ = [("decay", C.c_void_p), ("h_states", C.c_void_p), ("grad_h", C.c_void_p), ("d_chunk", C.c_void_p),
                ("d_decay", C.c_void_p), ("d_h_init", C.c_void_p), ("B", C.c_int64), ("K", C.c_int64),
                ("H", C.c_int64), ("PN", C.c_int64), ("dtype", C.c_int32)]


class LayerParams(C.Structure):
    _fields_ = [("H", C.c_int32), ("P", C.c_int32), ("N", C.c_int32), ("R", C.c_int32), ("G", C.c_int32),
                ("trapezoidal", C.c_int32), ("complex_ssm", C.c_int32), ("param_dtype", C.c_int32),
                ("norm_eps", C.c_float),
                ("A_log", C.c_void_p), ("D", C.c_void_p), ("dt_bias", C.c_void_p), ("B_norm_w", C.c_void_p),
                ("C_norm_w", C.c_void_p), ("B_bias", C.c_void_p), ("C_bias", C.c_void_p), ("mimo_x", C.c_void_p),
                ("mimo_z", C.c_void_p), ("mimo_down", C.c_void_p)]


class StepArgs(C.Structure):
    _fields_ = [("prm", LayerParams), ("batch", C.c_int64), ("proj", C.c_void_p), ("proj_stride", C.c_int64),
                ("act_dtype", C.c_int32), ("dt_scale", C.c_void_p), ("h", C.c_void_p), ("prev_bx", C.c_void_p),
                ("angle", C.c_void_p), ("angle_dtype", C.c_int32), ("h_out", C.c_void_p), ("bx_out", C.c_void_p),
                ("angle_out", C.c_void_p), ("y", C.c_void_p), ("prev_b", C.c_void_p), ("prev_x", C.c_void_p),
                ("prev_b_out", C.c_void_p), ("prev_x_out", C.c_void_p), ("workspace", C.c_void_p),
                ("workspace_bytes", C.c_size_t)]


class LayerFwdArgs(C.Structure):
    _fields_ = [("prm", LayerParams), ("batch", C.c_int64), ("seqlen", C.c_int64), ("proj", C.c_void_p),
                ("proj_stride", C.c_int64), ("act_dtype", C.c_int32), ("dt_scale", C.c_void_p),
                ("h_init", C.c_void_p), ("angle_init", C.c_void_p), ("prev_bx_init", C.c_void_p), ("y", C.c_void_p),
                ("h_final", C.c_void_p), ("angle_final", C.c_void_p), ("prev_bx_final", C.c_void_p),
                ("err", C.c_void_p), ("stage_events", C.POINTER(C.c_void_p)), ("algo", C.c_int32),
                ("state_only", C.c_int32), ("prev_b_final", C.c_void_p), ("prev_x_final", C.c_void_p),
                ("wait_limit_ns", C.c_int64), ("rms_in", C.c_void_p)]


class InProjArgs(C.Structure):
    _fields_ = [("rows", C.c_int64), ("d_model", C.c_int32), ("d_proj", C.c_int32), ("x", C.c_void_p),
                ("x_stride", C.c_int64), ("weight", C.c_void_p), ("bias", C.c_void_p), ("proj", C.c_void_p),
                ("proj_stride", C.c_int64), ("prm", LayerParams), ("rms", C.c_void_p), ("err", C.c_void_p),
                ("wait_limit_ns", C.c_int64)]


class SsdArgs(C.Structure):
    _fields_ = [("batch", C.c_int64), ("seqlen", C.c_int64), ("H", C.c_int32), ("P", C.c_int32), ("N", C.c_int32),
                ("R", C.c_int32), ("dtype", C.c_int32), ("x_g", C.c_void_p), ("x_b", C.c_void_p),
                ("B_g", C.c_void_p), ("B_b", C.c_void_p), ("C", C.c_void_p), ("x_raw", C.c_void_p),
                ("dt", C.c_void_p), ("dt_dtype", C.c_int32), ("A", C.c_void_p), ("D", C.c_void_p),
                ("ad_dtype", C.c_int32), ("h_init", C.c_void_p), ("y", C.c_void_p), ("h_final", C.c_void_p),
                ("err", C.c_void_p)]


class SsdBwdArgs(C.Structure):
    _fields_ = [("batch", C.c_int64), ("seqlen", C.c_int64), ("H", C.c_int32), ("P", C.c_int32), ("N", C.c_int32),
                ("R", C.c_int32), ("dtype", C.c_int32), ("x_g", C.c_void_p), ("x_b", C.c_void_p),
                ("B_g", C.c_void_p), ("B_b", C.c_void_p), ("C", C.c_void_p), ("x_raw", C.c_void_p),
                ("dt", C.c_void_p), ("dt_dtype", C.c_int32), ("A", C.c_void_p), ("D", C.c_void_p),
                ("ad_dtype", C.c_int32), ("h_init", C.c_void_p), ("dy", C.c_void_p), ("dh_final", C.c_void_p),
                ("dx_g", C.c_void_p), ("dx_b", C.c_void_p), ("dB_g", C.c_void_p), ("dB_b", C.c_void_p),
                ("dC", C.c_void_p), ("dx_raw", C.c_void_p), ("ddt", C.c_void_p), ("dA", C.c_void_p),
                ("dD", C.c_void_p), ("dh_init", C.c_void_p), ("algo", C.c_int32)]


class GateArgs(C.Structure):
    _fields_ = [("rows", C.c_int64), ("z_stride", C.c_int64), ("channels", C.c_int32), ("R", C.c_int32),
                ("dtype", C.c_int32), ("y", C.c_void_p), ("z", C.c_void_p), ("mimo_z", C.c_void_p),
                ("mimo_down", C.c_void_p), ("out", C.c_void_p), ("dout", C.c_void_p), ("dy", C.c_void_p),
                ("dz", C.c_void_p), ("d_mimo_z", C.c_void_p), ("d_mimo_down", C.c_void_p)]


class BcArgs(C.Structure):
    _fields_ = [("batch", C.c_int64), ("seqlen", C.c_int64), ("H", C.c_int32), ("G", C.c_int32), ("N", C.c_int32),
                ("R", C.c_int32), ("rotate", C.c_int32), ("shift", C.c_int32), ("dtype", C.c_int32),
                ("dt_dtype", C.c_int32), ("eps", C.c_float), ("bc_stride", C.c_int64), ("theta_stride", C.c_int64),
                ("Bf", C.c_void_p), ("Cf", C.c_void_p), ("theta", C.c_void_p), ("dt", C.c_void_p),
                ("wB", C.c_void_p), ("bB", C.c_void_p), ("wC", C.c_void_p), ("bC", C.c_void_p),
                ("B_g", C.c_void_p), ("B_b", C.c_void_p), ("C", C.c_void_p), ("dB_g", C.c_void_p),
                ("dB_b", C.c_void_p), ("dC", C.c_void_p), ("dBf", C.c_void_p), ("dCf", C.c_void_p),
                ("dtheta", C.c_void_p), ("ddt", C.c_void_p), ("dwB", C.c_void_p), ("dbB", C.c_void_p),
                ("dwC", C.c_void_p), ("dbC", C.c_void_p)]


class XprepArgs(C.Structure):
    _fields_ = [("batch", C.c_int64), ("seqlen", C.c_int64), ("H", C.c_int32), ("P", C.c_int32), ("R", C.c_int32),
                ("trapezoidal", C.c_int32), ("dtype", C.c_int32), ("dt_dtype", C.c_int32), ("a_dtype", C.c_int32),
                ("x_stride", C.c_int64), ("lam_stride", C.c_int64), ("xf", C.c_void_p), ("mimo_x", C.c_void_p),
                ("lam_raw", C.c_void_p), ("dt", C.c_void_p), ("A", C.c_void_p), ("x_raw", C.c_void_p),
                ("x_g", C.c_void_p), ("x_b", C.c_void_p), ("dx_raw", C.c_void_p), ("dx_g", C.c_void_p),
                ("dx_b", C.c_void_p), ("dxf", C.c_void_p), ("dmimo_x", C.c_void_p), ("dlam_raw", C.c_void_p),
                ("ddt", C.c_void_p), ("dA", C.c_void_p)]


class SeqparFoldArgs(C.Structure):
    _fields_ = [("summaries", C.c_void_p), ("rank_stride", C.c_int64), ("upto", C.c_int32), ("batch", C.c_int64),
                ("H", C.c_int32), ("P", C.c_int32), ("N", C.c_int32), ("h", C.c_void_p), ("angle", C.c_void_p),
                ("prev_bx", C.c_void_p)]


LAYER_FWD_STAGES = ("prep", "angle_prefix", "chunk_state", "scan", "chunk_out", "last_bx")


# every symbol include/mamba3_b200.h declares, with its ctypes signature
SIGNATURES = {
    "m3b_strerror": (C.c_char_p, [C.c_int]),
    "m3b_last_error": (C.c_char_p, []),
    "m3b_abi_version": (C.c_int, []),
    "m3b_scan_fwd": (C.c_int, [C.POINTER(ScanArgs), C.c_void_p]),
    "m3b_scan_bwd_workspace": (C.c_size_t, [C.POINTER(ScanBwdArgs)]),
    "m3b_scan_bwd": (C.c_int, [C.POINTER(ScanBwdArgs), C.c_void_p, C.c_size_t, C.c_void_p]),
    "m3b_step": (C.c_int, [C.POINTER(StepArgs), C.c_void_p]),
    "m3b_step_workspace": (C.c_size_t, [C.POINTER(StepArgs)]),
    "m3b_layer_fwd_workspace": (C.c_size_t, [C.POINTER(LayerFwdArgs)]),
    "m3b_layer_fwd": (C.c_int, [C.POINTER(LayerFwdArgs), C.c_void_p, C.c_size_t, C.c_void_p]),
    "m3b_layer_fwd_noalloc": (C.c_int, [C.POINTER(LayerFwdArgs), C.c_void_p]),
    "m3b_in_proj": (C.c_int, [C.POINTER(InProjArgs), C.c_void_p]),
    "m3b_seqpar_fold": (C.c_int, [C.POINTER(SeqparFoldArgs), C.c_void_p]),
    "m3b_copy_rows_async": (C.c_int, [C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t,
                                      C.c_void_p]),
    "m3b_chunked_ssd_workspace": (C.c_size_t, [C.POINTER(SsdArgs)]),
    "m3b_chunked_ssd": (C.c_int, [C.POINTER(SsdArgs), C.c_void_p, C.c_size_t, C.c_void_p]),
    "m3b_chunked_ssd_bwd_workspace": (C.c_size_t, [C.POINTER(SsdBwdArgs)]),
    "m3b_chunked_ssd_bwd": (C.c_int, [C.POINTER(SsdBwdArgs), C.c_void_p, C.c_size_t, C.c_void_p]),
    "m3b_gate_fwd": (C.c_int, [C.POINTER(GateArgs), C.c_void_p]),
    "m3b_gate_bwd_workspace": (C.c_size_t, [C.POINTER(GateArgs)]),
    "m3b_gate_bwd": (C.c_int, [C.POINTER(GateArgs), C.c_void_p, C.c_size_t, C.c_void_p]),
    "m3b_bc_fwd_workspace": (C.c_size_t, [C.POINTER(BcArgs)]),
    "m3b_bc_fwd": (C.c_int, [C.POINTER(BcArgs), C.c_void_p, C.c_size_t, C.c_void_p]),
    "m3b_bc_bwd_workspace": (C.c_size_t, [C.POINTER(BcArgs)]),
    "m3b_bc_bwd": (C.c_int, [C.POINTER(BcArgs), C.c_void_p, C.c_size_t, C.c_void_p]),
    "m3b_xprep_fwd": (C.c_int, [C.POINTER(XprepArgs), C.c_void_p]),
    "m3b_xprep_bwd_workspace": (C.c_size_t, [C.POINTER(XprepArgs)]),
    "m3b_xprep_bwd": (C.c_int, [C.POINTER(XprepArgs), C.c_void_p, C.c_size_t, C.c_void_p]),
    "m3b_rmsnorm": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int32, C.c_float, C.c_int32,
                              C.c_void_p]),
    "m3b_swiglu_act": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int32, C.c_void_p]),
    "m3b_scaled_add": (C.c_int, [C.c_void_p, C.c_void_p, C.c_float, C.c_void_p, C.c_int64, C.c_int32, C.c_void_p]),
    "m3b_swiglu_rows": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.c_int32, C.c_int32, C.c_void_p]),
    "m3b_add_rmsnorm": (C.c_int, [C.c_void_p, C.c_void_p, C.c_float, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64,
                                  C.c_int32, C.c_float, C.c_int32, C.c_void_p]),
    "m3b_selftest_umma": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]),
    "m3b_selftest_wait": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int64, C.c_void_p, C.c_void_p]),
}


def lib():
    """The loaded library (loaded once).  A library that is missing, or was built from other
    sources than the ones beside it (content digest), is compiled first; raises if that fails."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                from . import build as _build

                if not _build.is_current():
                    try:
                        _build.build()
                    except Exception as e:  # noqa: BLE001 - reported with the reason
                        raise M3bError(f"{LIB_PATH.name} is missing or stale and could not be built: {e}") from e
                h = C.CDLL(str(LIB_PATH))
                for name, (res, args) in SIGNATURES.items():
                    f = getattr(h, name)
                    f.restype = res
                    f.argtypes = args
                _lib = h
    return _lib


def _check(rc: int, what: str):
    if rc != 0:
        L = lib()
        raise M3bError(f"{what}: {L.m3b_strerror(rc).decode()} ({L.m3b_last_error().decode()})")


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _cuda(*ts):
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise M3bError("mamba3_b200 kernels need CUDA tensors (there is no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise M3bError(f"tensors on different devices: {dev} vs {t.device}")
    return dev


def _stream(dev):
    return C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def layer_params(H, P, N, R, G, trapezoidal, complex_ssm, norm_eps, A_log, D, dt_bias, B_norm_w, C_norm_w,
                 B_bias, C_bias, mimo_x, mimo_z, mimo_down):
    ps = [A_log, D, dt_bias, B_norm_w, C_norm_w, B_bias, C_bias, mimo_x, mimo_z, mimo_down]
    pdt = ps[0].dtype
    for t in ps:
        if t.dtype != pdt or not t.is_contiguous():
            raise M3bError("layer parameters must be contiguous and share one dtype")
    return LayerParams(H, P, N, R, G, int(bool(trapezoidal)), int(bool(complex_ssm)), dtype_code(pdt),
                       float(norm_eps), *[_ptr(t) for t in ps])


def scan_fwd(decay, h_chunk, h_init=None, h_states=None, h_final=None):
    """Launch the inter-chunk scan; decay (B,K,H) fp32, h_chunk (B,K,H,PN) fp32/bf16."""
    dev = _cuda(decay, h_chunk, h_init, h_states, h_final)
    B, K, H, PN = h_chunk.shape
    if h_states is None:
        h_states = torch.empty_like(h_chunk)
    a = ScanArgs(_ptr(decay), _ptr(h_chunk), _ptr(h_init), _ptr(h_states), _ptr(h_final), B, K, H, PN,
                 dtype_code(h_chunk.dtype))
    with torch.cuda.device(dev):
        _check(lib().m3b_scan_fwd(C.byref(a), _stream(dev)), "m3b_scan_fwd")
    return h_states


def scan_bwd(decay, h_states, grad_h, with_h_init=False):
    """Launch the scan backward; decay (B,K,H) fp32, h_states / grad_h (B,K,H,PN) of one dtype
    (fp32 or bf16).  Returns (d_decay fp32, d_chunk in grad_h's dtype, d_h_init fp32 or None)."""
    dev = _cuda(decay, h_states, grad_h)
    B, K, H, PN = h_states.shape
    if grad_h.shape != h_states.shape or grad_h.dtype != h_states.dtype or decay.shape != (B, K, H):
        raise M3bError("scan_bwd: decay (B,K,H) and h_states / grad_h (B,K,H,PN) of one dtype expected")
    d_chunk = torch.empty_like(grad_h)
    d_decay = torch.empty((B, K, H), dtype=torch.float32, device=dev)
    d_h_init = torch.empty((B, H, PN), dtype=torch.float32, device=dev) if with_h_init else None
    a = ScanBwdArgs(_ptr(decay), _ptr(h_states), _ptr(grad_h), _ptr(d_chunk), _ptr(d_decay), _ptr(d_h_init),
                    B, K, H, PN, dtype_code(grad_h.dtype))
    L = lib()
    nbytes = L.m3b_scan_bwd_workspace(C.byref(a))
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _check(L.m3b_scan_bwd(C.byref(a), _ptr(ws), nbytes, _stream(dev)), "m3b_scan_bwd")
    return d_decay, d_chunk, d_h_init


def step(prm: LayerParams, proj, dt_scale, h, prev_bx, angle, h_out, bx_out, angle_out, y, prev_b=None,
         prev_x=None, prev_b_out=None, prev_x_out=None, workspace=None, streaming=True):
    """One decode step.  Either prev_bx / bx_out (the reference's (P, N) previous-token state) or
    the compact prev_b / prev_x / prev_b_out / prev_x_out ((N, R) and (P, R)) are given.  Where
    the streaming two-kernel path applies (m3b_step_workspace > 0) it runs with `workspace`
    (uint8, allocated here when None); returns the workspace so callers can keep it.
    streaming=False runs the single-kernel path without a workspace."""
    dev = _cuda(proj, dt_scale, h, prev_bx, angle, h_out, bx_out, angle_out, y, prev_b, prev_x, prev_b_out,
                prev_x_out, workspace)
    a = StepArgs(prm, proj.shape[0], _ptr(proj), proj.stride(0), dtype_code(proj.dtype), _ptr(dt_scale), _ptr(h),
                 _ptr(prev_bx), _ptr(angle), dtype_code(angle.dtype), _ptr(h_out), _ptr(bx_out), _ptr(angle_out),
                 _ptr(y), _ptr(prev_b), _ptr(prev_x), _ptr(prev_b_out), _ptr(prev_x_out))
    L = lib()
    need = L.m3b_step_workspace(C.byref(a)) if streaming else 0
    if need:
        if workspace is None or workspace.numel() < need:
            workspace = torch.empty(need, dtype=torch.uint8, device=dev)
        a.workspace = _ptr(workspace)
        a.workspace_bytes = need
    with torch.cuda.device(dev):
        _check(L.m3b_step(C.byref(a), _stream(dev)), "m3b_step")
    return workspace


def layer_fwd(prm: LayerParams, proj, y, dt_scale=None, h_init=None, angle_init=None, prev_bx_init=None,
              h_final=None, angle_final=None, prev_bx_final=None, err=None, workspace=None, stage_events=None,
              algo=0, state_only=False, prev_b_final=None, prev_x_final=None, wait_limit_ns=0, rms_in=None):
    """Launch the chunked layer forward; proj (B,T,d_proj) with unit stride in the last dim.
    Without `err` the device's error word records expired device waits (check_device_errors);
    wait_limit_ns bounds each device wait (0: the library's 2 s); rms_in: the (B*T, G, 2) fp32
    1/rms rows of in_proj(..., prm=...), which spare the layer its own pass over B and C."""
    dev = _cuda(proj, y, dt_scale, h_init, angle_init, prev_bx_init, h_final, angle_final, prev_bx_final, err,
                rms_in)
    if err is None:
        err = device_err_word(dev)
    Bt, T, _ = proj.shape
    if proj.stride(2) != 1 or proj.stride(0) != T * proj.stride(1):
        raise M3bError("proj must be row-contiguous (B,T,d_proj)")
    a = LayerFwdArgs(prm, Bt, T, _ptr(proj), proj.stride(1), dtype_code(proj.dtype), _ptr(dt_scale), _ptr(h_init),
                     _ptr(angle_init), _ptr(prev_bx_init), _ptr(y), _ptr(h_final), _ptr(angle_final),
                     _ptr(prev_bx_final), _ptr(err))
    a.algo = int(algo)
    a.state_only = int(bool(state_only))
    a.prev_b_final = _ptr(prev_b_final)
    a.prev_x_final = _ptr(prev_x_final)
    a.wait_limit_ns = int(wait_limit_ns)
    if rms_in is not None:
        if rms_in.dtype != torch.float32 or not rms_in.is_contiguous() or rms_in.numel() != Bt * T * prm.G * 2:
            raise M3bError("rms_in must be a contiguous fp32 (B*T, G, 2) tensor")
        a.rms_in = _ptr(rms_in)
    if stage_events is not None:
        if len(stage_events) != len(LAYER_FWD_STAGES) + 1:
            raise M3bError("stage_events needs one event per stage plus one")
        arr = (C.c_void_p * len(stage_events))(*[e.cuda_event for e in stage_events])
        a.stage_events = C.cast(arr, C.POINTER(C.c_void_p))
    L = lib()
    need = L.m3b_layer_fwd_workspace(C.byref(a))
    if need == 0:
        _check(L.m3b_layer_fwd(C.byref(a), None, 0, None), "m3b_layer_fwd")  # reports the validation error
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _check(L.m3b_layer_fwd(C.byref(a), _ptr(workspace), need, _stream(dev)), "m3b_layer_fwd")
    _after_launch(dev)
    return workspace


def in_proj(x, weight, bias=None, proj=None, prm: LayerParams | None = None, rms=None, err=None):
    """proj = x weight^T (+ bias) on the tensor cores, bf16 (x: (..., d_model), any leading shape,
    unit stride in the last dim and one row stride).  With `prm` (the layer's dimensions and
    norm eps) the epilogue also writes `rms`, the (rows, G, 2) fp32 1/rms of each token's B and C
    rows, as layer_fwd(rms_in=...) takes it.  Returns (proj, rms)."""
    dev = _cuda(x, weight, bias, proj, rms, err)
    if err is None:
        err = device_err_word(dev)
    d_model = x.shape[-1]
    x2 = x.reshape(-1, d_model)
    if x2.stride(1) != 1 or weight.stride(1) != 1 or weight.stride(0) != d_model or weight.shape[1] != d_model:
        raise M3bError("in_proj: x and weight need unit stride in d_model, weight row-contiguous")
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16 or (bias is not None and bias.dtype != torch.bfloat16):
        raise M3bError("in_proj: bf16 x, weight and bias")
    rows, d_proj = x2.shape[0], weight.shape[0]
    if proj is None:
        proj = torch.empty(*x.shape[:-1], d_proj, dtype=torch.bfloat16, device=dev)
    p2 = proj.reshape(rows, d_proj)
    if p2.stride(1) != 1 or p2.data_ptr() != proj.data_ptr():
        raise M3bError("in_proj: proj must have unit stride in its last dim")
    if prm is not None and rms is None:
        rms = torch.empty(rows, prm.G, 2, dtype=torch.float32, device=dev)
    a = InProjArgs(rows, d_model, d_proj, _ptr(x2), x2.stride(0), _ptr(weight), _ptr(bias), _ptr(p2), p2.stride(0),
                   prm if prm is not None else LayerParams(), _ptr(rms) if prm is not None else None, _ptr(err), 0)
    with torch.cuda.device(dev):
        _check(lib().m3b_in_proj(C.byref(a), _stream(dev)), "m3b_in_proj")
    _after_launch(dev)
    return proj, (rms if prm is not None else None)


def chunked_ssd(x_g, x_b, B_g, B_b, Cm, dt, A, D, x_raw, y, h_init=None, h_final=None, err=None):
    """Launch the general chunked SSD; all activations contiguous and of one dtype."""
    dev = _cuda(x_g, x_b, B_g, B_b, Cm, dt, A, D, x_raw, y, h_init, h_final, err)
    if err is None:
        err = device_err_word(dev)
    Bt, T, H, P, R = x_g.shape
    N = B_g.shape[3]
    a = SsdArgs(Bt, T, H, P, N, R, dtype_code(x_g.dtype), _ptr(x_g), _ptr(x_b), _ptr(B_g), _ptr(B_b), _ptr(Cm),
                _ptr(x_raw), _ptr(dt), dtype_code(dt.dtype), _ptr(A), _ptr(D), dtype_code(A.dtype), _ptr(h_init),
                _ptr(y), _ptr(h_final), _ptr(err))
    L = lib()
    need = L.m3b_chunked_ssd_workspace(C.byref(a))
    if need == 0:
        _check(L.m3b_chunked_ssd(C.byref(a), None, 0, None), "m3b_chunked_ssd")
    ws = torch.empty(need, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _check(L.m3b_chunked_ssd(C.byref(a), _ptr(ws), need, _stream(dev)), "m3b_chunked_ssd")
    _after_launch(dev)


def chunked_ssd_bwd(x_g, x_b, B_g, B_b, Cm, dt, A, D, x_raw, dy, h_init=None, dh_final=None, algo=0):
    """Launch the chunked SSD backward.  Activations, dy contiguous and of one dtype (fp32 / bf16);
    dt fp32 / bf16 / fp16; A, D of one dtype; h_init, dh_final fp32 or None.  Returns a dict of
    gradients (x_g, x_b, B_g, B_b, C, x_raw in the activation dtype, dt in dt's dtype, A, D, h_init
    fp32; None for absent inputs).  algo 0: chunk-level products on tensor cores where they apply,
    1: the token sweeps."""
    dev = _cuda(x_g, x_b, B_g, B_b, Cm, dt, A, D, x_raw, dy, h_init, dh_final)
    Bt, T, H, P, R = x_g.shape
    N = B_g.shape[3]
    e = lambda t: None if t is None else torch.empty_like(t)  # noqa: E731
    g = dict(x_g=e(x_g), x_b=e(x_b), B_g=e(B_g), B_b=e(B_b), C=e(Cm), x_raw=e(x_raw), dt=e(dt),
             A=torch.empty(H, dtype=torch.float32, device=dev), D=torch.empty(H, dtype=torch.float32, device=dev),
             h_init=None if h_init is None else torch.empty(Bt, H, P, N, dtype=torch.float32, device=dev))
    a = SsdBwdArgs(Bt, T, H, P, N, R, dtype_code(x_g.dtype), _ptr(x_g), _ptr(x_b), _ptr(B_g), _ptr(B_b), _ptr(Cm),
                   _ptr(x_raw), _ptr(dt), dtype_code(dt.dtype), _ptr(A), _ptr(D), dtype_code(A.dtype), _ptr(h_init),
                   _ptr(dy), _ptr(dh_final), _ptr(g["x_g"]), _ptr(g["x_b"]), _ptr(g["B_g"]), _ptr(g["B_b"]),
                   _ptr(g["C"]), _ptr(g["x_raw"]), _ptr(g["dt"]), _ptr(g["A"]), _ptr(g["D"]), _ptr(g["h_init"]),
                   int(algo))
    L = lib()
    need = L.m3b_chunked_ssd_bwd_workspace(C.byref(a))
    if need == 0:
        _check(L.m3b_chunked_ssd_bwd(C.byref(a), None, 0, None), "m3b_chunked_ssd_bwd")
    ws = torch.empty(need, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _check(L.m3b_chunked_ssd_bwd(C.byref(a), _ptr(ws), need, _stream(dev)), "m3b_chunked_ssd_bwd")
    return g


def _gate_args(y, z, mimo_z, mimo_down):
    """(rows, channels, R) view of the gate operands: y (..., H, P, R) contiguous, z (..., H*P)
    with unit channel stride and a uniform row stride, parameters (H, P, R) contiguous."""
    H, P, R = mimo_z.shape
    Cn = H * P
    rows = y.numel() // (Cn * R) if Cn * R else 0
    if (not y.is_contiguous() or y.shape[-3:] != (H, P, R) or mimo_down.shape != (H, P, R)
            or not mimo_z.is_contiguous() or not mimo_down.is_contiguous()
            or len({y.dtype, z.dtype, mimo_z.dtype, mimo_down.dtype}) != 1):
        raise M3bError("gate: y (..., H, P, R) contiguous, parameters (H, P, R), one dtype expected")
    z2 = z.reshape(rows, Cn) if rows else z.reshape(0, Cn)
    if rows and (z2.stride(1) != 1 or z2.data_ptr() != z.data_ptr()):
        raise M3bError("gate: z must be a strided view of (rows, H*P) with unit channel stride")
    return GateArgs(rows, z2.stride(0) if rows else 0, Cn, R, dtype_code(y.dtype), _ptr(y), _ptr(z),
                    _ptr(mimo_z), _ptr(mimo_down))


def gate_fwd(y, z, mimo_z, mimo_down):
    """out = sum_r y * silu(z * mimo_z) * mimo_down over the rank -> (..., H*P) in y's dtype."""
    dev = _cuda(y, z, mimo_z, mimo_down)
    a = _gate_args(y, z, mimo_z, mimo_down)
    out = torch.empty(*y.shape[:-3], a.channels, dtype=y.dtype, device=dev)
    a.out = _ptr(out)
    with torch.cuda.device(dev):
        _check(lib().m3b_gate_fwd(C.byref(a), _stream(dev)), "m3b_gate_fwd")
    return out


def gate_bwd(y, z, mimo_z, mimo_down, dout):
    """Gradients of gate_fwd -> (dy like y, dz (..., H*P) contiguous, d_mimo_z, d_mimo_down)."""
    dev = _cuda(y, z, mimo_z, mimo_down, dout)
    a = _gate_args(y, z, mimo_z, mimo_down)
    dout = dout.contiguous()
    if dout.dtype != y.dtype or dout.numel() != a.rows * a.channels:
        raise M3bError("gate_bwd: dout of the forward output's shape and dtype expected")
    dy, dz = torch.empty_like(y), torch.empty(*y.shape[:-3], a.channels, dtype=y.dtype, device=dev)
    dmz, dmd = torch.empty_like(mimo_z), torch.empty_like(mimo_down)
    a.dout, a.dy, a.dz, a.d_mimo_z, a.d_mimo_down = _ptr(dout), _ptr(dy), _ptr(dz), _ptr(dmz), _ptr(dmd)
    L = lib()
    need = L.m3b_gate_bwd_workspace(C.byref(a))
    ws = torch.empty(max(need, 16), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _check(L.m3b_gate_bwd(C.byref(a), _ptr(ws), ws.numel(), _stream(dev)), "m3b_gate_bwd")
    return dy, dz, dmz, dmd


def _row_stride(t, what):
    """Element stride between the token rows of a (batch, seqlen, width) view with unit inner
    stride and uniformly spaced rows (a column slice of a contiguous projection)."""
    Bt, T, _ = t.shape
    if t.stride(2) != 1 or (Bt > 1 and T > 0 and t.stride(0) != T * t.stride(1)):
        raise M3bError(f"bc_prep: {what} must have unit inner stride and evenly spaced token rows")
    return t.stride(1)


def _bc_args(Bf, Cf, theta, dt, wB, bB, wC, bC, H, eps, shift):
    G, N, R = bB.shape
    Bt, T, _ = Bf.shape
    rotate = theta is not None
    params = (wB, bB, wC, bC)
    if (Bf.shape != (Bt, T, G * N * R) or Cf.shape != Bf.shape or wB.numel() != N * R or wC.numel() != N * R
            or bC.shape != bB.shape or any(t.dtype != Bf.dtype or not t.is_contiguous() for t in params)
            or Cf.dtype != Bf.dtype or dt.shape != (Bt, T, H) or not dt.is_contiguous()
            or (rotate and (theta.shape != (Bt, T, N // 2) or theta.dtype != Bf.dtype))):
        raise M3bError("bc_prep: inconsistent shapes or dtypes")
    bs = _row_stride(Bf, "Bf")
    if _row_stride(Cf, "Cf") != bs:
        raise M3bError("bc_prep: Bf and Cf must share a row stride")
    ts = _row_stride(theta, "theta") if rotate else 0
    return BcArgs(Bt, T, H, G, N, R, int(rotate), int(bool(shift)), dtype_code(Bf.dtype), dtype_code(dt.dtype),
                  float(eps), bs, ts, _ptr(Bf), _ptr(Cf), _ptr(theta), _ptr(dt), _ptr(wB), _ptr(bB), _ptr(wC),
                  _ptr(bC))


def bc_fwd(Bf, Cf, theta, dt, wB, bB, wC, bC, H, eps, shift):
    """B / C preparation (norm + bias, head broadcast, rotation when theta is given, previous-token
    shift) -> (B_g, B_b or an empty tensor, C), each (batch, seqlen, H, N, R)."""
    dev = _cuda(Bf, Cf, theta, dt, wB, bB, wC, bC)
    a = _bc_args(Bf, Cf, theta, dt, wB, bB, wC, bC, H, eps, shift)
    shape = (a.batch, a.seqlen, H, a.N, a.R)
    Bg, Co = torch.empty(shape, dtype=Bf.dtype, device=dev), torch.empty(shape, dtype=Bf.dtype, device=dev)
    Bb = torch.empty(shape if shift else (0,), dtype=Bf.dtype, device=dev)
    a.B_g, a.B_b, a.C = _ptr(Bg), _ptr(Bb) if shift else None, _ptr(Co)
    L = lib()
    need = L.m3b_bc_fwd_workspace(C.byref(a))
    ws = torch.empty(max(need, 16), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _check(L.m3b_bc_fwd(C.byref(a), _ptr(ws), ws.numel(), _stream(dev)), "m3b_bc_fwd")
    return Bg, Bb, Co


def bc_bwd(Bf, Cf, theta, dt, wB, bB, wC, bC, dB_g, dB_b, dC, H, eps, shift):
    """Gradients of bc_fwd -> (dBf, dCf, dtheta, ddt, dwB, dbB, dwC, dbC); dtheta / ddt are empty
    tensors without rotation."""
    dev = _cuda(Bf, Cf, theta, dt, wB, bB, wC, bC, dB_g, dB_b, dC)
    a = _bc_args(Bf, Cf, theta, dt, wB, bB, wC, bC, H, eps, shift)
    shape = (a.batch, a.seqlen, H, a.N, a.R)
    grads = [dB_g, dC] + ([dB_b] if shift else [])
    if any(g.shape != shape or g.dtype != Bf.dtype or not g.is_contiguous() for g in grads):
        raise M3bError("bc_bwd: gradients of the forward outputs' shape and dtype, contiguous, expected")
    rotate = theta is not None
    dBf = torch.empty(a.batch, a.seqlen, a.G * a.N * a.R, dtype=Bf.dtype, device=dev)
    dCf = torch.empty_like(dBf)
    dth = torch.empty((a.batch, a.seqlen, a.N // 2) if rotate else (0,), dtype=Bf.dtype, device=dev)
    ddt = torch.empty(dt.shape if rotate else (0,), dtype=dt.dtype, device=dev)
    dwB, dbB, dwC, dbC = (torch.empty_like(t) for t in (wB, bB, wC, bC))
    a.dB_g, a.dB_b, a.dC = _ptr(dB_g), _ptr(dB_b) if shift else None, _ptr(dC)
    a.dBf, a.dCf, a.dtheta, a.ddt = _ptr(dBf), _ptr(dCf), _ptr(dth) if rotate else None, _ptr(ddt) if rotate else None
    a.dwB, a.dbB, a.dwC, a.dbC = _ptr(dwB), _ptr(dbB), _ptr(dwC), _ptr(dbC)
    L = lib()
    need = L.m3b_bc_bwd_workspace(C.byref(a))
    ws = torch.empty(max(need, 16), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _check(L.m3b_bc_bwd(C.byref(a), _ptr(ws), ws.numel(), _stream(dev)), "m3b_bc_bwd")
    return dBf, dCf, dth, ddt, dwB, dbB, dwC, dbC


def _xprep_args(xf, mimo_x, lam_raw, dt, A):
    H, P, R = mimo_x.shape
    Bt, T, _ = xf.shape
    trap = lam_raw is not None
    if (xf.shape[2] != H * P or mimo_x.dtype != xf.dtype or not mimo_x.is_contiguous()
            or (trap and (lam_raw.shape != (Bt, T, H) or lam_raw.dtype != xf.dtype or dt.shape != (Bt, T, H)
                          or not dt.is_contiguous() or A.shape != (H,) or not A.is_contiguous()))):
        raise M3bError("xprep: inconsistent shapes or dtypes")
    return XprepArgs(Bt, T, H, P, R, int(trap), dtype_code(xf.dtype), dtype_code(dt.dtype) if trap else 0,
                     dtype_code(A.dtype) if trap else 0, _row_stride(xf, "xf"),
                     _row_stride(lam_raw, "lam_raw") if trap else 0, _ptr(xf), _ptr(mimo_x),
                     _ptr(lam_raw), _ptr(dt) if trap else None, _ptr(A) if trap else None)


def xprep_fwd(xf, mimo_x, lam_raw, dt, A):
    """x_raw = xf * mimo_x per rank; with lam_raw also x_g and x_b (trapezoid weights) ->
    (x_raw, x_g, x_b), each (batch, seqlen, H, P, R); x_g / x_b empty without lam_raw."""
    dev = _cuda(xf, mimo_x, lam_raw, dt, A)
    a = _xprep_args(xf, mimo_x, lam_raw, dt, A)
    shape = (a.batch, a.seqlen, a.H, a.P, a.R)
    trap = lam_raw is not None
    outs = [torch.empty(shape if (i == 0 or trap) else (0,), dtype=xf.dtype, device=dev) for i in range(3)]
    a.x_raw, a.x_g, a.x_b = _ptr(outs[0]), _ptr(outs[1]) if trap else None, _ptr(outs[2]) if trap else None
    with torch.cuda.device(dev):
        _check(lib().m3b_xprep_fwd(C.byref(a), _stream(dev)), "m3b_xprep_fwd")
    return tuple(outs)


def xprep_bwd(xf, mimo_x, lam_raw, dt, A, dx_raw, dx_g, dx_b):
    """Gradients of xprep_fwd -> (dxf, dmimo_x, dlam_raw, ddt, dA); the last three empty without
    lam_raw."""
    dev = _cuda(xf, mimo_x, lam_raw, dt, A, dx_raw, dx_g, dx_b)
    a = _xprep_args(xf, mimo_x, lam_raw, dt, A)
    shape = (a.batch, a.seqlen, a.H, a.P, a.R)
    trap = lam_raw is not None
    grads = [dx_raw] + ([dx_g, dx_b] if trap else [])
    if any(g.shape != shape or g.dtype != xf.dtype or not g.is_contiguous() for g in grads):
        raise M3bError("xprep_bwd: gradients of the forward outputs' shape and dtype, contiguous, expected")
    dxf = torch.empty(a.batch, a.seqlen, a.H * a.P, dtype=xf.dtype, device=dev)
    dmx = torch.empty_like(mimo_x)
    dlam = torch.empty((a.batch, a.seqlen, a.H) if trap else (0,), dtype=xf.dtype, device=dev)
    ddt = torch.empty(dt.shape if trap else (0,), dtype=dt.dtype, device=dev)
    dA = torch.empty(A.shape if trap else (0,), dtype=A.dtype, device=dev)
    a.dx_raw, a.dx_g, a.dx_b = _ptr(dx_raw), _ptr(dx_g) if trap else None, _ptr(dx_b) if trap else None
    a.dxf, a.dmimo_x = _ptr(dxf), _ptr(dmx)
    a.dlam_raw, a.ddt, a.dA = (_ptr(dlam), _ptr(ddt), _ptr(dA)) if trap else (None, None, None)
    L = lib()
    need = L.m3b_xprep_bwd_workspace(C.byref(a))
    ws = torch.empty(max(need, 16), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _check(L.m3b_xprep_bwd(C.byref(a), _ptr(ws), ws.numel(), _stream(dev)), "m3b_xprep_bwd")
    return dxf, dmx, dlam, ddt, dA


def rmsnorm(x, weight, eps, out=None):
    """RMSNorm over the last dim of x (contiguous) with weight (d,) of x's dtype."""
    dev = _cuda(x, weight, out)
    d = x.shape[-1]
    if x.stride(-1) != 1 or not x.is_contiguous() or weight.numel() != d or weight.dtype != x.dtype:
        raise M3bError("rmsnorm: contiguous x and a weight of x's dtype with x.shape[-1] entries expected")
    y = torch.empty_like(x) if out is None else out
    with torch.cuda.device(dev):
        _check(lib().m3b_rmsnorm(_ptr(x), _ptr(weight.contiguous()), _ptr(y), x.numel() // d, d, float(eps),
                                 dtype_code(x.dtype), _stream(dev)), "m3b_rmsnorm")
    return y


def _same(*ts):
    t0 = ts[0]
    for t in ts:
        if t.shape != t0.shape or t.dtype != t0.dtype or not t.is_contiguous():
            raise M3bError("element-wise op: contiguous tensors of one shape and dtype expected")


def swiglu_act(g, u, out=None):
    """silu(g) * u in g's dtype."""
    dev = _cuda(g, u, out)
    _same(g, u)
    out = torch.empty_like(g) if out is None else out
    with torch.cuda.device(dev):
        _check(lib().m3b_swiglu_act(_ptr(g), _ptr(u), _ptr(out), g.numel(), dtype_code(g.dtype), _stream(dev)),
               "m3b_swiglu_act")
    return out


def scaled_add(x, h, scale, out=None):
    """x + h * scale in x's dtype."""
    dev = _cuda(x, h, out)
    _same(x, h)
    out = torch.empty_like(x) if out is None else out
    with torch.cuda.device(dev):
        _check(lib().m3b_scaled_add(_ptr(x), _ptr(h), float(scale), _ptr(out), x.numel(), dtype_code(x.dtype),
                                    _stream(dev)), "m3b_scaled_add")
    return out


def swiglu_rows(gu, out=None):
    """silu(g) * u for gu (..., 2f) = [g | u] per row (one GEMM of the stacked gate / up weights)."""
    dev = _cuda(gu, out)
    if not gu.is_contiguous() or gu.shape[-1] % 2:
        raise M3bError("swiglu_rows: contiguous [g | u] rows expected")
    f = gu.shape[-1] // 2
    out = torch.empty(*gu.shape[:-1], f, dtype=gu.dtype, device=gu.device) if out is None else out
    with torch.cuda.device(dev):
        _check(lib().m3b_swiglu_rows(_ptr(gu), _ptr(out), gu.numel() // (2 * f), f, dtype_code(gu.dtype),
                                     _stream(dev)), "m3b_swiglu_rows")
    return out


def add_rmsnorm(x, h, scale, weight, eps, x_out=None, y=None):
    """x_out = x + h * scale (rounded as scaled_add stores it) and y = RMSNorm(x_out), one pass."""
    dev = _cuda(x, h, weight, x_out, y)
    _same(x, h)
    d = x.shape[-1]
    if weight.numel() != d or weight.dtype != x.dtype:
        raise M3bError("add_rmsnorm: a weight of x's dtype with x.shape[-1] entries expected")
    x_out = torch.empty_like(x) if x_out is None else x_out
    y = torch.empty_like(x) if y is None else y
    with torch.cuda.device(dev):
        _check(lib().m3b_add_rmsnorm(_ptr(x), _ptr(h), float(scale), _ptr(weight.contiguous()), _ptr(x_out), _ptr(y),
                                     x.numel() // d, d, float(eps), dtype_code(x.dtype), _stream(dev)),
               "m3b_add_rmsnorm")
    return x_out, y


def selftest_umma(A, B, mode):
    dev = _cuda(A, B)
    D = torch.empty(128, 64, dtype=torch.float32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        _check(lib().m3b_selftest_umma(_ptr(A), _ptr(B), _ptr(D), mode, _ptr(err), _stream(dev)), "selftest_umma")
    return D, err


def selftest_wait(flag, target, mode, limit_ns, err):
    """Bounded wait on `flag` >= target (mode 0) or on an mbarrier nothing completes (mode 1)."""
    dev = _cuda(flag, err)
    with torch.cuda.device(dev):
        _check(lib().m3b_selftest_wait(_ptr(flag), int(target), int(mode), int(limit_ns), _ptr(err), _stream(dev)),
               "selftest_wait")


# ---------------------------------------------------------------------------
# device error word
# ---------------------------------------------------------------------------
# Kernels that wait on the device (the fused layer kernel's pipeline and hand-off waits, the
# chunked kernels' tensor-core commits) give up after a bounded time and record
# M3B_ERR_TIMEOUT in an error word.  Every layer forward and chunked_ssd call of this module
# passes one word per device; it keeps the first error until check_device_errors() reads and
# clears it.  Reading it synchronises the device, so the calls themselves never do; set
# M3B_SYNC_CHECK=1 to check after every such call (debugging).
_err_words = {}
_SYNC_CHECK = __import__("os").environ.get("M3B_SYNC_CHECK", "0") not in ("", "0")


def device_err_word(dev):
    """The per-device int32 error word (allocated zeroed on first use; None when the first use
    falls inside a CUDA graph capture, which must not allocate)."""
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    w = _err_words.get(key)
    if w is None:
        if torch.cuda.is_current_stream_capturing():
            return None
        w = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", key))
        _err_words[key] = w
    return w


def check_device_errors(dev=None):
    """Synchronise `dev` (default: every device with an error word), read and clear its error
    word, and raise M3bError if a kernel recorded one (e.g. an expired bounded wait)."""
    keys = list(_err_words) if dev is None else [dev.index if dev.index is not None else torch.cuda.current_device()]
    for key in keys:
        w = _err_words.get(key)
        if w is None:
            continue
        code = int(w.item())
        if code != 0:
            w.zero_()
            L = lib()
            raise M3bError(f"device cuda:{key}: a kernel reported {L.m3b_strerror(code).decode()} (code {code})")


def _after_launch(dev):
    if _SYNC_CHECK:
        check_device_errors(dev)


def copy_token_range(dst, dst_t0, src, src_t0, ntok, stream):
    """dst[:, dst_t0:dst_t0+ntok] = src[:, src_t0:src_t0+ntok] for (batch, seqlen, d) tensors with
    contiguous last two dims, host or device on either side, asynchronously on `stream` (one
    strided copy for the whole batch)."""
    if dst.dim() != 3 or src.dim() != 3 or dst.shape[0] != src.shape[0] or dst.shape[2] != src.shape[2]:
        raise M3bError("copy_token_range: (batch, seqlen, d) tensors with equal batch and d expected")
    if dst.dtype != src.dtype:
        raise M3bError("copy_token_range: dtypes differ")
    for t in (dst, src):
        if t.stride(2) != 1 or t.stride(1) != t.shape[2]:
            raise M3bError("copy_token_range: the (seqlen, d) dims must be contiguous")
    es = src.element_size()
    row = ntok * src.shape[2] * es
    d_ptr = C.c_void_p(dst.data_ptr() + dst_t0 * dst.stride(1) * es)
    s_ptr = C.c_void_p(src.data_ptr() + src_t0 * src.stride(1) * es)
    _check(lib().m3b_copy_rows_async(d_ptr, dst.stride(0) * es, s_ptr, src.stride(0) * es, row, src.shape[0],
                                     C.c_void_p(stream.cuda_stream)), "m3b_copy_rows_async")


def seqpar_fold(summaries, upto: int, batch: int, H: int, P: int, N: int, h, angle, prev_bx):
    """m3b_seqpar_fold: the state entering shard `upto` from the summaries of shards 0 .. upto-1.
    summaries: (world, rank_stride) fp32 CUDA tensor (each row one rank's [S | PB | Om | Lam | c0]);
    h, prev_bx (batch, H, P, N) and angle (batch, H, N/2) fp32 outputs."""
    import torch

    for t in (summaries, h, angle, prev_bx):
        if not t.is_cuda or t.dtype != torch.float32 or not t.is_contiguous():
            raise M3bError("seqpar_fold: fp32 contiguous CUDA tensors required")
    a = SeqparFoldArgs(C.c_void_p(summaries.data_ptr()), summaries.stride(0) if summaries.dim() > 1 else 0,
                       upto, batch, H, P, N, C.c_void_p(h.data_ptr()), C.c_void_p(angle.data_ptr()),
                       C.c_void_p(prev_bx.data_ptr()))
    _check(lib().m3b_seqpar_fold(C.byref(a), _stream(h.device)), "m3b_seqpar_fold")
