"""The allocation-free layer forward, m3b_layer_fwd_noalloc, against m3b_layer_fwd.

Some callers cannot allocate device memory where they run the layer (for example a
plugin inside another runtime that owns the allocator and only hands over the input
and output buffers).  m3b_layer_fwd_noalloc serves them from a fixed static scratch
array inside the library.  This file checks, through the C ABI, that two calls in a
row give the same results as the allocating entry point, and that a problem too large
for the static scratch is refused.  It is collected last so that a failure here does
not hide the other tests' results.
"""

import ctypes as C

import pytest
import torch

from goldens import max_rel
from helpers import to_np

pytestmark = pytest.mark.gpu

TOL = 2e-2  # the bf16 tolerance used by the layer parity tests


def _layer(d_model=128):
    from mamba3_b200 import KulaMamba

    torch.manual_seed(3)
    return KulaMamba(d_model=d_model, d_state=128, headdim=64, mimo_rank=2).cuda().to(torch.bfloat16).eval()


def _args(m, proj, y, h_final, angle, prev_bx):
    from mamba3_b200 import _lib

    prm = _lib.layer_params(m.nheads, m.headdim, m.d_state, m.mimo_rank, m.ngroups, m.use_trapezoidal,
                            m.use_complex_ssm, m.B_norm.eps, *m._param_tensors())
    Bt, T, _ = proj.shape
    p = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    return _lib.LayerFwdArgs(prm, Bt, T, p(proj), proj.stride(1), _lib.BF16, None, None, None, None, p(y),
                             p(h_final), p(angle), p(prev_bx), None)


def _outputs(proj, H, P, N):
    Bt, T, _ = proj.shape
    f32 = dict(dtype=torch.float32, device="cuda")
    return (torch.empty(Bt, T, H * P, dtype=proj.dtype, device="cuda"), torch.empty(Bt, H, P, N, **f32),
            torch.empty(Bt, H, N // 2, **f32), torch.empty(Bt, H, P, N, **f32))


@pytest.mark.parametrize("d_model,B,T", [(128, 2, 150), (768, 8, 1000)], ids=["whole", "parts"])
def test_noalloc_matches_allocating_entry_point_twice(d_model, B, T):
    """"whole": 4 (batch, head) sequences, one per CTA.  "parts": 192 sequences of 16 chunks, more
    than the SMs, so the fused kernel cuts them into parts handed from CTA to CTA through the
    scratch (states, angles and the flags that order the hand-offs); the second call finds the
    first call's flags in the shared scratch and must not be misled by them."""
    from mamba3_b200 import _lib

    m = _layer(d_model)
    L = _lib.lib()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    H, P, N = m.nheads, m.headdim, m.d_state
    if d_model == 768:  # the workspace holds the part hand-off buffers and fits the static scratch
        proj0 = torch.empty(B, T, m.in_proj.out_features, dtype=torch.bfloat16, device="cuda")
        ws = L.m3b_layer_fwd_workspace(C.byref(_args(m, proj0, *_outputs(proj0, H, P, N))))
        assert B * H * P * N * 4 < ws <= (32 << 20), ws
    for call, seed in enumerate((11, 12)):
        g = torch.Generator().manual_seed(seed)
        x = torch.randn(B, T, d_model, generator=g).cuda().to(torch.bfloat16)
        with torch.no_grad():
            proj = m.in_proj(x).contiguous()
        ref = _outputs(proj, H, P, N)
        prm = _lib.layer_params(H, P, N, m.mimo_rank, m.ngroups, m.use_trapezoidal, m.use_complex_ssm,
                                m.B_norm.eps, *m._param_tensors())
        _lib.layer_fwd(prm, proj, ref[0], h_final=ref[1], angle_final=ref[2], prev_bx_final=ref[3])
        out = _outputs(proj, H, P, N)
        a = _args(m, proj, *out)
        rc = L.m3b_layer_fwd_noalloc(C.byref(a), stream)
        assert rc == 0, (call, L.m3b_last_error())
        torch.cuda.synchronize()
        for o, r in zip(out, ref):
            assert max_rel(to_np(o), to_np(r)) < TOL, call


def test_noalloc_rejects_problem_larger_than_scratch():
    from mamba3_b200 import _lib

    m = _layer()
    L = _lib.lib()
    # the chunk-parallel algorithm keeps every chunk state in scratch: 16 x 4096 tokens need far
    # more than the static array; refused on the host, nothing launched
    proj = torch.empty(16, 4096, m.in_proj.out_features, dtype=torch.bfloat16, device="cuda")
    out = _outputs(proj, m.nheads, m.headdim, m.d_state)
    a = _args(m, proj, *out)
    a.algo = 2
    assert L.m3b_layer_fwd_workspace(C.byref(a)) > (32 << 20)
    rc = L.m3b_layer_fwd_noalloc(C.byref(a), C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 6  # M3B_ERR_WORKSPACE
    assert b"static scratch" in L.m3b_last_error()
