"""Failure detection on the GPU without a GPU fault: every device-side wait of the library is
bounded, and one that runs out records M3B_ERR_TIMEOUT in an error word and lets the kernel
return.  These tests make a wait run out on purpose -- a flag nothing sets, an mbarrier nothing
arrives on -- with a limit of a few milliseconds, check that the status comes back, and that
the context is still usable afterwards."""

import time

import pytest
import torch

pytestmark = pytest.mark.gpu

M3B_ERR_TIMEOUT = 5


@pytest.mark.parametrize("mode", [0, 1], ids=["flag", "mbarrier"])
def test_expired_wait_reports_timeout(mode):
    from mamba3_b200 import _lib

    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    _lib.selftest_wait(flag, 1, mode, 5_000_000, err)  # 5 ms; nothing ever sets the flag / arrives
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert int(err.item()) == M3B_ERR_TIMEOUT
    assert waited < 1.0  # the limit, not the library's 2 s default, ended the wait
    # the context is still usable
    x = torch.arange(16, device="cuda", dtype=torch.float32)
    assert float(x.sum().item()) == 120.0


def test_satisfied_wait_reports_nothing():
    from mamba3_b200 import _lib

    flag = torch.full((1,), 3, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    _lib.selftest_wait(flag, 3, 0, 5_000_000, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0


def test_expired_wait_surfaces_through_device_error_word():
    """The word the layer forward and chunked_ssd calls pass by default: a timeout recorded in it
    turns into an M3bError at check_device_errors(), which then clears it."""
    from mamba3_b200 import KulaMamba, M3bError, _lib, check_device_errors

    torch.manual_seed(0)
    m = KulaMamba(d_model=128, d_state=128, headdim=64, mimo_rank=2).cuda().to(torch.bfloat16).eval()
    x = torch.randn(2, 300, 128, device="cuda").to(torch.bfloat16)
    with torch.no_grad():
        m(x)
    check_device_errors()  # a normal forward leaves the word clear
    word = _lib.device_err_word(x.device)
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    _lib.selftest_wait(flag, 1, 0, 2_000_000, word)
    with pytest.raises(M3bError, match="timed out"):
        check_device_errors()
    check_device_errors()  # cleared
    with torch.no_grad():
        m(x)
    check_device_errors()


def test_selftest_wait_rejects_bad_limits():
    from mamba3_b200 import M3bError, _lib

    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    for lim in (0, -1, 2_000_000_000):
        with pytest.raises(M3bError):
            _lib.selftest_wait(flag, 1, 0, lim, err)
