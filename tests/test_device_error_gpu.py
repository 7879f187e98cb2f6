"""Bounded device waits report through the error word instead of hanging.

Every mbarrier wait in the library's kernels has a wall-clock budget; on expiry the kernel records
OSAM_ERR_TIMEOUT in the library's device error word and returns.  This drives one wait to its limit in the
allowed form: a test-only kernel (one thread, no TMA, no TMEM) waits on an mbarrier that nothing arrives at,
under a short budget passed as an argument, and the host reads the code back through osam_device_error().
"""
import time

import pytest
import torch

from objectsam_b200 import _lib

pytestmark = pytest.mark.gpu


def test_bounded_wait_runs_out_and_reports_timeout(cuda_lib):
    assert _lib.device_error() == 0
    t0 = time.perf_counter()
    _lib.check(_lib.lib().osam_selftest_wait_timeout(20_000_000, _lib.stream_ptr()))  # 20 ms budget
    assert _lib.device_error() == _lib.OSAM_ERR_TIMEOUT
    assert time.perf_counter() - t0 < 5.0
    assert b"reported error 4" in _lib.lib().osam_last_error()
    # read and cleared: the next call sees a clean word, and the context is still usable
    assert _lib.device_error() == 0
    x = torch.ones(1024, device="cuda")
    assert x.sum().item() == 1024.0


def test_timeout_visible_without_synchronising(cuda_lib):
    """After the first plan exists the word is host-mapped: a finished kernel's timeout is visible to
    osam_device_error_peek() (no device synchronisation, no clearing) — what the ConvOp shim polls."""
    from objectsam_b200.conv import ConvGeom, ConvOp
    ConvOp().init(ConvGeom(1, 8, 8, 32, 32, 3, 3, 1, 1))  # plan creation sets up the mapped word
    assert _lib.device_error() == 0
    assert _lib.lib().osam_device_error_peek() == 0
    _lib.check(_lib.lib().osam_selftest_wait_timeout(10_000_000, _lib.stream_ptr()))
    torch.cuda.synchronize()
    assert _lib.lib().osam_device_error_peek() == _lib.OSAM_ERR_TIMEOUT
    assert _lib.lib().osam_device_error_peek() == _lib.OSAM_ERR_TIMEOUT  # peek does not clear
    assert _lib.device_error() == _lib.OSAM_ERR_TIMEOUT
    assert _lib.lib().osam_device_error_peek() == 0


def test_selftest_rejects_bad_budget(cuda_lib):
    assert _lib.lib().osam_selftest_wait_timeout(0, _lib.stream_ptr()) == _lib.OSAM_ERR_INVALID
    assert _lib.lib().osam_selftest_wait_timeout(10_000_000_000, _lib.stream_ptr()) == _lib.OSAM_ERR_INVALID
