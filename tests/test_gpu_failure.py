"""Failure detection on the GPU without a fault or a hang.

Every mbarrier wait of the library's kernels is bounded; when its budget
runs out the kernel raises the device error word (JT_B200_KERR_TIMEOUT),
drains and returns.  jt_b200_selftest_bounded_wait runs that wait on a
barrier nothing completes with a budget of about a millisecond: the test
checks that the host learns of it through jt_b200_sync_code, that the word
is cleared once read, and that the context then runs a kernel normally.
"""
import ctypes as C

import numpy as np
import pytest

from jimotono_b200 import JT_ERR_CUDA, JT_ERR_INVAL, lib

KERR_TIMEOUT = 0x71


@pytest.mark.gpu
def test_bounded_wait_runs_out_and_is_reported():
    from tests import _dev
    L = lib()
    code = C.c_int(-1)
    assert L.jt_b200_sync_code(C.byref(code)) == 0 and code.value == 0
    assert L.jt_b200_selftest_bounded_wait(2_000_000, _dev.stream()) == 0  # ~1 ms of SM cycles
    assert L.jt_b200_sync_code(C.byref(code)) == JT_ERR_CUDA
    assert code.value == KERR_TIMEOUT
    assert L.jt_b200_sync_code(C.byref(code)) == 0 and code.value == 0  # read once, then clear
    # the context is still usable: an int8 GEMM runs and is exact
    rng = np.random.default_rng(0)
    X = rng.integers(-127, 128, (16, 64), dtype=np.int8)
    W = rng.integers(-127, 128, (32, 64), dtype=np.int8)
    dX, dW = _dev.to_dev(X), _dev.to_dev(W)
    dC = _dev.zeros((16, 32), np.int32)
    assert L.jt_b200_w8a8_gemm_i32(dX.data_ptr(), 64, dW.data_ptr(), 64, dC.data_ptr(), 32, 16, 32, 64,
                                   _dev.stream()) == 0
    assert L.jt_b200_sync() == 0
    assert np.array_equal(_dev.host(dC), X.astype(np.int32) @ W.astype(np.int32).T)


def test_bounded_wait_budget_is_checked():
    # rejected before any device work, so no GPU is needed
    L = lib()
    assert L.jt_b200_selftest_bounded_wait(0, None) == JT_ERR_INVAL
    assert L.jt_b200_selftest_bounded_wait(5_000_000_000, None) == JT_ERR_INVAL
