"""jt_b200_w8a8_linear_noalloc: quantize + W8A8 GEMM with library-held
scratch, against the same work done through the existing entry points
(jt_w8a8_quant_per_channel for the per-token codes and scales, then
jt_b200_w8a8_gemm).  The arithmetic is identical, so the outputs must
agree to within 1e-6 relative (they are expected to be bit-identical).

Two calls in a row with different inputs check that nothing of the first
call leaks into the second through the shared scratch.  The file name
sorts last so it also runs after every other test in one session.
"""
import ctypes as C

import numpy as np
import pytest

from jimotono_b200 import JT_ERR_INVAL, lib

TOL = 1e-6


def _existing_path(x, W, sw):
    """Per-token quantization via the reference-compatible host API, GEMM
    via the device entry point."""
    from tests import _dev
    M, K = x.shape
    N = W.shape[0]
    q = np.empty((M, K), np.int8)
    sx = np.empty(M, np.float32)
    rc = lib().jt_w8a8_quant_per_channel(x.ctypes.data, M, K, q.ctypes.data, sx.ctypes.data)
    assert rc == 0
    dq, dsx, dW, dsw = _dev.to_dev(q), _dev.to_dev(sx), _dev.to_dev(W), _dev.to_dev(sw)
    dC = _dev.zeros((M, N), np.float32)
    rc = lib().jt_b200_w8a8_gemm(dq.data_ptr(), K, dsx.data_ptr(), dW.data_ptr(), K,
                                 dsw.data_ptr(), dC.data_ptr(), N, M, N, K, _dev.stream())
    assert rc == 0
    assert lib().jt_b200_sync() == 0
    return _dev.host(dC)


def _noalloc(x, W, sw):
    from tests import _dev
    M, K = x.shape
    N = W.shape[0]
    dx, dW, dsw = _dev.to_dev(x), _dev.to_dev(W), _dev.to_dev(sw)
    dC = _dev.zeros((M, N), np.float32)
    rc = lib().jt_b200_w8a8_linear_noalloc(dx.data_ptr(), M, K, dW.data_ptr(), K, dsw.data_ptr(),
                                           dC.data_ptr(), N, N, _dev.stream())
    assert rc == 0
    assert lib().jt_b200_sync() == 0
    return _dev.host(dC)


def _case(seed, M, N, K):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K)).astype(np.float32) * rng.uniform(0.1, 4.0, (M, 1)).astype(
        np.float32)
    W = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    sw = rng.uniform(0.001, 0.01, N).astype(np.float32)
    return x, W, sw


@pytest.mark.gpu
def test_noalloc_matches_existing_entry_points_twice():
    # Second call: more rows and a different K, so stale codes or scales
    # from the first call would show.
    for seed, (M, N, K) in ((11, (96, 384, 1024)), (12, (300, 256, 512))):
        x, W, sw = _case(seed, M, N, K)
        want = _existing_path(x, W, sw)
        got = _noalloc(x, W, sw)
        scale = max(float(np.abs(want).max()), 1e-30)
        assert float(np.abs(got - want).max()) / scale <= TOL


@pytest.mark.gpu
def test_noalloc_at_the_size_limit():
    M, K, N = 512, 4096, 256  # M * K == 2 MiB of codes
    x, W, sw = _case(13, M, N, K)
    want = _existing_path(x, W, sw)
    got = _noalloc(x, W, sw)
    assert float(np.abs(got - want).max()) / float(np.abs(want).max()) <= TOL


def test_noalloc_rejects_shapes_beyond_its_scratch():
    # Rejected before any device work, so no GPU is needed.
    f = lib().jt_b200_w8a8_linear_noalloc
    p = C.c_void_p(16)
    assert f(p, 4097, 16, p, 16, p, p, 16, 16, None) == JT_ERR_INVAL
    assert f(p, 513, 4096, p, 4096, p, p, 16, 16, None) == JT_ERR_INVAL
    assert f(p, 4, 24, p, 32, p, p, 16, 16, None) == JT_ERR_INVAL  # K not a multiple of 16


@pytest.mark.gpu
def test_noalloc_nonfinite_row_comes_out_nan_and_is_reported():
    from tests import _dev
    M, N, K = 64, 128, 256
    x, W, sw = _case(14, M, N, K)
    x[5, 17] = np.inf
    dx, dW, dsw = _dev.to_dev(x), _dev.to_dev(W), _dev.to_dev(sw)
    dC = _dev.zeros((M, N), np.float32)
    rc = lib().jt_b200_w8a8_linear_noalloc(dx.data_ptr(), M, K, dW.data_ptr(), K, dsw.data_ptr(),
                                           dC.data_ptr(), N, N, _dev.stream())
    assert rc == 0
    assert lib().jt_b200_sync() != 0  # the non-finite activation is reported ...
    assert lib().jt_b200_sync() == 0  # ... once
    got = _dev.host(dC)
    assert np.isnan(got[5]).all()
    x[5] = 0.0  # every other row is quantized on its own
    want = _existing_path(x, W, sw)
    keep = np.arange(M) != 5
    scale = float(np.abs(want[keep]).max())
    assert float(np.abs(got[keep] - want[keep]).max()) / scale <= TOL
    # the next call starts clean
    x2, W2, sw2 = _case(15, M, N, K)
    got2 = _noalloc(x2, W2, sw2)
    want2 = _existing_path(x2, W2, sw2)
    assert float(np.abs(got2 - want2).max()) / float(np.abs(want2).max()) <= TOL


def test_noalloc_rejects_misaligned_weights():
    f = lib().jt_b200_w8a8_linear_noalloc
    p, q = C.c_void_p(16), C.c_void_p(24)
    assert f(p, 4, 16, q, 16, p, p, 16, 16, None) == JT_ERR_INVAL
