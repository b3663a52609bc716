"""Batch-1 low-bit GEMV (jt_b200_lowbit_gemv) against the oracle's
restatement (jto_lowbit_gemv): int32 group partials and the fp32 fold in
group order are reproduced exactly, so the outputs are compared bit for bit.
"""
import numpy as np
import pytest

import oracle
from jimotono_b200 import JT_ERR_INVAL, lib

pytestmark = pytest.mark.gpu


def _rows(rng, n, K, bits):
    packed = rng.integers(0, 256, (n, K * bits // 8), dtype=np.uint8)
    scales = rng.uniform(0.01, 0.05, (n, K // 64)).astype(np.float16).view(np.uint16)
    return packed, scales


def _oracle(a, sa, packed, scales, bits):
    n, K = packed.shape[0], a.size
    y = np.zeros(n, np.float32)
    if n:
        oracle.oracle().jto_lowbit_gemv(a.ctypes.data, float(sa), packed.ctypes.data, scales.ctypes.data,
                                        n, K, bits, y.ctypes.data)
    return y


@pytest.mark.parametrize("n2,n4,K", [(256, 96, 2048), (70, 33, 1024), (64, 64, 4096), (0, 40, 2048),
                                     (37, 0, 192), (1, 1, 64),
                                     (20000, 7000, 256),    # many chunks per CTA: ring reuse
                                     (9472, 4736, 2048),    # 2 + 1 ring turns per SM
                                     (49152, 16384, 2048)])  # the batch-1 GEMV configuration in full
def test_lowbit_gemv_matches_oracle(n2, n4, K):
    from tests import _dev
    rng = np.random.default_rng(n2 * 7 + n4 + K)
    a = rng.integers(-127, 128, K, dtype=np.int8)
    sa = np.float32(rng.uniform(0.005, 0.02))
    w2, s2 = _rows(rng, n2, K, 2)
    w4, s4 = _rows(rng, n4, K, 4)
    want = np.concatenate([_oracle(a, sa, w2, s2, 2), _oracle(a, sa, w4, s4, 4)])
    da = _dev.to_dev(a)
    dw2, ds2 = (_dev.to_dev(w2), _dev.to_dev(s2)) if n2 else (None, None)
    dw4, ds4 = (_dev.to_dev(w4), _dev.to_dev(s4)) if n4 else (None, None)
    dy = _dev.zeros(n2 + n4, np.float32)
    rc = lib().jt_b200_lowbit_gemv(da.data_ptr(), float(sa),
                                   dw2.data_ptr() if n2 else None, ds2.data_ptr() if n2 else None, n2,
                                   dw4.data_ptr() if n4 else None, ds4.data_ptr() if n4 else None, n4,
                                   K, dy.data_ptr(), _dev.stream())
    assert rc == 0
    assert lib().jt_b200_sync() == 0
    got = _dev.host(dy)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
        f"mismatches {(got != want).sum()} max {np.abs(got - want).max()}"


def test_lowbit_gemv_rejects_bad_shapes():
    f = lib().jt_b200_lowbit_gemv
    assert f(None, 1.0, None, None, 0, None, None, 0, 64, None, None) == JT_ERR_INVAL
