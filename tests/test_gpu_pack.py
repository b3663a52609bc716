"""Weight preparation on the device against the CPU side.

* jt_b200_lowbit_pack (fp32 masters -> packed INT2/INT4 group-64 codes and
  fp16 scales) against the oracle's restatement of the level rule
  (jto_pack_lowbit, lowbit.c:78-88 per 64-element group), bit for bit, in
  both scale layouts; the inputs include all-zero groups, groups whose
  values sit exactly on level boundaries (where only the double expression
  decides the code), tiny and huge maxima.
* jt_b200_lowbit_planes_to_packed against the reference library itself:
  the bit planes of jt_lowbit_col_to_idx (lowbit.c:93-141) convert to the
  codes the oracle packs with one group spanning the column.
"""
import ctypes as C

import numpy as np
import pytest

import oracle
from jimotono_b200 import JT_ERR_INVAL, lib

pytestmark = pytest.mark.gpu


def _masters(rng, rows, K, bits):
    W = rng.standard_normal((rows, K)).astype(np.float32)
    nl1 = (1 << bits) - 1
    G = K // 64
    for r in range(rows):
        kind = r % 6
        g = r % G
        grp = W[r, 64 * g:64 * (g + 1)]
        if kind == 1:    # all zero
            grp[:] = 0.0
        elif kind == 2:  # integers with max |w| = n-1: every even step lands on a floor boundary
            grp[:] = rng.integers(-nl1, nl1 + 1, 64).astype(np.float32)
            grp[0] = nl1
        elif kind == 3:  # the same boundaries at another scale
            grp[:] = rng.integers(-nl1, nl1 + 1, 64).astype(np.float32) * np.float32(0.37)
            grp[1] = -nl1 * np.float32(0.37)
        elif kind == 4:  # tiny values: subnormal fp16 scales
            grp *= np.float32(1e-6)
        elif kind == 5:  # huge values: the fp16 scale overflows to infinity
            grp *= np.float32(1e6)
    return W


def _oracle_pack(W, bits, group):
    rows, K = W.shape
    packed = np.zeros((rows, K * bits // 8), np.uint8)
    scales = np.zeros((rows, K // group), np.uint16)
    assert oracle.oracle().jto_pack_lowbit(W.ctypes.data, rows, K, bits, group, packed.ctypes.data,
                                           scales.ctypes.data) == 0
    return packed, scales


def _group_major(scales, n_ch):
    rows, G = scales.shape
    return np.ascontiguousarray(scales.reshape(rows // n_ch, n_ch, G).transpose(0, 2, 1)).reshape(rows, G)


@pytest.mark.parametrize("bits", [2, 4])
@pytest.mark.parametrize("rows,K,n_ch", [(48, 2048, 0), (256, 1024, 128), (7, 64, 0), (192, 4096, 64),
                                         (1000, 256, 0)])
def test_pack_matches_oracle(bits, rows, K, n_ch):
    from tests import _dev
    rng = np.random.default_rng(rows * 31 + K + bits)
    W = _masters(rng, rows, K, bits)
    want_p, want_s = _oracle_pack(W, bits, 64)
    if n_ch:
        want_s = _group_major(want_s, n_ch)
    dW = _dev.to_dev(W)
    dp = _dev.zeros((rows, K * bits // 8), np.uint8)
    ds = _dev.zeros((rows, K // 64), np.uint16)
    rc = lib().jt_b200_lowbit_pack(dW.data_ptr(), rows, K, bits, n_ch, dp.data_ptr(), ds.data_ptr(),
                                   _dev.stream())
    assert rc == 0
    assert lib().jt_b200_sync() == 0
    got_p = _dev.host(dp)
    got_s = _dev.host(ds).view(np.uint16)
    assert np.array_equal(got_p, want_p), f"code bytes differ at {np.argwhere(got_p != want_p)[:5]}"
    assert np.array_equal(got_s, want_s), f"scales differ at {np.argwhere(got_s != want_s)[:5]}"


def test_packed_masters_feed_the_gemv():
    """Packed on the GPU, multiplied on the GPU: equal to the oracle's GEMV on
    the oracle's packing of the same masters."""
    from tests import _dev
    rng = np.random.default_rng(5)
    K, n2, n4 = 2048, 300, 100
    W2 = rng.standard_normal((n2, K)).astype(np.float32) * np.float32(0.02)
    W4 = rng.standard_normal((n4, K)).astype(np.float32) * np.float32(0.02)
    a = rng.integers(-127, 128, K, dtype=np.int8)
    sa = np.float32(0.0123)
    want = []
    for W, bits in ((W2, 2), (W4, 4)):
        p, s = _oracle_pack(W, bits, 64)
        y = np.zeros(W.shape[0], np.float32)
        oracle.oracle().jto_lowbit_gemv(a.ctypes.data, float(sa), p.ctypes.data, s.ctypes.data, W.shape[0], K,
                                        bits, y.ctypes.data)
        want.append(y)
    want = np.concatenate(want)
    dev = {}
    for name, W, bits in (("2", W2, 2), ("4", W4, 4)):
        dW = _dev.to_dev(W)
        dp = _dev.zeros((W.shape[0], K * bits // 8), np.uint8)
        ds = _dev.zeros((W.shape[0], K // 64), np.uint16)
        assert lib().jt_b200_lowbit_pack(dW.data_ptr(), W.shape[0], K, bits, 0, dp.data_ptr(), ds.data_ptr(),
                                         _dev.stream()) == 0
        dev[name] = (dW, dp, ds)
    da = _dev.to_dev(a)
    dy = _dev.zeros(n2 + n4, np.float32)
    assert lib().jt_b200_lowbit_gemv(da.data_ptr(), float(sa), dev["2"][1].data_ptr(), dev["2"][2].data_ptr(), n2,
                                     dev["4"][1].data_ptr(), dev["4"][2].data_ptr(), n4, K, dy.data_ptr(),
                                     _dev.stream()) == 0
    assert lib().jt_b200_sync() == 0
    got = _dev.host(dy)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.skipif(not oracle.have_ref(), reason="reference library not built")
@pytest.mark.parametrize("bits,cols,K,n_ch", [(2, 40, 2048, 0), (4, 33, 1024, 0), (2, 64, 256, 32),
                                              (4, 128, 64, 64)])
def test_planes_to_packed_matches_reference_planes(bits, cols, K, n_ch):
    from tests import _dev
    rng = np.random.default_rng(cols + K + bits)
    W = rng.standard_normal((cols, K)).astype(np.float32)
    W[1, :] = 0.0
    nl1 = (1 << bits) - 1
    W[2, :] = rng.integers(-nl1, nl1 + 1, K).astype(np.float32)
    W[2, 0] = nl1
    ref = oracle.ref()
    idx = np.zeros((cols, bits * K // 4), np.uint8)
    ws = np.zeros(cols, np.float32)
    for j in range(cols):
        col = np.ascontiguousarray(W[j])
        wsj = C.c_float(0.0)
        assert ref.jt_lowbit_col_to_idx(col.ctypes.data, K, bits, idx[j].ctypes.data, C.addressof(wsj)) == 0
        ws[j] = wsj.value
    want_p, _ = _oracle_pack(W, bits, K)  # one group spanning the column: the reference's codes
    want_s = np.repeat((np.float64(ws)[:, None] / nl1).astype(np.float32).astype(np.float16).view(np.uint16),
                       K // 64, axis=1)
    if n_ch:
        want_s = _group_major(want_s, n_ch)
    di, dws = _dev.to_dev(idx), _dev.to_dev(ws)
    dp = _dev.zeros((cols, K * bits // 8), np.uint8)
    ds = _dev.zeros((cols, K // 64), np.uint16)
    assert lib().jt_b200_lowbit_planes_to_packed(di.data_ptr(), dws.data_ptr(), cols, K, bits, n_ch, dp.data_ptr(),
                                                 ds.data_ptr(), _dev.stream()) == 0
    assert lib().jt_b200_sync() == 0
    assert np.array_equal(_dev.host(dp), want_p)
    assert np.array_equal(_dev.host(ds).view(np.uint16), want_s)
    # codes only
    dp2 = _dev.zeros((cols, K * bits // 8), np.uint8)
    assert lib().jt_b200_lowbit_planes_to_packed(di.data_ptr(), None, cols, K, bits, 0, dp2.data_ptr(), None,
                                                 _dev.stream()) == 0
    assert lib().jt_b200_sync() == 0
    assert np.array_equal(_dev.host(dp2), want_p)


def test_pack_reports_non_finite_masters():
    from tests import _dev
    W = np.ones((4, 128), np.float32)
    W[2, 77] = np.nan
    dW = _dev.to_dev(W)
    dp = _dev.zeros((4, 32), np.uint8)
    ds = _dev.zeros((4, 2), np.uint16)
    assert lib().jt_b200_lowbit_pack(dW.data_ptr(), 4, 128, 2, 0, dp.data_ptr(), ds.data_ptr(), _dev.stream()) == 0
    assert lib().jt_b200_sync() != 0
    assert lib().jt_b200_sync() == 0  # the error word was cleared by the first read


def test_pack_rejects_bad_arguments():
    L = lib()
    buf = np.zeros(64, np.uint8)
    p = buf.ctypes.data
    assert L.jt_b200_lowbit_pack(None, 4, 128, 2, 0, p, p, None) == JT_ERR_INVAL
    assert L.jt_b200_lowbit_pack(p, 4, 100, 2, 0, p, p, None) == JT_ERR_INVAL   # K % 64
    assert L.jt_b200_lowbit_pack(p, 4, 128, 3, 0, p, p, None) == JT_ERR_INVAL   # bits
    assert L.jt_b200_lowbit_pack(p, 6, 128, 2, 4, p, p, None) == JT_ERR_INVAL   # rows % n_ch
    assert L.jt_b200_lowbit_pack(p + 4, 4, 128, 2, 0, p, p, None) == JT_ERR_INVAL  # 8-byte alignment
    assert L.jt_b200_lowbit_planes_to_packed(p, None, 4, 128, 2, 0, p, p, None) == JT_ERR_INVAL  # scales w/o w_scale
    assert L.jt_b200_lowbit_planes_to_packed(p, p, 4, 128, 1, 0, p, p, None) == JT_ERR_INVAL
