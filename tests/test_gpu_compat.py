"""Reference-compatible routing, batch-sort, fp32 GEMM/transpose and
low-bit entry points (computed on the GPU) against the reference library
itself (oracle/_ref) and its known-answer cases: ids, perm/off/drop, codes
and GEMM/transpose results bit-exact; routing weights bit-exact on the
seeded cases (double exp of the GPU vs libm agree after the float
rounding)."""
import ctypes as C
import math

import numpy as np
import pytest

import oracle
from jimotono_b200 import JT_ERR_INVAL, lib

pytestmark = pytest.mark.gpu
needs_ref = pytest.mark.skipif(not oracle.have_ref(), reason="oracle/_ref not built")


def topk(fn, logits, k):
    lg = np.ascontiguousarray(logits, np.float32)
    ids = np.zeros(k, np.uint64)
    w = np.zeros(k, np.float32)
    rc = fn(lg.ctypes.data, lg.size, k, ids.ctypes.data, w.ctypes.data)
    return rc, ids, w


def test_topk_known_answers():
    f = lib().jt_routing_topk
    rc, ids, w = topk(f, [0.1, 2.0, 0.5, 3.0, 1.0], 2)
    assert rc == 0 and list(ids) == [3, 1] and abs(w[0] - 0.7310586) <= 1e-5
    rc, ids, w = topk(f, [0.1, 2.0, 0.5, 3.0, 1.0], 5)
    assert rc == 0 and list(ids) == [3, 1, 4, 2, 0]
    rc, ids, w = topk(f, [1.0, 1.0, 1.0], 2)
    assert rc == 0 and list(ids) == [0, 1] and np.allclose(w, 0.5)
    assert topk(f, [1.0, float("nan"), 0.5], 2)[0] == JT_ERR_INVAL
    assert topk(f, [math.inf, 1.0, 0.0], 2)[0] == JT_ERR_INVAL
    rc, ids, w = topk(f, [2.0, 1.0, -math.inf, -math.inf], 2)
    assert rc == 0 and list(ids) == [0, 1]
    rc, ids, w = topk(f, np.arange(4096) % 256, 16)
    assert rc == 0 and ids[0] == 255 and ids[15] == 4095
    assert topk(f, [1.0, 2.0], 3)[0] == JT_ERR_INVAL


@needs_ref
@pytest.mark.parametrize("n,k", [(64, 8), (1024, 8), (300, 100), (7, 7)])
def test_topk_vs_reference(n, k):
    rng = np.random.default_rng(n + k)
    for trial in range(5):
        lg = rng.standard_normal(n).astype(np.float32)
        if trial == 1:
            lg[::3] = 0.25  # ties
        r1 = topk(lib().jt_routing_topk, lg, k)
        r2 = topk(oracle.ref().jt_routing_topk, lg, k)
        assert r1[0] == r2[0] == 0
        assert np.array_equal(r1[1], r2[1])
        assert np.array_equal(r1[2].view(np.uint32), r2[2].view(np.uint32))


def _sort(fn, ids, T, k, E, cf):
    flat = np.ascontiguousarray(ids.reshape(-1).astype(np.uint64))
    perm = np.zeros(T * k, np.uint64)
    off = np.zeros(E + 1, np.uint64)
    drop = np.full(T * k, 9, np.uint8)
    kept, dropped = C.c_size_t(0), C.c_size_t(0)
    rc = fn(flat.ctypes.data, T, k, E, cf, perm.ctypes.data, off.ctypes.data, drop.ctypes.data,
            C.addressof(kept), C.addressof(dropped))
    return rc, perm[:kept.value], off, drop, kept.value, dropped.value


def test_batch_sort_known_answers():
    f = lib().jt_moe_batch_sort
    rc, perm, off, drop, kept, dropped = _sort(f, np.array([2, 0, 1, 2, 0, 1, 2, 1]), 4, 2, 3, 1.0)
    assert rc == 0 and list(perm) == [1, 4, 2, 5, 7, 0, 3, 6] and list(off) == [0, 2, 5, 8]
    assert kept == 8 and dropped == 0 and not drop.any()
    rc, perm, off, drop, kept, dropped = _sort(f, np.array([0, 0, 0, 0, 0, 1, 1, 1]), 4, 2, 2, 1.0)
    assert rc == 0 and list(perm) == [0, 1, 2, 3, 5, 6, 7] and list(off) == [0, 4, 7]
    assert list(drop) == [0, 0, 0, 0, 1, 0, 0, 0] and kept == 7 and dropped == 1
    assert _sort(f, np.array([0, 3]), 1, 2, 3, 1.0)[0] == JT_ERR_INVAL  # id out of range


@needs_ref
@pytest.mark.parametrize("T,k,E,cf", [(500, 8, 64, 1.0), (4096, 8, 256, 1.5), (77, 3, 5, 1.25)])
def test_batch_sort_vs_reference(T, k, E, cf):
    rng = np.random.default_rng(T)
    ids = ((rng.zipf(1.2, (T, k)) - 1) % E).astype(np.uint64)
    a = _sort(lib().jt_moe_batch_sort, ids, T, k, E, cf)
    b = _sort(oracle.ref().jt_moe_batch_sort, ids, T, k, E, cf)
    assert a[0] == b[0] == 0
    for x, y in zip(a[1:], b[1:]):
        assert np.array_equal(np.asarray(x), np.asarray(y))


@needs_ref
@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (13, 37, 129), (64, 256, 512), (200, 9, 33)])
def test_gemm_mat_f32_vs_reference(M, N, K):
    rng = np.random.default_rng(M * N + K)
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.standard_normal((K, N)).astype(np.float32)
    C1 = np.zeros((M, N), np.float32)
    C2 = np.zeros((M, N), np.float32)
    assert lib().jt_gemm_mat_f32(A.ctypes.data, B.ctypes.data, C1.ctypes.data, M, N, K) == 0
    assert oracle.ref().jt_gemm_mat_f32(A.ctypes.data, B.ctypes.data, C2.ctypes.data, M, N, K) == 0
    assert np.array_equal(C1.view(np.uint32), C2.view(np.uint32))


def test_transpose_f32():
    rng = np.random.default_rng(1)
    for r, c in [(1, 1), (33, 65), (128, 7)]:
        src = rng.standard_normal((r, c)).astype(np.float32)
        dst = np.zeros((c, r), np.float32)
        assert lib().jt_transpose_f32(src.ctypes.data, dst.ctypes.data, r, c) == 0
        assert np.array_equal(dst, src.T)


@needs_ref
@pytest.mark.parametrize("bits", [2, 4])
def test_lowbit_vs_reference(bits):
    rng = np.random.default_rng(bits)
    for n in (8, 256, 4096):
        w = (rng.standard_normal(n) * 0.3).astype(np.float32)
        w[n // 2] = -w.max() * 1.0001
        f1 = np.zeros(n, np.float32)
        f2 = np.zeros(n, np.float32)
        assert lib().jt_lowbit_fakequant(w.ctypes.data, f1.ctypes.data, n, bits) == 0
        assert oracle.ref().jt_lowbit_fakequant(w.ctypes.data, f2.ctypes.data, n, bits) == 0
        assert np.array_equal(f1.view(np.uint32), f2.view(np.uint32))
        i1 = np.zeros(bits * n // 4, np.uint8)
        i2 = np.zeros(bits * n // 4, np.uint8)
        s1, s2 = np.zeros(1, np.float32), np.zeros(1, np.float32)
        assert lib().jt_lowbit_col_to_idx(w.ctypes.data, n, bits, i1.ctypes.data, s1.ctypes.data) == 0
        assert oracle.ref().jt_lowbit_col_to_idx(w.ctypes.data, n, bits, i2.ctypes.data, s2.ctypes.data) == 0
        assert np.array_equal(i1, i2) and s1[0] == s2[0]


def test_lowbit_known_answers_and_modes():
    L = lib()
    col = np.arange(1, 9, dtype=np.float32)
    idx = np.zeros(8, np.uint8)
    ws = np.zeros(1, np.float32)
    assert L.jt_lowbit_col_to_idx(col.ctypes.data, 8, 4, idx.ctypes.data, ws.ctypes.data) == 0
    assert ws[0] == 8.0
    assert L.jt_lowbit_col_to_idx(col.ctypes.data, 7, 4, idx.ctypes.data, ws.ctypes.data) == JT_ERR_INVAL
    assert L.jt_lowbit_col_to_idx(col.ctypes.data, 8, 3, idx.ctypes.data, ws.ctypes.data) == JT_ERR_INVAL
    z = np.zeros(4, np.float32)
    fq = np.ones(4, np.float32)
    assert L.jt_lowbit_fakequant(z.ctypes.data, fq.ctypes.data, 4, 2) == 0 and not fq.any()
    bad = np.array([1.0, np.nan], np.float32)
    assert L.jt_lowbit_fakequant(bad.ctypes.data, fq.ctypes.data, 2, 2) == JT_ERR_INVAL
    b = C.c_int(0)
    assert L.jt_lowbit_bits_for(1, C.byref(b)) == 0 and b.value == 4
    assert L.jt_lowbit_bits_for(0, C.byref(b)) == 0 and b.value == 2
    assert L.jt_lowbit_set_mode(3) == JT_ERR_INVAL
    assert L.jt_lowbit_set_mode(2) == 0 and L.jt_lowbit_get_mode() == 2
    assert L.jt_lowbit_set_mode(0) == 0


# ---------------------------------------------------------------- T-MAC LUT (tmac.c, lowbit.c:158-267)
def _ctor(fn, act, n, k):
    a = np.ascontiguousarray(act, np.float32)
    q = np.full(n * (k // 4) * 8, 0x55, np.uint8).view(np.int8)
    sc = np.full(n * (k // 32), 7.0, np.float32)
    bi = np.full(n * (k // 32), 7.0, np.float32)
    rc = fn(a.ctypes.data, n, k, q.ctypes.data, sc.ctypes.data, bi.ctypes.data)
    return rc, q, sc, bi


def _lookup(fn, q, idx, sc, bi, ng, nb, bits, ws):
    out = np.full(1, 123.0, np.float32)
    rc = fn(q.ctypes.data, idx.ctypes.data, sc.ctypes.data, bi.ctypes.data, ng, nb, bits, ws, out.ctypes.data)
    return rc, out[0]


def test_tmac_known_answers():
    """tmac_lut.c:58-165: zero and single-activation tables, mirror sums,
    plane weighting, w_scale and bias."""
    L = lib()
    rc, q, sc, bi = _ctor(L.jt_tmac_lut_ctor, np.zeros(32), 1, 32)
    assert rc == 0 and sc[0] == 1.0 and bi[0] == 0.0 and not q.any()
    act = np.zeros(32, np.float32)
    act[0] = 8.0
    rc, q, sc, bi = _ctor(L.jt_tmac_lut_ctor, act, 1, 32)
    assert rc == 0 and sc[0] == np.float32(8.0 / 127.0) and bi[0] == 8.0
    assert list(q[:8]) == [-127, 127] * 4 and not q[8:].any()

    q = (np.arange(64) + 1).astype(np.int8)
    sc = np.ones(1, np.float32)
    bi = np.zeros(1, np.float32)
    for fill, want in ((15, 144.0), (0, -144.0), (8, 116.0), (7, -116.0), (0xA0, -144.0)):
        rc, out = _lookup(L.jt_tmac_lookup_accum, q, np.full(8, fill, np.uint8), sc, bi, 8, 1, 1, 1.0)
        assert rc == 0 and out == want
    idx = np.array([15] * 8 + [8] * 8, np.uint8)
    assert _lookup(L.jt_tmac_lookup_accum, q, idx, sc, bi, 8, 1, 2, 1.0) == (0, 376.0)
    idx = np.array([15] * 8 + [14] * 8 + [13] * 8, np.uint8)
    assert _lookup(L.jt_tmac_lookup_accum, q, idx, sc, bi, 8, 1, 3, 1.0) == (0, 968.0)
    idx = np.array([15] * 8 + [14] * 8 + [13] * 8 + [12] * 8, np.uint8)
    assert _lookup(L.jt_tmac_lookup_accum, q, idx, sc, bi, 8, 1, 4, 1.0) == (0, 2024.0)
    assert _lookup(L.jt_tmac_lookup_accum, q, idx, sc, bi, 8, 1, 4, 0.5) == (0, 1012.0)
    bi[0] = 4.0
    assert _lookup(L.jt_tmac_lookup_accum, q, idx, sc, bi, 8, 1, 4, 1.0) == (0, 2054.0)


def _acts(rng, kind, n, k):
    if kind == "normal":
        return rng.standard_normal((n, k)).astype(np.float32)
    if kind == "quarter":  # multiples of 1/4: many exact rounding ties
        return ((rng.integers(-6, 7, (n, k))) * 0.25).astype(np.float32)
    if kind == "sparse":
        a = rng.standard_normal((n, k)).astype(np.float32)
        a[rng.random((n, k)) < 0.7] = 0.0
        a[0, :32] = 0.0  # one all-zero block
        return a
    return (rng.standard_normal((n, k)) * 1e30).astype(np.float32)  # "huge"


@needs_ref
@pytest.mark.parametrize("kind", ["normal", "quarter", "sparse", "huge"])
@pytest.mark.parametrize("n,k", [(1, 32), (5, 256), (3, 2048)])
def test_tmac_ctor_vs_reference(kind, n, k):
    act = _acts(np.random.default_rng(n * k + len(kind)), kind, n, k)
    g = _ctor(lib().jt_tmac_lut_ctor, act, n, k)
    r = _ctor(oracle.ref().jt_tmac_lut_ctor, act, n, k)
    assert g[0] == r[0] == 0
    assert np.array_equal(g[1], r[1])
    assert np.array_equal(g[2].view(np.uint32), r[2].view(np.uint32))
    assert np.array_equal(g[3].view(np.uint32), r[3].view(np.uint32))


def test_tmac_ctor_errors():
    L = lib()
    act = np.ones((4, 64), np.float32)
    for bad in (np.nan, np.inf):
        a = act.copy()
        a[2, 40] = bad
        rc, q, sc, bi = _ctor(L.jt_tmac_lut_ctor, a, 4, 64)
        assert rc == JT_ERR_INVAL and (sc == 7.0).all()  # outputs untouched
    a = np.full((1, 32), 3e38, np.float32)  # block sum overflows float
    assert _ctor(L.jt_tmac_lut_ctor, a, 1, 32)[0] == JT_ERR_INVAL
    assert _ctor(L.jt_tmac_lut_ctor, act, 4, 48)[0] == JT_ERR_INVAL  # k % 32
    assert _ctor(L.jt_tmac_lut_ctor, act, 0, 64)[0] == JT_ERR_INVAL
    assert L.jt_tmac_lut_ctor(None, 1, 32, None, None, None) == JT_ERR_INVAL


@needs_ref
@pytest.mark.parametrize("bits", [1, 2, 3, 4])
@pytest.mark.parametrize("nb", [1, 3, 64, 300])
def test_tmac_lookup_vs_reference(bits, nb):
    rng = np.random.default_rng(bits * 1000 + nb)
    ng = nb * 8
    q = rng.integers(-128, 128, ng * 8).astype(np.int8)
    idx = rng.integers(0, 256, bits * ng).astype(np.uint8)
    sc = rng.uniform(1e-3, 0.1, nb).astype(np.float32)
    bi = rng.standard_normal(nb).astype(np.float32)
    for ws in (1.0, 0.37, -2.5):
        g = _lookup(lib().jt_tmac_lookup_accum, q, idx, sc, bi, ng, nb, bits, ws)
        r = _lookup(oracle.ref().jt_tmac_lookup_accum, q, idx, sc, bi, ng, nb, bits, ws)
        assert g[0] == r[0] == 0
        assert np.float32(g[1]).view(np.uint32) == np.float32(r[1]).view(np.uint32)


def test_tmac_lookup_errors():
    L = lib()
    q = np.ones(64, np.int8)
    idx = np.full(32, 15, np.uint8)
    sc = np.ones(1, np.float32)
    bi = np.zeros(1, np.float32)
    assert _lookup(L.jt_tmac_lookup_accum, q, idx, sc, bi, 8, 2, 1, 1.0)[0] == JT_ERR_INVAL  # ng != nb*8
    assert _lookup(L.jt_tmac_lookup_accum, q, idx, sc, bi, 8, 1, 5, 1.0)[0] == JT_ERR_INVAL
    assert _lookup(L.jt_tmac_lookup_accum, q, idx, sc, bi, 8, 1, 1, math.inf)[0] == JT_ERR_INVAL
    assert _lookup(L.jt_tmac_lookup_accum, q, idx, np.full(1, np.nan, np.float32), bi, 8, 1, 1, 1.0) == \
        (JT_ERR_INVAL, 123.0)
    big = np.full(1, 3e38, np.float32)  # float result overflows
    assert _lookup(L.jt_tmac_lookup_accum, q, idx, big, bi, 8, 1, 4, 1.0) == (JT_ERR_INVAL, 123.0)


def _gemm_lut(fn, X, W, me, h, k, bits):
    Y = np.full((max(me, 1), h), -7.0, np.float32)
    rc = fn(X.ctypes.data, W.ctypes.data, Y.ctypes.data, me, h, k, bits)
    return rc, Y


@needs_ref
@pytest.mark.parametrize("me,h,k,bits", [(3, 40, 64, 2), (7, 130, 256, 4), (2, 33, 2048, 2),
                                         (17, 64, 512, 4), (4, 20, 48, 2), (2, 5, 30, 4)])
def test_lowbit_gemm_lut_vs_reference(me, h, k, bits):
    """The LUT product (k % 32 == 0) and the double-accumulated fallback
    (k % 32 != 0), bit-exact."""
    rng = np.random.default_rng(me * h + k + bits)
    X = rng.standard_normal((me, k)).astype(np.float32)
    W = (rng.standard_normal((k, h)) * 0.05).astype(np.float32)
    W[:, 0] = 0.0  # an all-zero column (maxa 0)
    g = _gemm_lut(lib().jt_lowbit_gemm_lut, X, W, me, h, k, bits)
    r = _gemm_lut(oracle.ref().jt_lowbit_gemm_lut, X, W, me, h, k, bits)
    assert g[0] == r[0] == 0
    assert np.array_equal(g[1].view(np.uint32), r[1].view(np.uint32))


def test_lowbit_gemm_lut_errors():
    L = lib()
    X = np.ones((2, 64), np.float32)
    W = np.ones((64, 8), np.float32)
    assert _gemm_lut(L.jt_lowbit_gemm_lut, X, W, 0, 8, 64, 2)[0] == 0
    assert _gemm_lut(L.jt_lowbit_gemm_lut, X, W, 2, 8, 64, 3)[0] == JT_ERR_INVAL
    assert _gemm_lut(L.jt_lowbit_gemm_lut, X, W, -1, 8, 64, 2)[0] == JT_ERR_INVAL
    for arr in ("X", "W"):
        X2, W2 = X.copy(), W.copy()
        (X2 if arr == "X" else W2)[1, 3] = np.nan
        rc, Y = _gemm_lut(L.jt_lowbit_gemm_lut, X2, W2, 2, 8, 64, 2)
        assert rc == JT_ERR_INVAL and (Y == -7.0).all()
