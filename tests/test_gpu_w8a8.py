"""W8A8 tensor-core GEMM parity on the GPU (through the C ABI).

* int32 accumulators: bit-exact against the oracle's integer GEMM
  (restating w8a8.c:654-686).
* per-token x per-channel fp32 output: bit-exact against the oracle's
  epilogue ((float)acc * sx) * sw, and within 1e-6 relative of the
  reference's fp64 formula.
* reference-compatible jt_w8a8_gemm_per_channel / _per_tensor: bit-exact
  against the reference library itself (oracle/_ref), including the
  fail-closed error cases of test_w8a8.c:250-272.
"""
import ctypes as C

import numpy as np
import pytest

import oracle
from jimotono_b200 import lib

pytestmark = pytest.mark.gpu

SHAPES = [  # (M, N, K)
    (1, 128, 128), (16, 256, 256), (17, 200, 144), (64, 4096, 1024), (128, 512, 2048),
    (200, 384, 1040), (1000, 256, 512), (300, 130, 64), (512, 768, 1024), (1024, 1024, 256),
    (384, 640, 2176),
    # CTA-pair kernel: fewer tiles than pairs, ragged K, more tiles than pairs
    (512, 4096, 1024), (256, 2048, 512), (300, 520, 208), (2560, 2048, 384),
]


def _rand_s8(rng, shape):
    return rng.integers(-127, 128, size=shape, dtype=np.int8)


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_i32_accumulators_bit_exact(M, N, K):
    from tests import _dev
    rng = np.random.default_rng(1000 + M + N + K)
    X = _rand_s8(rng, (M, K))
    W = _rand_s8(rng, (N, K))
    want = np.empty((M, N), np.int32)
    oracle.oracle().jto_gemm_s8(oracle.ptr(X), oracle.ptr(W), oracle.ptr(want), M, N, K)
    dX, dW = _dev.to_dev(X), _dev.to_dev(W)
    dC = _dev.zeros((M, N), np.int32)
    rc = lib().jt_b200_w8a8_gemm_i32(dX.data_ptr(), K, dW.data_ptr(), K, dC.data_ptr(), N,
                                     M, N, K, _dev.stream())
    assert rc == 0
    assert lib().jt_b200_sync() == 0
    got = _dev.host(dC)
    assert np.array_equal(got, want), f"mismatches: {(got != want).sum()}"


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_token_channel_f32(M, N, K):
    from tests import _dev
    rng = np.random.default_rng(2000 + M + N + K)
    X = _rand_s8(rng, (M, K))
    W = _rand_s8(rng, (N, K))
    sx = rng.uniform(0.005, 0.02, M).astype(np.float32)
    sw = rng.uniform(0.001, 0.01, N).astype(np.float32)
    acc = np.empty((M, N), np.int32)
    o = oracle.oracle()
    o.jto_gemm_s8(oracle.ptr(X), oracle.ptr(W), oracle.ptr(acc), M, N, K)
    want = np.empty((M, N), np.float32)
    o.jto_w8a8_token_channel(oracle.ptr(acc), oracle.ptr(sx), oracle.ptr(sw), oracle.ptr(want),
                             M, N)
    d = [_dev.to_dev(a) for a in (X, sx, W, sw)]
    dC = _dev.zeros((M, N), np.float32)
    rc = lib().jt_b200_w8a8_gemm(d[0].data_ptr(), K, d[1].data_ptr(), d[2].data_ptr(), K,
                                 d[3].data_ptr(), dC.data_ptr(), N, M, N, K, _dev.stream())
    assert rc == 0 and lib().jt_b200_sync() == 0
    got = _dev.host(dC)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    # tolerance against the reference's fp64 dequant formula (north_star: 1e-3)
    ref64 = acc.astype(np.float64) * (sx.astype(np.float64)[:, None] * sw.astype(np.float64)[None, :])
    err = np.abs(got - ref64).max() / max(np.abs(ref64).max(), 1e-30)
    assert err < 1e-6


def test_pair_kernel_repeat_and_graph_replay():
    """The CTA-pair kernel (cluster launch) stays bit-exact over back-to-back
    launches and over replays of one captured CUDA graph."""
    import torch
    from tests import _dev
    M, N, K = 512, 4096, 1024
    rng = np.random.default_rng(77)
    X = _rand_s8(rng, (M, K))
    W = _rand_s8(rng, (N, K))
    want = np.empty((M, N), np.int32)
    oracle.oracle().jto_gemm_s8(oracle.ptr(X), oracle.ptr(W), oracle.ptr(want), M, N, K)
    dX, dW = _dev.to_dev(X), _dev.to_dev(W)
    dC = _dev.zeros((M, N), np.int32)

    def call():
        return lib().jt_b200_w8a8_gemm_i32(dX.data_ptr(), K, dW.data_ptr(), K, dC.data_ptr(), N,
                                           M, N, K, torch.cuda.current_stream().cuda_stream)
    for _ in range(3):
        dC.zero_()
        assert call() == 0
        assert lib().jt_b200_sync() == 0
        assert np.array_equal(_dev.host(dC), want)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            assert call() == 0
        for _ in range(3):
            dC.zero_()
            g.replay()
            torch.cuda.synchronize()
            assert lib().jt_b200_sync() == 0
            assert np.array_equal(_dev.host(dC), want)
    del g


@pytest.mark.skipif(not oracle.have_ref(), reason="reference library not built")
@pytest.mark.parametrize("M,N,K", [(4, 8, 16), (64, 4096, 1024), (33, 100, 77), (1, 1, 1),
                                   (257, 130, 4096)])
def test_compat_per_channel_matches_reference(M, N, K):
    rng = np.random.default_rng(3000 + M + N + K)
    Aq = _rand_s8(rng, (M, K))
    Bq = _rand_s8(rng, (K, N))
    sA = np.float32(rng.uniform(0.005, 0.02))
    sB = rng.uniform(0.001, 0.01, N).astype(np.float32)
    want = np.full((M, N), 7.0, np.float32)
    got = np.full((M, N), 7.0, np.float32)
    rr = oracle.ref().jt_w8a8_gemm_per_channel(oracle.ptr(Aq), oracle.ptr(Bq), float(sA),
                                               oracle.ptr(sB), oracle.ptr(want), M, N, K)
    rg = lib().jt_w8a8_gemm_per_channel(Aq.ctypes.data, Bq.ctypes.data, float(sA),
                                        sB.ctypes.data, got.ctypes.data, M, N, K)
    assert rr == rg == 0
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.skipif(not oracle.have_ref(), reason="reference library not built")
def test_compat_per_tensor_and_fail_closed():
    rng = np.random.default_rng(7)
    M, N, K = 12, 40, 96
    Aq = _rand_s8(rng, (M, K))
    Bq = _rand_s8(rng, (K, N))
    want = np.zeros((M, N), np.float32)
    got = np.zeros((M, N), np.float32)
    assert oracle.ref().jt_w8a8_gemm_per_tensor(oracle.ptr(Aq), oracle.ptr(Bq), 0.01, 0.003,
                                                oracle.ptr(want), M, N, K) == 0
    assert lib().jt_w8a8_gemm_per_tensor(Aq.ctypes.data, Bq.ctypes.data, 0.01, 0.003,
                                         got.ctypes.data, M, N, K) == 0
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    # -128 in A or B -> INVAL, output untouched (test_w8a8.c:266-270)
    keep = got.copy()
    Abad = Aq.copy()
    Abad[3, 5] = -128
    assert lib().jt_w8a8_gemm_per_tensor(Abad.ctypes.data, Bq.ctypes.data, 0.01, 0.003,
                                         got.ctypes.data, M, N, K) == 2
    Bbad = Bq.copy()
    Bbad[K - 1, N - 1] = -128
    sB = np.full(N, 0.003, np.float32)
    assert lib().jt_w8a8_gemm_per_channel(Aq.ctypes.data, Bbad.ctypes.data, 0.01,
                                          sB.ctypes.data, got.ctypes.data, M, N, K) == 2
    assert np.array_equal(got, keep)


@pytest.mark.skipif(not oracle.have_ref(), reason="reference library not built")
@pytest.mark.parametrize("rows,cols", [(1, 256), (8, 32), (64, 1024), (1, 100003), (3, 5)])
def test_compat_quant_matches_reference(rows, cols):
    rng = np.random.default_rng(rows * 7 + cols)
    x = (rng.standard_normal((rows, cols)) * 3).astype(np.float32)
    x[0, 0] = 0.5 * 3 / 127 * 11  # near-tie style value
    r = oracle.ref()
    if rows == 1:
        qw, qg = np.zeros(cols, np.int8), np.zeros(cols, np.int8)
        sw_, sg_ = np.zeros(1, np.float32), np.zeros(1, np.float32)
        assert r.jt_w8a8_quant_per_tensor(oracle.ptr(x), cols, oracle.ptr(qw), oracle.ptr(sw_)) == 0
        assert lib().jt_w8a8_quant_per_tensor(x.ctypes.data, cols, qg.ctypes.data,
                                              sg_.ctypes.data) == 0
    else:
        qw, qg = np.zeros((rows, cols), np.int8), np.zeros((rows, cols), np.int8)
        sw_, sg_ = np.zeros(rows, np.float32), np.zeros(rows, np.float32)
        assert r.jt_w8a8_quant_per_channel(oracle.ptr(x), rows, cols, oracle.ptr(qw),
                                           oracle.ptr(sw_)) == 0
        assert lib().jt_w8a8_quant_per_channel(x.ctypes.data, rows, cols, qg.ctypes.data,
                                               sg_.ctypes.data) == 0
    assert np.array_equal(qw, qg)
    assert np.array_equal(sw_.view(np.uint32), sg_.view(np.uint32))
    # fake-quant and dequant round trip
    fw, fg = np.zeros_like(x), np.zeros_like(x)
    assert r.jt_w8a8_fakequant_per_channel(oracle.ptr(x), rows, cols, oracle.ptr(fw)) == 0
    assert lib().jt_w8a8_fakequant_per_channel(x.ctypes.data, rows, cols, fg.ctypes.data) == 0
    assert np.array_equal(fw.view(np.uint32), fg.view(np.uint32))
    q = qw.reshape(rows, cols)
    dw, dg = np.zeros_like(x), np.zeros_like(x)
    s = sw_.reshape(-1)
    assert r.jt_w8a8_dequant_per_channel(oracle.ptr(q), oracle.ptr(s), rows, cols,
                                         oracle.ptr(dw)) == 0
    assert lib().jt_w8a8_dequant_per_channel(q.ctypes.data, s.ctypes.data, rows, cols,
                                             dg.ctypes.data) == 0
    assert np.array_equal(dw.view(np.uint32), dg.view(np.uint32))


def test_quant_nan_is_rejected_untouched():
    x = np.array([0.1, 0.2, np.nan, 0.4], np.float32)
    q = np.full(4, 9, np.int8)
    s = np.full(1, 3.0, np.float32)
    assert lib().jt_w8a8_quant_per_tensor(x.ctypes.data, 4, q.ctypes.data, s.ctypes.data) == 2
    assert (q == 9).all() and s[0] == 3.0


@pytest.mark.skipif(not oracle.have_ref(), reason="reference library not built")
@pytest.mark.parametrize("n", [1, 3, 256, 100003, 1 << 20])
def test_compat_per_tensor_dequant_and_fakequant_match_reference(n):
    """jt_w8a8_dequant_per_tensor (w8a8.c:749-785) and
    jt_w8a8_fakequant_per_tensor (w8a8.c:1074-1120) bit for bit against the
    reference library, including a whole-tensor zero input and the
    fail-closed cases (-128 code, non-positive / non-finite scale, NaN input:
    INVAL with the output untouched)."""
    rng = np.random.default_rng(n)
    r = oracle.ref()
    q = _rand_s8(rng, n)
    scale = np.float32(rng.uniform(0.001, 0.05))
    dw, dg = np.zeros(n, np.float32), np.zeros(n, np.float32)
    assert r.jt_w8a8_dequant_per_tensor(oracle.ptr(q), float(scale), n, oracle.ptr(dw)) == 0
    assert lib().jt_w8a8_dequant_per_tensor(q.ctypes.data, float(scale), n, dg.ctypes.data) == 0
    assert np.array_equal(dw.view(np.uint32), dg.view(np.uint32))
    x = (rng.standard_normal(n) * rng.uniform(0.1, 30.0)).astype(np.float32)
    fw, fg = np.zeros(n, np.float32), np.zeros(n, np.float32)
    assert r.jt_w8a8_fakequant_per_tensor(oracle.ptr(x), n, oracle.ptr(fw)) == 0
    assert lib().jt_w8a8_fakequant_per_tensor(x.ctypes.data, n, fg.ctypes.data) == 0
    assert np.array_equal(fw.view(np.uint32), fg.view(np.uint32))
    z = np.zeros(n, np.float32)
    fw[:] = 5.0
    fg[:] = 5.0
    assert r.jt_w8a8_fakequant_per_tensor(oracle.ptr(z), n, oracle.ptr(fw)) == 0
    assert lib().jt_w8a8_fakequant_per_tensor(z.ctypes.data, n, fg.ctypes.data) == 0
    assert np.array_equal(fw.view(np.uint32), fg.view(np.uint32))
    # fail-closed: each rejected call leaves its output as it was
    keep = dg.copy()
    qbad = q.copy()
    qbad[n // 2] = -128
    assert r.jt_w8a8_dequant_per_tensor(oracle.ptr(qbad), float(scale), n, oracle.ptr(dw)) == 2
    assert lib().jt_w8a8_dequant_per_tensor(qbad.ctypes.data, float(scale), n, dg.ctypes.data) == 2
    for bad_scale in (0.0, -1.0, float("inf"), float("nan")):
        assert r.jt_w8a8_dequant_per_tensor(oracle.ptr(q), bad_scale, n, oracle.ptr(dw)) == 2
        assert lib().jt_w8a8_dequant_per_tensor(q.ctypes.data, bad_scale, n, dg.ctypes.data) == 2
    assert np.array_equal(dg, keep)
    xbad = x.copy()
    xbad[n - 1] = np.nan
    keep = fg.copy()
    assert r.jt_w8a8_fakequant_per_tensor(oracle.ptr(xbad), n, oracle.ptr(fw)) == 2
    assert lib().jt_w8a8_fakequant_per_tensor(xbad.ctypes.data, n, fg.ctypes.data) == 2
    assert np.array_equal(fg, keep)


# Projection shapes of a Gated DeltaNet-2 attention layer (gdn2.h: head dims
# dk = dv = 128 by default, at most JT_GDN2_MAX_D = 1024) in front of and
# behind the MoE layer, d_model 1024 / 2048: fused q|k|v|w projection
# (4 x 16 heads x 128), b (erase) keys, per-head decay gates (16 outputs),
# and the output projection back to d_model; decode (M = 1) and prefill rows.
GDN2_SHAPES = [  # (M, N, K)
    (1, 8192, 2048), (1, 16, 2048), (1, 2048, 2048), (1, 1024, 1024),
    (7, 2048, 2048), (4096, 8192, 2048), (4096, 16, 2048), (4096, 2048, 2048),
    (2048, 4096, 1024), (2048, 1024, 1024), (300, 2048, 1024),
]


@pytest.mark.parametrize("M,N,K", GDN2_SHAPES)
def test_gdn2_projection_shapes(M, N, K):
    """The W8A8 GEMM at the attention-projection shapes of the GDN-2 path:
    int32 accumulators and the per-token x per-channel fp32 output bit for
    bit against the oracle."""
    from tests import _dev
    rng = np.random.default_rng(5000 + M + N + K)
    X = _rand_s8(rng, (M, K))
    W = _rand_s8(rng, (N, K))
    sx = rng.uniform(0.005, 0.02, M).astype(np.float32)
    sw = rng.uniform(0.001, 0.01, N).astype(np.float32)
    acc = np.empty((M, N), np.int32)
    want = np.empty((M, N), np.float32)
    o = oracle.oracle()
    o.jto_gemm_s8(oracle.ptr(X), oracle.ptr(W), oracle.ptr(acc), M, N, K)
    o.jto_w8a8_token_channel(oracle.ptr(acc), oracle.ptr(sx), oracle.ptr(sw), oracle.ptr(want), M, N)
    d = [_dev.to_dev(a) for a in (X, sx, W, sw)]
    dC = _dev.zeros((M, N), np.float32)
    dI = _dev.zeros((M, N), np.int32)
    assert lib().jt_b200_w8a8_gemm(d[0].data_ptr(), K, d[1].data_ptr(), d[2].data_ptr(), K,
                                   d[3].data_ptr(), dC.data_ptr(), N, M, N, K, _dev.stream()) == 0
    assert lib().jt_b200_w8a8_gemm_i32(d[0].data_ptr(), K, d[2].data_ptr(), K, dI.data_ptr(), N,
                                       M, N, K, _dev.stream()) == 0
    assert lib().jt_b200_sync() == 0
    assert np.array_equal(_dev.host(dI), acc)
    assert np.array_equal(_dev.host(dC).view(np.uint32), want.view(np.uint32))
