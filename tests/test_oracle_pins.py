"""Pins the CPU oracle (oracle/jt_oracle.c) to the reference.

Three kinds of evidence, all on the CPU:
  * the known-answer cases of the reference's own tests
    (bench/kernel/test_routing.c:28-189, test_moe_layer.c:668-728,
    test_lowbit.c:78-98 and :215-228, test_w8a8.c:78-104), applied to the
    oracle;
  * golden fixtures produced by the reference library
    (tests/golden/make_golden.py), reproduced bit for bit;
  * live comparisons against the reference library compiled from its own
    sources (oracle/_ref), on seeded random inputs, when it was built.
"""
import ctypes as C
import math
import os

import numpy as np
import pytest

import oracle

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
P = oracle.ptr


def topk(logits, k, bias=None):
    logits = np.ascontiguousarray(np.atleast_2d(logits).astype(np.float32))
    T, E = logits.shape
    ids = np.zeros((T, k), np.int32)
    w = np.zeros((T, k), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    rc = oracle.oracle().jto_route_topk(P(logits), None if b is None else P(b), T, E, k, P(ids), P(w))
    return rc, ids, w


def batch_sort(ids, T, k, E, cap):
    flat = np.ascontiguousarray(np.asarray(ids, np.int32).reshape(-1))
    perm = np.full(T * k, -7, np.int32)
    off = np.zeros(E + 1, np.int32)
    drop = np.full(T * k, 9, np.uint8)
    kept = C.c_int(0)
    rc = oracle.oracle().jto_batch_sort(P(flat), T, k, E, cap, P(perm), P(off), P(drop), C.addressof(kept))
    return rc, perm[:kept.value], off, drop, kept.value


# ---------------------------------------------------------------- known answers

def test_topk_known_answers():
    lg = [0.1, 2.0, 0.5, 3.0, 1.0]
    rc, ids, w = topk(lg, 2)
    assert rc == 0 and list(ids[0]) == [3, 1]
    assert abs(w[0, 0] - 0.7310586) <= 1e-5 and abs(w[0, 1] - 0.2689414) <= 1e-5
    assert abs(w[0].sum() - 1.0) <= 1e-6
    rc, ids, w = topk(lg, 1)
    assert rc == 0 and ids[0, 0] == 3 and abs(w[0, 0] - 1.0) <= 1e-6
    rc, ids, w = topk(lg, 5)
    assert rc == 0 and list(ids[0]) == [3, 1, 4, 2, 0] and abs(w[0].sum() - 1.0) <= 1e-6
    rc, ids, w = topk([1.0, 1.0, 1.0], 2)  # ties go to the lowest index
    assert rc == 0 and list(ids[0]) == [0, 1] and np.allclose(w[0], 0.5, atol=1e-6)


def test_topk_nonfinite_and_masks():
    assert topk([1.0, float("nan"), 0.5, 0.25], 2)[0] != 0
    rc, ids, w = topk([2.0, 1.0, -math.inf, -math.inf], 2)
    assert rc == 0 and list(ids[0]) == [0, 1] and abs(w[0].sum() - 1.0) <= 1e-6
    assert topk([math.inf, 1.0, 0.0], 2)[0] != 0


def test_topk_large_known_answers():
    rc, ids, w = topk(np.arange(512) % 64, 8)
    assert rc == 0 and ids[0, 0] == 63 and ids[0, 7] == 511
    assert abs(w[0].sum() - 1.0) <= 1e-5 and abs(w[0, 0] - 0.125) <= 1e-6
    rc, ids, w = topk(np.arange(4096) % 256, 16)
    assert rc == 0 and ids[0, 0] == 255 and ids[0, 15] == 4095
    assert abs(float(w[0].astype(np.float64).sum()) - 1.0) < 1e-5


def test_batch_sort_known_answers():
    rc, perm, off, drop, kept = batch_sort([2, 0, 1, 2, 0, 1, 2, 1], 4, 2, 3, 1.0)
    assert rc == 0 and kept == 8
    assert list(perm) == [1, 4, 2, 5, 7, 0, 3, 6] and list(off) == [0, 2, 5, 8]
    assert not drop.any()
    rc, perm, off, drop, kept = batch_sort([0, 0, 0, 0, 0, 1, 1, 1], 4, 2, 2, 1.0)
    assert rc == 0 and kept == 7
    assert list(perm) == [0, 1, 2, 3, 5, 6, 7] and list(off) == [0, 4, 7]
    assert list(drop) == [0, 0, 0, 0, 1, 0, 0, 0]


def test_lowbit_col_known_answer():
    # test_lowbit.c:215-228: column 1..8 at 4 bits has scale 8; codes on the
    # odd grid: li = floor(t*15/2 + 15/2 + 0.5), t = w/8
    col = np.arange(1, 9, dtype=np.float32)[None, :]
    packed = np.zeros(4, np.uint8)
    scales = np.zeros(1, np.uint16)
    assert oracle.oracle().jto_pack_lowbit(P(col), 1, 8, 4, 8, P(packed), P(scales)) == 0
    li = [oracle.oracle().jto_code_at(P(packed), 8, 4, 0, k) for k in range(8)]
    want = [math.floor((v / 8.0) * 7.5 + 7.5 + 0.5) for v in range(1, 9)]
    assert li == want
    assert oracle.oracle().jto_half_to_float(int(scales[0])) == np.float32(np.float16(8.0 / 15.0))


def test_quant_zero_block():
    x = np.zeros((1, 4), np.float32)
    q = np.full((1, 4), 9, np.int8)
    s = np.zeros(1, np.float32)
    assert oracle.oracle().jto_quant_blocks(P(x), 1, 4, 4, P(q), P(s)) == 0
    assert s[0] == 1.0 and not q.any()


# ---------------------------------------------------------------- golden fixtures

def test_golden_routing_and_sort():
    g = np.load(os.path.join(GOLD, "routing_sort.npz"))
    T, E, k = int(g["T"]), int(g["E"]), int(g["k"])
    rc, ids, w = topk(g["logits"], k, bias=g["bias"])
    assert rc == 0
    assert np.array_equal(ids, g["ids"])
    assert np.array_equal(w.view(np.uint32), g["w"].view(np.uint32))
    for tag, cap in (("c100", 1.0), ("c125", 1.25)):
        rc, perm, off, drop, kept = batch_sort(g["ids"], T, k, E, cap)
        assert rc == 0 and kept == int(g[f"kept_{tag}"])
        assert np.array_equal(perm, g[f"perm_{tag}"])
        assert np.array_equal(off, g[f"off_{tag}"])
        assert np.array_equal(drop, g[f"drop_{tag}"])


def test_golden_quant():
    g = np.load(os.path.join(GOLD, "quant.npz"))
    x = g["x"]
    rows, cols = x.shape
    q = np.zeros_like(g["q_pc"])
    s = np.zeros(rows, np.float32)
    assert oracle.oracle().jto_quant_blocks(P(x), rows, cols, cols, P(q), P(s)) == 0
    assert np.array_equal(q, g["q_pc"])
    assert np.array_equal(s.view(np.uint32), g["s_pc"].view(np.uint32))
    qt = np.zeros_like(g["q_pt"])
    st = np.zeros(1, np.float32)
    flat = np.ascontiguousarray(x.reshape(1, -1))
    assert oracle.oracle().jto_quant_blocks(P(flat), 1, rows * cols, rows * cols, P(qt), P(st)) == 0
    assert np.array_equal(qt, g["q_pt"]) and st[0] == g["s_pt"][0]


def test_golden_w8a8():
    g = np.load(os.path.join(GOLD, "w8a8.npz"))
    A, B = g["A"], g["B"]
    M, K = A.shape
    N = B.shape[1]
    W = np.ascontiguousarray(B.T)
    acc = np.zeros((M, N), np.int32)
    oracle.oracle().jto_gemm_s8(P(A), P(W), P(acc), M, N, K)
    # w8a8.c:664,676-677: C = (float)((double)acc * ((double)sA * (double)sB))
    ss = np.float64(g["sA"][0]) * g["sB"].astype(np.float64)
    C_pc = (acc.astype(np.float64) * ss[None, :]).astype(np.float32)
    assert np.array_equal(C_pc.view(np.uint32), g["C_pc"].view(np.uint32))
    ss_t = np.float64(g["sA"][0]) * np.float64(g["sB_pt"][0])
    C_pt = (acc.astype(np.float64) * ss_t).astype(np.float32)
    assert np.array_equal(C_pt.view(np.uint32), g["C_pt"].view(np.uint32))


@pytest.mark.parametrize("bits", [2, 4])
def test_golden_lowbit_levels(bits):
    # group = K: one scale per row, the reference's whole-column convention
    g = np.load(os.path.join(GOLD, "lowbit.npz"))
    W = g["W"]
    rows, K = W.shape
    packed = np.zeros(rows * K * bits // 8, np.uint8)
    scales = np.zeros(rows, np.uint16)
    assert oracle.oracle().jto_pack_lowbit(P(W), rows, K, bits, K, P(packed), P(scales)) == 0
    li = np.array([[oracle.oracle().jto_code_at(P(packed), K, bits, r, k) for k in range(K)]
                   for r in range(rows)], np.uint8)
    assert np.array_equal(li, g[f"li{bits}"])
    # dequantized value of the reference: (float)(((2li-(n-1))/(n-1)) * maxa)
    n = float((1 << bits) - 1)
    maxa = np.abs(W.astype(np.float64)).max(axis=1)
    fq = (((2.0 * li.astype(np.float64) - n) / n) * maxa[:, None]).astype(np.float32)
    assert np.array_equal(fq.view(np.uint32), g[f"fq{bits}"].view(np.uint32))
    assert np.array_equal(maxa.astype(np.float32), g[f"ws{bits}"])


# ---------------------------------------------------------------- deterministic exp

def test_expf_accuracy():
    x = np.linspace(-87.0, 88.0, 200001, dtype=np.float32)
    got = np.array([oracle.oracle().jto_expf(float(v)) for v in x[::97]], np.float32)
    want = np.exp(x[::97].astype(np.float64))
    rel = np.abs(got.astype(np.float64) - want) / want
    assert rel.max() < 4e-7  # within ~3 ulp of the true value


# ---------------------------------------------------------------- live reference

needs_ref = pytest.mark.skipif(not oracle.have_ref(), reason="oracle/_ref not built")


@needs_ref
@pytest.mark.parametrize("E,k", [(64, 8), (256, 8), (1024, 8), (7, 7)])
def test_live_topk_vs_reference(E, k):
    rng = np.random.default_rng(E * 10 + k)
    T = 64
    lg = rng.standard_normal((T, E)).astype(np.float32)
    lg[3, :] = 1.0
    rc, ids, w = topk(lg, k)
    assert rc == 0
    ref = oracle.ref()
    for t in range(T):
        row = np.ascontiguousarray(lg[t])
        ri = np.zeros(k, np.uint64)
        rw = np.zeros(k, np.float32)
        assert ref.jt_routing_topk(P(row), E, k, P(ri), P(rw)) == 0
        assert np.array_equal(ids[t], ri.astype(np.int32))
        assert np.array_equal(w[t].view(np.uint32), rw.view(np.uint32))


@needs_ref
@pytest.mark.parametrize("T,k,E,cap,s", [(500, 8, 64, 1.0, 1.2), (333, 2, 5, 1.5, 1.1), (64, 1, 3, 1.0, 0.0)])
def test_live_batch_sort_vs_reference(T, k, E, cap, s):
    rng = np.random.default_rng(T + E)
    if s > 0:
        ids = (rng.zipf(1.0 + s, (T, k)) - 1) % E
    else:
        ids = rng.integers(0, E, (T, k))
    ids = ids.astype(np.int32)
    rc, perm, off, drop, kept = batch_sort(ids, T, k, E, cap)
    assert rc == 0
    flat = np.ascontiguousarray(ids.reshape(-1).astype(np.uint64))
    rperm = np.zeros(T * k, np.uint64)
    roff = np.zeros(E + 1, np.uint64)
    rdrop = np.zeros(T * k, np.uint8)
    rk = C.c_size_t(0)
    rd = C.c_size_t(0)
    assert oracle.ref().jt_moe_batch_sort(P(flat), T, k, E, cap, P(rperm), P(roff), P(rdrop),
                                          C.addressof(rk), C.addressof(rd)) == 0
    assert kept == rk.value
    assert np.array_equal(perm, rperm[:kept].astype(np.int32))
    assert np.array_equal(off, roff.astype(np.int32))
    assert np.array_equal(drop, rdrop)


@needs_ref
def test_live_quant_vs_reference():
    rng = np.random.default_rng(7)
    rows, cols = 64, 1024
    x = (rng.standard_normal((rows, cols)) * rng.uniform(1e-3, 30.0, (rows, 1))).astype(np.float32)
    q = np.zeros((rows, cols), np.int8)
    s = np.zeros(rows, np.float32)
    assert oracle.oracle().jto_quant_blocks(P(x), rows, cols, cols, P(q), P(s)) == 0
    rq = np.zeros((rows, cols), np.int8)
    rs = np.zeros(rows, np.float32)
    assert oracle.ref().jt_w8a8_quant_per_channel(P(x), rows, cols, P(rq), P(rs)) == 0
    assert np.array_equal(q, rq) and np.array_equal(s.view(np.uint32), rs.view(np.uint32))


@needs_ref
@pytest.mark.parametrize("T,n,E,k", [(24, 256, 16, 4), (9, 130, 12, 3)])
def test_live_router_logits_vs_reference_layer(T, n, E, k):
    """jto_router_logits (4-lane double dot of moe_layer.c:67-86) feeding the
    pinned top-k gives the reference layer's routing: the same ids, and -
    for tokens without a capacity drop - the same weights bit for bit (a
    one-ulp change of a logit moves its softmax weight).  The sums are kept
    in double and rounded to float once, so another summation order would
    rarely change a logit; the restatement keeps the reference's order all
    the same.  n = 130 runs the scalar tail after the four lanes."""
    rng = np.random.default_rng(T * 7 + n)
    X = rng.standard_normal((T, n)).astype(np.float32)
    Wg8 = (rng.standard_normal((E, n)) * 0.3).astype(np.float32)
    h = 8
    We = [(rng.standard_normal((E, h, n)) * 0.05).astype(np.float32) for _ in range(3)]
    ref = oracle.ref()
    assert ref.jt_w8a8_set_enabled(0) == 0 and ref.jt_lowbit_set_mode(0) == 0
    Y = np.zeros((T, n), np.float32)
    ids = np.zeros(T * k, np.uint64)
    w = np.zeros(T * k, np.float32)
    drop = np.zeros(T * k, np.uint8)
    kept, dropped = C.c_size_t(0), C.c_size_t(0)
    rc = ref.jt_moe_fwd_batch_unchecked(P(X), P(Wg8), P(We[0]), P(We[1]), P(We[2]), None, None, None, P(Y),
                                        T, n, h, E, k, 0, P(ids), P(w), None, None, None, None, None,
                                        1.5, None, None, P(drop), C.addressof(kept),
                                        C.addressof(dropped))
    assert rc == 0
    logits = np.zeros((T, E), np.float32)
    assert oracle.oracle().jto_router_logits(P(X), P(Wg8), T, n, E, P(logits)) == 0
    rc, oids, ow = topk(logits, k)
    assert rc == 0
    assert np.array_equal(oids.reshape(-1).astype(np.uint64), ids)
    nodrop = ~drop.reshape(T, k).any(axis=1)
    assert nodrop.any()
    assert np.array_equal(ow.reshape(T, k)[nodrop].view(np.uint32), w.reshape(T, k)[nodrop].view(np.uint32))


def test_sampled_layer_equals_full_layer():
    """jto_moe_forward_sampled (the oracle form the benchmarked-shape GPU
    tests use) gives, for the rows and tokens it computes, exactly the
    values of jto_moe_forward."""
    from jimotono_b200.moe import WEIGHT_FIELDS, Dims, synth_inputs, synth_weights
    dm = Dims(96, 256, 128, 8, 4, 2, 256, 1.0)
    w = synth_weights(dm, seed=11)
    w = {n: np.ascontiguousarray(a.view(np.uint16) if a.dtype == np.float16 else a) for n, a in w.items()}
    x, logits, bias = synth_inputs(dm, dm.T, seed=12, zipf_s=1.1)
    od = oracle.MoeDims(dm.T, dm.d, dm.f, dm.E, dm.k, dm.S, dm.fs, dm.cap_factor)
    ow = oracle.MoeWeights(*[w[n].ctypes.data for n in WEIGHT_FIELDS])
    Tk = dm.T * dm.k
    full = {"ids": np.zeros(Tk, np.int32), "w": np.zeros(Tk, np.float32), "perm": np.zeros(Tk, np.int32),
            "off": np.zeros(dm.E + 1, np.int32), "drop": np.zeros(Tk, np.uint8),
            "xq": np.zeros(dm.T * dm.d, np.int8), "xs": np.zeros(dm.T, np.float32),
            "h": np.zeros(Tk * dm.f, np.uint16)}
    ft = oracle.MoeTrace(*[full[n].ctypes.data for n in ("ids", "w", "perm", "off", "drop", "xq", "xs",
                                                         "h")], None, None, 0)
    y = np.zeros((dm.T, dm.d), np.float32)
    o = oracle.oracle()
    assert o.jto_moe_forward(C.byref(od), C.byref(ow), P(x), P(logits), P(bias), P(y), C.byref(ft)) == 0
    kept = ft.kept
    assert full["drop"].sum() > 0
    samp = {n: np.zeros_like(full[n]) for n in ("ids", "w", "perm", "off", "drop", "xq", "xs")}
    st = oracle.MoeTrace(*[samp[n].ctypes.data for n in ("ids", "w", "perm", "off", "drop", "xq", "xs")],
                         None, None, None, 0)
    rows = np.array([0, 5, kept - 1, kept + 3, 2**31 - 2], np.int32)
    toks = np.array([0, 17, dm.T - 1], np.int32)
    h = np.zeros((len(rows), dm.f), np.uint16)
    ys = np.zeros((len(toks), dm.d), np.float32)
    assert o.jto_moe_forward_sampled(C.byref(od), C.byref(ow), P(x), P(logits), P(bias), P(rows), len(rows),
                                     P(h), P(toks), len(toks), P(ys), C.byref(st)) == 0
    assert st.kept == kept
    for n in ("ids", "w", "off", "drop", "xq", "xs"):
        assert np.array_equal(samp[n], full[n]), n
    assert np.array_equal(samp["perm"][:kept], full["perm"][:kept])
    assert list(rows) == [0, 5, kept - 1, 3, (2**31 - 2) % kept]
    fh = full["h"].reshape(Tk, dm.f)
    assert np.array_equal(h, fh[rows])
    assert np.array_equal(ys.view(np.uint32), y[toks].view(np.uint32))
