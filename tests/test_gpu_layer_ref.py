"""The reference-signature MoE layer (jt_moe_fwd_batch[_unchecked],
jt_moe_fwd) computed on the GPU against the reference library itself
(oracle/_ref) on the same seeded fp32 weights, in every mode the flags
select: fp32, W8A8, low-bit fake-quant (mode 1) and the T-MAC LUT (mode 2).

Routing ids, weights, perm/off/drop and the logits are compared bit for
bit.  Y and the caches are compared with max-abs-rel 1e-5 (the north-star
fp32 tolerance is 1e-3): the GEMM, quantization and combine arithmetic is
the reference's, and the remaining source of difference is the double
exp() of the SwiGLU (CUDA's vs libm's, both within 1 ulp), which changes
the float result only in rare rounding cases; the test also requires that
almost every element matches exactly."""
import ctypes as C

import numpy as np
import pytest

import oracle
from jimotono_b200 import JT_ERR_INVAL, lib

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not oracle.have_ref(), reason="oracle/_ref not built")]

F32, U64, U8 = np.float32, np.uint64, np.uint8


def _ptr(a):
    return None if a is None else a.ctypes.data


def _weights(rng, T, n, h, E, S):
    X = rng.standard_normal((T, n)).astype(F32)
    Wgate = (rng.standard_normal((E, n)) * 0.3).astype(F32)
    Wg = (rng.standard_normal((E, h, n)) * 0.08).astype(F32)
    Wu = (rng.standard_normal((E, h, n)) * 0.08).astype(F32)
    Wd = (rng.standard_normal((E, h, n)) * 0.08).astype(F32)
    if S:
        Ws = [(rng.standard_normal((S, h, n)) * 0.08).astype(F32) for _ in range(3)]
    else:
        Ws = [None, None, None]
    return X, Wgate, Wg, Wu, Wd, Ws


def _batch(L, args, T, n, h, E, k, S, cf, unchecked=False):
    X, Wgate, Wg, Wu, Wd, Ws = args
    o = dict(Y=np.full((T, n), -3.0, F32), ids=np.zeros(T * k, U64), w=np.zeros(T * k, F32),
             cG=np.zeros(T * k * h, F32), cU=np.zeros(T * k * h, F32), cY=np.zeros(T * k * n, F32),
             cGs=np.zeros(max(T * S * h, 1), F32), cUs=np.zeros(max(T * S * h, 1), F32),
             perm=np.zeros(T * k, U64), off=np.zeros(E + 1, U64), drop=np.full(T * k, 7, U8))
    kept, dropped = C.c_size_t(0), C.c_size_t(0)
    fn = L.jt_moe_fwd_batch_unchecked if unchecked else L.jt_moe_fwd_batch
    o["rc"] = fn(_ptr(X), _ptr(Wgate), _ptr(Wg), _ptr(Wu), _ptr(Wd), _ptr(Ws[0]), _ptr(Ws[1]), _ptr(Ws[2]),
                 _ptr(o["Y"]), T, n, h, E, k, S, _ptr(o["ids"]), _ptr(o["w"]), _ptr(o["cG"]), _ptr(o["cU"]),
                 _ptr(o["cY"]), _ptr(o["cGs"]) if S else None, _ptr(o["cUs"]) if S else None, cf,
                 _ptr(o["perm"]), _ptr(o["off"]), _ptr(o["drop"]), C.addressof(kept), C.addressof(dropped))
    o["kept"], o["dropped"] = kept.value, dropped.value
    return o


def _close(a, b, what, exact_frac=0.999):
    a = np.asarray(a, np.float32).ravel()
    b = np.asarray(b, np.float32).ravel()
    rel = np.max(np.abs(a.astype(np.float64) - b) / np.maximum(np.abs(b), 1e-6)) if a.size else 0.0
    same = np.mean(a.view(np.uint32) == b.view(np.uint32)) if a.size else 1.0
    assert rel <= 1e-5, f"{what}: max rel {rel}"
    assert same >= exact_frac, f"{what}: only {same:.4f} bit-exact"


@pytest.fixture
def modes():
    def set_modes(w8, lb):
        for L in (lib(), oracle.ref()):
            assert L.jt_w8a8_set_enabled(w8) == 0
            assert L.jt_lowbit_set_mode(lb) == 0
    yield set_modes
    set_modes(0, 0)


SHAPES = [  # T, n, h, E, k, S, cap_factor
    (16, 64, 32, 8, 2, 1, 1.0),
    (33, 40, 48, 6, 3, 2, 1.5),
    (1, 64, 64, 4, 2, 0, 1.0),
    (40, 96, 64, 16, 4, 2, 1.25),
]


@pytest.mark.parametrize("mode", ["fp32", "w8a8", "fq", "lut"])
@pytest.mark.parametrize("shape", SHAPES)
def test_fwd_batch_vs_reference(modes, mode, shape):
    T, n, h, E, k, S, cf = shape
    modes(1 if mode == "w8a8" else 0, {"fq": 1, "lut": 2}.get(mode, 0))
    args = _weights(np.random.default_rng(T * 7 + n + h + E), T, n, h, E, S)
    g = _batch(lib(), args, T, n, h, E, k, S, cf)
    r = _batch(oracle.ref(), args, T, n, h, E, k, S, cf)
    assert g["rc"] == r["rc"] == 0
    for key in ("ids", "perm", "off", "drop"):
        assert np.array_equal(g[key][:r["kept"]] if key == "perm" else g[key],
                              r[key][:r["kept"]] if key == "perm" else r[key]), key
    assert (g["kept"], g["dropped"]) == (r["kept"], r["dropped"])
    assert np.array_equal(g["w"].view(np.uint32), r["w"].view(np.uint32))
    _close(g["Y"], r["Y"], "Y")
    for key in ("cG", "cU", "cY") + (("cGs", "cUs") if S else ()):
        _close(g[key], r[key], key)


def test_fwd_batch_unchecked_matches_checked(modes):
    modes(0, 0)
    T, n, h, E, k, S, cf = SHAPES[0]
    args = _weights(np.random.default_rng(5), T, n, h, E, S)
    a = _batch(lib(), args, T, n, h, E, k, S, cf)
    b = _batch(lib(), args, T, n, h, E, k, S, cf, unchecked=True)
    assert a["rc"] == b["rc"] == 0 and np.array_equal(a["Y"], b["Y"])


def test_fwd_batch_fail_closed(modes):
    modes(0, 0)
    T, n, h, E, k, S, cf = SHAPES[0]
    X, Wgate, Wg, Wu, Wd, Ws = _weights(np.random.default_rng(9), T, n, h, E, S)
    bad = Wd.copy()
    bad[3, 1, 2] = np.nan
    o = _batch(lib(), (X, Wgate, Wg, Wu, bad, Ws), T, n, h, E, k, S, cf)
    assert o["rc"] == JT_ERR_INVAL and (o["Y"] == -3.0).all()
    X2 = X.copy()
    X2[0, 0] = np.inf
    o = _batch(lib(), (X2, Wgate, Wg, Wu, Wd, Ws), T, n, h, E, k, S, cf)
    assert o["rc"] == JT_ERR_INVAL and (o["Y"] == -3.0).all()
    assert _batch(lib(), (X, Wgate, Wg, Wu, Wd, Ws), T, n, h, E, k, S, 0.9)["rc"] == JT_ERR_INVAL
    assert _batch(lib(), (X, Wgate, Wg, Wu, Wd, [None] * 3), T, n, h, E, k, S, cf)["rc"] == JT_ERR_INVAL
    assert _batch(lib(), (X, Wgate, Wg, Wu, Wd, Ws), T, n, h, E, E + 1, S, cf)["rc"] == JT_ERR_INVAL


def _tok(L, args, n, h, E, k, S, unchecked=False):
    X, Wgate, Wg, Wu, Wd, Ws = args
    o = dict(Y=np.full(n, -3.0, F32), ids=np.zeros(k, U64), w=np.zeros(k, F32), lg=np.zeros(E, F32),
             cG=np.zeros(k * h, F32), cU=np.zeros(k * h, F32), cY=np.zeros(k * n, F32),
             cGs=np.zeros(max(S * h, 1), F32), cUs=np.zeros(max(S * h, 1), F32))
    fn = L.jt_moe_fwd_unchecked if unchecked else L.jt_moe_fwd
    o["rc"] = fn(_ptr(X), _ptr(Wgate), _ptr(Wg), _ptr(Wu), _ptr(Wd), _ptr(Ws[0]), _ptr(Ws[1]), _ptr(Ws[2]),
                 _ptr(o["Y"]), n, h, E, k, S, _ptr(o["ids"]), _ptr(o["w"]), _ptr(o["lg"]), _ptr(o["cG"]),
                 _ptr(o["cU"]), _ptr(o["cY"]), _ptr(o["cGs"]) if S else None, _ptr(o["cUs"]) if S else None)
    return o


@pytest.mark.parametrize("n,h,E,k,S", [(64, 32, 8, 2, 1), (37, 19, 5, 3, 0), (128, 96, 64, 8, 2)])
def test_fwd_single_token_vs_reference(modes, n, h, E, k, S):
    modes(1, 2)  # the single-token layer ignores the mode flags
    args = _weights(np.random.default_rng(n + h + E), 1, n, h, E, S)
    args = (args[0][0].copy(),) + args[1:]
    g = _tok(lib(), args, n, h, E, k, S)
    r = _tok(oracle.ref(), args, n, h, E, k, S)
    assert g["rc"] == r["rc"] == 0
    assert np.array_equal(g["ids"], r["ids"])
    assert np.array_equal(g["w"].view(np.uint32), r["w"].view(np.uint32))
    assert np.array_equal(g["lg"].view(np.uint32), r["lg"].view(np.uint32))
    _close(g["Y"], r["Y"], "Y", 0.99)
    for key in ("cG", "cU", "cY") + (("cGs", "cUs") if S else ()):
        _close(g[key], r[key], key, 0.99)
    X = args[0].copy()
    X[3] = np.nan
    bad = _tok(lib(), (X,) + args[1:], n, h, E, k, S)
    assert bad["rc"] == JT_ERR_INVAL and (bad["Y"] == -3.0).all()
