"""Quantized MoE layer on the GPU against the oracle restatement.

Bit-exact: routing ids, renormalized weights, perm / off / drop (the
reference's jt_routing_topk + jt_moe_batch_sort semantics), per-token codes
and scales.  Within oracle.h_mismatch's tolerance: the bf16 SwiGLU output h
of every kept (token, slot) row, whose gate/up sums of x * fp16 weight the
tensor cores (batched) or the integer partials (batch-1) form in fp32 in
their own order.  The layer output within the
north_star tolerance 1e-3 of its largest magnitude (the combine also adds
the k slot contributions with fp32 atomics in arbitrary order).
"""
import ctypes as C

import numpy as np
import pytest

import oracle
from jimotono_b200.moe import (DBG_DROP, DBG_H, DBG_IDS, DBG_META, DBG_OFF, DBG_PERM,
                               DBG_WEIGHTS, DBG_XQ, DBG_XS, WEIGHT_FIELDS, Dims, MoeWeights, Plan,
                               synth_inputs, synth_weights)

pytestmark = pytest.mark.gpu


def run_oracle(dm: Dims, w: dict, x, logits, bias):
    T = x.shape[0]
    od = oracle.MoeDims(T, dm.d, dm.f, dm.E, dm.k, dm.S, dm.fs, dm.cap_factor)
    ow = oracle.MoeWeights(*[w[n].ctypes.data for n in WEIGHT_FIELDS])
    Tk = T * dm.k
    tr = {
        "ids": np.zeros(Tk, np.int32), "w": np.zeros(Tk, np.float32),
        "perm": np.zeros(Tk, np.int32), "off": np.zeros(dm.E + 1, np.int32),
        "drop": np.zeros(Tk, np.uint8), "xq": np.zeros(T * dm.d, np.int8),
        "xs": np.zeros(T, np.float32), "h": np.zeros(Tk * dm.f, np.uint16),
        "ypair": np.zeros(Tk * dm.d, np.float32), "yshared": np.zeros(T * dm.d, np.float32),
    }
    ot = oracle.MoeTrace(*[tr[n].ctypes.data for n in ("ids", "w", "perm", "off", "drop", "xq",
                                                       "xs", "h", "ypair", "yshared")], 0)
    y = np.zeros((T, dm.d), np.float32)
    rc = oracle.oracle().jto_moe_forward(C.byref(od), C.byref(ow), x.ctypes.data,
                                         logits.ctypes.data,
                                         bias.ctypes.data if bias is not None else None,
                                         y.ctypes.data, C.byref(ot))
    assert rc == 0
    tr["kept"] = ot.kept
    return y, tr


def run_gpu(dm: Dims, w: dict, x, logits, bias, bf16=False):
    import torch
    from tests import _dev
    T = x.shape[0]
    dw = {n: _dev.to_dev(w[n]) for n in WEIGHT_FIELDS}
    wp = MoeWeights(*[dw[n].data_ptr() for n in WEIGHT_FIELDS])
    dx, dl = _dev.to_dev(x), _dev.to_dev(logits)
    db = _dev.to_dev(bias) if bias is not None else None
    y = torch.zeros((T, dm.d), dtype=torch.bfloat16 if bf16 else torch.float32, device="cuda")
    plan = Plan(dm)
    plan.forward(wp, dx.data_ptr(), dl.data_ptr(), db.data_ptr() if db is not None else None, T,
                 y.data_ptr(), bf16, _dev.stream())
    from jimotono_b200 import lib
    assert lib().jt_b200_sync() == 0
    Tk = T * dm.k
    meta = plan.debug(DBG_META, np.int32, 4)
    kept = int(meta[0])
    got = {
        "ids": plan.debug(DBG_IDS, np.int32, Tk), "w": plan.debug(DBG_WEIGHTS, np.float32, Tk),
        "perm": plan.debug(DBG_PERM, np.int32, kept), "off": plan.debug(DBG_OFF, np.int32, dm.E + 1),
        "drop": plan.debug(DBG_DROP, np.uint8, Tk), "xq": plan.debug(DBG_XQ, np.int8, T * dm.d),
        "xs": plan.debug(DBG_XS, np.float32, T), "h": plan.debug(DBG_H, np.uint16, kept * dm.f),
        "kept": kept,
    }
    yh = y.float().cpu().numpy()
    plan.close()
    return yh, got


CASES = [
    # (T, d, f, E, k, S, fs, cap, zipf)
    (37, 256, 128, 8, 2, 2, 256, 1.5, None),
    (1, 1024, 256, 64, 8, 2, 512, 1.5, None),  # decode shape of the batch-1 configuration
    (200, 128, 128, 4, 2, 0, 0, 1.0, 1.1),     # drops + renormalization, no shared experts
    (300, 512, 384, 16, 4, 1, 128, 1.25, 1.1),
    (130, 2048, 128, 32, 8, 2, 256, 1.5, 1.1),
    # shared gate/up on 256-token CTA-pair tiles: 3 channel tiles, ragged last token tile
    (600, 256, 128, 8, 2, 2, 384, 1.5, None),
    # batch-1 kernels: configuration 5's expert shapes, an odd multiple of 128
    # for d (K parts of 128 bytes), no shared experts with more than 64
    # experts (the pass-based top-k), a routing bias
    (1, 2048, 1536, 128, 8, 2, 4096, 1.5, None),
    (1, 384, 128, 16, 4, 1, 256, 1.0, None),
    (1, 256, 128, 200, 6, 0, 0, 1.5, None),
    (1, 1024, 256, 64, 8, 2, 512, 1.5, 1.1),
]


@pytest.mark.parametrize("T,d,f,E,k,S,fs,cap,zipf", CASES)
def test_moe_layer_matches_oracle(T, d, f, E, k, S, fs, cap, zipf):
    dm = Dims(T, d, f, E, k, S, fs, cap)
    w = synth_weights(dm, seed=T * 31 + d)
    x, logits, bias = synth_inputs(dm, T, seed=T * 7 + E, zipf_s=zipf)
    y_ref, tr = run_oracle(dm, w, x, logits, bias)
    y_gpu, got = run_gpu(dm, w, x, logits, bias)
    kept = tr["kept"]
    assert got["kept"] == kept
    assert np.array_equal(got["ids"], tr["ids"])
    assert np.array_equal(got["drop"], tr["drop"])
    assert np.array_equal(got["off"], tr["off"])
    assert np.array_equal(got["perm"], tr["perm"][:kept])
    assert np.array_equal(got["w"].view(np.uint32), tr["w"].view(np.uint32))
    assert np.array_equal(got["xq"], tr["xq"])
    assert np.array_equal(got["xs"].view(np.uint32), tr["xs"].view(np.uint32))
    bad = oracle.h_mismatch(got["h"], tr["h"][:kept * f])
    assert bad is None, bad
    scale = max(float(np.abs(y_ref).max()), 1e-30)
    err = float(np.abs(y_gpu - y_ref).max()) / scale
    assert err < oracle.Y_RTOL, err
    if zipf is not None and cap == 1.0:
        assert tr["drop"].sum() > 0  # the case exercises drops


def test_moe_bf16_output():
    dm = Dims(64, 256, 128, 8, 2, 2, 128, 1.5)
    w = synth_weights(dm, seed=5)
    x, logits, bias = synth_inputs(dm, 64, seed=6, zipf_s=1.1)
    y_ref, _ = run_oracle(dm, w, x, logits, bias)
    y_gpu, _ = run_gpu(dm, w, x, logits, bias, bf16=True)
    err = float(np.abs(y_gpu - y_ref).max()) / float(np.abs(y_ref).max())
    assert err < 1e-2  # north_star bf16 tolerance


def test_moe_nan_logits_rejected():
    from jimotono_b200 import lib
    dm = Dims(8, 128, 128, 4, 2, 0, 0, 1.5)
    w = synth_weights(dm, seed=1)
    x, logits, _ = synth_inputs(dm, 8, seed=2)
    logits[3, 1] = np.nan
    import torch
    from tests import _dev
    dw = {n: _dev.to_dev(w[n]) for n in WEIGHT_FIELDS}
    wp = MoeWeights(*[dw[n].data_ptr() for n in WEIGHT_FIELDS])
    y = torch.zeros((8, 128), device="cuda")
    plan = Plan(dm)
    dx, dl = _dev.to_dev(x), _dev.to_dev(logits)  # alive until the forward has run
    plan.forward(wp, dx.data_ptr(), dl.data_ptr(), None, 8, y.data_ptr(), False, _dev.stream())
    assert lib().jt_b200_sync() != 0  # kernel-reported routing fault surfaces as JT_ERR_CUDA
    assert lib().jt_b200_sync() == 0  # and is cleared
    plan.close()


def test_moe_routing_matches_reference_golden():
    """Routing and capacity sort of the GPU layer against fixtures produced
    by the reference's jt_routing_topk / jt_moe_batch_sort
    (tests/golden/make_golden.py); weights after renormalization against
    the oracle's restatement of moe_layer.c:1171-1201 applied to them."""
    import os
    g = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "routing_sort.npz"))
    T, E, k = int(g["T"]), int(g["E"]), int(g["k"])
    dm = Dims(T, 128, 128, E, k, 0, 0, 1.25)
    w = synth_weights(dm, seed=3)
    x, _, _ = synth_inputs(dm, T, seed=4)
    y_gpu, got = run_gpu(dm, w, x, np.ascontiguousarray(g["logits"]), np.ascontiguousarray(g["bias"]))
    assert np.array_equal(got["ids"].reshape(T, k), g["ids"])
    assert got["kept"] == int(g["kept_c125"])
    assert np.array_equal(got["perm"], g["perm_c125"])
    assert np.array_equal(got["off"], g["off_c125"])
    assert np.array_equal(got["drop"], g["drop_c125"])
    wr = np.ascontiguousarray(g["w"].reshape(-1).copy())
    drop = np.ascontiguousarray(g["drop_c125"])
    assert oracle.oracle().jto_renorm(wr.ctypes.data, drop.ctypes.data, T, k) == 0
    assert np.array_equal(got["w"].view(np.uint32), wr.view(np.uint32))


@pytest.mark.parametrize("T", [1, 37])
def test_moe_routing_with_negative_infinite_logits(T):
    """Logits of -inf (the router's masking value): the top-k follows the
    reference's passes (routing.c:38-52), including a pass that finds only
    -inf left; the rank-based selection for E <= 64 hands such rows to the
    passes."""
    dm = Dims(T, 128, 128, 16, 4, 1, 128, 1.5)
    w = synth_weights(dm, seed=T + 40)
    x, logits, _ = synth_inputs(dm, T, seed=T + 41)
    rng = np.random.default_rng(T)
    logits[rng.random(logits.shape) < 0.6] = -np.inf
    logits[:, 3] = rng.standard_normal(T).astype(np.float32)  # one finite logit per token at least
    if T > 1:
        logits[0, :] = -np.inf
        logits[0, 5] = 0.25  # a single finite logit: three passes see only -inf
    y_ref, tr = run_oracle(dm, w, x, logits, None)
    y_gpu, got = run_gpu(dm, w, x, logits, None)
    assert np.array_equal(got["ids"], tr["ids"])
    assert np.array_equal(got["w"].view(np.uint32), tr["w"].view(np.uint32))
    assert got["kept"] == tr["kept"]
    assert np.array_equal(got["perm"], tr["perm"][:tr["kept"]])
    scale = max(float(np.abs(y_ref).max()), 1e-30)
    assert float(np.abs(y_gpu - y_ref).max()) / scale < 1e-5
