"""The prepared MoE layer at the benchmarked shapes against the oracle.

The full CPU restatement of these layers would take from minutes to hours
on one core, so the oracle runs in its sampled form
(jto_moe_forward_sampled), which gives for the rows and tokens it computes
exactly the values of the full form (tests/test_oracle_pins.py checks that):

* in full and bit for bit: routing ids and renormalized weights, the
  capacity sort (perm / off / drop, kept count) and the per-token int8
  codes and scales of the activations;
* on a seeded sample of kept (token, slot) rows, within oracle.h_mismatch's
  tolerance: the bf16 SwiGLU output h of the routed gate/up GEMM, whose
  fp16-weight products the tensor cores sum in fp32 in their own order
  (every element within one bf16 ulp, at most 0.1 % of them differing);
* within tolerance on a seeded sample of tokens: the layer output (routed
  down projection, weighted combine and shared experts), the north_star
  tolerances 1e-3 of the sample's largest magnitude for fp32 output and
  1e-2 for bf16 output.

Cases: configuration 3 in full (T=4096, d=2048, 256 experts of ffn 1024,
two shared experts of ffn 2048, Zipf-skewed routing with drops, bf16 and
fp32 output); configuration 5's per-expert shapes at 1/8 of its size (T=2048,
128 experts of ffn 1536, shared ffn 4096); configuration 5 in full (T=16384,
1024 experts).  Weights are generated on the device with a seeded torch
generator and copied to the host for the oracle.
"""
import ctypes as C

import numpy as np
import pytest

import oracle
from jimotono_b200.moe import (DBG_DROP, DBG_H, DBG_IDS, DBG_META, DBG_OFF, DBG_PERM,
                               DBG_WEIGHTS, DBG_XQ, DBG_XS, WEIGHT_FIELDS, Dims, Plan,
                               synth_weights_dev, zipf_bias)

pytestmark = pytest.mark.gpu

N_ROWS, N_TOK = 48, 12


def _host_weights(dw):
    out = {}
    for n in WEIGHT_FIELDS:
        a = dw[n].cpu().numpy()
        out[n] = np.ascontiguousarray(a.view(np.uint16) if a.dtype == np.float16 else a)
    return out


def oracle_sampled(dm, hw, x, logits, bias, rows, toks):
    T, Tk = dm.T, dm.T * dm.k
    od = oracle.MoeDims(T, dm.d, dm.f, dm.E, dm.k, dm.S, dm.fs, dm.cap_factor)
    ow = oracle.MoeWeights(*[hw[n].ctypes.data for n in WEIGHT_FIELDS])
    tr = {"ids": np.zeros(Tk, np.int32), "w": np.zeros(Tk, np.float32),
          "perm": np.zeros(Tk, np.int32), "off": np.zeros(dm.E + 1, np.int32),
          "drop": np.zeros(Tk, np.uint8), "xq": np.zeros(T * dm.d, np.int8),
          "xs": np.zeros(T, np.float32)}
    ot = oracle.MoeTrace(*[tr[n].ctypes.data for n in ("ids", "w", "perm", "off", "drop", "xq", "xs")],
                         None, None, None, 0)
    rows = np.ascontiguousarray(rows, np.int32).copy()
    toks = np.ascontiguousarray(toks, np.int32)
    h = np.zeros((len(rows), dm.f), np.uint16)
    y = np.zeros((len(toks), dm.d), np.float32)
    rc = oracle.oracle().jto_moe_forward_sampled(
        C.byref(od), C.byref(ow), x.ctypes.data, logits.ctypes.data,
        bias.ctypes.data if bias is not None else None, rows.ctypes.data, len(rows), h.ctypes.data,
        toks.ctypes.data, len(toks), y.ctypes.data, C.byref(ot))
    assert rc == 0
    tr["kept"] = ot.kept
    tr["perm"] = tr["perm"][:ot.kept]
    return tr, rows, h, y


def gpu_forward(torch, dm, wp, dx, dl, db, bf16):
    from jimotono_b200 import lib
    y = torch.zeros((dm.T, dm.d), dtype=torch.bfloat16 if bf16 else torch.float32, device="cuda")
    plan = Plan(dm)
    plan.forward(wp, dx.data_ptr(), dl.data_ptr(), db.data_ptr() if db is not None else None, dm.T,
                 y.data_ptr(), bf16, torch.cuda.current_stream().cuda_stream)
    assert lib().jt_b200_sync() == 0
    Tk = dm.T * dm.k
    kept = int(plan.debug(DBG_META, np.int32, 4)[0])
    got = {"kept": kept, "ids": plan.debug(DBG_IDS, np.int32, Tk),
           "w": plan.debug(DBG_WEIGHTS, np.float32, Tk), "perm": plan.debug(DBG_PERM, np.int32, kept),
           "off": plan.debug(DBG_OFF, np.int32, dm.E + 1), "drop": plan.debug(DBG_DROP, np.uint8, Tk),
           "xq": plan.debug(DBG_XQ, np.int8, dm.T * dm.d), "xs": plan.debug(DBG_XS, np.float32, dm.T),
           "h": plan.debug(DBG_H, np.uint16, kept * dm.f).reshape(kept, dm.f)}
    plan.close()
    return y.float().cpu().numpy(), got


SHAPES = {
    # name: (T, d, f, E, k, S, fs, cap, zipf)
    "cfg3": (4096, 2048, 1024, 256, 8, 2, 2048, 1.5, 1.1),
    "cfg5_eighth": (2048, 2048, 1536, 128, 8, 2, 4096, 1.5, None),
    "cfg5": (16384, 2048, 1536, 1024, 8, 2, 4096, 1.5, None),
}


@pytest.mark.parametrize("name", list(SHAPES))
def test_moe_layer_benchmarked_shape(name):
    import torch
    T, d, f, E, k, S, fs, cap, zipf = SHAPES[name]
    dm = Dims(T, d, f, E, k, S, fs, cap)
    seed = sum(map(ord, name))
    dw, wp = synth_weights_dev(torch, dm, seed)
    hw = _host_weights(dw)
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, d), dtype=np.float32)
    logits = rng.standard_normal((T, E), dtype=np.float32)
    bias = zipf_bias(E, zipf, rng) if zipf is not None else None
    rows = rng.integers(0, 2**31 - 1, N_ROWS)
    toks = np.sort(rng.choice(T, N_TOK, replace=False)).astype(np.int32)
    tr, rows, h_ref, y_ref = oracle_sampled(dm, hw, x, logits, bias, rows, toks)

    dx, dl = torch.from_numpy(x).cuda(), torch.from_numpy(logits).cuda()
    db = torch.from_numpy(bias).cuda() if bias is not None else None
    y_gpu, got = gpu_forward(torch, dm, wp, dx, dl, db, bf16=False)

    kept = tr["kept"]
    assert got["kept"] == kept
    for n in ("ids", "drop", "off", "perm", "xq"):
        assert np.array_equal(got[n], tr[n]), n
    for n in ("w", "xs"):
        assert np.array_equal(got[n].view(np.uint32), tr[n].view(np.uint32)), n
    if zipf is not None:
        assert tr["drop"].sum() > 0  # the skewed case exercises drops and renormalization
    bad = oracle.h_mismatch(got["h"][rows], h_ref)
    assert bad is None, bad
    scale = max(float(np.abs(y_ref).max()), 1e-30)
    err = float(np.abs(y_gpu[toks] - y_ref).max()) / scale
    assert err < oracle.Y_RTOL, err

    if name == "cfg3":  # the configuration's own output type
        y16, _ = gpu_forward(torch, dm, wp, dx, dl, db, bf16=True)
        err16 = float(np.abs(y16[toks] - y_ref).max()) / scale
        assert err16 < 1e-2, err16
    del dw
    torch.cuda.empty_cache()
