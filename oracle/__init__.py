"""Parity checker (test infrastructure only).

Loads two CPU libraries with ctypes:
  * oracle/libjtoracle.so - the C restatement (oracle/jt_oracle.c);
  * oracle/_ref/libjtref.so - the reference's own hot-path sources compiled
    unmodified (oracle/Makefile `ref`), present when it was built here.
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use
this package.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_PATH = os.path.join(_HERE, "libjtoracle.so")
REF_PATH = os.path.join(_HERE, "_ref", "libjtref.so")

P, I, SZ, F = C.c_void_p, C.c_int, C.c_size_t, C.c_float

_ORACLE = None
_REF = None


def ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


class MoeDims(C.Structure):
    _fields_ = [("T", I), ("d", I), ("f", I), ("E", I), ("k", I), ("S", I), ("fs", I),
                ("cap_factor", F)]


class MoeWeights(C.Structure):
    _fields_ = [(n, P) for n in ("wg", "wu", "sg", "su", "wd", "sd", "wsg", "wsu", "ssg", "ssu",
                                 "wsd", "ssd")]


class MoeTrace(C.Structure):
    _fields_ = [(n, P) for n in ("ids", "w", "perm", "off", "drop", "xq", "xs", "h",
                                 "ypair", "yshared")] + [("kept", I)]


def oracle() -> C.CDLL:
    global _ORACLE
    if _ORACLE is None:
        h = C.CDLL(ORACLE_PATH, mode=C.RTLD_LOCAL)
        protos = {
            "jto_quant_blocks": (I, [P, I, I, I, P, P]),
            "jto_gemm_s8": (None, [P, P, P, I, I, I]),
            "jto_w8a8_token_channel": (None, [P, P, P, P, I, I]),
            "jto_router_logits": (I, [P, P, I, I, I, P]),
            "jto_route_topk": (I, [P, P, I, I, I, P, P]),
            "jto_batch_sort": (I, [P, I, I, I, F, P, P, P, P]),
            "jto_renorm": (I, [P, P, I, I]),
            "jto_half_to_float": (F, [C.c_uint16]),
            "jto_float_to_half": (C.c_uint16, [F]),
            "jto_bf16_to_float": (F, [C.c_uint16]),
            "jto_float_to_bf16": (C.c_uint16, [F]),
            "jto_pack_lowbit": (I, [P, I, I, I, I, P, P]),
            "jto_code_at": (I, [P, I, I, I, I]),
            "jto_expf": (F, [F]),
            "jto_swiglu": (F, [F, F]),
            "jto_lowbit_gemv": (None, [P, F, P, P, I, I, I, P]),
            "jto_lowbit_partials": (None, [P, P, I, I, I, P]),
            "jto_moe_forward": (I, [C.POINTER(MoeDims), C.POINTER(MoeWeights), P, P, P, P,
                                    C.POINTER(MoeTrace)]),
            "jto_moe_forward_sampled": (I, [C.POINTER(MoeDims), C.POINTER(MoeWeights), P, P, P,
                                            P, I, P, P, I, P, C.POINTER(MoeTrace)]),
        }
        for n, (r, a) in protos.items():
            fn = getattr(h, n)
            fn.restype = r
            fn.argtypes = a
        _ORACLE = h
    return _ORACLE


def have_ref() -> bool:
    return os.path.exists(REF_PATH)


def ref() -> C.CDLL:
    """The reference's own CPU library (compiled from its sources)."""
    global _REF
    if _REF is None:
        h = C.CDLL(REF_PATH, mode=C.RTLD_LOCAL)
        protos = {
            "jt_w8a8_quant_per_tensor": (I, [P, SZ, P, P]),
            "jt_w8a8_quant_per_channel": (I, [P, SZ, SZ, P, P]),
            "jt_w8a8_dequant_per_tensor": (I, [P, F, SZ, P]),
            "jt_w8a8_dequant_per_channel": (I, [P, P, SZ, SZ, P]),
            "jt_w8a8_gemm_per_tensor": (I, [P, P, F, F, P, I, I, I]),
            "jt_w8a8_gemm_per_channel": (I, [P, P, F, P, P, I, I, I]),
            "jt_w8a8_fakequant_per_tensor": (I, [P, SZ, P]),
            "jt_w8a8_fakequant_per_channel": (I, [P, SZ, SZ, P]),
            "jt_w8a8_set_enabled": (I, [I]),
            "jt_routing_topk": (I, [P, SZ, SZ, P, P]),
            "jt_moe_batch_sort": (I, [P, I, I, I, F, P, P, P, P, P]),
            "jt_lowbit_fakequant": (I, [P, P, SZ, I]),
            "jt_lowbit_col_to_idx": (I, [P, SZ, I, P, P]),
            "jt_lowbit_set_mode": (I, [I]),
            "jt_lowbit_gemm_lut": (I, [P, P, P, I, I, I, I]),
            "jt_tmac_lut_ctor": (I, [P, SZ, SZ, P, P, P]),
            "jt_tmac_qlut_bytes": (I, [SZ, SZ, P]),
            "jt_tmac_param_bytes": (I, [SZ, SZ, P]),
            "jt_tmac_lookup_accum": (I, [P, P, P, P, SZ, SZ, I, F, P]),
            "jt_gemm_mat_f32": (I, [P, P, P, I, I, I]),
            "jt_transpose_f32": (I, [P, P, I, I]),
            "jt_moe_fwd_batch": (I, [P] * 9 + [I] * 6 + [P] * 7 + [F] + [P] * 5),
            "jt_moe_fwd_batch_unchecked": (I, [P] * 9 + [I] * 6 + [P] * 7 + [F] + [P] * 5),
            "jt_moe_fwd": (I, [P] * 9 + [I] * 5 + [P] * 8),
        }
        for n, (r, a) in protos.items():
            fn = getattr(h, n)
            fn.restype = r
            fn.argtypes = a
        _REF = h
    return _REF


# Tolerances of the routed SwiGLU output h (bf16) against this restatement.
# The CUDA path accumulates x * fp16_rn(code * scale) in fp32 on the tensor
# cores (order chosen by the hardware), the restatement in double, so g and u
# agree to a few fp32 ulps and bf16(h) agrees except where h lies within that
# distance of a bf16 rounding tie: then the two differ by one bf16 ulp.
H_FLIP_FRAC = 1e-3
# The layer output: the north_star fp32 tolerance, relative to max |y|.
Y_RTOL = 1e-3


def bf16_to_f32(bits) -> np.ndarray:
    b = np.asarray(bits).astype(np.uint16).astype(np.uint32) << 16
    return b.view(np.float32)


def h_mismatch(h_got, h_want) -> str | None:
    """None when the routed h (bf16 bits) agrees within the tolerance above:
    every element within one bf16 ulp of the restatement's and at most
    H_FLIP_FRAC of them differing at all; else a one-line description."""
    g = np.asarray(h_got).astype(np.uint16).ravel()
    w = np.asarray(h_want).astype(np.uint16).ravel()
    if g.shape != w.shape:
        return "shape differs"
    if g.size == 0:
        return None
    gf, wf = bf16_to_f32(g).astype(np.float64), bf16_to_f32(w).astype(np.float64)
    if not np.all(np.isfinite(gf)):
        return "non-finite h"
    # one bf16 ulp at the larger magnitude of the pair (8 significant bits)
    mag = np.maximum(np.abs(gf), np.abs(wf))
    ulp = np.where(mag > 0, np.exp2(np.floor(np.log2(np.maximum(mag, 1e-38))) - 7), 0.0)
    d = np.abs(gf - wf)
    big = float((d / np.maximum(ulp, 1e-45)).max())
    frac = float((g != w).mean())
    if big > 1.0 + 1e-9 or frac > H_FLIP_FRAC:
        return f"h max diff {big:.3g} bf16 ulp, differing elements {frac:.3g}"
    return None
