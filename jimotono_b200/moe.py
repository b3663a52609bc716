"""Host-side view of the MoE device API (jt_b200_moe_* in jimotono_b200.h)
plus seeded synthetic inputs in the layouts the kernels consume.

The synthetic generators stand in for the benchmark configurations (there
are no checkpoints): packed INT2/INT4 codes uniform over their levels, fp16
group scales ~U[0.01, 0.05] as the configurations state, int8 shared-expert
weights uniform over [-127, 127] with per-channel scales of the size int8
quantization of N(0, 0.02) weights produces, activations and router logits
~N(0, 1), and for the skewed-routing configuration a per-expert bias
log(Zipf(s) pmf) over a seeded expert permutation.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import check, lib


class MoeDims(C.Structure):
    _fields_ = [("T", C.c_int), ("d", C.c_int), ("f", C.c_int), ("E", C.c_int), ("k", C.c_int),
                ("S", C.c_int), ("fs", C.c_int), ("cap_factor", C.c_float)]


class MoeWeights(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("wg", "wu", "sg", "su", "wd", "sd", "wsg", "wsu", "ssg",
                                          "ssu", "wsd", "ssd")]


WEIGHT_FIELDS = ("wg", "wu", "sg", "su", "wd", "sd", "wsg", "wsu", "ssg", "ssu", "wsd", "ssd")

DBG_IDS, DBG_WEIGHTS, DBG_PERM, DBG_OFF, DBG_DROP, DBG_XQ, DBG_XS, DBG_H = range(8)
DBG_META = 9


@dataclass
class Dims:
    T: int
    d: int
    f: int
    E: int
    k: int
    S: int
    fs: int
    cap_factor: float = 1.5

    def c(self) -> MoeDims:
        return MoeDims(self.T, self.d, self.f, self.E, self.k, self.S, self.fs, self.cap_factor)


def synth_weights(dm: Dims, seed: int) -> dict:
    rng = np.random.default_rng(seed)
    E, d, f, S, fs = dm.E, dm.d, dm.f, dm.S, max(dm.fs, 64)
    w = {
        "wg": rng.integers(0, 256, (E, f, d // 4), dtype=np.uint8),
        "wu": rng.integers(0, 256, (E, f, d // 4), dtype=np.uint8),
        "sg": rng.uniform(0.01, 0.05, (E, d // 64, f)).astype(np.float16),
        "su": rng.uniform(0.01, 0.05, (E, d // 64, f)).astype(np.float16),
        "wd": rng.integers(0, 256, (E, d, f // 2), dtype=np.uint8),
        "sd": rng.uniform(0.01, 0.05, (E, f // 64, d)).astype(np.float16),
        "wsg": rng.integers(-127, 128, (max(S, 1), fs, d), dtype=np.int8),
        "wsu": rng.integers(-127, 128, (max(S, 1), fs, d), dtype=np.int8),
        "ssg": rng.uniform(4e-4, 8e-4, (max(S, 1), fs)).astype(np.float32),
        "ssu": rng.uniform(4e-4, 8e-4, (max(S, 1), fs)).astype(np.float32),
        "wsd": rng.integers(-127, 128, (max(S, 1), d, fs), dtype=np.int8),
        "ssd": rng.uniform(4e-4, 8e-4, (max(S, 1), d)).astype(np.float32),
    }
    return w


def synth_weights_dev(torch, dm: Dims, seed: int):
    """The synth_weights distributions generated on the current CUDA device
    with a seeded torch generator (numpy takes minutes at the largest
    configurations).  Returns ({name: tensor}, MoeWeights of their device
    pointers); fp16 scales are torch.float16 tensors."""
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    E, d, f, S, fs = dm.E, dm.d, dm.f, max(dm.S, 1), max(dm.fs, 64)

    def u8(*shape):
        return torch.randint(0, 256, shape, dtype=torch.uint8, device="cuda", generator=g)

    def s8(*shape):
        return torch.randint(-127, 128, shape, dtype=torch.int8, device="cuda", generator=g)

    def uni(lo, hi, *shape, dtype=torch.float32):
        return (torch.rand(shape, device="cuda", generator=g) * (hi - lo) + lo).to(dtype)

    dw = {
        "wg": u8(E, f, d // 4), "wu": u8(E, f, d // 4),
        "sg": uni(0.01, 0.05, E, d // 64, f, dtype=torch.float16),
        "su": uni(0.01, 0.05, E, d // 64, f, dtype=torch.float16),
        "wd": u8(E, d, f // 2), "sd": uni(0.01, 0.05, E, f // 64, d, dtype=torch.float16),
        "wsg": s8(S, fs, d), "wsu": s8(S, fs, d), "ssg": uni(4e-4, 8e-4, S, fs),
        "ssu": uni(4e-4, 8e-4, S, fs), "wsd": s8(S, d, fs), "ssd": uni(4e-4, 8e-4, S, d),
    }
    return dw, MoeWeights(*[dw[n].data_ptr() for n in WEIGHT_FIELDS])


def zipf_bias(E: int, s: float, rng: np.random.Generator) -> np.ndarray:
    """Per-expert routing bias log(Zipf(s) pmf) over a seeded permutation of
    the experts (the skewed-load configuration)."""
    ranks = rng.permutation(E) + 1
    pmf = 1.0 / ranks.astype(np.float64) ** s
    pmf /= pmf.sum()
    return np.log(pmf).astype(np.float32)


def synth_inputs(dm: Dims, T: int, seed: int, zipf_s: float | None = None):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, dm.d), dtype=np.float32)
    logits = rng.standard_normal((T, dm.E), dtype=np.float32)
    bias = zipf_bias(dm.E, zipf_s, rng) if zipf_s is not None else None
    return x, logits, bias


class Plan:
    """Owns a jt_b200_moe_plan (device workspace of one layer shape)."""

    def __init__(self, dm: Dims):
        self.dm = dm
        self._c = dm.c()
        self.handle = C.c_void_p()
        check(lib().jt_b200_moe_plan_create(C.byref(self._c), C.byref(self.handle)),
              "jt_b200_moe_plan_create")

    def forward(self, wptrs: MoeWeights, x_ptr: int, logits_ptr: int, bias_ptr, T: int,
                y_ptr: int, y_bf16: bool, stream: int) -> None:
        check(lib().jt_b200_moe_forward(self.handle, C.byref(wptrs), x_ptr, logits_ptr,
                                        bias_ptr, T, y_ptr, int(y_bf16), stream),
              "jt_b200_moe_forward")

    def debug(self, what: int, dtype, count: int) -> np.ndarray:
        out = np.empty(count, dtype=dtype)
        if count:
            check(lib().jt_b200_moe_debug_copy(self.handle, what, out.ctypes.data, out.nbytes),
                  "jt_b200_moe_debug_copy")
        return out

    def bytes(self) -> int:
        return lib().jt_b200_moe_plan_bytes(self.handle)

    def close(self) -> None:
        if self.handle:
            lib().jt_b200_moe_plan_destroy(self.handle)
            self.handle = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------------- expert parallel
class EpComm:
    """NCCL communicator of the current CUDA device over `nranks` processes.
    `uid` is the 128-byte id from `EpComm.unique_id()` on one rank."""

    @staticmethod
    def unique_id() -> bytes:
        buf = C.create_string_buffer(128)
        check(lib().jt_b200_ep_unique_id(buf), "jt_b200_ep_unique_id")
        return buf.raw

    def __init__(self, uid: bytes, nranks: int, rank: int):
        assert len(uid) == 128
        self._uid = C.create_string_buffer(uid, 128)
        self.handle = C.c_void_p()
        self.nranks, self.rank = nranks, rank
        check(lib().jt_b200_ep_comm_create(self._uid, nranks, rank, C.byref(self.handle)),
              "jt_b200_ep_comm_create")

    def close(self) -> None:
        if self.handle:
            lib().jt_b200_ep_comm_destroy(self.handle)
            self.handle = C.c_void_p()


class EpPlan:
    """Expert-parallel layer plan: dm.T tokens per rank, dm.E global experts,
    weights of the rank's dm.E / nranks experts."""

    def __init__(self, dm: Dims, comm: EpComm):
        self.dm = dm
        self.comm = comm
        self._c = dm.c()
        self.handle = C.c_void_p()
        check(lib().jt_b200_moe_ep_plan_create(C.byref(self._c), comm.handle, C.byref(self.handle)),
              "jt_b200_moe_ep_plan_create")

    def forward(self, wptrs: MoeWeights, x_ptr: int, logits_ptr: int, bias_ptr, y_ptr: int,
                y_bf16: bool, stream: int) -> None:
        check(lib().jt_b200_moe_ep_forward(self.handle, C.byref(wptrs), x_ptr, logits_ptr, bias_ptr,
                                           y_ptr, int(y_bf16), stream), "jt_b200_moe_ep_forward")

    def debug(self, what: int, dtype, count: int) -> np.ndarray:
        out = np.empty(count, dtype=dtype)
        if count:
            check(lib().jt_b200_moe_ep_debug_copy(self.handle, what, out.ctypes.data, out.nbytes),
                  "jt_b200_moe_ep_debug_copy")
        return out

    def close(self) -> None:
        if self.handle:
            lib().jt_b200_moe_ep_plan_destroy(self.handle)
            self.handle = C.c_void_p()


def ep_layout(cnt: np.ndarray, rank: int, cap: int) -> dict:
    """Host exchange layout of `rank` from the gathered counts cnt [N][E]."""
    N, E = cnt.shape
    El = E // N
    cnt = np.ascontiguousarray(cnt, np.int32)
    out = {"gbase": np.zeros(E, np.int32), "send": np.zeros(N, np.int32),
           "recv": np.zeros(N, np.int32), "own_off": np.zeros(El + 1, np.int32),
           "own_tile_off": np.zeros(El + 1, np.int32), "gather": np.zeros((N, El, 4), np.int32)}
    check(lib().jt_b200_ep_layout(cnt.ctypes.data, N, E, rank, cap, out["gbase"].ctypes.data,
                                  out["send"].ctypes.data, out["recv"].ctypes.data,
                                  out["own_off"].ctypes.data, out["own_tile_off"].ctypes.data,
                                  out["gather"].ctypes.data), "jt_b200_ep_layout")
    return out
