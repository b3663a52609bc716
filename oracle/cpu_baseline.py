"""CPU baseline of the MoE layer: the reference's own implementation.

Used only by bench.py (its cpu_baseline object and the `--impl reference`
arm).  It runs the reference library compiled from the reference sources
(oracle/_ref/libjtref.so, `kind: reference`): jt_moe_fwd_batch_unchecked
with jt_lowbit_set_mode(2) (true T-MAC LUT routed experts) and
jt_w8a8_set_enabled(1) (W8A8 shared experts), the reference's quantized
inference path.

The expert-parallel configuration (16384 tokens, 1024 experts, ~39 GB of
fp32 master weights in the reference's API) cannot run in a bounded time on
a CPU, so the sample keeps the configuration's per-expert shapes (model dim
2048, expert ffn 1536, top-8) with 8 experts and 128 tokens per call: every
expert then sees 128 tokens per call, the configuration's average, so the
per-call weight preparation the reference does (moe_layer.c:1301-1397,
lowbit.c:228-237) is amortized as it would be at full size.  The
reference's API forces the shared experts' ffn to equal the routed one
(1536 instead of 4096), which favours the reference.
"""
from __future__ import annotations

import ctypes as C
import os
import threading
import time

import numpy as np

from . import have_ref, ref

N, H, E, K, S = 2048, 1536, 8, 8, 2


class _Sample:
    def __init__(self, seed: int = 0):
        rng = np.random.default_rng(seed)
        sc = np.float32(0.02)
        self.Wgate = (rng.standard_normal((E, N), dtype=np.float32) * sc)
        self.Wg = (rng.standard_normal((E, H, N), dtype=np.float32) * sc)
        self.Wu = (rng.standard_normal((E, H, N), dtype=np.float32) * sc)
        self.Wd = (rng.standard_normal((E, H, N), dtype=np.float32) * sc)
        self.Wgs = (rng.standard_normal((S, H, N), dtype=np.float32) * sc)
        self.Wus = (rng.standard_normal((S, H, N), dtype=np.float32) * sc)
        self.Wds = (rng.standard_normal((S, H, N), dtype=np.float32) * sc)
        r = ref()
        r.jt_lowbit_set_mode(2)
        r.jt_w8a8_set_enabled(1)

    def call(self, T: int, seed: int) -> float:
        rng = np.random.default_rng(seed)
        X = rng.standard_normal((T, N), dtype=np.float32)
        Y = np.zeros((T, N), np.float32)
        ids = np.zeros(T * K, np.uint64)
        w = np.zeros(T * K, np.float32)
        t0 = time.perf_counter()
        rc = ref().jt_moe_fwd_batch_unchecked(
            X.ctypes.data, self.Wgate.ctypes.data, self.Wg.ctypes.data, self.Wu.ctypes.data,
            self.Wd.ctypes.data, self.Wgs.ctypes.data, self.Wus.ctypes.data,
            self.Wds.ctypes.data, Y.ctypes.data, T, N, H, E, K, S, ids.ctypes.data,
            w.ctypes.data, None, None, None, None, None, C.c_float(1.5), None, None, None, None,
            None)
        dt = time.perf_counter() - t0
        if rc != 0:
            raise RuntimeError(f"reference layer returned {rc}")
        return dt


def cpu_baseline(seconds: float = 20.0) -> dict | None:
    """One core: a 128-token call of the sample (see module docstring)."""
    if not have_ref():
        return None
    smp = _Sample()
    T = 128
    dt = smp.call(T, 1)
    return {"value": round(T / dt, 3), "unit": "tokens/s", "cores": 1, "kind": "reference",
            "sample": f"reference jt_moe_fwd_batch_unchecked (LUT routed + W8A8 shared) at "
                      f"d=2048 f=1536 top-8, E=8, S=2 (ffn 1536), {T} tokens/call "
                      f"(128 tokens per expert as in the full config), 1 thread, {dt:.1f} s"}


def reference_arm(steps: int, warmup: int, metric: str) -> dict:
    """bench.py --impl reference: every host thread runs the sample call
    concurrently; one step = one round of calls."""
    if not have_ref():
        return {"impl": "reference", "unavailable": "oracle/_ref/libjtref.so not built"}
    smp = _Sample()
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    T = 128
    smp.call(1, 0)  # warm-up (page in weights, libm)
    times = []
    for s in range(steps):
        errs = []

        def work(i):
            try:
                smp.call(T, 100 * s + i)
            except Exception as e:  # pragma: no cover
                errs.append(e)
        th = [threading.Thread(target=work, args=(i,)) for i in range(cores)]
        t0 = time.perf_counter()
        for t in th:
            t.start()
        for t in th:
            t.join()
        times.append(time.perf_counter() - t0)
        if errs:
            raise errs[0]
    ms = 1e3 * sum(times) / len(times)
    value = cores * T / (ms / 1e3)
    return {"impl": "reference", "metric": metric, "value": round(value, 2), "unit": "tokens/s",
            "n_gpus": 0, "steps": steps, "warmup": warmup, "ms_per_step": round(ms, 1),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32+int8",
            "data": "synthetic",
            "config": {"workload": "cfg5 EP MoE layer: T=16384 d=2048 E=1024 f=1536 top-8 INT2/INT4 g64 + "
                                   "2 shared INT8 f=4096, cap 1.5",
                       "tokens": 16384, "parallelism": "host cores",
                       "measured_on": "a bounded sample of the workload's expert shapes (see cpu_baseline)"},
            "cpu_baseline": {"value": round(value, 2), "unit": "tokens/s", "cores": cores,
                             "kind": "reference",
                             "sample": f"{cores} threads x {T}-token calls, E=8 top-8 d=2048 f=1536"},
            "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
