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
lowbit.c:228-237) is amortized as it would be at full size (the reference
arm).  The single-core baseline uses 64-token calls, so that several timed
trials fit in its time budget; that amortizes the weight preparation over
half as many tokens, which is to the reference's disadvantage.  The
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


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as fh:
            for ln in fh:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def _median_mad(xs):
    xs = sorted(xs)
    med = xs[len(xs) // 2] if len(xs) % 2 else 0.5 * (xs[len(xs) // 2 - 1] + xs[len(xs) // 2])
    dev = sorted(abs(x - med) for x in xs)
    mad = dev[len(dev) // 2] if len(dev) % 2 else 0.5 * (dev[len(dev) // 2 - 1] + dev[len(dev) // 2])
    return med, mad


def trials(T: int, seconds: float, max_trials: int = 11, min_trials: int = 3) -> list:
    """Seconds per call of the sample at T tokens: at least min_trials calls,
    then more until `seconds` have passed or max_trials are done."""
    smp = _Sample()
    smp.call(1, 0)  # pages the weights in, loads libm
    out = []
    t_end = time.perf_counter() + seconds
    while len(out) < max_trials and (len(out) < min_trials or time.perf_counter() < t_end):
        out.append(smp.call(T, 1 + len(out)))
    return out


def cpu_baseline(seconds: float = 60.0, T: int = 64) -> dict | None:
    """One pinned core: the reference layer on the sample (module docstring),
    repeated while `seconds` last (3 to 11 trials), median and MAD of the
    per-call time.  Runs in a child process under taskset so the pinning does
    not touch the caller."""
    if not have_ref():
        return None
    import json
    import subprocess
    import sys
    cores = sorted(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else [0]
    core = cores[-1]
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = ("import json, sys; sys.path.insert(0, %r); from oracle.cpu_baseline import trials; "
            "print(json.dumps(trials(%d, %f)))" % (root, T, seconds))
    cmd = [sys.executable, "-c", code]
    pinned = False
    try:
        res = subprocess.run(["taskset", "-c", str(core)] + cmd, capture_output=True, text=True,
                             timeout=seconds * 4 + 300)
        pinned = res.returncode == 0
    except (OSError, subprocess.TimeoutExpired):
        res = None
    if not pinned:  # no taskset: unpinned child
        res = subprocess.run(cmd, capture_output=True, text=True, timeout=seconds * 4 + 300)
    times = json.loads(res.stdout.strip().splitlines()[-1])
    med, mad = _median_mad(times)
    return {"value": round(T / med, 3), "unit": "tokens/s", "cores": 1, "kind": "reference",
            "trials": len(times), "median_s_per_call": round(med, 3), "mad_s_per_call": round(mad, 3),
            "pinned": f"taskset -c {core}" if pinned else "unpinned", "cpu_model": cpu_model(),
            "host_cores": os.cpu_count(),
            "sample": f"reference jt_moe_fwd_batch_unchecked (LUT routed + W8A8 shared) at "
                      f"d=2048 f=1536 top-8, E=8, S=2 (ffn 1536), {T} tokens/call, 1 thread; "
                      f"{len(times)} trials, value = tokens / median seconds per call"}


def reference_arm(steps: int, warmup: int, metric: str) -> dict:
    """bench.py --impl reference: every host thread runs the sample call
    concurrently; one step = one round of calls."""
    if not have_ref():
        return {"impl": "reference", "unavailable": "oracle/_ref/libjtref.so not built"}
    smp = _Sample()
    cpus = sorted(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else list(range(os.cpu_count()))
    cores = len(cpus)
    T = 128
    smp.call(1, 0)  # warm-up (page in weights, libm)
    times = []
    for s in range(steps):
        errs = []

        def work(i):
            try:
                if hasattr(os, "sched_setaffinity"):  # this thread on its own core
                    os.sched_setaffinity(0, {cpus[i % len(cpus)]})
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
    med, mad = _median_mad(times)
    ms = 1e3 * med
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
                             "kind": "reference", "cpu_model": cpu_model(),
                             "median_ms_per_step": round(ms, 1), "mad_ms_per_step": round(1e3 * mad, 1),
                             "sample": f"{cores} threads (one per core, pinned) x {T}-token calls, "
                                       f"E=8 top-8 d=2048 f=1536; median over {len(times)} steps"},
            "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
