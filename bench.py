"""Benchmark of the B200 quantized-MoE hot path (one JSON line on rank 0).

Headline (`value`): MoE-layer tokens/s of the expert-parallel configuration
(T=16384 tokens, d=2048, 1024 routed experts of ffn 1536
top-8 with INT2 gate/up + INT4 down group-64, 2 shared INT8 experts of ffn
4096) on N GPUs, device-resident inputs, whole-job throughput.  `parts`
adds the other configurations' metrics on GPU 0: W8A8 TOPS (config 1),
batch-1 decode HBM GB/s (config 2), prefill tokens/s (config 3).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

N > 1 runs under torchrun, one rank per GPU: the expert-parallel layer
(E/N experts and T/N tokens per rank, NCCL send/recv dispatch and combine),
timed with CUDA events, the max over ranks.

`e2e` is the same metric through the public API with host buffers: every
step copies its inputs from pinned host memory and its output back, the
copies on their own streams overlapping the neighbouring steps' compute.

`--impl reference` times the reference's own CPU implementation
(oracle/_ref, the reference sources compiled unmodified) on the host cores.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CFG5 = dict(T=16384, d=2048, f=1536, E=1024, k=8, S=2, fs=4096, cap=1.5)
CFG3 = dict(T=4096, d=2048, f=1024, E=256, k=8, S=2, fs=2048, cap=1.5)
CFG2 = dict(T=1, d=1024, f=256, E=64, k=8, S=2, fs=512, cap=1.5)
# 1/8 of config 5 (same rows per expert, same shapes per expert): the case the
# profiler captures run on (`--small`), whose DRAM traffic scales by 8 to a
# full config-5 launch.
# rotating weight copies of the batch-1 timing (each forward touches 5.46 MB)
DEC_ROT = 48
CFG5_SMALL = dict(T=2048, d=2048, f=1536, E=128, k=8, S=2, fs=4096, cap=1.5)
METRIC = "MoE-layer tokens/s at 1/2/4/8 B200; W8A8 TOPS; decode HBM GB/s vs peak"
# DRAM bytes (read + write) of one routed gate/up launch at config 5: the ncu
# capture of `bench.py --small` (1/8 of config 5) gave 294.3 + 43.0 MB, scaled by 8.
GU_TRAFFIC_BYTES = 8 * 337_319_680


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            p = json.load(fh)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def tensor_peak():
    """Dense bf16/fp16 tensor-core peak (TFLOP/s) for the kind::f16 expert
    GEMMs: the measured cuBLAS bf16 burst figure (a kernel of a few ms timed
    inside a forward of a few ms, not a seconds-long loop)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            return float(json.load(fh)["bf16_tflops"]), "measured (cuBLAS bf16 burst)"
    except Exception:
        return 1590.0, "fallback"


# ----------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None

    def __enter__(self):
        self.first = []
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        # nvidia-smi takes a moment to start: wait (at most 5 s) for its first
        # sample so that the sampling covers the whole timed work that follows
        if self.proc is not None:
            import select
            ready, _, _ = select.select([self.proc.stdout], [], [], 5.0)
            if ready:
                self.first.append(self.proc.stdout.readline())
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in self.first + out.splitlines() if ln.strip()]

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for name, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------- device helpers
def dev_weights(torch, w: dict):
    from jimotono_b200.moe import WEIGHT_FIELDS, MoeWeights
    dw = {}
    for n in WEIGHT_FIELDS:
        a = w[n]
        if a.dtype == np.float16:
            a = a.view(np.int16)
        dw[n] = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return dw, MoeWeights(*[dw[n].data_ptr() for n in WEIGHT_FIELDS])


def synth_weights_dev(torch, dm, seed):
    from jimotono_b200.moe import synth_weights_dev as gen
    return gen(torch, dm, seed)


def weight_bytes(dm) -> int:
    routed = dm.E * (2 * dm.f * (dm.d // 4 + dm.d // 64 * 2) + dm.d * (dm.f // 2 + dm.f // 64 * 2))
    shared = dm.S * (2 * dm.fs * (dm.d + 4) + dm.d * (dm.fs + 4))
    return routed + shared


# ----------------------------------------------------------------- MoE layer timing
def time_layer(torch, cfg, rank, world, steps, warmup, seed, zipf=None, bf16=False, nrot=1,
               profile=True):
    from jimotono_b200 import lib
    from jimotono_b200.moe import Dims, Plan
    T = cfg["T"] // world if world > 1 else cfg["T"]
    dm = Dims(T, cfg["d"], cfg["f"], cfg["E"], cfg["k"], cfg["S"], cfg["fs"], cfg["cap"])
    rots = [synth_weights_dev(torch, dm, seed + 17 * r) for r in range(nrot)]
    g = torch.Generator(device="cuda")
    g.manual_seed(seed + 1000 * rank)
    x = torch.randn((T, dm.d), device="cuda", generator=g)
    logits = torch.randn((T, dm.E), device="cuda", generator=g)
    bias = None
    if zipf is not None:
        from jimotono_b200.moe import zipf_bias
        bias = torch.from_numpy(zipf_bias(dm.E, zipf, np.random.default_rng(seed))).cuda()
    y = torch.empty((T, dm.d), dtype=torch.bfloat16 if bf16 else torch.float32, device="cuda")
    plan = Plan(dm)
    stream = torch.cuda.current_stream().cuda_stream
    bp = bias.data_ptr() if bias is not None else None

    def step(i):
        plan.forward(rots[i % nrot][1], x.data_ptr(), logits.data_ptr(), bp, T, y.data_ptr(),
                     bf16, stream)

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    if lib().jt_b200_sync() != 0:
        raise RuntimeError("kernel fault during warm-up")
    if profile:
        assert lib().jt_b200_moe_profile_begin(plan.handle, steps) == 0
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        step(i)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    stage = None
    if profile:
        arr = (C.c_float * 7)()
        nsteps = C.c_int(0)
        assert lib().jt_b200_moe_profile_end(plan.handle, arr, 7, C.byref(nsteps)) == 0
        stage = [v / max(nsteps.value, 1) for v in arr]
    if lib().jt_b200_sync() != 0:
        raise RuntimeError("kernel fault during the timed region")
    meta = plan.debug(9, np.int32, 4)
    out = dict(T=T, ms_per_step=ms / steps, stage_ms=stage, kept=int(meta[0]), dims=dm, plan=plan,
               x=x, logits=logits, y=y, rots=rots, bias=bias, bf16=bf16)
    if nrot > 1:  # a token and router logits of its own for every weight copy
        out["x_rot"] = [torch.randn((T, dm.d), device="cuda", generator=g) for _ in range(nrot)]
        out["logits_rot"] = [torch.randn((T, dm.E), device="cuda", generator=g) for _ in range(nrot)]
    return out


def time_decode_graph(torch, st, reps=50, warm=False):
    """Batch-1 forwards captured in a CUDA graph and replayed: per-token
    device time without host launch overhead, microseconds per token.

    L2-cold (default): one forward per rotating weight copy, each with its
    own token and router logits (so each picks its own experts); the copies
    touch nrot x 5.46 MB, several times the 126 MB L2, so every forward
    streams its weights from HBM.  warm=True replays the first copy with
    the first token only (the same 5.46 MB every time, resident in L2)."""
    from jimotono_b200 import lib
    plan, rots, y = st["plan"], st["rots"], st["y"]
    xs, ls = st["x_rot"], st["logits_rot"]
    per_graph = len(rots)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for i in range(per_graph):
            j = 0 if warm else i
            plan.forward(rots[j][1], xs[j].data_ptr(), ls[j].data_ptr(), None, 1, y.data_ptr(), st["bf16"],
                         s.cuda_stream)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            cs = torch.cuda.current_stream().cuda_stream
            for i in range(per_graph):
                j = 0 if warm else i
                plan.forward(rots[j][1], xs[j].data_ptr(), ls[j].data_ptr(), None, 1, y.data_ptr(), st["bf16"], cs)
        for _ in range(5):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(reps):
            g.replay()
        e1.record(s)
        torch.cuda.synchronize()
    if lib().jt_b200_sync() != 0:
        raise RuntimeError("kernel fault in the decode graph")
    us = e0.elapsed_time(e1) / (reps * per_graph) * 1e3
    del g
    return us


def time_layer_ep(torch, cfg, rank, world, steps, warmup, seed):
    """Expert-parallel config 5 on `world` ranks: rank r owns tokens
    [r*T/N, (r+1)*T/N) and routed experts [r*E/N, (r+1)*E/N) (its weight
    shard generated on its GPU), shared experts replicated; dispatch and
    combine over NCCL inside every step."""
    from jimotono_b200 import lib
    from jimotono_b200.moe import Dims, EpComm, EpPlan
    T = cfg["T"] // world
    El = cfg["E"] // world
    dm_w = Dims(T, cfg["d"], cfg["f"], El, cfg["k"], cfg["S"], cfg["fs"], cfg["cap"])
    dw, wp = synth_weights_dev(torch, dm_w, seed + 101 * rank)
    dm = Dims(T, cfg["d"], cfg["f"], cfg["E"], cfg["k"], cfg["S"], cfg["fs"], cfg["cap"])
    g = torch.Generator(device="cuda")
    g.manual_seed(seed + 1000 * rank)
    x = torch.randn((T, dm.d), device="cuda", generator=g)
    logits = torch.randn((T, dm.E), device="cuda", generator=g)
    y = torch.empty((T, dm.d), device="cuda")
    uid = [EpComm.unique_id() if rank == 0 else None]
    torch.distributed.broadcast_object_list(uid, src=0)
    comm = EpComm(uid[0], world, rank)
    plan = EpPlan(dm, comm)
    stream = torch.cuda.current_stream().cuda_stream

    def step():
        plan.forward(wp, x.data_ptr(), logits.data_ptr(), None, y.data_ptr(), False, stream)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if lib().jt_b200_sync() != 0:
        raise RuntimeError("kernel fault during warm-up")
    torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    if lib().jt_b200_sync() != 0:
        raise RuntimeError("kernel fault during the timed region")
    meta = plan.debug(9, np.int32, 4)
    # end to end: pinned host x / logits in, y out, every step (pipelined
    # copies, e2e_pipelined); every rank starts its timed region together
    hx = x.cpu().pin_memory()
    hl = logits.cpu().pin_memory()

    def fwd(dx, dl, yy, stream):
        plan.forward(wp, dx.data_ptr(), dl.data_ptr(), None, yy.data_ptr(), False, stream)

    torch.distributed.barrier()
    e2e_ms, h2d, d2h = e2e_pipelined(torch, hx, hl, y, fwd, max(8, 2 * steps), 2)
    out = dict(T=T, ms_per_step=ms, e2e_ms=e2e_ms, h2d=h2d, d2h=d2h, kept_local=int(meta[0]),
               owned_rows=int(meta[1]), dims=dm)
    plan.close()
    comm.close()
    del dw
    return out


def e2e_pipelined(torch, hx, hl, y_like, forward, steps, warmup):
    """End to end through the public API with host buffers, as a serving
    loop runs it: every step copies its inputs (x, router logits) from
    pinned host memory, runs the forward and copies its output back.  The
    copies go on their own streams into double-buffered device buffers, so
    step i+1's inputs and step i-1's output cross PCIe while step i
    computes; every step's copies are inside the timed region, which ends
    when the last output has reached host memory, so the first step's input
    copy and the last step's output copy (together about 6 ms at config 5)
    are paid once per run: the run is long enough (twice the device-timed
    steps) for them to amortize as in a serving loop.  forward(dx, dl, y,
    stream) enqueues one forward on `stream`."""
    cs = torch.cuda.current_stream()
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    dx = [torch.empty(hx.shape, dtype=hx.dtype, device="cuda") for _ in range(2)]
    dl = [torch.empty(hl.shape, dtype=hl.dtype, device="cuda") for _ in range(2)]
    ys = [torch.empty_like(y_like) for _ in range(2)]
    hy = [torch.empty(y_like.shape, dtype=y_like.dtype, device="cpu").pin_memory() for _ in range(2)]
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_comp = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def step(i):
        b = i & 1
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_comp[b])  # step i-2 has consumed buffer b
            dx[b].copy_(hx, non_blocking=True)
            dl[b].copy_(hl, non_blocking=True)
            ev_in[b].record(s_in)
        cs.wait_event(ev_in[b])
        cs.wait_event(ev_out[b])  # step i-2's output has left buffer b
        forward(dx[b], dl[b], ys[b], cs.cuda_stream)
        ev_comp[b].record(cs)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_comp[b])
            hy[b].copy_(ys[b], non_blocking=True)
            ev_out[b].record(s_out)

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cs)
    s_in.wait_event(e0)
    s_out.wait_event(e0)
    for i in range(warmup, warmup + steps):
        step(i)
    cs.wait_event(ev_out[(warmup + steps - 1) & 1])
    e1.record(cs)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    h2d = hx.numel() * hx.element_size() + hl.numel() * hl.element_size()
    d2h = hy[0].numel() * hy[0].element_size()
    return ms, h2d, d2h


def e2e_layer(torch, st, steps, warmup):
    """The single-GPU layer end to end (e2e_pipelined)."""
    plan = st["plan"]
    T = st["T"]
    hx = st["x"].cpu().pin_memory()
    hl = st["logits"].cpu().pin_memory()
    bp = st["bias"].data_ptr() if st["bias"] is not None else None
    wp = st["rots"][0][1]

    def fwd(dx, dl, y, stream):
        plan.forward(wp, dx.data_ptr(), dl.data_ptr(), bp, T, y.data_ptr(), st["bf16"], stream)

    return e2e_pipelined(torch, hx, hl, st["y"], fwd, steps, warmup)


# ----------------------------------------------------------------- parts
def part_w8a8(torch, steps=200):
    from jimotono_b200 import lib
    L = lib()
    stream = torch.cuda.current_stream().cuda_stream
    res = {}
    for (M, N, K, rot) in [(64, 4096, 1024, 32), (4096, 4096, 4096, 4)]:
        bufs = []
        for _ in range(rot):
            X = torch.randint(-127, 128, (M, K), dtype=torch.int8, device="cuda")
            W = torch.randint(-127, 128, (N, K), dtype=torch.int8, device="cuda")
            sx = torch.rand(M, device="cuda") * 0.015 + 0.005
            sw = torch.rand(N, device="cuda") * 0.009 + 0.001
            Cm = torch.empty((M, N), device="cuda")
            bufs.append((X, W, sx, sw, Cm))

        def call(b):
            X, W, sx, sw, Cm = b
            return L.jt_b200_w8a8_gemm(X.data_ptr(), K, sx.data_ptr(), W.data_ptr(), K,
                                       sw.data_ptr(), Cm.data_ptr(), N, M, N, K, stream)
        for i in range(10):
            call(bufs[i % rot])
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(steps):
            call(bufs[i % rot])
        e1.record()
        torch.cuda.synchronize()
        assert L.jt_b200_sync() == 0
        us = e0.elapsed_time(e1) / steps * 1e3
        # the same calls captured in a CUDA graph: device time without the
        # per-call host work (ctypes, tensor-map encoding, launch)
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            cs = s.cuda_stream
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                for i in range(rot):
                    X, W, sx, sw, Cm = bufs[i]
                    L.jt_b200_w8a8_gemm(X.data_ptr(), K, sx.data_ptr(), W.data_ptr(), K, sw.data_ptr(),
                                        Cm.data_ptr(), N, M, N, K, torch.cuda.current_stream().cuda_stream)
            for _ in range(3):
                g.replay()
            torch.cuda.synchronize()
            reps = max(1, steps // rot)
            e0.record(s)
            for _ in range(reps):
                g.replay()
            e1.record(s)
            torch.cuda.synchronize()
        us_g = e0.elapsed_time(e1) / (reps * rot) * 1e3
        del g
        assert L.jt_b200_sync() == 0
        byts = M * K + N * K + 4 * M * N + 4 * (M + N)
        res[f"{M}x{N}x{K}"] = {"us": round(us, 3), "TOPS": round(2 * M * N * K / us / 1e6, 2),
                               "GBs": round(byts / us / 1e3, 1), "us_graph": round(us_g, 3),
                               "TOPS_graph": round(2 * M * N * K / us_g / 1e6, 2),
                               "frac_of_nominal_int8": round(2 * M * N * K / us / 1e6 / 4500.0, 4)}
        if M == 4096:
            # the same GEMM with int32 output, ours and cuBLASLt's (torch._int_mm),
            # as a measured int8 tensor-core comparator on this GPU
            Ci = torch.empty((M, N), dtype=torch.int32, device="cuda")

            def t_ev(fn, n):
                for i in range(5):
                    fn(i)
                torch.cuda.synchronize()
                e0.record()
                for i in range(n):
                    fn(i)
                e1.record()
                torch.cuda.synchronize()
                return e0.elapsed_time(e1) / n * 1e3

            us_i32 = t_ev(lambda i: L.jt_b200_w8a8_gemm_i32(
                bufs[i % rot][0].data_ptr(), K, bufs[i % rot][1].data_ptr(), K, Ci.data_ptr(), N,
                M, N, K, stream), steps)
            assert L.jt_b200_sync() == 0
            res[f"{M}x{N}x{K}"]["i32_us"] = round(us_i32, 3)
            try:
                us_lt = t_ev(lambda i: torch._int_mm(bufs[i % rot][0], bufs[i % rot][1].t()), steps)
                res[f"{M}x{N}x{K}"]["cublaslt_i32_us"] = round(us_lt, 3)
                res[f"{M}x{N}x{K}"]["cublaslt_TOPS"] = round(2 * M * N * K / us_lt / 1e6, 2)
            except RuntimeError as e:  # no int8 cuBLASLt kernel for this GPU / build
                res[f"{M}x{N}x{K}"]["cublaslt_i32_us"] = f"unavailable: {str(e).splitlines()[0][:80]}"
    return res


def part_gemv(torch, hbm_peak, steps=200, rot=4):
    """Config 4: batch-1 low-bit GEMV over INT2 [49152][2048] + INT4
    [16384][2048], group-64 fp16 scales; `rot` weight copies (185 MB > L2)
    cycled so every call streams its weights from HBM."""
    from jimotono_b200 import lib
    L = lib()
    K, n2, n4 = 2048, 49152, 16384
    g = torch.Generator(device="cuda")
    g.manual_seed(4)
    stream = torch.cuda.current_stream().cuda_stream
    a = torch.randint(-127, 128, (K,), dtype=torch.int8, device="cuda", generator=g)
    y = torch.empty(n2 + n4, device="cuda")
    copies = []
    for _ in range(rot):
        w2 = torch.randint(0, 256, (n2, K // 4), dtype=torch.uint8, device="cuda", generator=g)
        w4 = torch.randint(0, 256, (n4, K // 2), dtype=torch.uint8, device="cuda", generator=g)
        s2 = (torch.rand((n2, K // 64), device="cuda", generator=g) * 0.04 + 0.01).half()
        s4 = (torch.rand((n4, K // 64), device="cuda", generator=g) * 0.04 + 0.01).half()
        copies.append((w2, s2, w4, s4))

    def call(i):
        w2, s2, w4, s4 = copies[i % rot]
        return L.jt_b200_lowbit_gemv(a.data_ptr(), 0.0123, w2.data_ptr(), s2.data_ptr(), n2,
                                     w4.data_ptr(), s4.data_ptr(), n4, K, y.data_ptr(), stream)
    for i in range(10):
        assert call(i) == 0
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        call(i)
    e1.record()
    torch.cuda.synchronize()
    assert L.jt_b200_sync() == 0
    us = e0.elapsed_time(e1) / steps * 1e3
    byts = n2 * (K // 4 + K // 32) + n4 * (K // 2 + K // 32) + K + 4 * (n2 + n4)
    return {"us": round(us, 3), "bytes": byts, "GBs": round(byts / us / 1e3, 1),
            "frac_hbm": round(byts / us / 1e3 / hbm_peak, 4),
            "l2": f"{rot} rotating weight copies ({rot * byts / 1e6:.0f} MB > L2)"}


def main_ep(torch, args, rank, world, local, hbm_peak, peak_kind):
    """N > 1: the expert-parallel layer, max step time over ranks."""
    with ClockSampler(local) as clk:
        st = time_layer_ep(torch, CFG5, rank, world, args.steps, args.warmup, seed=5)
    t = torch.tensor([st["ms_per_step"], st["e2e_ms"]], device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms, e2e_ms = float(t[0].item()), float(t[1].item())
    kept = torch.tensor([st["kept_local"]], device="cuda")
    torch.distributed.all_reduce(kept)
    clocks = clk.summary()
    dm = st["dims"]
    T = CFG5["T"]
    kept_all = int(kept.item())
    ops = 2.0 * kept_all * (dm.d * 2 * dm.f + dm.f * dm.d) + 2.0 * T * dm.S * (3 * dm.fs * dm.d)
    t_peak, t_peak_kind = tensor_peak()
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(T / (ms / 1e3), 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f16/bf16 products of int8, INT2, INT4 codes; fp32 accumulate",
            "data": "synthetic (seeded; random-init packed weights)",
            "config": {"workload": "cfg5 EP MoE layer: T=16384 d=2048 E=1024 f=1536 top-8 INT2/INT4 g64 + 2 shared INT8 f=4096, cap 1.5",
                       "tokens": T, "parallelism": f"ep{world}: {CFG5['E'] // world} experts and {T // world} tokens per GPU, NCCL send/recv dispatch + combine",
                       "l2": "inputs larger than L2 (weights per GPU > 126 MB)"},
            "e2e": {"value": round(T / (e2e_ms / 1e3), 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": st["h2d"] * world, "d2h_bytes_per_step": st["d2h"] * world},
            "gpu_launches": args.steps * (15 + 3 * dm.S),
            "kept_pairs": kept_all,
            "roofline": {"bound": "tensor", "kernel": "whole expert-parallel layer (flops of all GPUs)",
                         "achieved": round(ops / (ms / 1e3) / 1e12, 2), "peak": round(t_peak * world, 1),
                         "unit": "TFLOP/s", "frac": round(ops / (ms / 1e3) / 1e12 / (t_peak * world), 4),
                         "peak_kind": t_peak_kind + " x GPUs", "traffic": None},
            "clocks": clocks, "hbm_peak_gbs": hbm_peak, "hbm_peak_kind": peak_kind, "cpu_baseline": None,
        }
        print(json.dumps(line), flush=True)
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-parts", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--small", action="store_true",
                    help="time only the MoE layer at 1/8 of config 5 (profiler captures)")
    ap.add_argument("--part", choices=["cfg1", "cfg2", "cfg3", "cfg4"],
                    help="time only one secondary configuration and print its JSON (profiler captures)")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        from oracle.cpu_baseline import reference_arm
        if rank == 0:
            print(json.dumps(reference_arm(args.steps, args.warmup, METRIC)), flush=True)
        return

    import torch
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    hbm_peak, peak_kind = peaks()
    if args.part:
        if args.part == "cfg1":
            out = part_w8a8(torch, steps=args.steps)
        elif args.part == "cfg4":
            out = part_gemv(torch, hbm_peak, steps=args.steps)
        elif args.part == "cfg2":
            st2 = time_layer(torch, CFG2, 0, 1, args.steps, args.warmup, seed=2, nrot=DEC_ROT, profile=False)
            reps = max(1, args.steps // DEC_ROT)
            out = {"us_per_token_stream": round(st2["ms_per_step"] * 1e3, 2),
                   "us_per_token_graph": round(time_decode_graph(torch, st2, reps=reps), 2),
                   "us_per_token_graph_l2_warm": round(time_decode_graph(torch, st2, reps=reps, warm=True), 2)}
        else:
            st3 = time_layer(torch, CFG3, 0, 1, args.steps, args.warmup, seed=3, zipf=1.1, bf16=True)
            out = {"ms_per_step": round(st3["ms_per_step"], 4), "stage_ms": [round(v, 4) for v in st3["stage_ms"]]}
        print(json.dumps({"part": args.part, **out}), flush=True)
        return
    if args.small:
        st = time_layer(torch, CFG5_SMALL, 0, 1, args.steps, args.warmup, seed=5)
        print(json.dumps({"case": "cfg5/8", "ms_per_step": round(st["ms_per_step"], 4),
                          "stage_ms": [round(v, 4) for v in st["stage_ms"]], "kept": st["kept"]}))
        return

    if world > 1:
        main_ep(torch, args, rank, world, local, hbm_peak, peak_kind)
        return
    with ClockSampler(local) as clk:
        st = time_layer(torch, CFG5, rank, world, args.steps, args.warmup, seed=5)
    ms = st["ms_per_step"]
    tokens = CFG5["T"] if world > 1 else st["T"]
    value = tokens / (ms / 1e3)
    dm = st["dims"]
    # dominant kernel: routed gate/up (int ops of the kept pairs)
    stage = st["stage_ms"]
    kept = st["kept"]
    ops_gu = 2.0 * kept * dm.d * (2 * dm.f)
    ops_dn = 2.0 * kept * dm.f * dm.d
    ops_sh = 2.0 * st["T"] * dm.S * (2 * dm.fs * dm.d + dm.d * dm.fs)
    e2e_ms, h2d, d2h = e2e_layer(torch, st, max(8, 2 * args.steps), 2)
    parts = {}
    if rank == 0 and not args.no_parts:
        st3 = time_layer(torch, CFG3, 0, 1, args.steps, args.warmup, seed=3, zipf=1.1, bf16=True)
        parts["cfg3_prefill"] = {
            "tokens_per_s": round(CFG3["T"] / (st3["ms_per_step"] / 1e3), 1),
            "ms_per_step": round(st3["ms_per_step"], 4),
            "stage_ms": [round(v, 4) for v in st3["stage_ms"]], "kept": st3["kept"],
            "routed_TOPS": round(2.0 * st3["kept"] * CFG3["d"] * 3 * CFG3["f"] /
                                 ((st3["stage_ms"][4] + st3["stage_ms"][5]) / 1e3) / 1e12, 1)}
        del st3
        st2 = time_layer(torch, CFG2, 0, 1, 200, 20, seed=2, nrot=DEC_ROT)
        dec_us = time_decode_graph(torch, st2, reps=10)
        dec_us_warm = time_decode_graph(torch, st2, reps=10, warm=True)
        dm2 = st2["dims"]
        per_tok = (dm2.k * (2 * dm2.f * (dm2.d // 4 + dm2.d // 64 * 2) + dm2.d * (dm2.f // 2 + dm2.f // 64 * 2))
                   + dm2.S * (2 * dm2.fs * (dm2.d + 4) + dm2.d * (dm2.fs + 4)) + dm2.d * 8)
        parts["cfg2_decode"] = {
            "us_per_token": round(dec_us, 2), "bytes_per_token": per_tok,
            "GBs": round(per_tok / (dec_us / 1e6) / 1e9, 1),
            "frac_hbm": round(per_tok / (dec_us / 1e6) / 1e9 / hbm_peak, 4),
            "us_per_token_l2_warm": round(dec_us_warm, 2),
            "timing": "CUDA graph of %d forward calls (2 kernels each: gate/up with the router, down), replayed; "
                      "stream-launched with per-stage events: %.2f us" % (DEC_ROT, st2["ms_per_step"] * 1e3),
            "l2": "%d rotating weight copies, each forward with its own token and logits: %d x 5.46 MB "
                  "touched per replay, > L2 (l2_warm: one copy, one token)" % (DEC_ROT, DEC_ROT)}
        del st2
        parts["cfg1_w8a8"] = part_w8a8(torch)
        parts["cfg4_gemv"] = part_gemv(torch, hbm_peak)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        from oracle.cpu_baseline import cpu_baseline
        cpu = cpu_baseline(seconds=60.0)
    clocks = clk.summary()
    if rank == 0:
        gu_ms = stage[4]
        t_peak, t_peak_kind = tensor_peak()
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16/bf16 products of int8, INT2, INT4 codes; fp32 accumulate",
            "data": "synthetic (seeded; random-init packed weights)",
            "config": {"workload": "cfg5 EP MoE layer: T=16384 d=2048 E=1024 f=1536 top-8 INT2/INT4 g64 + 2 shared INT8 f=4096, cap 1.5",
                       "tokens": tokens, "parallelism": f"replicas{world}" if world > 1 else "single GPU",
                       "l2": "inputs larger than L2 (3.6 GB weights, 134 MB activations)"},
            "e2e": {"value": round(tokens / (e2e_ms / 1e3) if world == 1 else st["T"] / (e2e_ms / 1e3), 1),
                    "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": args.steps * (9 + 3 * dm.S),
            "stage_ms": {n: round(v, 4) for n, v in zip(
                ["route", "sort", "dispatch", "shared", "gateup", "down", "output"], stage)},
            "kept_pairs": kept,
            "roofline": {"bound": "tensor", "kernel": "routed gate/up (k_moe_gu16, tcgen05 kind::f16)",
                         "achieved": round(ops_gu / (gu_ms / 1e3) / 1e12, 2), "peak": t_peak,
                         "unit": "TFLOP/s", "frac": round(ops_gu / (gu_ms / 1e3) / 1e12 / t_peak, 4),
                         "peak_kind": t_peak_kind,
                         "traffic": GU_TRAFFIC_BYTES,
                         "traffic_note": "ncu dram read+write of one launch at 1/8 of config 5, x8"},
            "layer_TOPS": round((ops_gu + ops_dn + ops_sh) / (ms / 1e3) / 1e12, 1),
            "clocks": clocks, "hbm_peak_gbs": hbm_peak, "hbm_peak_kind": peak_kind,
            "parts": parts, "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    del st
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
