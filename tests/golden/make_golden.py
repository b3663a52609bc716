"""Generate the golden fixtures in this folder from the reference's own CPU
library (oracle/_ref/libjtref.so, compiled from the reference sources by
`make -C oracle ref`).

    python tests/golden/make_golden.py

Every array is produced by a reference entry point on seeded inputs; the
tests compare the oracle restatement (CPU) and the B200 library (GPU)
against these files, so they also run where the reference is absent.
"""
import ctypes as C
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle  # noqa: E402


def p(a):
    return a.ctypes.data


def routing_and_sort(ref):
    """routing.c:16-76 top-k + softmax per token, then moe_layer.c:895-978."""
    rng = np.random.default_rng(101)
    T, E, k = 300, 16, 4
    logits = rng.standard_normal((T, E)).astype(np.float32)
    logits[7] = 0.5          # a fully tied token: ids 0..k-1
    logits[9, 3] = logits[9, 11] = 4.0  # a tie inside the top-k
    bias = np.log(np.maximum(rng.zipf(1.3, E).astype(np.float64), 1.0) / 40.0).astype(np.float32)
    lb = (logits + bias[None, :]).astype(np.float32)  # bias added in float before the call
    ids = np.zeros((T, k), np.uint64)
    w = np.zeros((T, k), np.float32)
    for t in range(T):
        row = np.ascontiguousarray(lb[t])
        idt = np.zeros(k, np.uint64)
        wt = np.zeros(k, np.float32)
        assert ref.jt_routing_topk(p(row), E, k, p(idt), p(wt)) == 0
        ids[t], w[t] = idt, wt
    out = {"logits": logits, "bias": bias, "ids": ids.astype(np.int32), "w": w, "T": T, "E": E, "k": k}
    for tag, cap in (("c100", 1.0), ("c125", 1.25)):
        perm = np.zeros(T * k, np.uint64)
        off = np.zeros(E + 1, np.uint64)
        drop = np.zeros(T * k, np.uint8)
        kept = C.c_size_t(0)
        dropped = C.c_size_t(0)
        flat = np.ascontiguousarray(ids.reshape(-1))
        assert ref.jt_moe_batch_sort(p(flat), T, k, E, cap, p(perm), p(off), p(drop),
                                     C.addressof(kept), C.addressof(dropped)) == 0
        out[f"perm_{tag}"] = perm[:kept.value].astype(np.int32)
        out[f"off_{tag}"] = off.astype(np.int32)
        out[f"drop_{tag}"] = drop
        out[f"kept_{tag}"] = kept.value
    np.savez_compressed(os.path.join(HERE, "routing_sort.npz"), **out)


def quant(ref):
    """w8a8.c:688-855 per-tensor and per-channel quantization."""
    rng = np.random.default_rng(202)
    rows, cols = 33, 256
    x = (rng.standard_normal((rows, cols)) * rng.uniform(0.01, 8.0, (rows, 1))).astype(np.float32)
    x[5] = 0.0                      # zero row -> scale 1, codes 0
    x[6, :] = 0.5 * (np.arange(cols) % 7 - 3) * (1.0 / 127.0)  # exact ties on the grid
    q = np.zeros((rows, cols), np.int8)
    s = np.zeros(rows, np.float32)
    assert ref.jt_w8a8_quant_per_channel(p(x), rows, cols, p(q), p(s)) == 0
    qt = np.zeros(rows * cols, np.int8)
    st = np.zeros(1, np.float32)
    assert ref.jt_w8a8_quant_per_tensor(p(x), rows * cols, p(qt), p(st)) == 0
    np.savez_compressed(os.path.join(HERE, "quant.npz"), x=x, q_pc=q, s_pc=s, q_pt=qt.reshape(rows, cols),
                        s_pt=st)


def w8a8(ref):
    """w8a8.c:955-1072 GEMMs with fp64 dequantization."""
    rng = np.random.default_rng(303)
    M, K, N = 17, 272, 96
    A = rng.integers(-127, 128, (M, K), dtype=np.int8)
    B = rng.integers(-127, 128, (K, N), dtype=np.int8)  # reference layout [K][N]
    sA = np.float32(0.0123)
    sB = rng.uniform(0.001, 0.01, N).astype(np.float32)
    Cpc = np.zeros((M, N), np.float32)
    assert ref.jt_w8a8_gemm_per_channel(p(A), p(B), sA, p(sB), p(Cpc), M, N, K) == 0
    Cpt = np.zeros((M, N), np.float32)
    assert ref.jt_w8a8_gemm_per_tensor(p(A), p(B), sA, np.float32(0.0071), p(Cpt), M, N, K) == 0
    np.savez_compressed(os.path.join(HERE, "w8a8.npz"), A=A, B=B, sA=np.array([sA]), sB=sB, C_pc=Cpc,
                        C_pt=Cpt, sB_pt=np.array([np.float32(0.0071)]))


def lowbit(ref):
    """lowbit.c:47-141 level rule: fake-quant values and bit-plane codes."""
    rng = np.random.default_rng(404)
    rows, K = 12, 256
    W = (rng.standard_normal((rows, K)) * rng.uniform(0.01, 2.0, (rows, 1))).astype(np.float32)
    W[3, ::5] = W[3].max()          # repeated maxima
    out = {"W": W}
    for bits in (2, 4):
        li = np.zeros((rows, K), np.uint8)
        ws = np.zeros(rows, np.float32)
        fq = np.zeros((rows, K), np.float32)
        for r in range(rows):
            col = np.ascontiguousarray(W[r])
            idx = np.zeros(bits * K // 4, np.uint8)
            wsr = np.zeros(1, np.float32)
            assert ref.jt_lowbit_col_to_idx(p(col), K, bits, p(idx), p(wsr)) == 0
            planes = idx.reshape(bits, K // 4)
            for k in range(K):
                v = 0
                for b in range(bits):
                    v |= ((int(planes[b, k // 4]) >> (k % 4)) & 1) << b
                li[r, k] = v
            ws[r] = wsr[0]
            fqr = np.zeros(K, np.float32)
            assert ref.jt_lowbit_fakequant(p(col), p(fqr), K, bits) == 0
            fq[r] = fqr
        out[f"li{bits}"] = li
        out[f"ws{bits}"] = ws
        out[f"fq{bits}"] = fq
    np.savez_compressed(os.path.join(HERE, "lowbit.npz"), **out)


def main():
    if not oracle.have_ref():
        sys.exit("oracle/_ref/libjtref.so is missing: run `make -C oracle ref` first")
    ref = oracle.ref()
    routing_and_sort(ref)
    quant(ref)
    w8a8(ref)
    lowbit(ref)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
