// jt_decode.cu - batch-1 (T = 1) path of the prepared MoE layer.
//
// One token selects k distinct experts and every expert's capacity is at
// least one pair (cap = ceil(cap_factor * k / E) >= 1), so nothing is
// dropped, the routing weights are final and the expert GEMMs degenerate to
// matrix-vector products over the selected experts' rows.  The whole step
// is a latency-bound walk through a few MB, spread over many SMs, in two
// kernels:
//
//   k_dec_gateup  work units of 128 weight rows: 64 gate rows over the same
//                 64 up rows of one expert, four threads per row.  Routed
//                 unit (slot, 64-channel block): INT2 rows; the four threads
//                 of a row take interleaved groups, each group's exact
//                 integer partials give its dot with the fp16 weights
//                 fp16_rn(code * scale) of the batched kernel (jt_moe_gu16.cu),
//                 passed by shuffle so that the fold runs in fp32 in group
//                 order; then SwiGLU (moe_layer.c:146-148), h in bf16.
//                 Shared-expert unit (expert, 64-channel block, K part of up
//                 to 1024 bytes, a quarter per thread): for d <= 1024 one CTA
//                 takes the whole row and its quad sum is the dot; for longer
//                 rows ksplit CTAs each take a K part, their exact int32
//                 partial dots meet in a device accumulator through integer
//                 atomic adds, and the CTA that arrives last (ticket counter,
//                 no waiting) takes the totals - resetting the accumulator
//                 for the next call - and finishes the unit.  Every CTA quantizes the
//                 token itself (w8a8.c:688-747); routed CTAs route it first
//                 (jt_topk.cuh), which only they need, and the token's
//                 quantization runs while their weight loads are in flight.
//   k_dec_down    eight output channels per CTA.  Before it waits for the
//                 gate/up grid (programmatic dependent launch) it routes the
//                 token again (same function, same experts) with the
//                 softmax and pulls its down weight rows - those of the
//                 selected routed experts and of the shared experts, with
//                 their scales - into shared memory with bulk copies, so
//                 after the wait only the h rows (a few KB, from L2) are
//                 read.  Then one thread per dot product (routed: a whole
//                 INT4 row with its group fold; shared: the int32 partials of
//                 two groups) and one thread per channel for the combine in
//                 double in slot order and the shared experts
//                 (moe_layer.c:1443-1463, :1549-1559), fp32 or bf16 out.
//
// Every phase issues all of its loads before it uses any: the chain token
// -> routing -> selected rows is the critical path.
//
// The gate/up CTA (slot 0, block 0) also writes the per-token results the
// batched chain would produce for one token (perm, pos, off, drop, kept, xq,
// xs), so the layer's debug views are the same on both paths.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "jt_internal.h"
#include "jt_ptx.cuh"
#include "jt_quant.cuh"
#include "jt_runtime.cuh"
#include "jt_swiglu.cuh"
#include "jt_topk.cuh"

namespace {

constexpr int kMaxD = 4096;        // token width handled (d <= 4096)
constexpr int kMaxF = 4096;        // expert ffn handled (f, fs <= 4096)
constexpr int kMaxE = 4096;        // experts
constexpr int kGuThreads = 512;       // four threads per weight row of a unit
constexpr int kSharedPartMax = 1024;  // bytes of one shared-expert row per K part (at most)
constexpr int kSharedQuarter = kSharedPartMax / 4;  // of which one thread takes a quarter
constexpr int kDnWarps = 8;        // output channels per down CTA
constexpr size_t kDnSmemMax = 200 * 1024;

struct DecParams {
    CUtensorMap tmG, tmU;    // routed gate / up rows [E*f][d/4], 64-row x 128-byte boxes, 128B swizzle
    int tma;                 // 1: routed rows by tensor map (d % 512 == 0), 0: register loads
    const float *x;          // [d] token row
    const float *logits;     // [E] router logits
    const float *bias;       // [E] or NULL
    int32_t *ids;            // [k] selected experts (slot order)
    float *w;                // [k] routing weights (final: nothing is dropped)
    const uint8_t *wg, *wu;  // [E][f][d/4] INT2
    const __half *sg, *su;   // [E][d/64][f]
    const uint8_t *wd;       // [E][d][f/2] INT4
    const __half *sd;        // [E][f/64][d]
    const int8_t *wsg, *wsu; // [S][fs][d]
    const float *ssg, *ssu;  // [S][fs]
    const int8_t *wsd;       // [S][d][fs]
    const float *ssd;        // [S][d]
    int d, f, E, k, S, fs;
    int n_routed_units;      // k * (f / 64)
    int ksplit;              // K parts of a shared-expert row
    int32_t *acc_s;          // [S][2][fs] shared partial dots (zero between calls)
    int32_t *cnt_s;          // [S][fs/64] arrival tickets (zero between calls)
    // outputs of the gate/up kernel (and debug copies of the batched path)
    int8_t *xq;
    float *xs;
    uint16_t *h;             // [k][f] routed h, bf16, rows in expert order
    uint16_t *hb_s;          // [S][fs] shared h, bf16
    int32_t *perm, *pos, *off, *tile_off, *meta;
    uint8_t *drop;
    float *w_fin;
    // down output
    float *y;                // [d] fp32 (or NULL)
    uint16_t *y_bf16;        // [d] bf16 (or NULL)
    int *err;
};

// dp4a of unsigned bytes a against signed bytes b (the masked INT2 fields
// reach 192, beyond a signed byte).
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Sorted row of slot p: experts ascending, as the capacity sort orders the
// kept pairs of one token.
__device__ __forceinline__ int slot_rank(const int32_t *ids, int k, int p) {
    const int e = ids[p];
    int r = 0;
    for (int q = 0; q < k; ++q) r += ids[q] < e;
    return r;
}

// Group partials of one INT2 group (16 packed bytes, codes li little-endian
// along K) against the token: byte b of word i holds the codes of
// k = 16i + 4b + j in bits 2j, so field j of every byte pairs with the
// activation word xp[4i + j] = {x[16i+j], x[16i+4+j], x[16i+8+j],
// x[16i+12+j]}.  Each bit of a field is used in place (times 2^(2j) or
// 2^(2j+1)) and the sums are scaled back exactly: with li = b0 + 2 b1,
//   P  = sum x c            = 2 B0 + 4 B1 - 3 X   (c = 2 li - 3)
//   A3 = sum x [|c| = 3] sgn(c) = B0 + B1 - X       ([li=3] - [li=0] = b0 + b1 - 1)
// with B0 = sum x b0, B1 = sum x b1, X = sum x.  The routed gate/up weight
// of code c is fp16_rn(c s) = c s + [|c| = 3] sgn(c) (t - 3 s) with
// t = fp16_rn(3 s), so the group's dot with the weights is s P + (t - 3s) A3.
__device__ __forceinline__ int2 int2_group(const uint4 w, const uint32_t *xp, int gs) {
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
    int l0 = 0, l1 = 0, l2 = 0, l3 = 0, h0 = 0, h1 = 0, h2 = 0, h3 = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint4 xv = *reinterpret_cast<const uint4 *>(xp + 4 * i);
        l0 = dp4a_us(ww[i] & 0x01010101u, xv.x, l0);
        h0 = dp4a_us(ww[i] & 0x02020202u, xv.x, h0);
        l1 = dp4a_us(ww[i] & 0x04040404u, xv.y, l1);
        h1 = dp4a_us(ww[i] & 0x08080808u, xv.y, h1);
        l2 = dp4a_us(ww[i] & 0x10101010u, xv.z, l2);
        h2 = dp4a_us(ww[i] & 0x20202020u, xv.z, h2);
        l3 = dp4a_us(ww[i] & 0x40404040u, xv.w, l3);
        h3 = dp4a_us(ww[i] & 0x80808080u, xv.w, h3);
    }
    const int b0 = l0 + (l1 >> 2) + (l2 >> 4) + (l3 >> 6);
    const int b1 = (h0 >> 1) + (h1 >> 3) + (h2 >> 5) + (h3 >> 7);
    return make_int2(2 * b0 + 4 * b1 - 3 * gs, b0 + b1 - gs);
}

// fp32 dot of one group with its fp16 weights: s P + (t - 3s) A3 (see
// int2_group; t - 3s is exact in fp32).
__device__ __forceinline__ float int2_fold(float acc, int2 pa, __half sg) {
    const float s = __half2float(sg);
    const float s3 = 3.0f * s;
    const float dt = __half2float(__float2half_rn(s3)) - s3;
    return fmaf((float)pa.y, dt, fmaf((float)pa.x, s, acc));
}

// SwiGLU of the 64 channels staged in gu, rounded to bf16 into h[0..63].
// Warps 0 and 1, one channel per thread (a single exp chain each).
__device__ __forceinline__ void swiglu_bf16_64(const float (&gu)[2][64], uint16_t *h, int *err) {
    const int c = threadIdx.x;  // 0..63
    const float hv = jt::swiglu(gu[0][c], gu[1][c]);
    if (__any_sync(0xffffffffu, !isfinite(hv)) && (c & 31) == 0) atomicExch(err, JT_KERR_NONFINITE);
    h[c] = __bfloat16_as_ushort(__float2bfloat16_rn(hv));
}

// grid n_routed_units + S * (fs/64) * ksplit, kGuThreads threads: four
// per weight row (thread t: row t / 4, quarter t % 4).
//
// The token row is read once, as float4 per thread, and kept in registers;
// the weight rows of a shared expert (which depend neither on the token nor
// on the routing) are loaded before the wait for the previous kernel of the
// stream.  At most 96 registers per thread (a few bytes spill), so that a
// CTA of the down kernel, launched early as a programmatic dependent, fits
// on the same SM: 16.4 us per token against 18.2 us at 128 registers.
__global__ void __maxnreg__(96) k_dec_gateup(const __grid_constant__ DecParams p) {
    __shared__ __align__(16) int8_t sx[kMaxD];
    __shared__ __align__(16) uint32_t xp[kMaxD / 4];
    __shared__ int gsum[kMaxD / 64];
    __shared__ float gu[2][64];
    __shared__ __align__(16) uint32_t taken[kMaxE / 32];
    __shared__ int32_t sids[64], ssel[64];
    __shared__ float sw[64], sselv[64];
    __shared__ float wm[kGuThreads / 32];
    __shared__ int wb[kGuThreads / 32];
    __shared__ int ticket;
    __shared__ uint64_t wbar;
    __shared__ int abort_flag;
    // routed units: the unit's 64 gate then 64 up rows as 64-row x 128-byte
    // boxes (1024-byte aligned for the swizzle)
    extern __shared__ __align__(1024) uint8_t wsm_raw[];
    uint8_t *wsm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(wsm_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    // the down kernel may launch now; it waits for this grid before reading
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int d = p.d, ng = d / 64;
    const bool routed = (int)blockIdx.x < p.n_routed_units;
    const int r = threadIdx.x >> 2;  // 0..63 gate rows, 64..127 up rows
    const int qd = threadIdx.x & 3;  // quarter of the row
    const bool up = r >= 64;
    int slot = 0, cb = 0, s = 0, kq = 0;
    if (routed) {
        const int nb = p.f / 64;
        slot = blockIdx.x / nb;
        cb = blockIdx.x % nb;
    } else {
        const int u = blockIdx.x - p.n_routed_units;
        const int nb = p.fs / 64;
        s = u / (nb * p.ksplit);
        cb = (u / p.ksplit) % nb;
        kq = u % p.ksplit;
    }
    // shared units: the row's K part [kq part_bytes, +part_bytes), a quarter
    // of it per thread (qbytes = part_bytes / 4, 32..256 bytes)
    const int part_bytes = d / p.ksplit, qbytes = part_bytes / 4;
    if (threadIdx.x == 0) {
        abort_flag = 0;
        jt::mbar_init(&wbar, 1);
        jt::fence_mbar_init();
    }
    uint4 wv[kSharedQuarter / 16];
    if (!routed) {
        const int c = cb * 64 + (r & 63);
        const uint4 *wrow = reinterpret_cast<const uint4 *>(
            reinterpret_cast<const uint8_t *>((up ? p.wsu : p.wsg) + ((size_t)s * p.fs + c) * d) + kq * part_bytes +
            qd * qbytes);
#pragma unroll
        for (int j = 0; j < kSharedQuarter / 16; ++j)
            if (16 * j < qbytes) wv[j] = __ldg(wrow + j);
    }
    // this grid is itself launched as a dependent of the previous kernel of
    // the stream (the previous token's down kernel in a decode loop): wait
    // for it before reading the token or writing hq/hs
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // ---- the token row, once, into registers (indices clamped so every
    // load is issued unconditionally)
    constexpr int kXv = kMaxD / 4 / kGuThreads;
    const int nx4 = d / 4;
    float4 xv[kXv];
#pragma unroll
    for (int i = 0; i < kXv; ++i) {
        const int j = threadIdx.x + i * kGuThreads;
        xv[i] = reinterpret_cast<const float4 *>(p.x)[j < nx4 ? j : nx4 - 1];
    }
    if (routed && warp == 0) {
        sids[lane] = lane;  // fallback on a routing fault: experts 0..k-1 stay in range
        sids[lane + 32] = lane + 32;
        __syncwarp();
        jt::warp_topk_softmax(p.logits, p.bias, p.E, p.k, taken, ssel, sselv, sids, sw, p.err, false);
        __syncwarp();
        // the selected expert's 64 gate and 64 up rows: 64-row x 128-byte
        // boxes of the tensor maps, 128-byte swizzled in shared memory
        if (p.tma && lane == 0) {
            int e = sids[slot];
            e = (e < 0 || e >= p.E) ? 0 : e;
            const int nbox = d / 512;
            jt::mbar_arrive_expect_tx(&wbar, 2u * 64u * (uint32_t)(d / 4));
            for (int j = 0; j < nbox; ++j) {
                jt::tma_load_2d(wsm + (size_t)j * 8192, &p.tmG, &wbar, 128 * j, e * p.f + cb * 64);
                jt::tma_load_2d(wsm + (size_t)(nbox + j) * 8192, &p.tmU, &wbar, 128 * j, e * p.f + cb * 64);
            }
        }
    }
    float m = 0.0f;
    int bad = 0;
#pragma unroll
    for (int i = 0; i < kXv; ++i) {
        if (threadIdx.x + i * kGuThreads < nx4) {
            const float4 v = xv[i];
            bad |= !isfinite(v.x) | !isfinite(v.y) | !isfinite(v.z) | !isfinite(v.w);
            m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        bad |= __shfl_xor_sync(0xffffffffu, bad, o);
    }
    if (lane == 0) {
        wm[warp] = m;
        wb[warp] = bad;
    }
    __syncthreads();
    // ---- routed units: the raw fp16 scales of this thread's groups
    // g = qd + 4 i (coalesced over the block's 64 channels)
    uint32_t sv[kMaxD / 256];
    const __half *srow = nullptr;
    const uint4 *grow = nullptr;
    if (routed) {
        int e = sids[slot];
        e = (e < 0 || e >= p.E) ? 0 : e;
        const int c = cb * 64 + (r & 63);
        srow = (up ? p.su : p.sg) + (size_t)e * ng * p.f + c;
        grow = reinterpret_cast<const uint4 *>((up ? p.wu : p.wg) + ((size_t)e * p.f + c) * (d / 4));
#pragma unroll
        for (int i = 0; i < kMaxD / 256; ++i) {
            const int g = qd + 4 * i;
            sv[i] = g < ng ? (uint32_t)__half_as_ushort(srow[(size_t)g * p.f]) : 0u;
        }
    }
    // ---- quantize the token (w8a8.c:688-747) from the registers, in the
    // single-precision form of the quantizer: the same codes and stored scale
    // as the double formula (jt_quant.cuh), without double divisions
    m = 0.0f;
    bad = 0;
    for (int i = 0; i < kGuThreads / 32; ++i) {
        m = fmaxf(m, wm[i]);
        bad |= wb[i];
    }
    const jt::QuantBlockF qb = jt::quant_block_f(bad ? 0.0f : m);
    if (bad && threadIdx.x == 0) atomicExch(p.err, 0x85);
#pragma unroll
    for (int i = 0; i < kXv; ++i) {
        const int j = threadIdx.x + i * kGuThreads;
        if (j < nx4) {
            const float4 v = xv[i];
            uint32_t w4 = 0u;
            if (!bad)
                w4 = (uint32_t)(uint8_t)(int8_t)jt::quant_code_f(v.x, qb) |
                     ((uint32_t)(uint8_t)(int8_t)jt::quant_code_f(v.y, qb) << 8) |
                     ((uint32_t)(uint8_t)(int8_t)jt::quant_code_f(v.z, qb) << 16) |
                     ((uint32_t)(uint8_t)(int8_t)jt::quant_code_f(v.w, qb) << 24);
            reinterpret_cast<uint32_t *>(sx)[j] = w4;
        }
    }
    const float xs = qb.scale_f;
    __syncthreads();
    if (routed) {
        // activation words permuted for the INT2 fields: 16-byte block w gives
        // xp[4w + j] = bytes {j, 4+j, 8+j, 12+j}; group sums by dp4a
        for (int w = threadIdx.x; w < d / 16; w += kGuThreads) {
            const uint4 v = reinterpret_cast<const uint4 *>(sx)[w];
            const uint32_t lo01 = __byte_perm(v.x, v.y, 0x5140), lo23 = __byte_perm(v.z, v.w, 0x5140);
            const uint32_t hi01 = __byte_perm(v.x, v.y, 0x7362), hi23 = __byte_perm(v.z, v.w, 0x7362);
            uint4 o;
            o.x = __byte_perm(lo01, lo23, 0x5410);
            o.y = __byte_perm(lo01, lo23, 0x7632);
            o.z = __byte_perm(hi01, hi23, 0x5410);
            o.w = __byte_perm(hi01, hi23, 0x7632);
            reinterpret_cast<uint4 *>(xp)[w] = o;
        }
        for (int g = threadIdx.x; g < ng; g += kGuThreads) {
            const int4 *q4 = reinterpret_cast<const int4 *>(sx + 64 * g);
            int sm = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int4 v = q4[j];
                sm = __dp4a(v.x, 0x01010101, sm);
                sm = __dp4a(v.y, 0x01010101, sm);
                sm = __dp4a(v.z, 0x01010101, sm);
                sm = __dp4a(v.w, 0x01010101, sm);
            }
            gsum[g] = sm;
        }
        __syncthreads();
        if (p.tma && !jt::mbar_wait(&wbar, 0, &abort_flag, p.err)) return;
        // the four threads of a row take groups qd, qd + 4, ...: each group's
        // exact integer partials, then the fold of every group in ascending
        // order (all four lanes run it on the partials passed by shuffle;
        // lane qd == 0 keeps the result).  Row rr of a weight box holds its
        // 16-byte chunk c at chunk c ^ (rr % 8).
        const int rr = r & 63, nbox = d / 512;
        const uint8_t *rowb = wsm + (size_t)(up ? nbox : 0) * 8192 + (size_t)rr * 128;
        float acc = 0.0f;
#pragma unroll
        for (int i = 0; i < kMaxD / 256; ++i) {
            const int g0 = 4 * i;
            if (g0 >= ng) break;  // uniform over the CTA
            const int g = g0 + qd;
            // the group's owner converts once: its partials and the fold
            // constants s and t - 3s of int2_fold
            float pf = 0.0f, af = 0.0f, sf = 0.0f, dtf = 0.0f;
            if (g < ng) {
                const uint4 w = p.tma ? *reinterpret_cast<const uint4 *>(rowb + (size_t)(g >> 3) * 8192 +
                                                                         (((g & 7) ^ (rr & 7)) << 4))
                                      : __ldg(grow + g);
                const int2 pa = int2_group(w, xp + 16 * g, gsum[g]);
                pf = (float)pa.x;
                af = (float)pa.y;
                sf = __half2float(__ushort_as_half((unsigned short)sv[i]));
                const float s3 = 3.0f * sf;
                dtf = __half2float(__float2half_rn(s3)) - s3;
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int src = (lane & ~3) | j;
                const float P = __shfl_sync(0xffffffffu, pf, src);
                const float A3 = __shfl_sync(0xffffffffu, af, src);
                const float S = __shfl_sync(0xffffffffu, sf, src);
                const float D = __shfl_sync(0xffffffffu, dtf, src);
                if (g0 + j < ng) acc = fmaf(A3, D, fmaf(P, S, acc));  // int2_fold
            }
        }
        if (qd == 0) gu[up][rr] = __fmul_rn(acc, xs);
        __syncthreads();
        if (warp < 2) {
            const int row = slot_rank(sids, p.k, slot);
            swiglu_bf16_64(gu, p.h + (size_t)row * p.f + cb * 64, p.err);
        }
        if (blockIdx.x == 0) {
            // the batched path's per-token results for one token
            for (int i = threadIdx.x; i < d / 16; i += kGuThreads)
                reinterpret_cast<int4 *>(p.xq)[i] = reinterpret_cast<const int4 *>(sx)[i];
            if (threadIdx.x == 0) {
                p.xs[0] = xs;
                p.meta[0] = p.k;
                p.meta[1] = p.k;
                p.meta[2] = 1;
            }
            if (threadIdx.x < p.k) {
                const int q = threadIdx.x;
                const int row = slot_rank(sids, p.k, q);
                p.ids[q] = sids[q];
                p.perm[row] = q;
                p.pos[q] = row;
                p.drop[q] = 0;
            }
            for (int ex = threadIdx.x; ex <= p.E; ex += kGuThreads) {
                int n = 0;
                for (int q = 0; q < p.k; ++q) n += sids[q] < ex;
                p.off[ex] = n;
                p.tile_off[ex] = n;
            }
        }
        return;
    }
    // ---- shared-expert unit: exact int32 partial dot over this K part, a
    // quarter per thread, summed over the row's four lanes
    int dot = 0;
    {
        const int8_t *xk = sx + kq * part_bytes + qd * qbytes;
#pragma unroll
        for (int j = 0; j < kSharedQuarter / 16; ++j) {
            if (16 * j < qbytes) {
                const int4 xk4 = *reinterpret_cast<const int4 *>(xk + 16 * j);
                dot = __dp4a((int)wv[j].x, xk4.x, dot);
                dot = __dp4a((int)wv[j].y, xk4.y, dot);
                dot = __dp4a((int)wv[j].z, xk4.z, dot);
                dot = __dp4a((int)wv[j].w, xk4.w, dot);
            }
        }
        dot += __shfl_xor_sync(0xffffffffu, dot, 1);
        dot += __shfl_xor_sync(0xffffffffu, dot, 2);
    }
    int32_t *acc = p.acc_s + ((size_t)s * 2 + up) * p.fs + cb * 64 + (r & 63);
    int total = dot;
    if (p.ksplit > 1) {
        if (qd == 0) atomicAdd(acc, dot);
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) ticket = atomicAdd(&p.cnt_s[s * (p.fs / 64) + cb], 1);
        __syncthreads();
        if (ticket != p.ksplit - 1) return;  // another CTA of the unit finishes it
        __threadfence();
        if (qd == 0) total = atomicExch(acc, 0);  // the sum of every part; cleared for the next call
        if (threadIdx.x == 0) p.cnt_s[s * (p.fs / 64) + cb] = 0;
    }
    if (qd == 0) {
        const int c = cb * 64 + (r & 63);
        const float cs = (up ? p.ssu : p.ssg)[(size_t)s * p.fs + c];
        gu[up][r & 63] = __fmul_rn(__fmul_rn(__int2float_rn(total), xs), cs);
    }
    __syncthreads();
    if (warp < 2) swiglu_bf16_64(gu, p.hb_s + (size_t)s * p.fs + cb * 64, p.err);
}

// Layout of the down kernel's dynamic shared memory (byte offsets).  Rows
// are padded by 16 bytes so that rows read by neighbouring threads start in
// different banks.
struct DnLayout {
    uint32_t wr, wsc, ws, ssc, hr, hqs, hss, racc, sp, bar, total;
};

__host__ __device__ inline uint32_t dn_take(uint32_t &o, uint32_t bytes) {
    const uint32_t at = o;
    o = (o + bytes + 15u) & ~15u;
    return at;
}

__host__ __device__ inline DnLayout dn_layout(int k, int f, int S, int fs) {
    DnLayout L;
    uint32_t o = 0;
    L.wr = dn_take(o, (uint32_t)k * kDnWarps * (f / 2 + 16));      // routed down rows [k][8], padded
    L.wsc = dn_take(o, (uint32_t)k * (f / 64) * kDnWarps * 2);     // their fp16 scales [k][f/64][8]
    L.ws = dn_take(o, (uint32_t)S * kDnWarps * (fs + 16));         // shared down rows [S][8], padded
    L.ssc = dn_take(o, (uint32_t)S * kDnWarps * 4);                // their channel scales [S][8]
    L.hr = dn_take(o, (uint32_t)k * (2 * f + 16));                 // routed h rows, bf16 [k], padded
    L.hqs = dn_take(o, (uint32_t)S * fs);                          // shared h codes [S][fs]
    L.hss = dn_take(o, (uint32_t)S * 4);                           // shared h row scales [S]
    L.racc = dn_take(o, (uint32_t)kDnWarps * k * (f / 64) * 4);    // routed group dots [8][k][f/64]
    L.sp = dn_take(o, (uint32_t)kDnWarps * S * (fs / 64) * 4);     // shared group partials [8][S][fs/64]
    L.bar = dn_take(o, 8);
    L.total = o;
    return L;
}

// grid d / 8, 256 threads: output channels blockIdx.x*8 .. +7.
__global__ void __launch_bounds__(kDnWarps * 32) k_dec_down(const __grid_constant__ DecParams p) {
    // the next token's gate/up kernel may launch on the SMs left free; it
    // waits for this grid before its first global access
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    extern __shared__ __align__(16) uint8_t dsm[];
    __shared__ uint32_t taken[kMaxE / 32];
    __shared__ int32_t sids[64], ssel[64], srank[64];
    __shared__ float sw[64], sselv[64];
    __shared__ unsigned smax[8];  // shared h row maxima (float bits), S <= 8
    __shared__ double terms[kDnWarps][64 + 8];  // combine terms [channel][k slots, then S shared experts]
    __shared__ int abort_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int d = p.d, f = p.f, fs = p.fs, k = p.k, S = p.S, gf = f / 64;
    const int o0 = blockIdx.x * kDnWarps;
    const DnLayout L = dn_layout(k, f, S, fs);
    uint64_t *bar = reinterpret_cast<uint64_t *>(dsm + L.bar);
    if (threadIdx.x < 64) {
        sids[threadIdx.x] = threadIdx.x;
        sw[threadIdx.x] = 0.0f;
    }
    if (threadIdx.x < 8) smax[threadIdx.x] = 0u;
    if (threadIdx.x == 0) {
        abort_flag = 0;
        jt::mbar_init(bar, 1);
        jt::fence_mbar_init();
    }
    __syncthreads();
    // ---- independent of the gate/up grid: routing with the softmax (the same
    // function on the same logits as the gate/up grid), then this CTA's down
    // weights into shared memory
    if (warp == 0) jt::warp_topk_softmax(p.logits, p.bias, p.E, k, taken, ssel, sselv, sids, sw, p.err);
    __syncthreads();
    if (threadIdx.x < k) {
        const int q = threadIdx.x;
        const int e = sids[q];
        sids[q] = (e < 0 || e >= p.E) ? 0 : e;
        if (blockIdx.x == 0) {
            p.w[q] = sw[q];
            p.w_fin[q] = sw[q];
        }
    }
    __syncthreads();
    if (threadIdx.x < k) srank[threadIdx.x] = slot_rank(sids, k, threadIdx.x);
    if (warp == 0) {
        const uint32_t rbytes = (uint32_t)(f / 2), rstride = rbytes + 16u;
        const uint32_t sstride = (uint32_t)fs + 16u;
        const uint32_t tx = (uint32_t)k * kDnWarps * rbytes + (uint32_t)k * gf * 16u +
                            (uint32_t)S * kDnWarps * (fs + 4);
        if (lane == 0) jt::mbar_arrive_expect_tx(bar, tx);
        __syncwarp();
        // lane l issues the copies l, l + 32, ... of: k * 8 routed rows,
        // k * gf scale pieces, S * 8 shared rows, S shared scale pieces
        const int n_rows = k * kDnWarps, n_sc = k * gf, n_srows = S * kDnWarps;
        for (int i = lane; i < n_rows + n_sc + n_srows + S; i += 32) {
            if (i < n_rows) {
                const int q = i / kDnWarps, j = i % kDnWarps;
                jt::bulk_load(dsm + L.wr + (size_t)i * rstride, p.wd + ((size_t)sids[q] * d + o0 + j) * (f / 2),
                              rbytes, bar);
            } else if (i < n_rows + n_sc) {
                const int u = i - n_rows, q = u / gf, g = u % gf;
                jt::bulk_load(dsm + L.wsc + (size_t)u * 16, p.sd + ((size_t)sids[q] * gf + g) * d + o0, 16, bar);
            } else if (i < n_rows + n_sc + n_srows) {
                const int u = i - n_rows - n_sc, sh = u / kDnWarps, j = u % kDnWarps;
                jt::bulk_load(dsm + L.ws + (size_t)u * sstride, p.wsd + ((size_t)sh * d + o0 + j) * fs, fs, bar);
            } else {
                const int sh = i - n_rows - n_sc - n_srows;
                jt::bulk_load(dsm + L.ssc + (size_t)sh * kDnWarps * 4, p.ssd + (size_t)sh * d + o0, kDnWarps * 4, bar);
            }
        }
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // ---- h of the routed rows (bf16, rank order) into shared memory; the
    // shared h rows (bf16) quantized per row (w8a8.c:688-747 over the fs
    // channels, one scale per shared expert) into shared memory.  Every
    // global load of this phase first (one round trip to L2).
    uint8_t *hr = dsm + L.hr;
    int8_t *hqs = reinterpret_cast<int8_t *>(dsm + L.hqs);
    float *hss = reinterpret_cast<float *>(dsm + L.hss);
    const int nck = f / 8;   // 16-byte chunks of a routed h row
    constexpr int kHr = 6;   // routed h chunks per thread (k * f / 8 <= 1536 below)
    constexpr int kHs = 4;   // shared h chunks per thread (S * fs / 8 <= 1024 below)
    uint4 hv[kHr], sv[kHs];
    const int n_hr = k * nck, n_hs = S * fs / 8;
#pragma unroll
    for (int t = 0; t < kHr; ++t) {
        const int i = threadIdx.x + t * (int)blockDim.x;
        const int ii = i < n_hr ? i : 0;
        hv[t] = reinterpret_cast<const uint4 *>(p.h + (size_t)(ii / nck) * f)[ii % nck];
    }
#pragma unroll
    for (int t = 0; t < kHs; ++t) {
        const int i = threadIdx.x + t * (int)blockDim.x;
        if (i < n_hs) sv[t] = reinterpret_cast<const uint4 *>(p.hb_s)[i];
    }
#pragma unroll
    for (int t = 0; t < kHr; ++t) {
        const int i = threadIdx.x + t * (int)blockDim.x;
        if (i < n_hr) reinterpret_cast<uint4 *>(hr + (size_t)(i / nck) * (2 * f + 16))[i % nck] = hv[t];
    }
    // row maxima of the shared h (|bf16| as float bits order like the values):
    // 16 consecutive chunks lie in one row (fs / 8 is a multiple of 16), so
    // one shared-memory atomic per half warp and chunk round
#pragma unroll
    for (int t = 0; t < kHs; ++t) {
        const int i = threadIdx.x + t * (int)blockDim.x;
        if (t * (int)blockDim.x >= n_hs) break;  // uniform over the block
        float m = 0.0f;
        if (i < n_hs) {
            const uint32_t w4[4] = {sv[t].x, sv[t].y, sv[t].z, sv[t].w};
#pragma unroll
            for (int e = 0; e < 4; ++e)
                m = fmaxf(m, fmaxf(fabsf(__uint_as_float(w4[e] << 16)), fabsf(__uint_as_float(w4[e] & 0xFFFF0000u))));
        }
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if ((lane & 15) == 0 && i < n_hs) atomicMax(&smax[i / (fs / 8)], __float_as_uint(m));
    }
    __syncthreads();
#pragma unroll
    for (int t = 0; t < kHs; ++t) {
        const int i = threadIdx.x + t * (int)blockDim.x;
        if (i < n_hs) {
            const int sh = i / (fs / 8);
            const jt::QuantBlockF qb = jt::quant_block_f(__uint_as_float(smax[sh]));
            const uint32_t w4[4] = {sv[t].x, sv[t].y, sv[t].z, sv[t].w};
            uint32_t q[2] = {0u, 0u};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int q0 = jt::quant_code_f(__uint_as_float(w4[e] << 16), qb);
                const int q1 = jt::quant_code_f(__uint_as_float(w4[e] & 0xFFFF0000u), qb);
                q[e >> 1] |= ((uint32_t)(uint8_t)(int8_t)q0 | ((uint32_t)(uint8_t)(int8_t)q1 << 8)) << (16 * (e & 1));
            }
            reinterpret_cast<uint2 *>(hqs)[i] = make_uint2(q[0], q[1]);
            if (i % (fs / 8) == 0) hss[sh] = qb.scale_f;
        }
    }
    __syncthreads();
    if (!jt::mbar_wait(bar, 0, &abort_flag, p.err)) return;
    // ---- one thread per dot product.  Routed item (slot q, channel j): the
    // INT4 row's 64 codes of group g, as the bf16 weights
    // bf16_rn(code * bf16_rn(s_g)) of the batched kernel (jt_moe_dn16.cu),
    // against its bf16 h, summed in fp32 (the row's group dots are added in
    // group order in the combine).  Shared item (128-byte
    // part, expert sh, channel j): the int32 partials of its two groups.
    // Neighbouring threads take neighbouring (padded) rows.
    const uint32_t *wr = reinterpret_cast<const uint32_t *>(dsm + L.wr);
    const __half *wsc = reinterpret_cast<const __half *>(dsm + L.wsc);
    const int8_t *ws = reinterpret_cast<const int8_t *>(dsm + L.ws);
    const float *ssc = reinterpret_cast<const float *>(dsm + L.ssc);
    float *racc = reinterpret_cast<float *>(dsm + L.racc);
    int *sp = reinterpret_cast<int *>(dsm + L.sp);
    const int gs = fs / 64;
    const int n_rows = kDnWarps * k, n_r = n_rows * gf, n_s = kDnWarps * S * (fs / 128);
    for (int it = threadIdx.x; it < n_r + n_s; it += blockDim.x) {
        if (it < n_r) {  // routed item: group g of row (slot q, channel j)
            const int g = it / n_rows, q = (it % n_rows) / kDnWarps, j = it % kDnWarps;
            const int rr = srank[q];
            const uint4 *row = reinterpret_cast<const uint4 *>(wr + ((size_t)q * kDnWarps + j) * (f / 8 + 4));
            const uint4 *hrow = reinterpret_cast<const uint4 *>(hr + (size_t)rr * (2 * f + 16));
            const __nv_bfloat162 s2 = __bfloat162bfloat162(
                __float2bfloat16_rn(__half2float(wsc[((size_t)q * gf + g) * kDnWarps + j])));
            float acc0 = 0.0f, acc1 = 0.0f;
#pragma unroll
            for (int c = 0; c < 2; ++c) {  // 4 words = 32 codes
                const uint4 v = row[2 * g + c];
                const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {  // 8 codes against 8 h values
                    uint32_t wb[4];
                    jt::int4_bf16x8(wv[i], s2, wb);
                    const uint4 h8 = hrow[8 * g + 4 * c + i];
                    const uint32_t hb[4] = {h8.x, h8.y, h8.z, h8.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        acc0 = fmaf(__uint_as_float(hb[e] << 16), __uint_as_float(wb[e] << 16), acc0);
                        acc1 = fmaf(__uint_as_float(hb[e] & 0xFFFF0000u), __uint_as_float(wb[e] & 0xFFFF0000u), acc1);
                    }
                }
            }
            racc[(j * k + q) * gf + g] = acc0 + acc1;
        } else {
            const int u = it - n_r;
            const int pt = u / (S * kDnWarps), sh = (u / kDnWarps) % S, j = u % kDnWarps;
            const int4 *row = reinterpret_cast<const int4 *>(ws + ((size_t)sh * kDnWarps + j) * (fs + 16) + 128 * pt);
            const int4 *h = reinterpret_cast<const int4 *>(hqs + (size_t)sh * fs + 128 * pt);
#pragma unroll
            for (int g = 0; g < 2; ++g) {
                int part = 0;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const int4 wv = row[4 * g + c], hv = h[4 * g + c];
                    part = __dp4a(wv.x, hv.x, part);
                    part = __dp4a(wv.y, hv.y, part);
                    part = __dp4a(wv.z, hv.z, part);
                    part = __dp4a(wv.w, hv.w, part);
                }
                sp[(j * S + sh) * gs + 2 * pt + g] = part;
            }
        }
    }
    __syncthreads();
    // ---- the combine in double (moe_layer.c:1443-1463, :1549-1559): first
    // every term at once, one thread per (channel, term) - routed slot q:
    // w_q * (the row's group dots added in group order); shared expert sh:
    // ((float)acc * hs) * ssd[o] with its exact int32 dot summed over the
    // groups - then one thread per output channel adds them, routed rows in
    // slot order, then the shared experts in s order
    const int nterm = k + S;
    for (int it = threadIdx.x; it < kDnWarps * nterm; it += blockDim.x) {
        const int jj = it / nterm, t = it % nterm;
        double v;
        if (t < k) {
            float yp = 0.0f;
            for (int g = 0; g < gf; ++g) yp += racc[(jj * k + t) * gf + g];
            v = __dmul_rn((double)sw[t], (double)yp);
        } else {
            const int sh = t - k;
            int acc = 0;
            for (int g = 0; g < gs; ++g) acc += sp[(jj * S + sh) * gs + g];
            v = (double)__fmul_rn(__fmul_rn((float)acc, hss[sh]), ssc[sh * kDnWarps + jj]);
        }
        terms[jj][t] = v;
    }
    __syncthreads();
    if (threadIdx.x >= kDnWarps) return;
    const int j = threadIdx.x, o = o0 + j;
    if (o >= d) return;
    double ya = 0.0;
    for (int t = 0; t < nterm; ++t) ya = __dadd_rn(ya, terms[j][t]);
    const float yv = (float)ya;
    if (p.y) p.y[o] = yv;
    if (p.y_bf16) p.y_bf16[o] = __bfloat16_as_ushort(__float2bfloat16_rn(yv));
}

bool aligned16(const void *q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; }

}  // namespace

// Batch-1 layer after the router.  Returns -1 when the shape is outside
// what this path handles (the caller then runs the batched chain).
extern "C" int jtk_moe_decode(const float *x, const float *logits, const float *bias, int32_t *ids, float *w,
                              const uint8_t *wg, const uint8_t *wu, const void *sg, const void *su,
                              const uint8_t *wd, const void *sd, const int8_t *wsg, const int8_t *wsu,
                              const float *ssg, const float *ssu, const int8_t *wsd, const float *ssd, int d,
                              int f, int E, int k, int S, int fs, int8_t *xq, float *xs, uint16_t *h,
                              uint16_t *hb_s, int32_t *acc_s,
                              int32_t *cnt_s, int32_t *perm, int32_t *pos, int32_t *off, int32_t *tile_off,
                              int32_t *meta, uint8_t *drop, float *w_fin, float *y, uint16_t *y_bf16,
                              cudaStream_t stream) {
    const int fs_eff = S > 0 ? fs : 128;
    if (d <= 0 || d > kMaxD || d % 128 || f <= 0 || f > kMaxF || f % 64 || E <= 0 || E > kMaxE || k <= 0 ||
        k > 64 || k > E || S < 0 || (S > 0 && (fs <= 0 || fs > kMaxF || fs % 128)))
        return -1;
    // bulk copies and 16-byte loads need 16-byte aligned bases
    if (!aligned16(x) || !aligned16(wg) || !aligned16(wu) || !aligned16(sg) || !aligned16(su) ||
        !aligned16(wd) || !aligned16(sd) ||
        !aligned16(h) ||
        (S > 0 && (!aligned16(wsg) || !aligned16(wsu) || !aligned16(wsd) || !aligned16(ssd) || !aligned16(hb_s))))
        return -1;
    const DnLayout L = dn_layout(k, f, S, fs_eff);
    if (L.total > kDnSmemMax) return -1;
    // the down kernel stages h in one pass of its 256 threads: at most 6
    // routed and 4 shared 16-byte chunks per thread
    if (k * (f / 8) > 6 * kDnWarps * 32 || S * fs_eff / 8 > 4 * kDnWarps * 32 || S > 8) return -1;
    DecParams p{};
    p.tma = d % 512 == 0;
    if (p.tma && (!jt::make_tmap_2d_u8(&p.tmG, wg, (uint64_t)(d / 4), (uint64_t)E * f, (uint64_t)(d / 4), 128, 64, true) ||
                  !jt::make_tmap_2d_u8(&p.tmU, wu, (uint64_t)(d / 4), (uint64_t)E * f, (uint64_t)(d / 4), 128, 64, true)))
        return -2;
    const size_t gu_smem = p.tma ? 128 * (size_t)(d / 4) + 1024 : 0;
    p.x = x;
    p.logits = logits;
    p.bias = bias;
    p.ids = ids;
    p.w = w;
    p.wg = wg;
    p.wu = wu;
    p.sg = static_cast<const __half *>(sg);
    p.su = static_cast<const __half *>(su);
    p.wd = wd;
    p.sd = static_cast<const __half *>(sd);
    p.wsg = wsg;
    p.wsu = wsu;
    p.ssg = ssg;
    p.ssu = ssu;
    p.wsd = wsd;
    p.ssd = ssd;
    p.d = d;
    p.f = f;
    p.E = E;
    p.k = k;
    p.S = S;
    p.fs = fs_eff;
    p.n_routed_units = k * (f / 64);
    // K parts of the largest of 1024, 512, 256, 128 bytes that divides d
    {
        int part = kSharedPartMax;
        while (d % part) part /= 2;
        p.ksplit = d / part;
    }
    p.acc_s = acc_s;
    p.cnt_s = cnt_s;
    p.xq = xq;
    p.xs = xs;
    p.h = h;
    p.hb_s = hb_s;
    p.perm = perm;
    p.pos = pos;
    p.off = off;
    p.tile_off = tile_off;
    p.meta = meta;
    p.drop = drop;
    p.w_fin = w_fin;
    p.y = y;
    p.y_bf16 = y_bf16;
    p.err = jtk_error_word();
    const int n_shared_units = S * (fs_eff / 64) * p.ksplit;
    static bool attr_set = false;
    if (!attr_set) {
        if (cudaFuncSetAttribute(k_dec_down, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kDnSmemMax) !=
                cudaSuccess ||
            cudaFuncSetAttribute(k_dec_gateup, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)(128 * (kMaxD / 4) + 1024)) != cudaSuccess)
            return -3;
        attr_set = true;
    }
    {
        cudaLaunchConfig_t gcfg{};
        gcfg.gridDim = dim3(p.n_routed_units + n_shared_units);
        gcfg.blockDim = dim3(kGuThreads);
        gcfg.dynamicSmemBytes = gu_smem;
        gcfg.stream = stream;
        cudaLaunchAttribute gattr[1];
        gattr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        gattr[0].val.programmaticStreamSerializationAllowed = 1;
        gcfg.attrs = gattr;
        gcfg.numAttrs = 1;
        if (cudaLaunchKernelEx(&gcfg, k_dec_gateup, p) != cudaSuccess) return -4;
    }
    // down: programmatic dependent launch, so its launch, routing and weight
    // copies overlap the gate/up grid (it waits on griddepcontrol.wait before
    // any read of that grid's results)
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((d + kDnWarps - 1) / kDnWarps);
    cfg.blockDim = dim3(kDnWarps * 32);
    cfg.dynamicSmemBytes = L.total;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, k_dec_down, p) != cudaSuccess) return -4;
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}
