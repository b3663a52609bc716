// jt_decode.cu - batch-1 (T = 1) path of the prepared MoE layer.
//
// One token selects k distinct experts and every expert's capacity is at
// least one pair (cap = ceil(cap_factor * k / E) >= 1), so nothing is
// dropped, the routing weights are final and the expert GEMMs degenerate to
// matrix-vector products over the selected experts' rows.  The batched
// chain (sort, dispatch, persistent tensor-core kernels per projection)
// spends its time in launches and pipeline fill at this size; this path is
// two kernels after the router:
//
//   k_dec_gateup  one CTA per (expert slot, 64-channel block): quantizes the
//                 token (w8a8.c:688-747), computes the 64 gate and 64 up rows
//                 (INT2 group-64 with the same fp32 fold as the grouped
//                 kernel, or int8 rows of a shared expert), SwiGLU
//                 (moe_layer.c:146-148) and the per-64-channel requantization
//                 of h; CTA 0 also writes the sort results (perm, pos, off,
//                 drop, kept) the batched path would produce for one token.
//   k_dec_down    one warp per output channel: the down rows of every
//                 selected expert (INT4 group-64 fold, or int8 rows of a
//                 shared expert with the activation group scales) and the
//                 combine in double in slot order, then the shared experts
//                 (moe_layer.c:1443-1463, :1549-1559), fp32 or bf16 out.
//
// Integer dot products use dp4a on codes taken from the packed words in
// place: for an INT2 word (16 codes, byte b holds k0+4b .. k0+4b+3), the
// j-th 2-bit field of every byte is the code of k0+4b+j, so it pairs with
// the activation word {x[k0+j], x[k0+4+j], x[k0+8+j], x[k0+12+j]}; the
// signed code c = 2 li - (2^bits - 1) enters as 2 dot(li, x) - (2^bits - 1)
// sum(x) over the 64-element group.
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

constexpr int kMaxD = 4096;    // token width handled (d <= 4096)
constexpr int kMaxF = 4096;    // expert ffn handled (f, fs <= 4096)
constexpr int kMaxE = 4096;    // experts
constexpr int kGuThreads = 512;

struct DecParams {
    const float *x;          // [d] token row
    const float *logits;     // [E] router logits
    const float *bias;       // [E] or NULL
    int32_t *ids;            // [k] selected experts (slot order), written by CTA (0, 0)
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
    int hs_ld, hs_ld_s;      // row strides of the h scales (routed, shared)
    // outputs of the gate/up kernel (and debug copies of the batched path)
    int8_t *xq;
    float *xs;
    int8_t *hq;              // [k][f] routed h codes, rows in expert order
    float *hs;               // [k][hs_ld]
    int8_t *hq_s;            // [S][fs]
    float *hs_s;             // [S][hs_ld_s]
    int32_t *perm, *pos, *off, *tile_off, *meta;
    uint8_t *drop;
    float *w_fin;
    // down output
    float *y;                // [d] fp32 (or NULL)
    uint16_t *y_bf16;        // [d] bf16 (or NULL)
    int *err;
};

// Per-token int8 quantization of x (w8a8.c:688-747, as k_quant_dispatch):
// codes into sx (shared memory), scale returned; a non-finite value raises
// the error word and gives an all-zero row.  With `route`, warp 0 runs the
// router (jt_topk.cuh, results in sids / sw) while the other warps take the
// max-abs pass, so the two latencies overlap.
__device__ float quant_token(const float *__restrict__ x, int d, int8_t *sx, int *err, bool route,
                             const DecParams &p, uint32_t *taken, int32_t *ssel, float *sselv, int32_t *sids,
                             float *sw) {
    __shared__ float wm[kGuThreads / 32];
    __shared__ int wb[kGuThreads / 32];
    const int warp = threadIdx.x >> 5;
    float m = 0.0f;
    int bad = 0;
    if (route && warp == 0) {
        sids[threadIdx.x] = threadIdx.x;  // fallback: experts 0..31 (k <= 64 below)
        sids[threadIdx.x + 32] = threadIdx.x + 32;
        sw[threadIdx.x] = 0.0f;
        sw[threadIdx.x + 32] = 0.0f;
        __syncwarp();
        // the experts only: the weights are needed by the down kernel, which
        // computes them itself before it waits for this grid
        jt::warp_topk_softmax(p.logits, p.bias, p.E, p.k, taken, ssel, sselv, sids, sw, err, false);
    } else {
        const int t0 = route ? threadIdx.x - 32 : threadIdx.x;
        const int nt = route ? blockDim.x - 32 : blockDim.x;
        for (int i = t0; i < d; i += nt) {
            const float v = x[i];
            bad |= !isfinite(v);
            m = fmaxf(m, fabsf(v));
        }
        for (int o = 16; o > 0; o >>= 1) {
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            bad |= __shfl_xor_sync(0xffffffffu, bad, o);
        }
    }
    if ((threadIdx.x & 31) == 0) {
        wm[warp] = m;
        wb[warp] = bad;
    }
    __syncthreads();
    m = 0.0f;
    bad = 0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) {
        m = fmaxf(m, wm[i]);
        bad |= wb[i];
    }
    const jt::QuantBlock qb = jt::quant_block(bad ? 0.0f : m);
    if (bad && threadIdx.x == 0) atomicExch(err, 0x85);
    for (int i = threadIdx.x; i < d; i += blockDim.x) sx[i] = bad ? 0 : (int8_t)jt::quant_code(x[i], qb);
    __syncthreads();
    return qb.scale_f;
}

// Activation words permuted for INT2 words: xp[4w + j] = bytes
// {x[16w+j], x[16w+4+j], x[16w+8+j], x[16w+12+j]}; gsum[g] = sum of the 64
// codes of group g.
__device__ void permute_int2(const int8_t *sx, int d, uint32_t *xp, int *gsum) {
    for (int i = threadIdx.x; i < d / 4; i += blockDim.x) {
        const int w = i >> 2, j = i & 3;
        const uint8_t *b = reinterpret_cast<const uint8_t *>(sx) + 16 * w + j;
        xp[i] = (uint32_t)b[0] | ((uint32_t)b[4] << 8) | ((uint32_t)b[8] << 16) | ((uint32_t)b[12] << 24);
    }
    for (int g = threadIdx.x; g < d / 64; g += blockDim.x) {
        int s = 0;
        for (int i = 0; i < 64; ++i) s += sx[64 * g + i];
        gsum[g] = s;
    }
    __syncthreads();
}

// RB INT2 rows (d/4 packed bytes each, fp16 scales srow[i][g * sstride])
// against the permuted activation, all rows' loads in flight together.  Per
// row the fold r = fmaf((float)P_g, s_g, r) runs over the groups in
// ascending order, identically in every lane.  Lane l takes 8-byte chunks
// l, l+32, ... (chunk c covers half of group c/2) and, per pass of 32
// chunks, the scale of group g0 + l for l < 16.
template <int RB>
__device__ __forceinline__ void rows_int2(const uint8_t *const (&row)[RB], const __half *const (&srow)[RB],
                                          int sstride, int d, const uint32_t *xp, const int *gsum, int lane,
                                          float (&r)[RB]) {
    const int nchunk = d / 32;
    const int ng = d / 64;
#pragma unroll
    for (int i = 0; i < RB; ++i) r[i] = 0.0f;
    for (int c0 = 0; c0 < nchunk; c0 += 32) {
        const int c = c0 + lane, g0 = c0 / 2;
        uint2 wv[RB];
        float sv[RB];
#pragma unroll
        for (int i = 0; i < RB; ++i) {
            wv[i] = c < nchunk ? __ldg(reinterpret_cast<const uint2 *>(row[i]) + c) : make_uint2(0u, 0u);
            sv[i] = (lane < 16 && g0 + lane < ng) ? __half2float(srow[i][(size_t)(g0 + lane) * sstride]) : 0.0f;
        }
        int part[RB];
#pragma unroll
        for (int i = 0; i < RB; ++i) {
            part[i] = 0;
            const uint32_t *xw = xp + 8 * (c < nchunk ? c : 0);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                part[i] = __dp4a((int)((wv[i].x >> (2 * j)) & 0x03030303u), (int)xw[j], part[i]);
                part[i] = __dp4a((int)((wv[i].y >> (2 * j)) & 0x03030303u), (int)xw[4 + j], part[i]);
            }
            part[i] += __shfl_xor_sync(0xffffffffu, part[i], 1);  // the two halves of a group
        }
        for (int gi = 0; gi < 16 && g0 + gi < ng; ++gi) {
            const int gs = 3 * gsum[g0 + gi];
#pragma unroll
            for (int i = 0; i < RB; ++i) {
                const int P = 2 * __shfl_sync(0xffffffffu, part[i], 2 * gi) - gs;
                r[i] = fmaf((float)P, __shfl_sync(0xffffffffu, sv[i], gi), r[i]);
            }
        }
    }
}

// RB int8 rows of K = d bytes: exact int32 dots, reduced over the warp.
template <int RB>
__device__ __forceinline__ void rows_int8(const int8_t *const (&row)[RB], int d, const int8_t *sx, int lane,
                                          int (&acc)[RB]) {
#pragma unroll
    for (int i = 0; i < RB; ++i) acc[i] = 0;
    for (int k0 = lane * 16; k0 < d; k0 += 32 * 16) {
        int4 wv[RB];
#pragma unroll
        for (int i = 0; i < RB; ++i) wv[i] = __ldg(reinterpret_cast<const int4 *>(row[i] + k0));
        const int4 xv = *reinterpret_cast<const int4 *>(sx + k0);
#pragma unroll
        for (int i = 0; i < RB; ++i) {
            acc[i] = __dp4a(wv[i].x, xv.x, acc[i]);
            acc[i] = __dp4a(wv[i].y, xv.y, acc[i]);
            acc[i] = __dp4a(wv[i].z, xv.z, acc[i]);
            acc[i] = __dp4a(wv[i].w, xv.w, acc[i]);
        }
    }
#pragma unroll
    for (int i = 0; i < RB; ++i)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
}


// Sorted row of slot p: experts ascending, as the capacity sort orders the
// kept pairs of one token.
__device__ __forceinline__ int slot_rank(const int32_t *ids, int k, int p) {
    const int e = ids[p];
    int r = 0;
    for (int q = 0; q < k; ++q) r += ids[q] < e;
    return r;
}

// grid (max(f, fs)/64, k + S), 256 threads.  blockIdx.y < k: routed slot,
// else shared expert blockIdx.y - k.
__global__ void __launch_bounds__(kGuThreads) k_dec_gateup(const __grid_constant__ DecParams p) {
    __shared__ __align__(16) int8_t sx[kMaxD];
    __shared__ __align__(16) uint32_t xp[kMaxD / 4];
    __shared__ int gsum[kMaxD / 64];
    __shared__ float gu[2][64];
    __shared__ uint32_t taken[kMaxE / 32];
    __shared__ int32_t sids[64], ssel[64];
    __shared__ float sw[64], sselv[64];
    const int slot = blockIdx.y, cb = blockIdx.x;
    const bool shared = slot >= p.k;
    const int n_ch = shared ? p.fs : p.f;
    // the down kernel may launch now; it waits for this grid before reading
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // this grid is itself launched as a dependent of the previous kernel of
    // the stream (the previous token's down kernel in a decode loop): wait
    // for it before touching global memory (it reads hq/hs, written below)
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (cb * 64 >= n_ch) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // routed CTAs: the router (every routed CTA alike, jt_topk.cuh) overlaps
    // the max-abs pass; on a NaN logit or a bad softmax (error word raised)
    // the slots fall back to experts 0..k-1 with zero weight so every index
    // stays in range
    const float xs = quant_token(p.x, p.d, sx, p.err, !shared, p, taken, ssel, sselv, sids, sw);
    int e = 0;
    if (!shared) {
        e = sids[slot];
        if (slot == 0 && cb == 0 && threadIdx.x < p.k) p.ids[threadIdx.x] = sids[threadIdx.x];
    }
    if (!shared) permute_int2(sx, p.d, xp, gsum);
    // 128 rows: 0..63 gate, 64..127 up of channels cb*64 + (row & 63); each
    // warp takes kRB consecutive rows per step
    constexpr int kRB = 8;
    for (int r0 = warp * kRB; r0 < 128; r0 += (kGuThreads / 32) * kRB) {
        const bool up = r0 >= 64;
        const int c0 = cb * 64 + (r0 & 63);
        float v[kRB];
        if (!shared) {
            const uint8_t *wrow[kRB];
            const __half *srow[kRB];
#pragma unroll
            for (int i = 0; i < kRB; ++i) {
                wrow[i] = (up ? p.wu : p.wg) + ((size_t)e * p.f + c0 + i) * (p.d / 4);
                srow[i] = (up ? p.su : p.sg) + (size_t)e * (p.d / 64) * p.f + c0 + i;
            }
            float r[kRB];
            rows_int2<kRB>(wrow, srow, p.f, p.d, xp, gsum, lane, r);
#pragma unroll
            for (int i = 0; i < kRB; ++i) v[i] = __fmul_rn(r[i], xs);
        } else {
            const int s = slot - p.k;
            const int8_t *wrow[kRB];
#pragma unroll
            for (int i = 0; i < kRB; ++i) wrow[i] = (up ? p.wsu : p.wsg) + ((size_t)s * p.fs + c0 + i) * p.d;
            int acc[kRB];
            rows_int8<kRB>(wrow, p.d, sx, lane, acc);
#pragma unroll
            for (int i = 0; i < kRB; ++i) {
                const float cs = (up ? p.ssu : p.ssg)[(size_t)s * p.fs + c0 + i];
                v[i] = __fmul_rn(__fmul_rn(__int2float_rn(acc[i]), xs), cs);
            }
        }
        if (lane == 0)
#pragma unroll
            for (int i = 0; i < kRB; ++i) gu[up][(r0 & 63) + i] = v[i];
    }
    __syncthreads();
    if (warp == 0) {
        // h = SwiGLU(g, u) of channels 2l, 2l+1, requantized per 64 channels
        const float h0 = jt::swiglu(gu[0][2 * lane], gu[1][2 * lane]);
        const float h1 = jt::swiglu(gu[0][2 * lane + 1], gu[1][2 * lane + 1]);
        const bool bad = !isfinite(h0) || !isfinite(h1);
        float m = fmaxf(fabsf(h0), fabsf(h1));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (__any_sync(0xffffffffu, bad) && lane == 0) atomicExch(p.err, JT_KERR_NONFINITE);
        const jt::QuantBlockF qb = jt::quant_block_f(m);
        const int q0 = jt::quant_code_f(h0, qb), q1 = jt::quant_code_f(h1, qb);
        const uint16_t pair = (uint16_t)(uint8_t)(int8_t)q0 | ((uint16_t)(uint8_t)(int8_t)q1 << 8);
        int8_t *hq;
        float *hs;
        if (!shared) {
            const int row = slot_rank(sids, p.k, slot);
            hq = p.hq + (size_t)row * p.f;
            hs = p.hs + (size_t)row * p.hs_ld;
        } else {
            const int s = slot - p.k;
            hq = p.hq_s + (size_t)s * p.fs;
            hs = p.hs_s + (size_t)s * p.hs_ld_s;
        }
        *reinterpret_cast<uint16_t *>(hq + cb * 64 + 2 * lane) = pair;
        if (lane == 0) hs[cb] = qb.scale_f;
    }
    if (slot == 0 && cb == 0) {
        // the batched path's per-token results for one token
        for (int i = threadIdx.x; i < p.d; i += blockDim.x) p.xq[i] = sx[i];
        if (threadIdx.x == 0) {
            p.xs[0] = xs;
            p.meta[0] = p.k;
            p.meta[1] = p.k;
            p.meta[2] = 1;
        }
        if (threadIdx.x < p.k) {
            const int q = threadIdx.x;
            const int row = slot_rank(sids, p.k, q);
            p.perm[row] = q;
            p.pos[q] = row;
            p.drop[q] = 0;
        }
        for (int ex = threadIdx.x; ex <= p.E; ex += blockDim.x) {
            int n = 0;
            for (int q = 0; q < p.k; ++q) n += sids[q] < ex;
            p.off[ex] = n;
            p.tile_off[ex] = n;
        }
    }
}


constexpr int kDnWarps = 8;
constexpr int kMaxHp = 8192;  // permuted h words of the routed rows (k * f <= 32768)

// grid d / 8, 256 threads: warp w computes output channel blockIdx.x*8 + w.
__global__ void __launch_bounds__(kDnWarps * 32) k_dec_down(const __grid_constant__ DecParams p) {
    // the next token's gate/up kernel may launch on the SMs left free; it
    // waits for this grid before its first global access
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    __shared__ uint32_t taken[kMaxE / 32];
    __shared__ int32_t sids[64], ssel[64];
    __shared__ float sw[64], sselv[64];
    {
        // Everything here is independent of the gate/up grid, which may still
        // be running: the router again (the same function on the same
        // logits, so the same experts as the gate/up grid), then the down
        // rows this warp will read are pulled into L2.
        if (threadIdx.x < 64) {
            sids[threadIdx.x] = threadIdx.x;
            sw[threadIdx.x] = 0.0f;
        }
        __syncthreads();
        if ((threadIdx.x >> 5) == 0)
            jt::warp_topk_softmax(p.logits, p.bias, p.E, p.k, taken, ssel, sselv, sids, sw, p.err);
        __syncthreads();
        // the routing weights (final: nothing is dropped for one token); the
        // gate/up grid neither reads nor writes them
        if (blockIdx.x == 0 && threadIdx.x < p.k) {
            p.w[threadIdx.x] = sw[threadIdx.x];
            p.w_fin[threadIdx.x] = sw[threadIdx.x];
        }
        const int o = blockIdx.x * kDnWarps + (threadIdx.x >> 5);
        const int lane = threadIdx.x & 31;
        if (o < p.d) {
            const int gf = p.f / 64;
            for (int q = 0; q < p.k; ++q) {
                int e = sids[q];
                e = (e < 0 || e >= p.E) ? 0 : e;
                const uint8_t *row = p.wd + ((size_t)e * p.d + o) * (p.f / 2);
                for (int b = lane * 128; b < p.f / 2; b += 32 * 128)
                    asm volatile("prefetch.global.L2 [%0];" ::"l"(row + b));
                if (lane < gf)
                    asm volatile("prefetch.global.L2 [%0];" ::"l"(p.sd + ((size_t)e * gf + lane) * p.d + o));
            }
            for (int s = 0; s < p.S; ++s)
                for (int b = lane * 128; b < p.fs; b += 32 * 128)
                    asm volatile("prefetch.global.L2 [%0];" ::"l"(p.wsd + ((size_t)s * p.d + o) * p.fs + b));
        }
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // routed h rows (sorted rank order) permuted for INT4 words: for packed
    // word w (codes 8w .. 8w+7, even k in the low nibbles) hp[2w] holds the
    // even codes {h[8w], h[8w+2], h[8w+4], h[8w+6]} and hp[2w+1] the odd ones
    __shared__ uint32_t hp[kMaxHp];
    __shared__ int hsum[kMaxHp / 16];  // per (row, 64-group) sum of codes
    const int nw = p.f / 8;            // packed INT4 words per row
    const int gf = p.f / 64;
    for (int i = threadIdx.x; i < p.k * nw; i += blockDim.x) {
        const int r = i / nw, w = i % nw;
        const uint8_t *b = reinterpret_cast<const uint8_t *>(p.hq) + (size_t)r * p.f + 8 * w;
        hp[2 * i] = (uint32_t)b[0] | ((uint32_t)b[2] << 8) | ((uint32_t)b[4] << 16) | ((uint32_t)b[6] << 24);
        hp[2 * i + 1] = (uint32_t)b[1] | ((uint32_t)b[3] << 8) | ((uint32_t)b[5] << 16) | ((uint32_t)b[7] << 24);
    }
    for (int i = threadIdx.x; i < p.k * gf; i += blockDim.x) {
        const int8_t *h = p.hq + (size_t)(i / gf) * p.f + 64 * (i % gf);
        int sm = 0;
        for (int j = 0; j < 64; ++j) sm += h[j];
        hsum[i] = sm;
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int o = blockIdx.x * kDnWarps + warp;
    if (o >= p.d) return;
    double ya = 0.0;
    // routed pairs in slot order (moe_layer.c:1443-1463), eight rows' loads
    // in flight at a time
    constexpr int kRB = 8;
    for (int q0 = 0; q0 < p.k; q0 += kRB) {
        const uint32_t *row[kRB];
        const __half *sdo[kRB];
        const float *hsr[kRB];
        int rr[kRB];
        float acc[kRB];
#pragma unroll
        for (int i = 0; i < kRB; ++i) {
            const int q = q0 + i < p.k ? q0 + i : p.k - 1;
            int e = sids[q];
            e = (e < 0 || e >= p.E) ? 0 : e;
            rr[i] = p.pos[q];
            row[i] = reinterpret_cast<const uint32_t *>(p.wd + ((size_t)e * p.d + o) * (p.f / 2));
            sdo[i] = p.sd + (size_t)e * gf * p.d + o;
            hsr[i] = p.hs + (size_t)rr[i] * p.hs_ld;
            acc[i] = 0.0f;
        }
        for (int c0 = 0; c0 < nw; c0 += 32) {  // 4-byte chunks, 8 per group
            const int c = c0 + lane, g0 = c0 / 8;
            uint32_t wv[kRB];
            float sv[kRB], hv[kRB];
#pragma unroll
            for (int i = 0; i < kRB; ++i) {
                wv[i] = c < nw ? __ldg(row[i] + c) : 0u;
                const bool gl = lane < 4 && g0 + lane < gf;
                sv[i] = gl ? __half2float(sdo[i][(size_t)(g0 + lane) * p.d]) : 0.0f;
                hv[i] = gl ? hsr[i][g0 + lane] : 0.0f;
            }
            int part[kRB];
#pragma unroll
            for (int i = 0; i < kRB; ++i) {
                const uint32_t *hw = hp + 2 * ((size_t)rr[i] * nw + (c < nw ? c : 0));
                part[i] = __dp4a((int)(wv[i] & 0x0F0F0F0Fu), (int)hw[0], 0);
                part[i] = __dp4a((int)((wv[i] >> 4) & 0x0F0F0F0Fu), (int)hw[1], part[i]);
                part[i] += __shfl_xor_sync(0xffffffffu, part[i], 1);
                part[i] += __shfl_xor_sync(0xffffffffu, part[i], 2);
                part[i] += __shfl_xor_sync(0xffffffffu, part[i], 4);
            }
            for (int gi = 0; gi < 4 && g0 + gi < gf; ++gi) {
#pragma unroll
                for (int i = 0; i < kRB; ++i) {
                    const int P = 2 * __shfl_sync(0xffffffffu, part[i], 8 * gi) - 15 * hsum[rr[i] * gf + g0 + gi];
                    const float t = __fmul_rn((float)P, __shfl_sync(0xffffffffu, sv[i], gi));
                    acc[i] = fmaf(t, __shfl_sync(0xffffffffu, hv[i], gi), acc[i]);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < kRB; ++i)
            if (q0 + i < p.k) ya = __dadd_rn(ya, __dmul_rn((double)sw[q0 + i], (double)acc[i]));
    }
    // shared experts in s order (moe_layer.c:1549-1559)
    for (int s = 0; s < p.S; ++s) {
        const int8_t *row = p.wsd + ((size_t)s * p.d + o) * p.fs;
        const int8_t *h = p.hq_s + (size_t)s * p.fs;
        const float *hss = p.hs_s + (size_t)s * p.hs_ld_s;
        const int nb = p.fs / 64;
        float acc = 0.0f;
        for (int c0 = 0; c0 < p.fs / 4; c0 += 32) {  // 4-byte chunks, 16 per block
            const int c = c0 + lane;
            int part = 0;
            if (c < p.fs / 4)
                part = __dp4a(__ldg(reinterpret_cast<const int *>(row) + c), __ldg(reinterpret_cast<const int *>(h) + c), 0);
#pragma unroll
            for (int m = 1; m < 16; m <<= 1) part += __shfl_xor_sync(0xffffffffu, part, m);
            const int b0 = c0 / 16;
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                if (b0 + i >= nb) break;
                const int P = __shfl_sync(0xffffffffu, part, 16 * i);
                acc = fmaf((float)P, hss[b0 + i], acc);
            }
        }
        ya = __dadd_rn(ya, (double)__fmul_rn(acc, p.ssd[(size_t)s * p.d + o]));
    }
    if (lane == 0) {
        const float yv = (float)ya;
        if (p.y) p.y[o] = yv;
        if (p.y_bf16) p.y_bf16[o] = __bfloat16_as_ushort(__float2bfloat16_rn(yv));
    }
}

}  // namespace

// Batch-1 layer after the router.  Returns -1 when the shape is outside
// what this path handles (the caller then runs the batched chain).
extern "C" int jtk_moe_decode(const float *x, const float *logits, const float *bias, int32_t *ids, float *w,
                              const uint8_t *wg, const uint8_t *wu, const void *sg, const void *su,
                              const uint8_t *wd, const void *sd, const int8_t *wsg, const int8_t *wsu,
                              const float *ssg, const float *ssu, const int8_t *wsd, const float *ssd, int d,
                              int f, int E, int k, int S, int fs, int8_t *xq, float *xs, int8_t *hq, float *hs,
                              int hs_ld, int8_t *hq_s, float *hs_s, int hs_ld_s, int32_t *perm, int32_t *pos,
                              int32_t *off, int32_t *tile_off, int32_t *meta, uint8_t *drop, float *w_fin,
                              float *y, uint16_t *y_bf16, cudaStream_t stream) {
    if (d <= 0 || d > kMaxD || d % 128 || f <= 0 || f > kMaxF || f % 64 || E <= 0 || E > kMaxE || k <= 0 ||
        k > 64 || k > E || (long long)k * (f / 8) * 2 > kMaxHp || (long long)k * (f / 64) > kMaxHp / 16 ||
        S < 0 || (S > 0 && (fs <= 0 || fs > kMaxF || fs % 64)))
        return -1;
    DecParams p{};
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
    p.fs = S > 0 ? fs : 64;
    p.hs_ld = hs_ld;
    p.hs_ld_s = hs_ld_s;
    p.xq = xq;
    p.xs = xs;
    p.hq = hq;
    p.hs = hs;
    p.hq_s = hq_s;
    p.hs_s = hs_s;
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
    const int nmax = (S > 0 && fs > f) ? fs : f;
    {
        cudaLaunchConfig_t gcfg{};
        gcfg.gridDim = dim3(nmax / 64, k + S);
        gcfg.blockDim = dim3(kGuThreads);
        gcfg.dynamicSmemBytes = 0;
        gcfg.stream = stream;
        cudaLaunchAttribute gattr[1];
        gattr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        gattr[0].val.programmaticStreamSerializationAllowed = 1;
        gcfg.attrs = gattr;
        gcfg.numAttrs = 1;
        if (cudaLaunchKernelEx(&gcfg, k_dec_gateup, p) != cudaSuccess) return -4;
    }
    if (cudaGetLastError() != cudaSuccess) return -4;
    // down: programmatic dependent launch, so its launch and prologue overlap
    // the gate/up grid (it waits on griddepcontrol.wait before any read of
    // that grid's results)
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((d + kDnWarps - 1) / kDnWarps);
    cfg.blockDim = dim3(kDnWarps * 32);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, k_dec_down, p) != cudaSuccess) return -4;
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}
