// jt_route.cu - MoE routing on the GPU: top-k + softmax, the stable
// capacity sort with drop, the conditional renormalization, and the fused
// per-token quantization + dispatch that feeds the expert GEMMs.
//
//   k_route_topk     routing.c:16-76      (one warp per token)
//   k_sort_count     moe_layer.c:944-946  (per-chunk expert histograms)
//   k_sort_scan      moe_layer.c:931-954  (capacity, kept counts, offsets, GEMM tiles)
//   k_sort_scatter   moe_layer.c:955-970  (stable placement / drop) fused with
//                    the renormalization of moe_layer.c:1171-1201
//   k_quant_dispatch w8a8.c:688-747 per token + copy of each token's codes to
//                    its kept (token, slot) rows in expert order
//
// Integer results (ids, perm, off, drop) are bit-identical to the reference;
// the softmax uses double exp like routing.c:59-70.
#include <cuda_runtime.h>
#include <stdint.h>

#include "jt_internal.h"
#include "jt_quant.cuh"
#include "jt_topk.cuh"

namespace {

constexpr int kChunkTok = 64;  // tokens per sort chunk (chunks are token aligned)

// ------------------------------------------------------------------ top-k
// One warp per token (jt_topk.cuh).
__global__ void k_route_topk(const float *__restrict__ logits, const float *__restrict__ bias,
                             int T, int E, int k, int32_t *__restrict__ ids,
                             float *__restrict__ w, int *err) {
    const int warps = blockDim.x >> 5;
    const int t = blockIdx.x * warps + (threadIdx.x >> 5);
    if (t >= T) return;
    extern __shared__ __align__(16) uint32_t taken_all[];  // warps * topk_scratch_words(E)
    uint32_t *taken = taken_all + (threadIdx.x >> 5) * jt::topk_scratch_words(E);
    int32_t sel[64];
    float selv[64];
    jt::warp_topk_softmax(logits + (size_t)t * E, bias, E, k, taken, sel, selv, ids + (size_t)t * k,
                          w + (size_t)t * k, err);
}

// ------------------------------------------------------------------ sort
// hist[c][e] = number of pairs of chunk c routed to expert e.
__global__ void k_sort_count(const int32_t *__restrict__ ids, int T, int k, int E,
                             int32_t *__restrict__ hist, int *err) {
    extern __shared__ int32_t cnt[];
    const int c = blockIdx.x;
    for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    const int t0 = c * kChunkTok;
    const int t1 = min(T, t0 + kChunkTok);
    for (int q = t0 * k + threadIdx.x; q < t1 * k; q += blockDim.x) {
        const int e = ids[q];
        if (e < 0 || e >= E) {
            atomicExch(err, 0x83);
            continue;
        }
        atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) hist[(size_t)c * E + e] = cnt[e];
}

// One CTA.  base[c][e] = pairs of expert e in chunks < c; kept[e] =
// min(count, cap); off = exclusive scan of kept; tile_off = exclusive scan
// of ceil(kept/JT_TILE_ROWS) (token tiles of the expert GEMMs).
// meta[0] = kept total, meta[1] = total token tiles, meta[2] = max kept.
__global__ void k_sort_scan(int32_t *__restrict__ hist_base, int nchunks, int E, int cap,
                            const int32_t *__restrict__ gbase,
                            int32_t *__restrict__ off, int32_t *__restrict__ tile_off,
                            int32_t *__restrict__ meta) {
    extern __shared__ int32_t sm[];  // 2 * blockDim.x
    const int tid = threadIdx.x, nt = blockDim.x;
    const int per = (E + nt - 1) / nt;
    int kept_local[8];
    int ks = 0, ts = 0, mx = 0;
    for (int j = 0; j < per; ++j) {
        const int e = tid * per + j;
        int kc = 0;
        if (e < E) {
            // exclusive scan of the column over the chunks; sixteen loads
            // in flight at a time instead of one dependent round trip each
            int run = 0;
            int c = 0;
            for (; c + 16 <= nchunks; c += 16) {
                int h[16];
#pragma unroll
                for (int u = 0; u < 16; ++u) h[u] = hist_base[(size_t)(c + u) * E + e];
#pragma unroll
                for (int u = 0; u < 16; ++u) {
                    hist_base[(size_t)(c + u) * E + e] = run;  // becomes base[c][e]
                    run += h[u];
                }
            }
            for (; c < nchunks; ++c) {
                const int h = hist_base[(size_t)c * E + e];
                hist_base[(size_t)c * E + e] = run;
                run += h;
            }
            // gbase[e]: pairs of expert e ahead of this token range (other
            // ranks of an expert-parallel layer); they take capacity first
            const int cap_e = gbase ? max(cap - gbase[e], 0) : cap;
            kc = run < cap_e ? run : cap_e;
        }
        kept_local[j] = kc;
        ks += kc;
        ts += (kc + JT_TILE_ROWS - 1) / JT_TILE_ROWS;
        mx = kc > mx ? kc : mx;
    }
    sm[tid] = ks;
    sm[nt + tid] = ts;
    __syncthreads();
    // inclusive Hillis-Steele scans over threads (nt <= 1024)
    for (int o = 1; o < nt; o <<= 1) {
        int a = 0, b = 0;
        if (tid >= o) {
            a = sm[tid - o];
            b = sm[nt + tid - o];
        }
        __syncthreads();
        sm[tid] += a;
        sm[nt + tid] += b;
        __syncthreads();
    }
    int run_k = sm[tid] - ks, run_t = sm[nt + tid] - ts;
    for (int j = 0; j < per; ++j) {
        const int e = tid * per + j;
        if (e < E) {
            off[e] = run_k;
            tile_off[e] = run_t;
        }
        run_k += kept_local[j];
        run_t += (kept_local[j] + JT_TILE_ROWS - 1) / JT_TILE_ROWS;
    }
    if (tid == nt - 1) {
        off[E] = sm[tid];
        tile_off[E] = sm[nt + tid];
        meta[0] = sm[tid];
        meta[1] = sm[nt + tid];
    }
    // max kept per expert
    __syncthreads();
    sm[tid] = mx;
    __syncthreads();
    for (int o = nt / 2; o > 0; o >>= 1) {
        if (tid < o) sm[tid] = max(sm[tid], sm[tid + o]);
        __syncthreads();
    }
    if (tid == 0) meta[2] = sm[0];
}

// Token-tile table of the expert GEMMs: entry v = {expert, first row,
// expert's end row, 0} for the JT_TILE_ROWS-row tiles of every expert in order, so a
// GEMM CTA finds its tile with one load instead of a search.
__global__ void k_build_tiles(const int32_t *__restrict__ off, const int32_t *__restrict__ tile_off,
                              int E, int4 *__restrict__ tiles) {
    for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < E; e += gridDim.x * blockDim.x) {
        const int r0 = off[e], r1 = off[e + 1], t0 = tile_off[e];
        for (int j = 0; r0 + JT_TILE_ROWS * j < r1; ++j)
            tiles[t0 + j] = make_int4(e, r0 + JT_TILE_ROWS * j, r1, 0);
    }
}

// The JT_SUB_ROWS-row tiles of the tile table, in order: entry i of the
// table yields ceil(min(rows, JT_TILE_ROWS) / JT_SUB_ROWS) of them (a block
// scan of those counts, 1024 entries at a time, gives their positions).
__global__ void __launch_bounds__(1024) k_split_tiles(const int4 *__restrict__ tiles,
                                                     const int32_t *__restrict__ ntiles,
                                                     int4 *__restrict__ out, int32_t *__restrict__ nout) {
    __shared__ int sm[1024];
    __shared__ int carry;
    const int n = *ntiles, tid = threadIdx.x;
    if (tid == 0) carry = 0;
    __syncthreads();
    for (int b = 0; b < n; b += 1024) {
        const int i = b + tid;
        int4 te = make_int4(0, 0, 0, 0);
        int ns = 0;
        if (i < n) {
            te = tiles[i];
            ns = (min(te.z - te.y, JT_TILE_ROWS) + JT_SUB_ROWS - 1) / JT_SUB_ROWS;
        }
        sm[tid] = ns;
        __syncthreads();
        for (int o = 1; o < 1024; o <<= 1) {  // inclusive Hillis-Steele scan
            const int v = tid >= o ? sm[tid - o] : 0;
            __syncthreads();
            sm[tid] += v;
            __syncthreads();
        }
        const int pos = carry + sm[tid] - ns;
        for (int j = 0; j < ns; ++j) out[pos + j] = make_int4(te.x, te.y + JT_SUB_ROWS * j, te.z, 0);
        __syncthreads();  // every thread has read carry
        if (tid == 1023) carry += sm[1023];
        __syncthreads();
    }
    if (tid == 0) *nout = carry;
}

// One warp per chunk, pairs visited in q order 32 at a time; lanes routed
// to the same expert are ranked by __match_any_sync, so placement is the
// sequential scan of moe_layer.c:955-970.  Then renormalization of the
// chunk's tokens (moe_layer.c:1171-1201) with the final weights in wout.
__global__ void k_sort_scatter(const int32_t *__restrict__ ids, const float *__restrict__ win,
                               int T, int k, int E, int cap, const int32_t *__restrict__ gbase,
                               const int32_t *__restrict__ base, const int32_t *__restrict__ off,
                               int32_t *__restrict__ perm, int32_t *__restrict__ pos,
                               uint8_t *__restrict__ drop, float *__restrict__ wout, int *err) {
    extern __shared__ int32_t run[];  // E
    const int c = blockIdx.x, lane = threadIdx.x;
    for (int e = lane; e < E; e += 32) run[e] = 0;
    __syncwarp();
    const int t0 = c * kChunkTok, t1 = min(T, t0 + kChunkTok);
    const int q0 = t0 * k, q1 = t1 * k;
    for (int qb = q0; qb < q1; qb += 32) {
        const int q = qb + lane;
        const bool act = q < q1;
        int e = act ? ids[q] : -1 - lane;  // unique negative keys for idle lanes
        if (act && (e < 0 || e >= E)) {        // counted as an error by k_sort_count
            e = -1 - lane;
            if (act) {
                pos[q] = -1;
                drop[q] = 1;
            }
        }
        const bool valid = act && e >= 0;
        const unsigned same = __match_any_sync(0xffffffffu, e);
        const unsigned lt = (1u << lane) - 1u;
        int rank = 0;
        if (valid) rank = run[e] + __popc(same & lt);
        __syncwarp();
        if (valid && (same & lt) == 0) run[e] += __popc(same);  // group leader
        __syncwarp();
        if (valid) {
            const int g = base[(size_t)c * E + e] + rank;
            if (g < (gbase ? max(cap - gbase[e], 0) : cap)) {
                const int p = off[e] + g;
                perm[p] = q;
                pos[q] = p;
                drop[q] = 0;
            } else {
                pos[q] = -1;
                drop[q] = 1;
            }
        }
    }
    __syncwarp();
    for (int t = t0 + lane; t < t1; t += 32) {
        double s = 0.0;
        int nd = 0;
        for (int p = 0; p < k; ++p) {
            const size_t q = (size_t)t * k + p;
            if (drop[q]) nd++;
            else s += (double)win[q];
        }
        const bool rn = nd > 0 && s > 0.0;
        if (rn && !isfinite(s)) atomicExch(err, 0x84);
        for (int p = 0; p < k; ++p) {
            const size_t q = (size_t)t * k + p;
            float v = win[q];
            if (rn && !drop[q]) v = __double2float_rn(__ddiv_rn((double)v, s));
            wout[q] = v;
        }
    }
}

// ------------------------------------------------------------------ quant + dispatch
// One CTA per token: per-token int8 quantization of x (w8a8.c:688-747),
// written to xq[t] (shared experts) and to every kept (t, p) row of the
// expert-ordered activation matrix xd, with that row's metadata.
// Row metadata of the expert GEMMs, one 16-byte record per row:
// {activation scale, combine weight, token index (as bits), 0}.
__global__ void __launch_bounds__(256)
    k_quant_dispatch(const float *__restrict__ x, int T, int d, int k,
                     const int32_t *__restrict__ pos, const float *__restrict__ wfin,
                     int8_t *__restrict__ xq, float *__restrict__ xs, uint16_t *__restrict__ xd,
                     float4 *__restrict__ row_meta, float4 *__restrict__ sh_meta, int *err) {
    const int t = blockIdx.x;
    if (t >= T) return;
    const float *row = x + (size_t)t * d;
    __shared__ float wm[8];
    __shared__ int wb[8];
    __shared__ int sdst[64];
    // 16-byte loads when the row allows them (d % 8 == 0, x 16-byte aligned)
    const bool vec = (d % 8) == 0 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0;
    float m = 0.0f;
    int bad = 0;
    if (vec) {
        const float4 *row4 = reinterpret_cast<const float4 *>(row);
        for (int i = threadIdx.x; i < d / 4; i += blockDim.x) {
            const float4 v = __ldg(row4 + i);
            bad |= !isfinite(v.x) | !isfinite(v.y) | !isfinite(v.z) | !isfinite(v.w);
            m = fmaxf(fmaxf(m, fmaxf(fabsf(v.x), fabsf(v.y))), fmaxf(fabsf(v.z), fabsf(v.w)));
        }
    } else {
        for (int i = threadIdx.x; i < d; i += blockDim.x) {
            const float v = row[i];
            bad |= !isfinite(v);
            m = fmaxf(m, fabsf(v));
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        bad |= __shfl_xor_sync(0xffffffffu, bad, o);
    }
    if ((threadIdx.x & 31) == 0) {
        wm[threadIdx.x >> 5] = m;
        wb[threadIdx.x >> 5] = bad;
    }
    __syncthreads();
    m = 0.0f;
    bad = 0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) {
        m = fmaxf(m, wm[i]);
        bad |= wb[i];
    }
    const jt::QuantBlock qb = jt::quant_block(bad ? 0.0f : m);
    // Row metadata first: even on a rejected (non-finite) token every kept
    // row must name this token, so later kernels never index a stale token.
    int nd = 0;
    if (pos) {
        // the kept rows of this token, in slot order, shared by the CTA
        for (int p = 0; p < k; ++p) {
            const int ps = pos[(size_t)t * k + p];
            if (ps >= 0) {
                if (threadIdx.x == 0) sdst[nd] = ps;
                ++nd;
            }
        }
        if (threadIdx.x < k) {
            const int ps = pos[(size_t)t * k + threadIdx.x];
            if (ps >= 0)
                row_meta[ps] = make_float4(qb.scale_f, wfin[(size_t)t * k + threadIdx.x],
                                           __int_as_float(t), 0.0f);
        }
    }
    if (threadIdx.x == 0) {
        xs[t] = qb.scale_f;
        if (sh_meta) sh_meta[t] = make_float4(qb.scale_f, 1.0f, __int_as_float(t), 0.0f);
    }
    if (bad) {
        if (threadIdx.x == 0) atomicExch(err, 0x85);
        return;
    }
    __syncthreads();  // sdst
    // 16 codes per thread per step: xq in natural order, the kept rows xd as
    // exact fp16 values in the K order of the routed gate/up GEMM's INT2
    // unpack (jt::kX16Order)
    for (int i = threadIdx.x * 16; i < d; i += blockDim.x * 16) {
        float v[16];
        if (vec) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float4 a = __ldg(reinterpret_cast<const float4 *>(row + i + 4 * j));
                v[4 * j] = a.x;
                v[4 * j + 1] = a.y;
                v[4 * j + 2] = a.z;
                v[4 * j + 3] = a.w;
            }
        } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = row[i + j];
        }
        uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
        for (int j = 0; j < 16; ++j)
            w[j >> 2] |= (uint32_t)(uint8_t)(int8_t)jt::quant_code(v[j], qb) << (8 * (j & 3));
        *reinterpret_cast<uint4 *>(xq + (size_t)t * d + i) = make_uint4(w[0], w[1], w[2], w[3]);
        if (nd > 0) {
            uint4 lo, hi;
            jt::x16_block(w[0], w[1], w[2], w[3], lo, hi);
            for (int j = 0; j < nd; ++j) {
                uint4 *dst = reinterpret_cast<uint4 *>(xd + (size_t)sdst[j] * d + i);
                dst[0] = lo;
                dst[1] = hi;
            }
        }
    }
}

}  // namespace

extern "C" int jtk_route_topk(const float *logits, const float *bias, int T, int E, int k,
                              int32_t *ids, float *w, cudaStream_t stream) {
    if (T <= 0 || E <= 0 || k <= 0 || k > E || k > 64) return -1;
    const int warps = 4;
    const size_t sm = (size_t)warps * jt::topk_scratch_words(E) * sizeof(uint32_t);
    k_route_topk<<<(T + warps - 1) / warps, warps * 32, sm, stream>>>(logits, bias, T, E, k, ids,
                                                                      w, jtk_error_word());
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int jtk_sort_chunks(int T) { return (T + kChunkTok - 1) / kChunkTok; }

extern "C" int jtk_moe_sort(const int32_t *ids, const float *w_in, int T, int k, int E, int cap,
                            const int32_t *gbase,
                            int32_t *hist, int32_t *off, int32_t *tile_off, int4 *tiles,
                            int32_t *meta, int32_t *perm, int32_t *pos, uint8_t *drop,
                            float *w_out, cudaStream_t stream) {
    if (T <= 0 || k <= 0 || E <= 0 || E > 4096 || cap <= 0) return -1;
    const int nch = jtk_sort_chunks(T);
    int *err = jtk_error_word();
    k_sort_count<<<nch, 256, (size_t)E * sizeof(int32_t), stream>>>(ids, T, k, E, hist, err);
    int nt = 1024;
    while (nt / 2 >= E && nt > 32) nt /= 2;
    k_sort_scan<<<1, nt, 2 * nt * sizeof(int32_t), stream>>>(hist, nch, E, cap, gbase, off, tile_off,
                                                             meta);
    k_build_tiles<<<(E + 255) / 256, 256, 0, stream>>>(off, tile_off, E, tiles);
    k_sort_scatter<<<nch, 32, (size_t)E * sizeof(int32_t), stream>>>(
        ids, w_in, T, k, E, cap, gbase, hist, off, perm, pos, drop, w_out, err);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int jtk_split_tiles(const int4 *tiles, const int32_t *ntiles, int4 *out, int32_t *nout,
                               cudaStream_t stream) {
    k_split_tiles<<<1, 1024, 0, stream>>>(tiles, ntiles, out, nout);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int jtk_build_tiles(const int32_t *off, const int32_t *tile_off, int E, int4 *tiles,
                               cudaStream_t stream) {
    if (E <= 0) return -1;
    k_build_tiles<<<(E + 255) / 256, 256, 0, stream>>>(off, tile_off, E, tiles);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int jtk_quant_dispatch(const float *x, int T, int d, int k, const int32_t *pos,
                                  const float *wfin, int8_t *xq, float *xs, uint16_t *xd,
                                  float4 *row_meta, float4 *sh_meta, cudaStream_t stream) {
    if (T <= 0 || d <= 0 || (d % 16) != 0 || k > 64) return -1;
    // one thread per 16 codes of the row where that fits in 64..256 threads
    // (every thread busy in the quantize-and-store phase); at least k
    // threads, which write the row metadata
    int thr = d / 16;
    thr = thr < 64 ? 64 : (thr > 256 ? 256 : thr);
    thr = (thr + 31) & ~31;
    k_quant_dispatch<<<T, thr, 0, stream>>>(x, T, d, k, pos, wfin, xq, xs, xd, row_meta, sh_meta,
                                            jtk_error_word());
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}
