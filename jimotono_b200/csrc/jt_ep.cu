// jt_ep.cu - device kernels of the expert-parallel MoE layer (the exchange
// steps around the expert GEMMs; the NCCL calls and the bookkeeping are in
// jt_ep.c / jt_ep_layout.c).
#include <cuda_runtime.h>
#include <stdint.h>

#include "jt_internal.h"
#include "jt_quant.cuh"

namespace {

// cnt[e] += number of (token, slot) pairs routed to expert e (cnt zeroed).
__global__ void k_ep_count(const int32_t *__restrict__ ids, int n, int E, int32_t *__restrict__ cnt) {
    extern __shared__ int32_t c[];
    for (int e = threadIdx.x; e < E; e += blockDim.x) c[e] = 0;
    __syncthreads();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const int e = ids[i];
        if (e >= 0 && e < E) atomicAdd(&c[e], 1);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x)
        if (c[e]) atomicAdd(&cnt[e], c[e]);
}

// Token rows.  A token goes to an owner once, whatever number of its slots
// that owner's experts hold; the owner sums the weighted down-projection
// rows of those slots into one returned row.  trow[t*N + o] = position of
// token t among this rank's tokens with a routed slot on owner o (ascending
// t), or -1; ntok[o] = their number.  One CTA per owner; a block-wide scan
// over the tokens in chunks of blockDim.x.
__global__ void k_ep_tokens(const int32_t *__restrict__ ids, int T, int k, int El, int N,
                            int32_t *__restrict__ trow, int32_t *__restrict__ ntok) {
    __shared__ int32_t wsum[32];
    const int o = blockIdx.x;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int base = 0;
    for (int t0 = 0; t0 < T; t0 += blockDim.x) {
        const int t = t0 + threadIdx.x;
        int has = 0;
        if (t < T)
            for (int p = 0; p < k; ++p) {
                const int e = ids[(size_t)t * k + p];
                has |= (e >= 0 && e / El == o);
            }
        const unsigned bal = __ballot_sync(0xffffffffu, has);
        const int in_warp = __popc(bal & ((1u << lane) - 1u));
        if (lane == 0) wsum[wid] = __popc(bal);
        __syncthreads();
        int before = 0, total = 0;
        for (int i = 0; i < nw; ++i) {
            const int c = wsum[i];
            before += (i < wid) ? c : 0;
            total += c;
        }
        if (t < T) trow[(size_t)t * N + o] = has ? base + before + in_warp : -1;
        base += total;
        __syncthreads();
    }
    if (threadIdx.x == 0) ntok[o] = base;
}

// Send buffers of token t: its int8 codes once per owner it has a slot on
// (row tsoff[o] + trow[t][o] of send_tok), and the metadata of each kept
// pair at its send position: {token scale, combine weight, token row at the
// owner (trow), 0}.
__global__ void k_ep_pack(const int8_t *__restrict__ xq, const float *__restrict__ xs, int T, int d,
                          int k, int El, int N, const int32_t *__restrict__ ids,
                          const int32_t *__restrict__ pos, const float *__restrict__ wfin,
                          const int32_t *__restrict__ trow, const int32_t *__restrict__ tsoff,
                          int8_t *__restrict__ send_tok, float4 *__restrict__ row_meta) {
    const int t = blockIdx.x;
    if (t >= T) return;
    if (threadIdx.x < k) {
        const int q = t * k + threadIdx.x;
        const int ps = pos[q];
        if (ps >= 0) {
            const int o = ids[q] / El;
            row_meta[ps] = make_float4(xs[t], wfin[q], __int_as_float(trow[(size_t)t * N + o]), 0.0f);
        }
    }
    const uint4 *src = reinterpret_cast<const uint4 *>(xq + (size_t)t * d);
    const int nv = d / 16;
    for (int o = 0; o < N; ++o) {
        const int r = trow[(size_t)t * N + o];
        if (r < 0) continue;
        uint4 *dst = reinterpret_cast<uint4 *>(send_tok + (size_t)(tsoff[o] + r) * d);
        for (int i = threadIdx.x; i < nv; i += blockDim.x) dst[i] = src[i];
    }
}

// One CTA per (source, expert) block of received pairs: each pair's token
// row (received once per token) is copied to the pair's expert-contiguous
// row; the metadata's third field becomes the received token row, which is
// where the down projection adds that pair's weighted output.
__global__ void k_ep_gather(const int4 *__restrict__ ent, const int8_t *__restrict__ rtok,
                            const float4 *__restrict__ src_meta, int d, uint16_t *__restrict__ dst_x,
                            float4 *__restrict__ dst_meta) {
    // {first received pair, first owned row, pairs, first received token row of the source}
    const int4 g = ent[blockIdx.x];
    const int nv = d / 16;
    for (int r = 0; r < g.z; ++r) {
        const int tr = g.w + __float_as_int(src_meta[g.x + r].z);
        const uint4 *s = reinterpret_cast<const uint4 *>(rtok + (size_t)tr * d);
        uint4 *t = reinterpret_cast<uint4 *>(dst_x + (size_t)(g.y + r) * d);
        // the owner's expert rows as fp16 in the K order of the routed gate/up GEMM
        for (int i = threadIdx.x; i < nv; i += blockDim.x) {
            const uint4 v = s[i];
            jt::x16_block(v.x, v.y, v.z, v.w, t[2 * i], t[2 * i + 1]);
        }
    }
    for (int r = threadIdx.x; r < g.z; r += blockDim.x) {
        float4 m = src_meta[g.x + r];
        m.z = __int_as_float(g.w + __float_as_int(m.z));
        dst_meta[g.y + r] = m;
    }
}

// y[t] += back[tsoff[o] + trow[t][o]] for o = 0..N-1 in order (one returned
// row per owner holding slots of t): a fixed summation order per token.
__global__ void k_ep_combine(const int32_t *__restrict__ trow, const int32_t *__restrict__ tsoff,
                             int T, int N, const float *__restrict__ back, int d,
                             float *__restrict__ y) {
    for (int t = blockIdx.x; t < T; t += gridDim.x) {
        float4 *dst = reinterpret_cast<float4 *>(y + (size_t)t * d);
        for (int i = threadIdx.x; i < d / 4; i += blockDim.x) {
            float4 v = dst[i];
            for (int o = 0; o < N; ++o) {
                const int r = trow[(size_t)t * N + o];
                if (r < 0) continue;
                const float4 b = reinterpret_cast<const float4 *>(back + (size_t)(tsoff[o] + r) * d)[i];
                v.x = __fadd_rn(v.x, b.x);
                v.y = __fadd_rn(v.y, b.y);
                v.z = __fadd_rn(v.z, b.z);
                v.w = __fadd_rn(v.w, b.w);
            }
            dst[i] = v;
        }
    }
}

}  // namespace

extern "C" int jtk_ep_count(const int32_t *ids, int n, int E, int32_t *cnt, cudaStream_t stream) {
    if (n < 0 || E <= 0 || E > 8192) return -1;
    if (cudaMemsetAsync(cnt, 0, (size_t)E * sizeof(int32_t), stream) != cudaSuccess) return -4;
    if (n == 0) return 0;
    int grid = (n + 1023) / 1024;
    if (grid > 2 * jtk_num_sms()) grid = 2 * jtk_num_sms();
    k_ep_count<<<grid, 1024, (size_t)E * sizeof(int32_t), stream>>>(ids, n, E, cnt);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int jtk_ep_tokens(const int32_t *ids, int T, int k, int El, int N, int32_t *trow,
                             int32_t *ntok, cudaStream_t stream) {
    if (T <= 0 || k <= 0 || El <= 0 || N <= 0 || N > 64) return -1;
    k_ep_tokens<<<N, 1024, 0, stream>>>(ids, T, k, El, N, trow, ntok);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int jtk_ep_pack(const int8_t *xq, const float *xs, int T, int d, int k, int El, int N,
                           const int32_t *ids, const int32_t *pos, const float *wfin,
                           const int32_t *trow, const int32_t *tsoff, int8_t *send_tok,
                           float4 *row_meta, cudaStream_t stream) {
    if (T <= 0 || d <= 0 || d % 16 || k <= 0 || k > 256 || El <= 0 || N <= 0) return -1;
    k_ep_pack<<<T, 256, 0, stream>>>(xq, xs, T, d, k, El, N, ids, pos, wfin, trow, tsoff, send_tok,
                                     row_meta);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int jtk_ep_gather(const int4 *ent, int n_ent, const int8_t *rtok, const float4 *src_meta,
                             int d, uint16_t *dst_x, float4 *dst_meta, cudaStream_t stream) {
    if (n_ent < 0 || d <= 0 || d % 16) return -1;
    if (n_ent == 0) return 0;
    k_ep_gather<<<n_ent, 256, 0, stream>>>(ent, rtok, src_meta, d, dst_x, dst_meta);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int jtk_ep_combine(const int32_t *trow, const int32_t *tsoff, int T, int N, const float *back,
                              int d, float *y, cudaStream_t stream) {
    if (T < 0 || N <= 0 || d <= 0 || d % 4) return -1;
    if (T == 0) return 0;
    int grid = T < 4 * jtk_num_sms() ? T : 4 * jtk_num_sms();
    k_ep_combine<<<grid, 256, 0, stream>>>(trow, tsoff, T, N, back, d, y);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}
