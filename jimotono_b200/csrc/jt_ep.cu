// jt_ep.cu - device kernels of the expert-parallel MoE layer (the exchange
// steps around the expert GEMMs; the NCCL calls and the bookkeeping are in
// jt_ep.c / jt_ep_layout.c).
#include <cuda_runtime.h>
#include <stdint.h>

#include "jt_internal.h"

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

// One CTA per (source, expert) block of received rows: copy `count` rows of
// codes (d bytes) and metadata to their expert-contiguous position; the
// metadata's third field becomes the received row index, which is where
// the down projection writes that row's output.
__global__ void k_ep_gather(const int4 *__restrict__ ent, const int8_t *__restrict__ src_codes,
                            const float4 *__restrict__ src_meta, int d, int8_t *__restrict__ dst_codes,
                            float4 *__restrict__ dst_meta) {
    const int4 g = ent[blockIdx.x];  // {first received row, first owned row, rows, 0}
    const int nv = d / 16;
    for (int r = 0; r < g.z; ++r) {
        const uint4 *s = reinterpret_cast<const uint4 *>(src_codes + (size_t)(g.x + r) * d);
        uint4 *t = reinterpret_cast<uint4 *>(dst_codes + (size_t)(g.y + r) * d);
        for (int i = threadIdx.x; i < nv; i += blockDim.x) t[i] = s[i];
    }
    for (int r = threadIdx.x; r < g.z; r += blockDim.x) {
        float4 m = src_meta[g.x + r];
        m.z = __int_as_float(g.x + r);
        dst_meta[g.y + r] = m;
    }
}

// y[t] += back[j] for every kept local pair j (send order = perm order),
// t = perm[j] / k: the combine of the rows the owners sent back.
__global__ void k_ep_combine(const int32_t *__restrict__ perm, int kept, int k,
                             const float *__restrict__ back, int d, float *__restrict__ y) {
    for (int j = blockIdx.x; j < kept; j += gridDim.x) {
        const int t = perm[j] / k;
        const float4 *s = reinterpret_cast<const float4 *>(back + (size_t)j * d);
        float *dst = y + (size_t)t * d;
        for (int i = threadIdx.x; i < d / 4; i += blockDim.x) {
            const float4 v = s[i];
            atomicAdd(reinterpret_cast<float4 *>(dst) + i, v);
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

extern "C" int jtk_ep_gather(const int4 *ent, int n_ent, const int8_t *src_codes, const float4 *src_meta,
                             int d, int8_t *dst_codes, float4 *dst_meta, cudaStream_t stream) {
    if (n_ent < 0 || d <= 0 || d % 16) return -1;
    if (n_ent == 0) return 0;
    k_ep_gather<<<n_ent, 256, 0, stream>>>(ent, src_codes, src_meta, d, dst_codes, dst_meta);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int jtk_ep_combine(const int32_t *perm, int kept, int k, const float *back, int d, float *y,
                              cudaStream_t stream) {
    if (kept < 0 || k <= 0 || d <= 0 || d % 4) return -1;
    if (kept == 0) return 0;
    int grid = kept < 4 * jtk_num_sms() ? kept : 4 * jtk_num_sms();
    k_ep_combine<<<grid, 256, 0, stream>>>(perm, kept, k, back, d, y);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}
