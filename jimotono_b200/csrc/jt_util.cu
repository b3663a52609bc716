// jt_util.cu - small device kernels used by the reference-compatible entry
// points: int8 transpose with the symmetric-range check (q = -128 is
// rejected like w8a8.c:1041-1060), padded row copy with the same check, and
// a finiteness scan of an fp32 result (the reference's per-element
// isfinite() guards, w8a8.c:676-681).
#include <cuda_runtime.h>
#include <stdint.h>

#include "jt_internal.h"

namespace {

// dst[n][k] = src[k][n] for k < K, 0 for K <= k < Kp.  Sets *bad when any
// source byte equals -128.  32x32 tiles through shared memory.
__global__ void k_transpose_s8(const int8_t *__restrict__ src, int K, int N,
                               int8_t *__restrict__ dst, int Kp, int *bad) {
    __shared__ int8_t tile[32][33];
    const int n0 = blockIdx.x * 32, k0 = blockIdx.y * 32;
    const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
    int found = 0;
    for (int r = ty; r < 32; r += 8) {
        const int k = k0 + r, n = n0 + tx;
        int8_t v = 0;
        if (k < K && n < N) {
            v = src[(size_t)k * N + n];
            found |= (v == -128);
        }
        tile[r][tx] = v;
    }
    __syncthreads();
    for (int r = ty; r < 32; r += 8) {
        const int n = n0 + r, k = k0 + tx;
        if (n < N && k < Kp) dst[(size_t)n * Kp + k] = tile[tx][r];
    }
    if (found) atomicExch(bad, 1);
}

// dst[m][k] = src[m][k] (k < K), 0 for K <= k < Kp; flags -128.
__global__ void k_pad_rows_s8(const int8_t *__restrict__ src, int M, int K,
                              int8_t *__restrict__ dst, int Kp, int *bad) {
    const size_t total = (size_t)M * Kp;
    int found = 0;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        const int m = (int)(i / Kp), k = (int)(i % Kp);
        int8_t v = 0;
        if (k < K) {
            v = src[(size_t)m * K + k];
            found |= (v == -128);
        }
        dst[i] = v;
    }
    if (found) atomicExch(bad, 1);
}

__global__ void k_check_s8(const int8_t *__restrict__ p, size_t n, int *bad) {
    int found = 0;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        found |= (p[i] == -128);
    if (found) atomicExch(bad, 1);
}

__global__ void k_check_finite_f32(const float *__restrict__ p, size_t n, int *bad) {
    int found = 0;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        found |= !isfinite(p[i]);
    if (found) atomicExch(bad, 1);
}

int grid_for(size_t n) {
    size_t g = (n + 255) / 256;
    const size_t cap = (size_t)jtk_num_sms() * 8;
    if (g > cap) g = cap;
    if (g < 1) g = 1;
    return (int)g;
}

}  // namespace

extern "C" int jtk_transpose_s8(const int8_t *src, int K, int N, int8_t *dst, int Kp, int *bad,
                                cudaStream_t stream) {
    dim3 grid((N + 31) / 32, (Kp + 31) / 32), block(32, 8);
    k_transpose_s8<<<grid, block, 0, stream>>>(src, K, N, dst, Kp, bad);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int jtk_pad_rows_s8(const int8_t *src, int M, int K, int8_t *dst, int Kp, int *bad,
                               cudaStream_t stream) {
    k_pad_rows_s8<<<grid_for((size_t)M * Kp), 256, 0, stream>>>(src, M, K, dst, Kp, bad);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int jtk_check_s8(const int8_t *p, size_t n, int *bad, cudaStream_t stream) {
    k_check_s8<<<grid_for(n), 256, 0, stream>>>(p, n, bad);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int jtk_check_finite_f32(const float *p, size_t n, int *bad, cudaStream_t stream) {
    k_check_finite_f32<<<grid_for(n), 256, 0, stream>>>(p, n, bad);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

namespace {
// fp32 -> bf16, round to nearest even (the rounding a bf16 output of the
// layer gets; the reference commits Y = (float)yacc, moe_layer.c:1568-1574).
__global__ void k_f32_to_bf16(const float *__restrict__ src, uint16_t *__restrict__ dst, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        const uint32_t b = __float_as_uint(src[i]);
        uint16_t h;
        if ((b & 0x7fffffffu) > 0x7f800000u) h = (uint16_t)((b >> 16) | 0x40u);  // quiet NaN
        else h = (uint16_t)((b + 0x7fffu + ((b >> 16) & 1u)) >> 16);
        dst[i] = h;
    }
}
}  // namespace

extern "C" int jtk_f32_to_bf16(const float *src, uint16_t *dst, size_t n, cudaStream_t stream) {
    size_t g = (n + 255) / 256;
    const size_t cap = (size_t)jtk_num_sms() * 8;
    if (g > cap) g = cap;
    if (g < 1) g = 1;
    k_f32_to_bf16<<<(int)g, 256, 0, stream>>>(src, dst, n);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

namespace {
}  // namespace

