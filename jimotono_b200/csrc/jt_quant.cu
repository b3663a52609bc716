// jt_quant.cu - quantize / dequantize / fake-quantize kernels with the
// reference's exact arithmetic (w8a8.c:688-907, w8a8.c:1074-1200).
//
// A "block" is a contiguous run of `blk` elements inside a row: per-tensor
// quantization is one row with blk = n, per-channel / per-token is
// blk = cols, and the MoE requantization uses 128-element blocks.
#include <cuda_runtime.h>
#include <stdint.h>

#include "jt_internal.h"
#include "jt_quant.cuh"

namespace {

constexpr int kThreads = 256;

// Fake-quant value (float)(qd * scale_d) of w8a8.c:1105-1115.  qd is the
// double round() result, so a small negative input gives qd = -0.0 and the
// product keeps that sign; an all-zero tensor writes +0.0 (w8a8.c:1097-1102).
__device__ __forceinline__ float fq_value(float x, int c, float maxabs, const jt::QuantBlock &qb) {
    if (maxabs == 0.0f) return 0.0f;
    if (c == 0) return copysignf(0.0f, x);
    return __double2float_rn(__dmul_rn((double)c, qb.scale_d));
}

__device__ __forceinline__ float block_absmax(const float *p, int n, int *nonfinite) {
    float m = 0.0f;
    int bad = 0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = p[i];
        bad |= !isfinite(v);
        m = fmaxf(m, fabsf(v));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        bad |= __shfl_xor_sync(0xffffffffu, bad, o);
    }
    __shared__ float wm[kThreads / 32];
    __shared__ int wb[kThreads / 32];
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) {
        wm[w] = m;
        wb[w] = bad;
    }
    __syncthreads();
    if (w == 0) {
        m = l < (int)(blockDim.x >> 5) ? wm[l] : 0.0f;
        bad = l < (int)(blockDim.x >> 5) ? wb[l] : 0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            bad |= __shfl_xor_sync(0xffffffffu, bad, o);
        }
        if (l == 0) {
            wm[0] = m;
            wb[0] = bad;
        }
    }
    __syncthreads();
    m = wm[0];
    *nonfinite = wb[0];
    __syncthreads();
    return m;
}

// One CTA per (row, block).  mode 0: write int8 codes + scale;
// mode 1: write fake-quantized floats (float)(qd * scale_d).
__global__ void __launch_bounds__(kThreads)
    k_quant_blocks(const float *__restrict__ x, int rows, int cols, int blk, int mode,
                   int8_t *__restrict__ q, float *__restrict__ scales, float *__restrict__ fq,
                   int *bad) {
    const int nblk = cols / blk;
    const int row = blockIdx.x / nblk, b = blockIdx.x % nblk;
    if (row >= rows) return;
    const size_t base = (size_t)row * cols + (size_t)b * blk;
    int nonfinite = 0;
    const float maxabs = block_absmax(x + base, blk, &nonfinite);
    if (nonfinite) {
        if (threadIdx.x == 0) atomicExch(bad, 1);
        return;
    }
    const jt::QuantBlock qb = jt::quant_block(maxabs);
    if (maxabs != 0.0f && !(qb.scale_f > 0.0f)) {  // float scale underflow (w8a8.c:730-733)
        if (threadIdx.x == 0) atomicExch(bad, 2);
        return;
    }
    if (mode == 0 && threadIdx.x == 0) scales[(size_t)row * nblk + b] = qb.scale_f;
    for (int i = threadIdx.x; i < blk; i += blockDim.x) {
        const int c = jt::quant_code(x[base + i], qb);
        if (mode == 0) {
            q[base + i] = (int8_t)c;
        } else {
            fq[base + i] = fq_value(x[base + i], c, maxabs, qb);
        }
    }
}

// Global max |x| over n elements for per-tensor mode with n too long for
// one CTA: positive floats order like their bit patterns, so an integer
// atomicMax on the bits is an exact float max.
__global__ void k_absmax_all(const float *__restrict__ x, size_t n, unsigned *maxbits, int *bad) {
    float m = 0.0f;
    int nf = 0;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        const float v = x[i];
        nf |= !isfinite(v);
        m = fmaxf(m, fabsf(v));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        nf |= __shfl_xor_sync(0xffffffffu, nf, o);
    }
    if ((threadIdx.x & 31) == 0) {
        atomicMax(maxbits, __float_as_uint(m));
        if (nf) atomicExch(bad, 1);
    }
}

__global__ void k_quant_all(const float *__restrict__ x, size_t n, const unsigned *maxbits,
                            int mode, int8_t *__restrict__ q, float *__restrict__ scale,
                            float *__restrict__ fq, int *bad) {
    const float maxabs = __uint_as_float(*maxbits);
    const jt::QuantBlock qb = jt::quant_block(maxabs);
    if (maxabs != 0.0f && !(qb.scale_f > 0.0f)) {
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicExch(bad, 2);
        return;
    }
    if (mode == 0 && blockIdx.x == 0 && threadIdx.x == 0) *scale = qb.scale_f;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        const int c = jt::quant_code(x[i], qb);
        if (mode == 0)
            q[i] = (int8_t)c;
        else
            fq[i] = fq_value(x[i], c, maxabs, qb);
    }
}

// dst[r][c] = (float)((double)src[r][c] * (double)scales[r / ... ]) with the
// -128 check of w8a8.c:765-772 / :885-893.  `rows` scale entries, `cols`
// elements each (per-tensor = 1 row).
__global__ void k_dequant_rows(const int8_t *__restrict__ src, const float *__restrict__ scales,
                               size_t rows, size_t cols, float *__restrict__ dst, int *bad) {
    const size_t n = rows * cols;
    int found = 0, nf = 0;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        const int v = src[i];
        found |= (v == -128);
        const float f = __double2float_rn(__dmul_rn((double)v, (double)scales[i / cols]));
        nf |= !isfinite(f);
        dst[i] = f;
    }
    if (found) atomicExch(bad, 1);
    if (nf) atomicExch(bad, 2);
}

int grid_for(size_t n) {
    size_t g = (n + kThreads - 1) / kThreads;
    const size_t cap = (size_t)jtk_num_sms() * 8;
    if (g > cap) g = cap;
    if (g < 1) g = 1;
    return (int)g;
}

}  // namespace

extern "C" int jtk_quant_blocks(const float *x, int rows, int cols, int blk, int mode, int8_t *q,
                                float *scales, float *fq, int *bad, cudaStream_t stream) {
    if (rows <= 0 || cols <= 0 || blk <= 0 || cols % blk != 0) return -1;
    const long long nb = (long long)rows * (cols / blk);
    if (nb > 0x7fffffffLL) return -1;
    k_quant_blocks<<<(int)nb, kThreads, 0, stream>>>(x, rows, cols, blk, mode, q, scales, fq,
                                                     bad);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int jtk_quant_tensor(const float *x, size_t n, int mode, int8_t *q, float *scale,
                                float *fq, unsigned *maxbits_scratch, int *bad,
                                cudaStream_t stream) {
    if (n == 0) return -1;
    if (cudaMemsetAsync(maxbits_scratch, 0, sizeof(unsigned), stream) != cudaSuccess) return -4;
    k_absmax_all<<<grid_for(n), kThreads, 0, stream>>>(x, n, maxbits_scratch, bad);
    k_quant_all<<<grid_for(n), kThreads, 0, stream>>>(x, n, maxbits_scratch, mode, q, scale, fq,
                                                      bad);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int jtk_dequant_rows(const int8_t *src, const float *scales, size_t rows, size_t cols,
                                float *dst, int *bad, cudaStream_t stream) {
    k_dequant_rows<<<grid_for(rows * cols), kThreads, 0, stream>>>(src, scales, rows, cols, dst,
                                                                   bad);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}
