// jt_compat.cu - kernels behind the remaining reference-compatible host
// entry points (jt_api_compat.c): single-token top-k + softmax of any k,
// the exact fp32 GEMM / transpose of moe_gemm.c, and the low-bit level rule
// of lowbit.c (fake-quant values and bit-plane codes).  All arithmetic is
// the reference's: sequential k-order fp32 sums without fusion, double
// precision where the reference uses double.
#include <cuda_runtime.h>
#include <stdint.h>

#include "jt_internal.h"

namespace {

// ---------------------------------------------------------------- top-k
// One CTA: k passes of a block-wide (value, index) argmax over logits[0..n)
// with the selection rule of routing.c:38-52 (first index seeds `best`,
// then strictly greater values replace it, so ties go to the lowest index
// and taken entries count as -inf).  Then the softmax of routing.c:54-73 by
// thread 0: float max, double exp sum, w = (float)e * (float)(1/sum).
// flag[0] = 1 when the softmax sum is not finite and positive.
__global__ void __launch_bounds__(1024) k_topk_any(const float *__restrict__ logits, int n, int k,
                                                   uint32_t *__restrict__ taken, int32_t *__restrict__ ids,
                                                   float *__restrict__ w, int *flag) {
    __shared__ float sv[32];
    __shared__ int si[32];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int i = threadIdx.x; i < (n + 31) / 32; i += blockDim.x) taken[i] = 0;
    __syncthreads();
    for (int p = 0; p < k; ++p) {
        // per thread: best over its strided elements, "unset" = index n
        float bv = 0.0f;
        int bi = n;
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            const bool tk = (taken[i >> 5] >> (i & 31)) & 1u;
            const float v = tk ? -INFINITY : logits[i];
            if (bi == n || v > bv) {
                bv = v;
                bi = i;
            }
        }
        // combine candidates in index order semantics: a candidate (v, i)
        // wins over (v2, i2) when v > v2, or v == v2 and i < i2 (what the
        // sequential scan yields); an unset candidate never wins
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi != n && (bi == n || ov > bv || (ov == bv && oi < bi))) {
                bv = ov;
                bi = oi;
            }
        }
        if (lane == 0) {
            sv[wid] = bv;
            si[wid] = bi;
        }
        __syncthreads();
        if (wid == 0) {
            bv = lane < nw ? sv[lane] : 0.0f;
            bi = lane < nw ? si[lane] : n;
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (oi != n && (bi == n || ov > bv || (ov == bv && oi < bi))) {
                    bv = ov;
                    bi = oi;
                }
            }
            if (lane == 0) {
                ids[p] = bi;
                taken[bi >> 5] |= 1u << (bi & 31);
            }
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        float mx = logits[ids[0]];
        for (int p = 1; p < k; ++p) {
            const float v = logits[ids[p]];
            mx = v > mx ? v : mx;
        }
        double sum = 0.0;
        for (int p = 0; p < k; ++p) {
            const double e = exp((double)logits[ids[p]] - (double)mx);
            sum += e;
            w[p] = (float)e;
        }
        if (!(sum > 0.0) || !isfinite(sum)) {
            flag[0] = 1;
            return;
        }
        const float inv = (float)(1.0 / sum);
        for (int p = 0; p < k; ++p) w[p] = __fmul_rn(w[p], inv);
    }
}

// ---------------------------------------------------------------- fp32 GEMM
// C[m][n] = sum_k A[m][k] * B[k][n] in ascending k, one rounding per
// multiply and per add (moe_gemm.c:44-170: no fused multiply-add).
__global__ void k_gemm_f32_seq(const float *__restrict__ A, const float *__restrict__ B,
                               float *__restrict__ C, int M, int N, int K) {
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    const int m = blockIdx.y;
    if (n >= N || m >= M) return;
    const float *a = A + (size_t)m * K;
    float acc = 0.0f;
    for (int kk = 0; kk < K; ++kk) acc = __fadd_rn(acc, __fmul_rn(a[kk], B[(size_t)kk * N + n]));
    C[(size_t)m * N + n] = acc;
}

__global__ void k_transpose_f32(const float *__restrict__ src, float *__restrict__ dst, int rows, int cols) {
    __shared__ float tile[32][33];
    const int c = blockIdx.x * 32 + threadIdx.x, r = blockIdx.y * 32 + threadIdx.y;
    for (int j = 0; j < 32; j += 8)
        if (r + j < rows && c < cols) tile[threadIdx.y + j][threadIdx.x] = src[(size_t)(r + j) * cols + c];
    __syncthreads();
    const int c2 = blockIdx.y * 32 + threadIdx.x, r2 = blockIdx.x * 32 + threadIdx.y;
    for (int j = 0; j < 32; j += 8)
        if (r2 + j < cols && c2 < rows) dst[(size_t)(r2 + j) * rows + c2] = tile[threadIdx.x][threadIdx.y + j];
}

// ---------------------------------------------------------------- low-bit
// max |w| in double over n values (positive doubles order like their bits),
// bad = 1 on a non-finite value.
__global__ void k_absmax_d(const float *__restrict__ w, size_t n, unsigned long long *maxbits, int *bad) {
    double m = 0.0;
    int nf = 0;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const double v = (double)w[i];
        nf |= !isfinite(v);
        m = fmax(m, fabs(v));
    }
    for (int o = 16; o > 0; o >>= 1) {
        m = fmax(m, __shfl_xor_sync(0xffffffffu, m, o));
        nf |= __shfl_xor_sync(0xffffffffu, nf, o);
    }
    if ((threadIdx.x & 31) == 0) {
        atomicMax(maxbits, (unsigned long long)__double_as_longlong(m));
        if (nf) atomicExch(bad, 1);
    }
}

// level index of lowbit.c:78-88: t = w / maxa (double), li = floor(t(n-1)/2
// + (n-1)/2 + 0.5) clamped to [0, n-1]
__device__ __forceinline__ int level(float wv, double maxa, int nl) {
    const double t = maxa == 0.0 ? 0.0 : __ddiv_rn((double)wv, maxa);
    const double li = floor(__dadd_rn(__dadd_rn(__ddiv_rn(__dmul_rn(t, (double)(nl - 1)), 2.0),
                                                 (double)(nl - 1) / 2.0),
                                      0.5));
    long l = (long)li;
    l = l < 0 ? 0 : l;
    l = l > nl - 1 ? nl - 1 : l;
    return (int)l;
}

// fq[i] = (float)(((2li - (n-1)) / (n-1)) * maxa), all-zero input -> 0
__global__ void k_lowbit_fq(const float *__restrict__ w, size_t n, int bits,
                            const unsigned long long *maxbits, float *__restrict__ fq) {
    const double maxa = __longlong_as_double((long long)*maxbits);
    const int nl = 1 << bits;
    const double nd = (double)(nl - 1);
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        if (maxa == 0.0) {
            fq[i] = 0.0f;
            continue;
        }
        const int l = level(w[i], maxa, nl);
        const double lv = __ddiv_rn(__dsub_rn(2.0 * (double)l, nd), nd);
        fq[i] = (float)__dmul_rn(lv, maxa);
    }
}

// bit planes of lowbit.c:117-137: idx[b*(k/4) + g] bit j = bit b of li(4g+j)
__global__ void k_lowbit_idx(const float *__restrict__ col, size_t k, int bits,
                             const unsigned long long *maxbits, uint8_t *__restrict__ idx) {
    const double maxa = __longlong_as_double((long long)*maxbits);
    const int nl = 1 << bits;
    const size_t ng = k / 4;
    for (size_t g = blockIdx.x * (size_t)blockDim.x + threadIdx.x; g < ng; g += (size_t)gridDim.x * blockDim.x) {
        int li[4];
        for (int j = 0; j < 4; ++j) li[j] = level(col[g * 4 + j], maxa, nl);
        for (int b = 0; b < bits; ++b) {
            unsigned p = 0;
            for (int j = 0; j < 4; ++j)
                if (((unsigned)li[j] >> b) & 1u) p |= 1u << j;
            idx[(size_t)b * ng + g] = (uint8_t)p;
        }
    }
}

int grid_for(size_t n, int threads) {
    size_t g = (n + threads - 1) / threads;
    const size_t cap = (size_t)jtk_num_sms() * 8;
    if (g > cap) g = cap;
    return g < 1 ? 1 : (int)g;
}

}  // namespace

extern "C" int jtk_topk_any(const float *logits, int n, int k, uint32_t *taken, int32_t *ids, float *w,
                            int *flag, cudaStream_t stream) {
    if (n <= 0 || k <= 0 || k > n) return -1;
    k_topk_any<<<1, 1024, 0, stream>>>(logits, n, k, taken, ids, w, flag);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int jtk_gemm_f32_seq(const float *A, const float *B, float *C, int M, int N, int K,
                                cudaStream_t stream) {
    if (M <= 0 || N <= 0 || K <= 0 || M > 65535) return -1;
    dim3 grid((N + 127) / 128, M);
    k_gemm_f32_seq<<<grid, 128, 0, stream>>>(A, B, C, M, N, K);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int jtk_transpose_f32(const float *src, float *dst, int rows, int cols, cudaStream_t stream) {
    if (rows <= 0 || cols <= 0 || (rows + 31) / 32 > 65535) return -1;
    dim3 grid((cols + 31) / 32, (rows + 31) / 32);
    k_transpose_f32<<<grid, dim3(32, 8), 0, stream>>>(src, dst, rows, cols);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int jtk_lowbit_absmax(const float *w, size_t n, unsigned long long *maxbits, int *bad,
                                 cudaStream_t stream) {
    if (n == 0) return -1;
    if (cudaMemsetAsync(maxbits, 0, sizeof(unsigned long long), stream) != cudaSuccess) return -4;
    k_absmax_d<<<grid_for(n, 256), 256, 0, stream>>>(w, n, maxbits, bad);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int jtk_lowbit_fq(const float *w, size_t n, int bits, const unsigned long long *maxbits, float *fq,
                             cudaStream_t stream) {
    k_lowbit_fq<<<grid_for(n, 256), 256, 0, stream>>>(w, n, bits, maxbits, fq);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int jtk_lowbit_idx(const float *col, size_t k, int bits, const unsigned long long *maxbits,
                              uint8_t *idx, cudaStream_t stream) {
    k_lowbit_idx<<<grid_for(k / 4, 256), 256, 0, stream>>>(col, k, bits, maxbits, idx);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}
