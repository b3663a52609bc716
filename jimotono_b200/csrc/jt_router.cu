// jt_router.cu - router logits of the MoE layer (moe_layer.c:1114-1137):
//   logits[t][e] = (float) dot(x[t], wgate[e])
// with the dot product accumulated in double in the order of the
// reference's AVX2 build (moe_layer.c:67-86): lane l sums the products of
// the elements j = l mod 4 in ascending j, and the lanes combine as
// (l0 + l1) + (l2 + l3).  A product of two floats is exact in double, so
// fma(x, w, lane) rounds exactly like lane + x*w; the logits are therefore
// bit-identical to the reference's and the top-k that follows selects the
// same experts.
//
// Tiled GEMM on the FP64 pipe (one DFMA per product; the tensor cores'
// FP64 path accumulates in another order): a 256-thread block computes 32
// tokens x 64 experts, staging 32-element K chunks of both operands in
// shared memory as doubles (converted once per element and block); each
// thread holds 2 tokens x 4 experts x 4 lanes of accumulators.
#include <cuda_runtime.h>
#include <stdint.h>

#include "jt_internal.h"
#include "jt_ptx.cuh"

namespace {

constexpr int kTT = 32;  // tokens per block
constexpr int kTE = 64;  // experts per block
constexpr int kKC = 32;  // K elements per chunk (a multiple of 4: lanes stay j mod 4)
constexpr int kLd = kKC + 1;

__global__ void __launch_bounds__(256) k_router_logits(const float *__restrict__ x, const float *__restrict__ wg,
                                                       int T, int d, int E, float *__restrict__ logits, int *err) {
    __shared__ double xs[kTT][kLd];
    __shared__ double ws[kTE][kLd];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;  // experts tx + 16i, tokens ty + 16u
    const int t0 = blockIdx.y * kTT, e0 = blockIdx.x * kTE;
    double acc[2][4][4];
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int l = 0; l < 4; ++l) acc[u][i][l] = 0.0;

    for (int k0 = 0; k0 < d; k0 += kKC) {
        // stage: 32 x 32 activations and 64 x 32 gate weights, four
        // consecutive K elements per thread and step (16-byte loads)
        for (int i = threadIdx.x; i < kTT * kKC / 4; i += 256) {
            const int r = i / (kKC / 4), c = 4 * (i % (kKC / 4));
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (t0 + r < T) v = __ldg(reinterpret_cast<const float4 *>(x + (size_t)(t0 + r) * d + k0 + c));
            xs[r][c] = v.x, xs[r][c + 1] = v.y, xs[r][c + 2] = v.z, xs[r][c + 3] = v.w;
        }
        for (int i = threadIdx.x; i < kTE * kKC / 4; i += 256) {
            const int r = i / (kKC / 4), c = 4 * (i % (kKC / 4));
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (e0 + r < E) v = __ldg(reinterpret_cast<const float4 *>(wg + (size_t)(e0 + r) * d + k0 + c));
            ws[r][c] = v.x, ws[r][c + 1] = v.y, ws[r][c + 2] = v.z, ws[r][c + 3] = v.w;
        }
        __syncthreads();
#pragma unroll 2
        for (int j = 0; j < kKC; j += 4) {
#pragma unroll
            for (int l = 0; l < 4; ++l) {
                const double a0 = xs[ty][j + l], a1 = xs[ty + 16][j + l];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const double b = ws[tx + 16 * i][j + l];
                    acc[0][i][l] = __fma_rn(a0, b, acc[0][i][l]);
                    acc[1][i][l] = __fma_rn(a1, b, acc[1][i][l]);
                }
            }
        }
        __syncthreads();
    }
    bool bad = false;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int t = t0 + ty + 16 * u;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int e = e0 + tx + 16 * i;
            const double s = __dadd_rn(__dadd_rn(acc[u][i][0], acc[u][i][1]), __dadd_rn(acc[u][i][2], acc[u][i][3]));
            const float f = __double2float_rn(s);
            if (t < T && e < E) {
                bad |= !isfinite(s) || !isfinite(f);
                logits[(size_t)t * E + e] = f;
            }
        }
    }
    if (bad && err) atomicExch(err, JT_KERR_NONFINITE);
}

}  // namespace

extern "C" int jtk_router_logits(const float *x, const float *wgate, int T, int d, int E, float *logits,
                                 cudaStream_t stream) {
    if (!x || !wgate || !logits || T <= 0 || d <= 0 || E <= 0 || d % kKC ||
        ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(wgate)) & 15u))
        return -1;
    const dim3 grid((E + kTE - 1) / kTE, (T + kTT - 1) / kTT);
    if (grid.y > 65535u) return -1;
    k_router_logits<<<grid, 256, 0, stream>>>(x, wgate, T, d, E, logits, jtk_error_word());
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}
