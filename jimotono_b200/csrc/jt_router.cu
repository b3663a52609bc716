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
// FP64 path accumulates in another order): a 256-thread block computes 64
// tokens x 64 experts, staging 32-element K chunks of both operands in
// shared memory as doubles (converted once per element and block); each
// thread holds 4 tokens x 4 experts x 4 lanes of accumulators and reads its
// operands as 16-byte pairs, one shared-memory load per four DFMA.  Up to 32768
// logits (decode) a chain kernel with one thread per (logit, lane) is used
// instead.
#include <cuda_runtime.h>
#include <stdint.h>

#include "jt_internal.h"
#include "jt_ptx.cuh"

namespace {

constexpr int kTT = 64;  // tokens per block
constexpr int kTE = 64;  // experts per block
constexpr int kKC = 32;  // K elements per chunk (a multiple of 4: lanes stay j mod 4)
constexpr int kLd = kKC + 2;  // row stride in doubles: 16-byte loads of neighbouring rows hit other banks

__global__ void __launch_bounds__(256) k_router_logits(const float *__restrict__ x, const float *__restrict__ wg,
                                                       int T, int d, int E, float *__restrict__ logits, int *err) {
    __shared__ __align__(16) double xs[kTT][kLd];
    __shared__ __align__(16) double ws[kTE][kLd];
    // experts tx + 16i, tokens ty + 16u; a warp covers 8 expert rows x 4
    // token rows, so each of its 16-byte operand loads is one wavefront
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tx = (warp & 1) * 8 + (lane & 7), ty = (warp >> 1) * 4 + (lane >> 3);
    const int t0 = blockIdx.y * kTT, e0 = blockIdx.x * kTE;
    double acc[4][4][4];  // [token u][expert i][lane l]
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int l = 0; l < 4; ++l) acc[u][i][l] = 0.0;

    // staging: each thread moves two 16-byte pieces of the activation tile
    // and two of the weight tile per chunk (rows sr and sr + 32, elements
    // sc .. sc+3); the next chunk is loaded into registers while the current
    // one is multiplied
    const int sr = threadIdx.x >> 3, sc = 4 * (threadIdx.x & 7);
    const bool x0in = t0 + sr < T, x1in = t0 + sr + 32 < T, w0in = e0 + sr < E, w1in = e0 + sr + 32 < E;
    const float *xp0 = x + (size_t)(x0in ? t0 + sr : 0) * d + sc;
    const float *xp1 = x + (size_t)(x1in ? t0 + sr + 32 : 0) * d + sc;
    const float *wp0 = wg + (size_t)(w0in ? e0 + sr : 0) * d + sc;
    const float *wp1 = wg + (size_t)(w1in ? e0 + sr + 32 : 0) * d + sc;
    const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 px0 = x0in ? __ldg(reinterpret_cast<const float4 *>(xp0)) : z4;
    float4 px1 = x1in ? __ldg(reinterpret_cast<const float4 *>(xp1)) : z4;
    float4 pw0 = w0in ? __ldg(reinterpret_cast<const float4 *>(wp0)) : z4;
    float4 pw1 = w1in ? __ldg(reinterpret_cast<const float4 *>(wp1)) : z4;
    for (int k0 = 0; k0 < d; k0 += kKC) {
        *reinterpret_cast<double2 *>(&xs[sr][sc]) = make_double2(px0.x, px0.y);
        *reinterpret_cast<double2 *>(&xs[sr][sc + 2]) = make_double2(px0.z, px0.w);
        *reinterpret_cast<double2 *>(&xs[sr + 32][sc]) = make_double2(px1.x, px1.y);
        *reinterpret_cast<double2 *>(&xs[sr + 32][sc + 2]) = make_double2(px1.z, px1.w);
        *reinterpret_cast<double2 *>(&ws[sr][sc]) = make_double2(pw0.x, pw0.y);
        *reinterpret_cast<double2 *>(&ws[sr][sc + 2]) = make_double2(pw0.z, pw0.w);
        *reinterpret_cast<double2 *>(&ws[sr + 32][sc]) = make_double2(pw1.x, pw1.y);
        *reinterpret_cast<double2 *>(&ws[sr + 32][sc + 2]) = make_double2(pw1.z, pw1.w);
        __syncthreads();
        if (k0 + kKC < d) {
            const int kn = k0 + kKC;
            px0 = x0in ? __ldg(reinterpret_cast<const float4 *>(xp0 + kn)) : z4;
            px1 = x1in ? __ldg(reinterpret_cast<const float4 *>(xp1 + kn)) : z4;
            pw0 = w0in ? __ldg(reinterpret_cast<const float4 *>(wp0 + kn)) : z4;
            pw1 = w1in ? __ldg(reinterpret_cast<const float4 *>(wp1 + kn)) : z4;
        }
        // four K elements (one per lane) per step, ascending j in every lane
#pragma unroll 1
        for (int j = 0; j < kKC; j += 4) {
            double a[4][4], b[4][4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const double2 lo = *reinterpret_cast<const double2 *>(&xs[ty + 16 * u][j]);
                const double2 hi = *reinterpret_cast<const double2 *>(&xs[ty + 16 * u][j + 2]);
                a[u][0] = lo.x, a[u][1] = lo.y, a[u][2] = hi.x, a[u][3] = hi.y;
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const double2 lo = *reinterpret_cast<const double2 *>(&ws[tx + 16 * i][j]);
                const double2 hi = *reinterpret_cast<const double2 *>(&ws[tx + 16 * i][j + 2]);
                b[i][0] = lo.x, b[i][1] = lo.y, b[i][2] = hi.x, b[i][3] = hi.y;
            }
#pragma unroll
            for (int l = 0; l < 4; ++l)
#pragma unroll
                for (int u = 0; u < 4; ++u)
#pragma unroll
                    for (int i = 0; i < 4; ++i) acc[u][i][l] = __fma_rn(a[u][l], b[i][l], acc[u][i][l]);
        }
        __syncthreads();
    }
    bool bad = false;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
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

// Few logits (decode): one thread per (token, expert, lane) runs the lane's
// chain over j = lane mod 4 straight from global memory (L1/L2), and the
// four lanes of a logit - four neighbouring threads - combine through
// shuffles in the reference's order: (l0 + l1) + (l2 + l3).  The latency is
// one chain of d/4 fused multiply-adds instead of the tiled kernel's d/32
// staging rounds.
__global__ void __launch_bounds__(256) k_router_chains(const float *__restrict__ x, const float *__restrict__ wg,
                                                       int T, int d, int E, float *__restrict__ logits, int *err) {
    const long long gid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int l = static_cast<int>(gid & 3);
    const long long o = gid >> 2;
    const bool live = o < static_cast<long long>(T) * E;
    const int t = live ? static_cast<int>(o / E) : 0, e = live ? static_cast<int>(o % E) : 0;
    const float *xr = x + (size_t)t * d + l;
    const float *wr = wg + (size_t)e * d + l;
    double acc = 0.0;
#pragma unroll 8
    for (int j = 0; j < d; j += 4) acc = __fma_rn((double)__ldg(xr + j), (double)__ldg(wr + j), acc);
    // lanes 0/1 and 2/3 pair up (an exact, symmetric add), then the pairs
    const double s01 = __dadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 1));
    const double s23 = __shfl_xor_sync(0xffffffffu, s01, 2);
    if (live && l == 0) {
        const double s = __dadd_rn(s01, s23);
        const float f = __double2float_rn(s);
        if ((!isfinite(s) || !isfinite(f)) && err) atomicExch(err, JT_KERR_NONFINITE);
        logits[o] = f;
    }
}

}  // namespace

extern "C" int jtk_router_logits(const float *x, const float *wgate, int T, int d, int E, float *logits,
                                 cudaStream_t stream) {
    if (!x || !wgate || !logits || T <= 0 || d <= 0 || E <= 0 || d % kKC ||
        ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(wgate)) & 15u))
        return -1;
    const long long n = static_cast<long long>(T) * E;
    if (n <= 32768) {  // decode-sized: chains (at most 512 CTAs of 256 threads)
        k_router_chains<<<static_cast<unsigned>((4 * n + 255) / 256), 256, 0, stream>>>(x, wgate, T, d, E, logits,
                                                                                      jtk_error_word());
        return cudaGetLastError() == cudaSuccess ? 0 : -4;
    }
    const dim3 grid((E + kTE - 1) / kTE, (T + kTT - 1) / kTT);
    if (grid.y > 65535u) return -1;
    k_router_logits<<<grid, 256, 0, stream>>>(x, wgate, T, d, E, logits, jtk_error_word());
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}
