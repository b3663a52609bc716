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
// thread holds one lane's partial sums for 8 tokens x 8 experts and reads
// its operands as 16-byte pairs, one shared-memory load per eight DFMA
// (the shared-memory pipe, not the FP64 pipe, bounded a layout with four
// lanes per thread).  Up to 32768
// logits (decode) a chain kernel with one thread per (logit, lane) is used
// instead.
#include <cuda_runtime.h>
#include <stdint.h>

#include "jt_internal.h"
#include "jt_ptx.cuh"

namespace {

constexpr int kTT = 64;  // tokens per block
constexpr int kTE = 64;  // experts per block
constexpr int kKC = 32;  // K elements per chunk (a multiple of 8: two per lane and load)
constexpr int kLS = kKC / 4 + 2;  // lane stride in doubles (8 elements + pad)
constexpr int kRS = 4 * kLS;      // row stride in doubles: [row][lane][element]

// Thread t: lane l = t % 4 of the reference's accumulation (elements
// j = l mod 4), tokens tu + 8m (tu = (t / 4) % 8) and experts ti + 8n
// (ti = t / 32, the warp) of the block, m, n = 0..7.  The chunk lives in
// shared memory lane-major (element k of row r at [r][k % 4][k / 4]), so
// one 16-byte load gives a row's next two elements of one lane; per two
// K steps a thread issues 16 such loads for 128 DFMA.  With the 10-double
// lane pitch and token rows interleaved by 8, the eight 16-byte reads of a
// load phase fall in distinct banks.
__global__ void __launch_bounds__(256) k_router_logits(const float *__restrict__ x, const float *__restrict__ wg,
                                                       int T, int d, int E, float *__restrict__ logits, int *err) {
    __shared__ __align__(16) double xs[kTT * kRS];
    __shared__ __align__(16) double ws[kTE * kRS];
    const int l = threadIdx.x & 3, tu = (threadIdx.x >> 2) & 7, ti = threadIdx.x >> 5;
    const int t0 = blockIdx.y * kTT, e0 = blockIdx.x * kTE;
    double acc[8][8];  // [token m][expert n], lane l's partial sum
#pragma unroll
    for (int m = 0; m < 8; ++m)
#pragma unroll
        for (int n = 0; n < 8; ++n) acc[m][n] = 0.0;

    // staging: each thread moves elements sc .. sc+3 of rows sr and sr + 32
    // of both tiles per chunk; the next chunk is loaded into registers while
    // the current one is multiplied
    const int sr = threadIdx.x >> 3, sq = threadIdx.x & 7, sc = 4 * sq;
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
    auto put = [&](double *base, int row, float4 v) {  // elements sc..sc+3 -> lanes 0..3, position sq
        double *q = base + row * kRS + sq;
        q[0] = v.x;
        q[kLS] = v.y;
        q[2 * kLS] = v.z;
        q[3 * kLS] = v.w;
    };
    const double *xr = xs + tu * kRS + l * kLS;  // + 8m rows
    const double *wr = ws + ti * kRS + l * kLS;  // + 8n rows
    for (int k0 = 0; k0 < d; k0 += kKC) {
        put(xs, sr, px0);
        put(xs, sr + 32, px1);
        put(ws, sr, pw0);
        put(ws, sr + 32, pw1);
        __syncthreads();
        if (k0 + kKC < d) {
            const int kn = k0 + kKC;
            px0 = x0in ? __ldg(reinterpret_cast<const float4 *>(xp0 + kn)) : z4;
            px1 = x1in ? __ldg(reinterpret_cast<const float4 *>(xp1 + kn)) : z4;
            pw0 = w0in ? __ldg(reinterpret_cast<const float4 *>(wp0 + kn)) : z4;
            pw1 = w1in ? __ldg(reinterpret_cast<const float4 *>(wp1 + kn)) : z4;
        }
        // two of the lane's elements per step pair, ascending
#pragma unroll 1
        for (int sp = 0; sp < kKC / 8; ++sp) {
            double2 a[8];
#pragma unroll
            for (int m = 0; m < 8; ++m) a[m] = *reinterpret_cast<const double2 *>(xr + 8 * m * kRS + 2 * sp);
#pragma unroll
            for (int n = 0; n < 8; ++n) {
                const double2 b = *reinterpret_cast<const double2 *>(wr + 8 * n * kRS + 2 * sp);
#pragma unroll
                for (int m = 0; m < 8; ++m) acc[m][n] = __fma_rn(a[m].x, b.x, acc[m][n]);
#pragma unroll
                for (int m = 0; m < 8; ++m) acc[m][n] = __fma_rn(a[m].y, b.y, acc[m][n]);
            }
        }
        __syncthreads();
    }
    // the four lanes of a logit are neighbouring threads: (l0 + l1) + (l2 + l3)
    bool bad = false;
#pragma unroll
    for (int m = 0; m < 8; ++m) {
        const int t = t0 + tu + 8 * m;
#pragma unroll
        for (int n = 0; n < 8; ++n) {
            const int e = e0 + ti + 8 * n;
            const double s01 = __dadd_rn(acc[m][n], __shfl_xor_sync(0xffffffffu, acc[m][n], 1));
            const double s23 = __shfl_xor_sync(0xffffffffu, s01, 2);
            const double sum = __dadd_rn(s01, s23);
            const float f = __double2float_rn(sum);
            if (l == 0 && t < T && e < E) {
                bad |= !isfinite(sum) || !isfinite(f);
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
