// jt_gemv.cu - batch-1 low-bit GEMV: y[n] = sa * fold_g(P[n][g] * s[n][g])
// over INT2 and INT4 weight rows packed little-endian along K with one fp16
// scale per 64 K (the decode replacement of the reference's LUT path,
// lowbit.c:158-267 / tmac.c:387-506):
//   P[n][g] = sum_{k in group g} a[k] * c[n][k]   (int32, exact)
//   c = 2*li - (2^bits - 1)
//   r = 0; for g ascending: r = fmaf((float)P[n][g], s[n][g], r); y[n] = r * sa
//
// HBM-bound: every weight byte is read once.  One warp streams 32 rows at a
// time with 128-bit coalesced loads; lane l owns 64-K group l of each row
// (16 bytes of an INT2 row, 32 bytes of an INT4 row), extracts the unsigned
// codes of four K positions per byte lane with one shift+mask and feeds them
// to dp4a against activation words permuted to match, so
//   P = 2 * sum(dp4a(li, a')) - (2^bits - 1) * sum(a)   (exact in int32).
// The 32 group partials of each row go through shared memory so that the
// sequential fp32 fold runs lane-per-row.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "jt_internal.h"
#include "jt_ptx.cuh"

namespace {

constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kRows = 32;    // rows per warp task
// rows loaded ahead: 8 INT2 rows (16 B per lane each) or 4 INT4 rows (32 B)
template <int BITS>
struct Ahead {
    static constexpr int v = BITS == 2 ? 8 : 4;
};
constexpr int kMaxG = 64;    // K <= 4096

__device__ __forceinline__ uint32_t byte_of(const int8_t *a, int k) {
    return static_cast<uint32_t>(static_cast<uint8_t>(a[k]));
}

// Activation words of group g permuted to the code order of one packed
// 32-bit word: INT2 word w holds codes k = 16w + 4b + j at bits 2j of byte b,
// so (w >> 2j) & 0x03030303 pairs with bytes a[16w + j], a[16w+4+j],
// a[16w+8+j], a[16w+12+j]; INT4 word w holds k = 8w + 2b (low nibble) and
// 8w + 2b + 1 (high nibble).
template <int BITS>
__device__ __forceinline__ void perm_acts(const int8_t *a, int k0, uint32_t (&ap)[16], int &asum) {
    asum = 0;
    for (int i = 0; i < 64; ++i) asum += a[k0 + i];
    if (BITS == 2) {
#pragma unroll
        for (int w = 0; w < 4; ++w)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int b0 = k0 + 16 * w + j;
                ap[4 * w + j] = byte_of(a, b0) | (byte_of(a, b0 + 4) << 8) | (byte_of(a, b0 + 8) << 16) |
                                (byte_of(a, b0 + 12) << 24);
            }
    } else {
#pragma unroll
        for (int w = 0; w < 8; ++w)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int b0 = k0 + 8 * w + h;
                ap[2 * w + h] = byte_of(a, b0) | (byte_of(a, b0 + 2) << 8) | (byte_of(a, b0 + 4) << 16) |
                                (byte_of(a, b0 + 6) << 24);
            }
    }
}

// Group partial of one row from this lane's packed bytes.
template <int BITS>
__device__ __forceinline__ int group_partial(const uint4 (&q)[BITS / 2], const uint32_t (&ap)[16], int asum) {
    int acc = 0;
    if (BITS == 2) {
        const uint32_t w[4] = {q[0].x, q[0].y, q[0].z, q[0].w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j)
                acc = __dp4a(static_cast<int>((w[i] >> (2 * j)) & 0x03030303u), static_cast<int>(ap[4 * i + j]), acc);
        return 2 * acc - 3 * asum;
    } else {
        const uint32_t w[8] = {q[0].x, q[0].y, q[0].z, q[0].w, q[1].x, q[1].y, q[1].z, q[1].w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            acc = __dp4a(static_cast<int>(w[i] & 0x0F0F0F0Fu), static_cast<int>(ap[2 * i]), acc);
            acc = __dp4a(static_cast<int>((w[i] >> 4) & 0x0F0F0F0Fu), static_cast<int>(ap[2 * i + 1]), acc);
        }
        return 2 * acc - 15 * asum;
    }
}

template <int BITS>
__device__ __forceinline__ void load_row(const uint8_t *row, int g, bool on, uint4 (&q)[BITS / 2]) {
    if (!on) {
#pragma unroll
        for (int i = 0; i < BITS / 2; ++i) q[i] = make_uint4(0, 0, 0, 0);
        return;
    }
    const uint4 *p = reinterpret_cast<const uint4 *>(row + g * (64 * BITS / 8));
#pragma unroll
    for (int i = 0; i < BITS / 2; ++i) q[i] = __ldcs(p + i);  // streamed once
}

// One warp task: rows [r0, r0 + nrows) of one segment.
template <int BITS>
__device__ void gemv_task(const int8_t *a, float sa, const uint8_t *w, const uint16_t *s, int r0,
                          int nrows, int K, float *y, int32_t *Ps) {
    constexpr int kAhead = Ahead<BITS>::v;
    const int lane = jt::lane_id();
    const int G = K / 64;
    const int rowbytes = K * BITS / 8;
    for (int gp = 0; gp < G; gp += 32) {
        const int g = gp + lane;
        const bool on = g < G;
        uint32_t ap[16];
        int asum = 0;
        if (on) perm_acts<BITS>(a, 64 * g, ap, asum);
        uint4 cur[kAhead][BITS / 2];
#pragma unroll
        for (int i = 0; i < kAhead; ++i)
            load_row<BITS>(w + (size_t)(r0 + i) * rowbytes, g, on && i < nrows, cur[i]);
        for (int rb = 0; rb < kRows; rb += kAhead) {
            uint4 nxt[kAhead][BITS / 2];
#pragma unroll
            for (int i = 0; i < kAhead; ++i) {
                const int rr = rb + kAhead + i;
                load_row<BITS>(w + (size_t)(r0 + rr) * rowbytes, g, on && rr < nrows, nxt[i]);
            }
#pragma unroll
            for (int i = 0; i < kAhead; ++i)
                if (on) Ps[(rb + i) * (kMaxG + 1) + g] = group_partial<BITS>(cur[i], ap, asum);
#pragma unroll
            for (int i = 0; i < kAhead; ++i)
#pragma unroll
                for (int h = 0; h < BITS / 2; ++h) cur[i][h] = nxt[i][h];
        }
    }
    __syncwarp();
    // fold: lane = row, groups ascending
    if (lane < nrows) {
        const int n = r0 + lane;
        const uint16_t *sr = s + (size_t)n * G;
        float r = 0.0f;
        for (int g = 0; g < G; ++g)
            r = __fmaf_rn((float)Ps[lane * (kMaxG + 1) + g], __half2float(__ushort_as_half(__ldg(sr + g))), r);
        y[n] = __fmul_rn(r, sa);
    }
    __syncwarp();
}

__global__ void __launch_bounds__(kThreads) k_lowbit_gemv(const int8_t *__restrict__ a, float sa,
                                                         const uint8_t *__restrict__ w2,
                                                         const uint16_t *__restrict__ s2, int n2,
                                                         const uint8_t *__restrict__ w4,
                                                         const uint16_t *__restrict__ s4, int n4, int K,
                                                         float *__restrict__ y) {
    extern __shared__ int32_t smem[];
    int32_t *Ps = smem + jt::warp_id() * kRows * (kMaxG + 1);
    const int t2 = (n2 + kRows - 1) / kRows, t4 = (n4 + kRows - 1) / kRows;
    const int gw = blockIdx.x * kWarps + jt::warp_id();
    const int nw = gridDim.x * kWarps;
    for (int t = gw; t < t2 + t4; t += nw) {
        if (t < t2) {
            const int r0 = t * kRows;
            gemv_task<2>(a, sa, w2, s2, r0, min(kRows, n2 - r0), K, y, Ps);
        } else {
            const int r0 = (t - t2) * kRows;
            gemv_task<4>(a, sa, w4, s4, r0, min(kRows, n4 - r0), K, y + n2, Ps);
        }
    }
}

}  // namespace

// y[0..n2) from the INT2 rows, y[n2..n2+n4) from the INT4 rows.  K % 64 == 0,
// K <= 4096, packed rows 16-byte aligned (K/4 and K/2 bytes per row).
extern "C" int jtk_lowbit_gemv(const int8_t *a, float sa, const uint8_t *w2, const uint16_t *s2,
                               int n2, const uint8_t *w4, const uint16_t *s4, int n4, int K,
                               float *y, cudaStream_t stream) {
    if (K <= 0 || K % 64 || K / 64 > kMaxG || n2 < 0 || n4 < 0 || (n2 > 0 && (!w2 || !s2)) ||
        (n4 > 0 && (!w4 || !s4)) || !a || !y)
        return -1;
    if (n2 + n4 == 0) return 0;
    const size_t smem = (size_t)kWarps * kRows * (kMaxG + 1) * sizeof(int32_t);
    static bool attr = false;
    if (!attr) {
        if (cudaFuncSetAttribute(k_lowbit_gemv, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
            return -3;
        attr = true;
    }
    const int tasks = (n2 + kRows - 1) / kRows + (n4 + kRows - 1) / kRows;
    int grid = jtk_num_sms();
    if (grid * kWarps > tasks) grid = (tasks + kWarps - 1) / kWarps;
    k_lowbit_gemv<<<grid, kThreads, smem, stream>>>(a, sa, w2, s2, n2, w4, s4, n4, K, y);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}
