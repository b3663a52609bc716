// jt_pack.cu - weight preparation on the device: fp32 master weights to the
// packed INT2/INT4 group-64 format that the routed-expert GEMMs and the
// batch-1 GEMV read, and the reference's bit-plane index to the same codes.
//
// Level rule (lowbit.c:103-137, applied per 64-element K group instead of
// per whole column): maxa = max |w| over the group (double), t = w / maxa
// (0 for an all-zero group), li = floor(t*(n-1)/2 + (n-1)/2 + 0.5) clamped
// to [0, n-1] with n = 2^bits, all in double; the group's fp16 scale is
// (half)(float)(maxa / (n-1)), so code li stands for (2*li - (n-1)) * scale.
// Codes are little-endian along K: INT2 element k at bits 2*(k%4) of byte
// k/4, INT4 element k in the low (k even) or high (k odd) nibble of byte k/2.
//
// The level is first estimated in fp32 (error < 4e-6 on a value below 16);
// only when that estimate lies within 1e-4 of an integer, where floor()
// could go either way, is the double expression evaluated - the codes are
// those of the double formula in every case.
//
// HBM-bound: one warp per (row, group) reads the group's 256 bytes once
// with 8-byte loads and writes 16 (INT2) or 32 (INT4) code bytes and one
// fp16 scale.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "jt_internal.h"
#include "jt_ptx.cuh"

namespace {

// li of w for a group with max |w| = maxa (> 0 or == 0), n - 1 = NL1.
template <int NL1>
__device__ __forceinline__ int level_of(float w, float maxa_f, float inv_half) {
    constexpr float kC0 = NL1 / 2.0f + 0.5f;  // 2.0 (INT2) or 8.0 (INT4), exact
    if (maxa_f == 0.0f) return NL1 / 2 + (NL1 % 2);  // floor((n-1)/2 + 0.5)
    const float y = __fadd_rn(__fmul_rn(w, inv_half), kC0);
    const float fl = floorf(y);
    const float fr = __fsub_rn(y, fl);
    int li;
    if (fr > 1e-4f && fr < 0.9999f) {
        li = static_cast<int>(fl);
    } else {
        const double maxa = static_cast<double>(maxa_f);
        const double t = __ddiv_rn(static_cast<double>(w), maxa);
        const double yd = __dadd_rn(__dadd_rn(__ddiv_rn(__dmul_rn(t, (double)NL1), 2.0), NL1 / 2.0), 0.5);
        li = static_cast<int>(floor(yd));
    }
    li = li < 0 ? 0 : li;
    return li > NL1 ? NL1 : li;
}

// W [rows][K] fp32 -> packed [rows][K*BITS/8], scales fp16: row-major
// [rows][K/64] when n_ch == 0, else group-major per block of n_ch rows
// ([rows/n_ch][K/64][n_ch]).
template <int BITS>
__global__ void __launch_bounds__(256) k_pack_lowbit(const float *__restrict__ W, int rows, int K, int n_ch,
                                                     uint8_t *__restrict__ packed, __half *__restrict__ scales,
                                                     int *err) {
    constexpr int NL1 = (1 << BITS) - 1;
    const int lane = jt::lane_id();
    const int G = K / 64;
    const long long nwork = static_cast<long long>(rows) * G;
    const long long nwarps = static_cast<long long>(gridDim.x) * (blockDim.x / 32);
    for (long long wi = static_cast<long long>(blockIdx.x) * (blockDim.x / 32) + jt::warp_id(); wi < nwork;
         wi += nwarps) {
        const int r = static_cast<int>(wi / G), g = static_cast<int>(wi % G);
        const float2 v = __ldg(reinterpret_cast<const float2 *>(W + static_cast<size_t>(r) * K + 64 * g) + lane);
        const bool bad = !isfinite(v.x) || !isfinite(v.y);
        float m = fmaxf(fabsf(v.x), fabsf(v.y));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (__any_sync(0xffffffffu, bad) && lane == 0 && err) atomicExch(err, JT_KERR_NONFINITE);
        // (float)(0.5 * (n-1) / maxa): the fp32 estimate's multiplier
        const float inv_half = m == 0.0f ? 0.0f : __double2float_rn(__ddiv_rn(NL1 / 2.0, (double)m));
        const int l0 = level_of<NL1>(v.x, m, inv_half);
        const int l1 = level_of<NL1>(v.y, m, inv_half);
        const size_t row_bytes = static_cast<size_t>(K) * BITS / 8;
        uint8_t *dst = packed + static_cast<size_t>(r) * row_bytes + static_cast<size_t>(g) * (8 * BITS);
        if (BITS == 4) {
            dst[lane] = static_cast<uint8_t>(l0 | (l1 << 4));
        } else {
            const int nib = l0 | (l1 << 2);  // elements 2*lane, 2*lane + 1
            const int hi = __shfl_down_sync(0xffffffffu, nib, 1);
            if ((lane & 1) == 0) dst[lane >> 1] = static_cast<uint8_t>(nib | (hi << 4));
        }
        if (lane == 0) {
            const __half s = __float2half_rn(__double2float_rn(__ddiv_rn(static_cast<double>(m), (double)NL1)));
            size_t si;
            if (n_ch == 0)
                si = static_cast<size_t>(r) * G + g;
            else
                si = (static_cast<size_t>(r / n_ch) * G + g) * n_ch + (r % n_ch);
            scales[si] = s;
        }
    }
}

// Reference bit planes (jt_lowbit_col_to_idx, lowbit.c:117-137): column j
// owns idx[j*BITS*K/4 ...]; byte b*K/4 + q of it holds, in bit i, bit b of
// the code of element 4q + i.  One thread per packed output byte.
template <int BITS>
__global__ void k_planes_to_packed(const uint8_t *__restrict__ idx, int cols, int K, uint8_t *__restrict__ packed) {
    const size_t row_bytes = static_cast<size_t>(K) * BITS / 8;
    const size_t total = static_cast<size_t>(cols) * row_bytes;
    const size_t nq = static_cast<size_t>(K) / 4;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t j = i / row_bytes, m = i % row_bytes;
        const uint8_t *col = idx + j * BITS * nq;
        uint32_t out = 0;
        if (BITS == 2) {  // byte m = elements 4m .. 4m+3, all in plane byte m
            const uint32_t p0 = col[m], p1 = col[nq + m];
#pragma unroll
            for (int e = 0; e < 4; ++e) out |= (((p0 >> e) & 1u) | (((p1 >> e) & 1u) << 1)) << (2 * e);
        } else {  // byte m = elements 2m, 2m+1: plane byte m/2, bits 2(m%2), 2(m%2)+1
            const size_t q = m >> 1;
            const int e0 = static_cast<int>(m & 1) * 2;
            uint32_t l0 = 0, l1 = 0;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const uint32_t pb = col[b * nq + q];
                l0 |= ((pb >> e0) & 1u) << b;
                l1 |= ((pb >> (e0 + 1)) & 1u) << b;
            }
            out = l0 | (l1 << 4);
        }
        packed[i] = static_cast<uint8_t>(out);
    }
}

// Group scales of whole-column planes: every group of column j gets
// (half)(float)(w_scale[j] / (n-1)) - the packer's rule with one group
// spanning the column.  Same layouts as k_pack_lowbit.
__global__ void k_column_scales(const float *__restrict__ w_scale, int cols, int K, int n_ch, int nl1,
                                __half *__restrict__ scales, int *err) {
    const int G = K / 64;
    const size_t total = static_cast<size_t>(cols) * G;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int j = static_cast<int>(i / G), g = static_cast<int>(i % G);
        const float ws = w_scale[j];
        if (!(ws >= 0.0f) || !isfinite(ws)) {
            if (err) atomicExch(err, JT_KERR_NONFINITE);
        }
        const __half s = __float2half_rn(__double2float_rn(__ddiv_rn(static_cast<double>(ws), (double)nl1)));
        size_t si;
        if (n_ch == 0)
            si = static_cast<size_t>(j) * G + g;
        else
            si = (static_cast<size_t>(j / n_ch) * G + g) * n_ch + (j % n_ch);
        scales[si] = s;
    }
}

int grid_for(size_t work, int per_block) {
    const size_t blocks = (work + per_block - 1) / per_block;
    const size_t cap = static_cast<size_t>(jtk_num_sms()) * 16;
    return static_cast<int>(blocks < cap ? (blocks < 1 ? 1 : blocks) : cap);
}

}  // namespace

extern "C" int jtk_pack_lowbit(const float *W, int rows, int K, int bits, int n_ch, uint8_t *packed,
                               uint16_t *scales, cudaStream_t stream) {
    if (!W || !packed || !scales || rows <= 0 || K <= 0 || K % 64 || (bits != 2 && bits != 4) || n_ch < 0 ||
        (n_ch > 0 && rows % n_ch) || (reinterpret_cast<uintptr_t>(W) & 7u))
        return -1;
    const size_t warps = static_cast<size_t>(rows) * (K / 64);
    const int grid = grid_for(warps, 8);
    __half *s = reinterpret_cast<__half *>(scales);
    int *errw = jtk_error_word();
    if (bits == 2)
        k_pack_lowbit<2><<<grid, 256, 0, stream>>>(W, rows, K, n_ch, packed, s, errw);
    else
        k_pack_lowbit<4><<<grid, 256, 0, stream>>>(W, rows, K, n_ch, packed, s, errw);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int jtk_planes_to_packed(const uint8_t *idx, const float *w_scale, int cols, int K, int bits,
                                    int n_ch, uint8_t *packed, uint16_t *scales, cudaStream_t stream) {
    if (!idx || !packed || cols <= 0 || K <= 0 || K % 64 || (bits != 2 && bits != 4) || n_ch < 0 ||
        (n_ch > 0 && cols % n_ch) || ((w_scale == nullptr) != (scales == nullptr)))
        return -1;
    const size_t bytes = static_cast<size_t>(cols) * K * bits / 8;
    const int grid = grid_for(bytes, 256);
    if (bits == 2)
        k_planes_to_packed<2><<<grid, 256, 0, stream>>>(idx, cols, K, packed);
    else
        k_planes_to_packed<4><<<grid, 256, 0, stream>>>(idx, cols, K, packed);
    if (cudaGetLastError() != cudaSuccess) return -4;
    if (w_scale) {
        const size_t n = static_cast<size_t>(cols) * (K / 64);
        k_column_scales<<<grid_for(n, 256), 256, 0, stream>>>(w_scale, cols, K, n_ch, (1 << bits) - 1,
                                                              reinterpret_cast<__half *>(scales), jtk_error_word());
        if (cudaGetLastError() != cudaSuccess) return -4;
    }
    return 0;
}
