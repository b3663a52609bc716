// jt_shared.cu - the shared experts of the prepared MoE layer (batched path).
//
// Arithmetic of one shared expert s on token t (moe_layer.c:1468-1559 with
// the W8A8 projections of w8a8.c:1021-1072 and per-token activation scales):
//   g[t][c] = ((float)acc_g * xs[t]) * ssg[c],  u likewise      (int32 acc, exact)
//   hb[t][c] = bf16_rn(SwiGLU(g, u))                             (moe_layer.c:146-148)
//   hq[t][:], hs[t] = the symmetric int8 quantization of the row hb[t][:]
//                     (w8a8.c:688-747 over all fs channels, one scale per row)
//   y[t][o] (+)= ((float)acc_d * hs[t]) * ssd[o]                (acc_d = sum hq * wsd)
// so the down projection is a plain per-token x per-channel W8A8 GEMM.
//
// Pipeline per shared expert:
//   T >= 256: the CTA-pair gate/up kernel (jt_shared_pair.cu) writes hb and
//             the row maxima of |hb| directly;
//   T <  256: two dense W8A8 GEMMs (gate, up; fp32 out) and k_shared_swiglu;
//   k_shared_quant: the rows' codes and scales;
//   the dense W8A8 GEMM (jt_w8a8.cu) of the down projection, storing into y
//   for the first expert and adding for the others.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "jt_internal.h"
#include "jt_ptx.cuh"
#include "jt_quant.cuh"
#include "jt_swiglu.cuh"

namespace {

// hb = bf16(SwiGLU(g, u)) and the row maxima of |hb|; one CTA per token row,
// eight channels per thread step.
__global__ void __launch_bounds__(256) k_shared_swiglu(const float *__restrict__ g, const float *__restrict__ u,
                                                       int fs, uint16_t *__restrict__ hb,
                                                       float *__restrict__ rowmax, int *err) {
    const size_t row = blockIdx.x;
    float m = 0.0f;
    bool bad = false;
    for (int c = threadIdx.x * 8; c < fs; c += blockDim.x * 8) {
        const float4 *gp = reinterpret_cast<const float4 *>(g + row * fs + c);
        const float4 *up = reinterpret_cast<const float4 *>(u + row * fs + c);
        const float4 g0 = gp[0], g1 = gp[1], u0 = up[0], u1 = up[1];
        const float2 a = jt::swiglu2(make_float2(g0.x, g0.y), make_float2(u0.x, u0.y));
        const float2 b = jt::swiglu2(make_float2(g0.z, g0.w), make_float2(u0.z, u0.w));
        const float2 cc = jt::swiglu2(make_float2(g1.x, g1.y), make_float2(u1.x, u1.y));
        const float2 dd = jt::swiglu2(make_float2(g1.z, g1.w), make_float2(u1.z, u1.w));
        const __nv_bfloat162 v[4] = {__floats2bfloat162_rn(a.x, a.y), __floats2bfloat162_rn(b.x, b.y),
                                     __floats2bfloat162_rn(cc.x, cc.y), __floats2bfloat162_rn(dd.x, dd.y)};
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            w[i] = *reinterpret_cast<const uint32_t *>(&v[i]);
            const float lo = __uint_as_float(w[i] << 16), hi = __uint_as_float(w[i] & 0xFFFF0000u);
            bad |= !isfinite(lo) | !isfinite(hi);
            m = fmaxf(m, fmaxf(fabsf(lo), fabsf(hi)));
        }
        *reinterpret_cast<uint4 *>(hb + row * fs + c) = make_uint4(w[0], w[1], w[2], w[3]);
    }
    for (int o = 16; o > 0; o >>= 1) {
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        bad |= __shfl_xor_sync(0xffffffffu, (int)bad, o) != 0;
    }
    if ((threadIdx.x & 31) == 0) {
        atomicMax(reinterpret_cast<unsigned int *>(rowmax) + row, __float_as_uint(m));
        if (bad) atomicExch(err, JT_KERR_NONFINITE);
    }
}

// Row requantization: hq[t][:] = codes of hb[t][:] with the scale of the
// row maximum (w8a8.c:688-747), hs[t] = that scale, written over rowmax[t].
// One CTA per token row, 16 channels per thread step.
__global__ void __launch_bounds__(256) k_shared_quant(const uint16_t *__restrict__ hb, float *rowmax, int fs,
                                                      int8_t *__restrict__ hq) {
    const size_t row = blockIdx.x;
    const jt::QuantBlockF qb = jt::quant_block_f(rowmax[row]);
    for (int c = threadIdx.x * 16; c < fs; c += blockDim.x * 16) {
        const uint4 *src = reinterpret_cast<const uint4 *>(hb + row * fs + c);
        const uint4 a = src[0], b = src[1];
        const uint32_t hw[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        uint32_t q[4] = {0u, 0u, 0u, 0u};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int q0 = jt::quant_code_f(__uint_as_float(hw[i] << 16), qb);
            const int q1 = jt::quant_code_f(__uint_as_float(hw[i] & 0xFFFF0000u), qb);
            q[i >> 1] |= ((uint32_t)(uint8_t)(int8_t)q0 | ((uint32_t)(uint8_t)(int8_t)q1 << 8)) << (16 * (i & 1));
        }
        *reinterpret_cast<uint4 *>(hq + row * fs + c) = make_uint4(q[0], q[1], q[2], q[3]);
    }
    __syncthreads();  // every thread has read rowmax[row]
    if (threadIdx.x == 0) rowmax[row] = qb.scale_f;
}

}  // namespace

// The S shared experts on T token rows (codes xq [T][d], scales xs [T],
// sh_meta [T] = {xs, 1, t, 0}) into y [T][d] (stored by the first expert,
// added by the others).  Scratch: hb [T][fs] bf16, hq [T][fs], hs [T];
// g32 / u32 [T][fs] fp32 only when T < 256 (may be NULL otherwise).
extern "C" int jtk_moe_shared(const int8_t *wsg, const int8_t *wsu, const float *ssg, const float *ssu,
                              const int8_t *wsd, const float *ssd, int S, int fs, int d, const int8_t *xq,
                              const float *xs, const float4 *sh_meta, int T, uint16_t *hb, int8_t *hq,
                              float *hs, float *g32, float *u32, float *y, cudaStream_t stream) {
    if (S <= 0 || fs <= 0 || fs % 16 || d <= 0 || d % 16 || T <= 0) return -1;
    int *err = jtk_error_word();
    for (int s = 0; s < S; ++s) {
        const int8_t *g_w = wsg + (size_t)s * fs * d, *u_w = wsu + (size_t)s * fs * d;
        const float *g_s = ssg + (size_t)s * fs, *u_s = ssu + (size_t)s * fs;
        if (cudaMemsetAsync(hs, 0, (size_t)T * sizeof(float), stream) != cudaSuccess) return -4;
        int r = jtk_shared_gu_pair(g_w, u_w, g_s, u_s, fs, d, xq, sh_meta, T, hb, hs, stream);
        if (r == -1) {  // shape outside the pair kernel: gate and up as dense GEMMs
            if (g32 == NULL || u32 == NULL) return -1;
            r = jtk_w8a8_gemm(xq, d, g_w, d, T, fs, d, xs, g_s, 0.0, g32, fs, JTK_EPI_TOKEN_CHANNEL_F32, stream);
            if (r == 0)
                r = jtk_w8a8_gemm(xq, d, u_w, d, T, fs, d, xs, u_s, 0.0, u32, fs, JTK_EPI_TOKEN_CHANNEL_F32,
                                  stream);
            if (r == 0) {
                k_shared_swiglu<<<T, 256, 0, stream>>>(g32, u32, fs, hb, hs, err);
                r = cudaGetLastError() == cudaSuccess ? 0 : -4;
            }
        }
        if (r != 0) return r;
        k_shared_quant<<<T, 256, 0, stream>>>(hb, hs, fs, hq);
        if (cudaGetLastError() != cudaSuccess) return -4;
        r = jtk_w8a8_gemm(hq, fs, wsd + (size_t)s * d * fs, fs, T, d, fs, hs, ssd + (size_t)s * d, 0.0, y, d,
                          s == 0 ? JTK_EPI_TOKEN_CHANNEL_F32 : JTK_EPI_TOKEN_CHANNEL_F32_ACC, stream);
        if (r != 0) return r;
    }
    return 0;
}
