// jt_swiglu.cuh - the SwiGLU of moe_layer.c:146-148
//   sig = 1 / (1 + exp(-g)),  silu = g * sig,  s = silu * u
// evaluated in fp32 with an exp built only from IEEE basic operations
// (Cody-Waite reduction with a 15-bit head of ln 2, degree-7 Taylor
// polynomial of e^r in Horner form, scaling by 2^k in two exact steps), so
// the GPU result is bit-identical to the CPU restatement used as the parity
// oracle.  The library is compiled with --fmad=false; every fused operation
// below is an explicit __fmaf_rn.
#pragma once

namespace jt {

__device__ __forceinline__ float det_expf(float x) {
    if (x != x) return x;
    x = fminf(x, 89.0f);
    x = fmaxf(x, -104.0f);
    const float kLog2e = 0x1.715476p+0f;
    const float kLn2Hi = 0x1.62e4p-1f;
    const float kLn2Lo = 0x1.7f7d1cp-20f;
    // k = rint(x * log2 e) by the magic-number addition (|x log2 e| < 151):
    // the same integer as rintf (ties to even) without a conversion
    // instruction; k itself is read from the sum's bit pattern
    const float tm = __fadd_rn(__fmul_rn(x, kLog2e), 12582912.0f);
    const float kf = __fsub_rn(tm, 12582912.0f);
    float r = __fmaf_rn(-kf, kLn2Hi, x);
    r = __fmaf_rn(-kf, kLn2Lo, r);
    float p = 0x1.a01a02p-13f;
    p = __fmaf_rn(p, r, 0x1.6c16c2p-10f);
    p = __fmaf_rn(p, r, 0x1.111112p-7f);
    p = __fmaf_rn(p, r, 0x1.555556p-5f);
    p = __fmaf_rn(p, r, 0x1.555556p-3f);
    p = __fmaf_rn(p, r, 0x1.0p-1f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const int k = __float_as_int(tm) - 0x4B400000;
    const int k1 = k >> 1, k2 = k - k1;
    const float s1 = __int_as_float((k1 + 127) << 23);
    const float s2 = __int_as_float((k2 + 127) << 23);
    return __fmul_rn(__fmul_rn(p, s1), s2);
}

// silu(g) = g * sig with sig = 1/(1 + exp(-g)); the reciprocal is the
// correctly rounded 1/den, identical to the IEEE division 1.0f / den.
__device__ __forceinline__ float silu(float g) {
    const float e = det_expf(-g);
    const float den = __fadd_rn(1.0f, e);
    const float sig = __frcp_rn(den);
    return __fmul_rn(g, sig);
}

__device__ __forceinline__ float swiglu(float g, float u) { return __fmul_rn(silu(g), u); }

// Two lanes of det_expf at once with packed f32x2 arithmetic for the
// products and the polynomial, bit for bit the scalar results: the same
// clamps, rounding of k, two-step reduction, polynomial and scaling.  (A NaN
// input gives a finite value here; the callers' SwiGLU result is NaN either
// way.)
__device__ __forceinline__ float2 det_expf2(float2 x) {
    x.x = fmaxf(fminf(x.x, 89.0f), -104.0f);
    x.y = fmaxf(fminf(x.y, 89.0f), -104.0f);
    const float2 kLog2e = make_float2(0x1.715476p+0f, 0x1.715476p+0f);
    // the rounding to an integer in scalar additions (as det_expf): the
    // packed f32x2 add did not give these bits for the magic-number form
    const float2 t = __fmul2_rn(x, kLog2e);
    const float2 tm = make_float2(__fadd_rn(t.x, 12582912.0f), __fadd_rn(t.y, 12582912.0f));
    const float2 kf = make_float2(__fsub_rn(tm.x, 12582912.0f), __fsub_rn(tm.y, 12582912.0f));
    const float2 nkf = make_float2(-kf.x, -kf.y);
    float2 r = __ffma2_rn(nkf, make_float2(0x1.62e4p-1f, 0x1.62e4p-1f), x);
    r = __ffma2_rn(nkf, make_float2(0x1.7f7d1cp-20f, 0x1.7f7d1cp-20f), r);
    float2 p = make_float2(0x1.a01a02p-13f, 0x1.a01a02p-13f);
    p = __ffma2_rn(p, r, make_float2(0x1.6c16c2p-10f, 0x1.6c16c2p-10f));
    p = __ffma2_rn(p, r, make_float2(0x1.111112p-7f, 0x1.111112p-7f));
    p = __ffma2_rn(p, r, make_float2(0x1.555556p-5f, 0x1.555556p-5f));
    p = __ffma2_rn(p, r, make_float2(0x1.555556p-3f, 0x1.555556p-3f));
    p = __ffma2_rn(p, r, make_float2(0x1.0p-1f, 0x1.0p-1f));
    p = __ffma2_rn(p, r, make_float2(1.0f, 1.0f));
    p = __ffma2_rn(p, r, make_float2(1.0f, 1.0f));
    const int k0 = __float_as_int(tm.x) - 0x4B400000, k1 = __float_as_int(tm.y) - 0x4B400000;
    const int a0 = k0 >> 1, b0 = k0 - a0, a1 = k1 >> 1, b1 = k1 - a1;
    const float2 s1 = make_float2(__int_as_float((a0 + 127) << 23), __int_as_float((a1 + 127) << 23));
    const float2 s2 = make_float2(__int_as_float((b0 + 127) << 23), __int_as_float((b1 + 127) << 23));
    return __fmul2_rn(__fmul2_rn(p, s1), s2);
}

// swiglu() of two lanes at once, bit for bit.
__device__ __forceinline__ float2 swiglu2(float2 g, float2 u) {
    const float2 e = det_expf2(make_float2(-g.x, -g.y));
    const float2 den = __fadd2_rn(make_float2(1.0f, 1.0f), e);
    const float2 sig = make_float2(__frcp_rn(den.x), __frcp_rn(den.y));
    return __fmul2_rn(__fmul2_rn(g, sig), u);
}

}  // namespace jt
