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
    const float kf = rintf(__fmul_rn(x, kLog2e));
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
    const int k = static_cast<int>(kf);
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

}  // namespace jt
