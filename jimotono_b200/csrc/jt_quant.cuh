// jt_quant.cuh - device form of the reference's symmetric int8 quantizer
// (w8a8.c:688-747): scale_d = maxabs / 127 (double), q = clamp(round(x /
// scale_d), -127, 127) with round() = half away from zero, zero block ->
// scale 1, q 0.  Codes are bit-identical to the reference.
//
// The division is done in fp32 first (x * (float)(127/maxabs)); that
// estimate is within 2^-23 * 127 < 2e-5 of the exact quotient, so whenever
// it lies farther than 1e-3 from a rounding tie the rounded code is already
// exact.  Only the rare near-tie case runs the double division the
// reference uses.  The fast path rounds with the magic-number addition
// (FMA pipe) rather than floor/convert instructions, which issue at a
// fraction of the FMA rate.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

namespace jt {

// K order inside every 16-element block of the expert-ordered token rows
// (xd, fp16) that feed the routed gate/up GEMM: position p of the block holds
// element kX16Order[p] = 4 (p % 4) + p / 4 of the block (a 4 x 4 transpose),
// the order in which that GEMM's INT2 unpack produces the weight values.
constexpr int kX16Order[16] = {0, 4, 8, 12, 1, 5, 9, 13, 2, 6, 10, 14, 3, 7, 11, 15};

// Byte i of word a and byte i of word b as the fp16 pair (a_i, b_i) (exact):
// the byte q is biased to the fp16 bit pattern of 1152 + q, then 1152 is
// subtracted.
__device__ __forceinline__ uint32_t x16_pair(uint32_t a, uint32_t b, uint32_t i) {
    const uint32_t t = __byte_perm(a, b, i | (i << 4) | ((4u + i) << 8) | ((4u + i) << 12));
    uint32_t r = (t & 0x00FF00FFu) ^ 0x64806480u;
    const __half2 h = __hsub2(*reinterpret_cast<const __half2 *>(&r), __half2half2(__ushort_as_half(0x6480u)));
    r = *reinterpret_cast<const uint32_t *>(&h);
    return r;
}

// 16 int8 codes in natural order (four little-endian words) -> 16 exact fp16
// values in kX16Order, positions 0-7 in lo and 8-15 in hi.
__device__ __forceinline__ void x16_block(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3, uint4 &lo,
                                          uint4 &hi) {
    lo = make_uint4(x16_pair(w0, w1, 0), x16_pair(w2, w3, 0), x16_pair(w0, w1, 1), x16_pair(w2, w3, 1));
    hi = make_uint4(x16_pair(w0, w1, 2), x16_pair(w2, w3, 2), x16_pair(w0, w1, 3), x16_pair(w2, w3, 3));
}

// Eight INT4 codes (one packed word: element 2b in the low nibble of byte
// b, 2b + 1 in the high nibble) -> the eight bf16 weights
// bf16_rn((2 li - 15) * s) in order, as four words, for a scale s already in
// bf16 (s2 = (s, s)): 2 li is moved into the low byte of each 16-bit lane of
// 0x4300 (bf16 128 + 2 li, exact), minus 143 gives the code exactly, and one
// bf16 multiply rounds the product.
__device__ __forceinline__ void int4_bf16x8(uint32_t w, __nv_bfloat162 s2, uint32_t (&o)[4]) {
    const uint32_t lo2 = (w << 1) & 0x1E1E1E1Eu;  // 2 li of the even elements, one per byte
    const uint32_t hi2 = (w >> 3) & 0x1E1E1E1Eu;  // 2 li of the odd elements
    const uint32_t k143u = 0x430F430Fu;           // bf16 (143, 143)
    const __nv_bfloat162 k143 = *reinterpret_cast<const __nv_bfloat162 *>(&k143u);
#pragma unroll
    for (int b = 0; b < 4; ++b) {
        // lanes (low 16 bits, high 16 bits) = bf16 (128 + 2 li_2b, 128 + 2 li_2b+1)
        const uint32_t t = (__byte_perm(lo2, hi2, b | ((4 + b) << 8)) & 0x00FF00FFu) | 0x43004300u;
        const __nv_bfloat162 c = __hsub2(*reinterpret_cast<const __nv_bfloat162 *>(&t), k143);
        const __nv_bfloat162 v = __hmul2(c, s2);
        o[b] = *reinterpret_cast<const uint32_t *>(&v);
    }
}

struct QuantBlock {
    double scale_d;   // maxabs / 127 (0 when maxabs == 0)
    float inv;        // (float)(127 / maxabs), fast-path multiplier
    float scale_f;    // stored scale: (float)scale_d, or 1.0f for a zero block
};

__device__ __forceinline__ QuantBlock quant_block(float maxabs) {
    QuantBlock b;
    if (maxabs == 0.0f) {
        b.scale_d = 0.0;
        b.inv = 0.0f;
        b.scale_f = 1.0f;
    } else {
        b.scale_d = __ddiv_rn((double)maxabs, 127.0);
        b.inv = __double2float_rn(__ddiv_rn(127.0, (double)maxabs));
        b.scale_f = __double2float_rn(b.scale_d);
    }
    return b;
}

// Exact reference rounding, used only near a rounding tie (kept out of line
// so callers do not carry the double-division code and its registers).
static __device__ __noinline__ int quant_code_exact(float x, double scale_d) {
    return static_cast<int>(round(__ddiv_rn((double)x, scale_d)));
}

// Nearest integer of an estimate y (|y| < 2^22) on the FMA pipe: y + 1.5*2^23
// rounds y to an integer (ties to even) and its bit pattern carries that
// integer; the distance |y - round(y)| is exact.  Away from a tie (distance
// below 0.499) round-to-even equals the reference's half-away-from-zero
// rounding.  A non-finite y gives a NaN distance, which takes the exact path.
__device__ __forceinline__ bool round_fast(float y, int &q) {
    const float t = __fadd_rn(y, 12582912.0f);
    const float dist = fabsf(__fsub_rn(y, __fsub_rn(t, 12582912.0f)));
    q = __float_as_int(t) - 0x4B400000;
    return dist < 0.499f;
}

__device__ __forceinline__ int quant_code(float x, const QuantBlock &b) {
    if (b.scale_d == 0.0) return 0;
    const float y = __fmul_rn(x, b.inv);
    int q;
    if (!round_fast(y, q)) q = quant_code_exact(x, b.scale_d);
    q = q > 127 ? 127 : q;
    q = q < -127 ? -127 : q;
    return q;
}

// Light form for the fused requantization of the expert GEMMs: the same
// codes and stored scale with single-precision divisions.  For a finite
// m > 0, (float)((double)m / 127) equals the correctly rounded float
// quotient m / 127: the two can differ only when the double quotient lands
// exactly on a float rounding midpoint, and since m has 24 significant bits
// that happens only when m / 127 is itself that midpoint, where both round
// to even.  The double scale is formed only on the rare near-tie path.
struct QuantBlockF {
    float maxabs;   // 0 for an all-zero block
    float inv;      // 127 / maxabs, fast-path multiplier
    float scale_f;  // stored scale (1.0f for a zero block)
};

__device__ __forceinline__ QuantBlockF quant_block_f(float maxabs) {
    QuantBlockF b;
    b.maxabs = maxabs;
    if (maxabs == 0.0f) {
        b.inv = 0.0f;
        b.scale_f = 1.0f;
    } else {
        b.inv = __fdiv_rn(127.0f, maxabs);
        b.scale_f = __fdiv_rn(maxabs, 127.0f);
    }
    return b;
}

static __device__ __noinline__ int quant_code_exact_m(float x, float maxabs) {
    const double scale_d = __ddiv_rn((double)maxabs, 127.0);
    return static_cast<int>(round(__ddiv_rn((double)x, scale_d)));
}

__device__ __forceinline__ int quant_code_f(float x, const QuantBlockF &b) {
    if (b.maxabs == 0.0f) return 0;
    const float y = __fmul_rn(x, b.inv);
    int q;
    if (!round_fast(y, q)) q = quant_code_exact_m(x, b.maxabs);
    q = q > 127 ? 127 : q;
    q = q < -127 ? -127 : q;
    return q;
}

}  // namespace jt
