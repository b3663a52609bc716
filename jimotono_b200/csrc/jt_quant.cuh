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
#include <cstdint>

namespace jt {

// K order inside every 16-byte block of the expert-ordered token rows (xd)
// that feed the routed gate/up GEMM: position p of the block holds element
// kInt2Order16[p] of the block, the order in which the INT2 unpack of that
// GEMM produces the weight codes.  int2_order16 applies it to one block held
// as four 32-bit words (natural order in, stored order out).
constexpr int kInt2Order16[16] = {0, 1, 4, 5, 8, 9, 12, 13, 2, 3, 6, 7, 10, 11, 14, 15};

__host__ __device__ __forceinline__ uint4 int2_order16(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3) {
#ifdef __CUDA_ARCH__
    return make_uint4(__byte_perm(w0, w1, 0x5410), __byte_perm(w2, w3, 0x5410), __byte_perm(w0, w1, 0x7632),
                      __byte_perm(w2, w3, 0x7632));
#else
    return make_uint4((w0 & 0xFFFFu) | (w1 << 16), (w2 & 0xFFFFu) | (w3 << 16), (w0 >> 16) | (w1 & 0xFFFF0000u),
                      (w2 >> 16) | (w3 & 0xFFFF0000u));
#endif
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
