/* jt_oracle.c - CPU restatement of the quantized MoE / W8A8 hot path.
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker for tests/, the smoke test
 * and bench.py's cpu_baseline leg.  The shipped library never links it.
 * Every function names the reference lines it restates; see jt_oracle.h
 * for which parts are pinned to the reference and which parts this file
 * specifies (formats the reference does not have).
 *
 * Build: oracle/Makefile, -std=c11 -O2 -ffp-contract=off (no implicit FMA:
 * every fused multiply-add below is an explicit fmaf()). */
#include "jt_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------ quantization */

/* w8a8.c:688-747 (jt_w8a8_quant_per_tensor) applied per block. */
int jto_quant_blocks(const float *x, int rows, int cols, int blk, int8_t *q, float *scales) {
    if (!x || !q || !scales || rows <= 0 || cols <= 0 || blk <= 0 || cols % blk) return 2;
    const int nb = cols / blk;
    for (int r = 0; r < rows; r++) {
        for (int b = 0; b < nb; b++) {
            const float *src = x + (size_t)r * cols + (size_t)b * blk;
            int8_t *dst = q + (size_t)r * cols + (size_t)b * blk;
            double maxabs = 0.0;
            for (int i = 0; i < blk; i++) {
                if (!isfinite((double)src[i])) return 2;
                double a = fabs((double)src[i]);
                if (a > maxabs) maxabs = a;
            }
            if (maxabs == 0.0) {
                scales[(size_t)r * nb + b] = 1.0f;
                memset(dst, 0, (size_t)blk);
                continue;
            }
            double scale_d = maxabs / 127.0;
            float scale_f = (float)scale_d;
            if (!isfinite(scale_d) || scale_d <= 0.0 || !(scale_f > 0.0f)) return 2;
            scales[(size_t)r * nb + b] = scale_f;
            for (int i = 0; i < blk; i++) {
                double qd = round((double)src[i] / scale_d);
                if (qd > 127.0) qd = 127.0;
                if (qd < -127.0) qd = -127.0;
                dst[i] = (int8_t)(int)qd;
            }
        }
    }
    return 0;
}

/* Integer part of w8a8.c:654-686 with B[k][n] = W[n][k]. */
void jto_gemm_s8(const int8_t *A, const int8_t *W, int32_t *acc, int M, int N, int K) {
    for (int m = 0; m < M; m++) {
        const int8_t *a = A + (size_t)m * K;
        for (int n = 0; n < N; n++) {
            const int8_t *w = W + (size_t)n * K;
            int32_t s = 0;
            for (int k = 0; k < K; k++) s += (int32_t)a[k] * (int32_t)w[k];
            acc[(size_t)m * N + n] = s;
        }
    }
}

void jto_w8a8_token_channel(const int32_t *acc, const float *sx, const float *sw, float *C,
                            int M, int N) {
    for (int m = 0; m < M; m++)
        for (int n = 0; n < N; n++) {
            float v = (float)acc[(size_t)m * N + n];
            v = v * sx[m];
            v = v * sw[n];
            C[(size_t)m * N + n] = v;
        }
}

/* ------------------------------------------------------------ routing */

/* routing.c:16-76 per token; bias added in float before the call, the way a
 * caller of jt_routing_topk adds a selection bias. */
/* moe_layer.c:67-86 (jt_moe_avx2_dot) and :1114-1137. */
int jto_router_logits(const float *x, const float *wgate, int T, int d, int E, float *logits) {
    if (!x || !wgate || !logits || T <= 0 || d <= 0 || E <= 0) return 2;
    const int d4 = d & ~3;
    for (int t = 0; t < T; t++) {
        const float *xt = x + (size_t)t * d;
        for (int e = 0; e < E; e++) {
            const float *we = wgate + (size_t)e * d;
            double lane[4] = {0.0, 0.0, 0.0, 0.0};
            int j = 0;
            for (; j < d4; j += 4)
                for (int l = 0; l < 4; l++) lane[l] = lane[l] + (double)xt[j + l] * (double)we[j + l];
            double s = (lane[0] + lane[1]) + (lane[2] + lane[3]);
            for (; j < d; j++) s += (double)xt[j] * (double)we[j];
            if (!isfinite(s)) return 2;
            const float f = (float)s;
            if (!isfinite(f)) return 2;
            logits[(size_t)t * E + e] = f;
        }
    }
    return 0;
}

int jto_route_topk(const float *logits, const float *bias, int T, int E, int k, int32_t *ids,
                   float *w) {
    if (!logits || !ids || !w || T <= 0 || E <= 0 || k <= 0 || k > E) return 2;
    float *l = (float *)malloc((size_t)E * sizeof(float));
    if (!l) return 1;
    for (int t = 0; t < T; t++) {
        for (int e = 0; e < E; e++) {
            float v = logits[(size_t)t * E + e];
            if (bias) v = v + bias[e];
            if (isnan(v)) {
                free(l);
                return 2;
            }
            l[e] = v;
        }
        int32_t *oid = ids + (size_t)t * k;
        float *ow = w + (size_t)t * k;
        for (int p = 0; p < k; p++) {
            int best = E;
            float best_v = 0.0f;
            for (int i = 0; i < E; i++) {
                int taken = 0;
                for (int q = 0; q < p; q++) taken |= (oid[q] == i);
                float v = taken ? -INFINITY : l[i];
                int better = (best == E) ? 1 : (v > best_v);
                best = better ? i : best;
                best_v = better ? v : best_v;
            }
            oid[p] = best;
        }
        float mx = l[oid[0]];
        for (int p = 1; p < k; p++) {
            float v = l[oid[p]];
            mx = (v > mx) ? v : mx;
        }
        double sum = 0.0;
        for (int p = 0; p < k; p++) {
            double e = exp((double)l[oid[p]] - (double)mx);
            sum += e;
            ow[p] = (float)e;
        }
        if (!(sum > 0.0) || !isfinite(sum)) {
            free(l);
            return 2;
        }
        float inv = (float)(1.0 / sum);
        for (int p = 0; p < k; p++) ow[p] *= inv;
    }
    free(l);
    return 0;
}

/* moe_layer.c:895-978 (jt_moe_batch_sort). */
int jto_batch_sort(const int32_t *ids, int T, int k, int E, float cap_factor, int32_t *perm,
                   int32_t *off, uint8_t *drop, int *out_kept) {
    if (!ids || !perm || !off || !drop || T <= 0 || k <= 0 || E <= 0 || k > E) return 2;
    if (!(cap_factor >= 1.0f) || !(cap_factor <= 1.5f)) return 2;
    const size_t Tk = (size_t)T * k;
    for (size_t q = 0; q < Tk; q++)
        if (ids[q] < 0 || ids[q] >= E) return 2;
    double capd = ceil((double)cap_factor * (double)Tk / (double)E);
    if (!isfinite(capd) || capd < 1.0) return 2;
    const size_t cap = (size_t)capd;
    size_t *cnt = (size_t *)calloc((size_t)E, sizeof(size_t));
    if (!cnt) return 1;
    for (size_t q = 0; q < Tk; q++) cnt[ids[q]]++;
    off[0] = 0;
    for (int e = 0; e < E; e++) off[e + 1] = off[e] + (int32_t)(cnt[e] < cap ? cnt[e] : cap);
    for (int e = 0; e < E; e++) cnt[e] = (size_t)off[e];
    for (size_t q = 0; q < Tk; q++) {
        int e = ids[q];
        if ((int32_t)cnt[e] < off[e + 1]) {
            perm[cnt[e]] = (int32_t)q;
            cnt[e]++;
            drop[q] = 0;
        } else {
            drop[q] = 1;
        }
    }
    if (out_kept) *out_kept = off[E];
    free(cnt);
    return 0;
}

/* moe_layer.c:1171-1201. */
int jto_renorm(float *w, const uint8_t *drop, int T, int k) {
    for (int t = 0; t < T; t++) {
        double s = 0.0;
        int nd = 0;
        for (int p = 0; p < k; p++) {
            size_t q = (size_t)t * k + p;
            if (drop[q])
                nd++;
            else
                s += (double)w[q];
        }
        if (nd > 0 && s > 0.0) {
            if (!isfinite(s)) return 2;
            for (int p = 0; p < k; p++) {
                size_t q = (size_t)t * k + p;
                if (drop[q]) continue;
                double rw = (double)w[q] / s;
                if (!isfinite(rw) || rw < 0.0) return 2;
                w[q] = (float)rw;
            }
        }
    }
    return 0;
}

/* ------------------------------------------------------------ fp16 */

float jto_half_to_float(uint16_t h) {
    const uint32_t s = (uint32_t)(h >> 15) & 1u, e = (uint32_t)(h >> 10) & 31u,
                   m = (uint32_t)h & 1023u;
    float v;
    if (e == 0)
        v = ldexpf((float)m, -24);
    else if (e == 31)
        v = m ? NAN : INFINITY;
    else
        v = ldexpf((float)(m | 1024u), (int)e - 25);
    return s ? -v : v;
}

uint16_t jto_float_to_half(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    float a = fabsf(f);
    if (isnan(f)) return (uint16_t)(sign | 0x7e00u);
    if (a >= 65520.0f) return (uint16_t)(sign | 0x7c00u);
    if (a < ldexpf(1.0f, -14)) { /* subnormal half: units of 2^-24 */
        float u = a * 16777216.0f; /* exact scaling by 2^24 */
        uint32_t m = (uint32_t)nearbyintf(u);
        return (uint16_t)(sign | m);
    }
    int e;
    float fr = frexpf(a, &e); /* a = fr * 2^e, fr in [0.5,1) */
    float mant = ldexpf(fr, 11); /* [1024, 2048) */
    uint32_t m = (uint32_t)nearbyintf(mant);
    int he = e - 1 + 15;
    if (m == 2048u) {
        m = 1024u;
        he++;
    }
    if (he >= 31) return (uint16_t)(sign | 0x7c00u);
    return (uint16_t)(sign | ((uint32_t)he << 10) | (m & 1023u));
}

float jto_bf16_to_float(uint16_t h) {
    const uint32_t x = (uint32_t)h << 16;
    float f;
    memcpy(&f, &x, 4);
    return f;
}

uint16_t jto_float_to_bf16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    if (isnan(f)) return (uint16_t)((x >> 16) | 0x40u);
    x += 0x7FFFu + ((x >> 16) & 1u); /* round to nearest even (overflow to inf) */
    return (uint16_t)(x >> 16);
}

/* ------------------------------------------------------------ low-bit format */

/* Level rule of lowbit.c:78-88 applied per `group` elements along K. */
int jto_pack_lowbit(const float *W, int rows, int K, int bits, int group, uint8_t *packed,
                    uint16_t *scales) {
    if (!W || !packed || !scales || rows <= 0 || K <= 0 || group <= 0 || K % group) return 2;
    if (bits != 2 && bits != 4) return 2;
    const int nl = 1 << bits, per_byte = 8 / bits, ng = K / group;
    const size_t row_bytes = (size_t)K / per_byte;
    memset(packed, 0, row_bytes * rows);
    for (int r = 0; r < rows; r++) {
        for (int g = 0; g < ng; g++) {
            const float *src = W + (size_t)r * K + (size_t)g * group;
            double maxa = 0.0;
            for (int i = 0; i < group; i++) {
                if (!isfinite((double)src[i])) return 2;
                double a = fabs((double)src[i]);
                if (a > maxa) maxa = a;
            }
            scales[(size_t)r * ng + g] = jto_float_to_half((float)(maxa / (double)(nl - 1)));
            for (int i = 0; i < group; i++) {
                double t = (maxa == 0.0) ? 0.0 : (double)src[i] / maxa;
                double li = floor(t * (double)(nl - 1) / 2.0 + (double)(nl - 1) / 2.0 + 0.5);
                long l = (long)li;
                if (l < 0) l = 0;
                if (l > nl - 1) l = nl - 1;
                const int k = g * group + i;
                packed[(size_t)r * row_bytes + (size_t)(k / per_byte)] |=
                    (uint8_t)((unsigned)l << (bits * (k % per_byte)));
            }
        }
    }
    return 0;
}

int jto_code_at(const uint8_t *packed, int K, int bits, int r, int k) {
    const int per_byte = 8 / bits;
    const size_t row_bytes = (size_t)K / per_byte;
    const uint8_t b = packed[(size_t)r * row_bytes + (size_t)(k / per_byte)];
    return (b >> (bits * (k % per_byte))) & ((1 << bits) - 1);
}

/* ------------------------------------------------------------ SwiGLU */

/* exp(x) in fp32 from IEEE basic operations only, so the CPU and the GPU
 * produce identical bits: Cody-Waite reduction x = k ln2 + r with a 15-bit
 * head of ln2 (k*LN2_HI exact for |k| < 512), |r| <= ln2/2, then the
 * degree-7 Taylor polynomial of e^r in Horner form (truncation error
 * < 6e-9 relative) and scaling by 2^k in two exact power-of-two steps. */
float jto_expf(float x) {
    if (x != x) return x;
    if (x > 89.0f) x = 89.0f;
    if (x < -104.0f) x = -104.0f;
    const float kLog2e = 0x1.715476p+0f;
    const float kLn2Hi = 0x1.62e4p-1f;
    const float kLn2Lo = 0x1.7f7d1cp-20f;
    const float kf = rintf(x * kLog2e);
    float r = fmaf(-kf, kLn2Hi, x);
    r = fmaf(-kf, kLn2Lo, r);
    float p = 0x1.a01a02p-13f;    /* 1/7! */
    p = fmaf(p, r, 0x1.6c16c2p-10f); /* 1/6! */
    p = fmaf(p, r, 0x1.111112p-7f);  /* 1/5! */
    p = fmaf(p, r, 0x1.555556p-5f);  /* 1/4! */
    p = fmaf(p, r, 0x1.555556p-3f);  /* 1/3! */
    p = fmaf(p, r, 0x1.0p-1f);       /* 1/2! */
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const int k = (int)kf;
    const int k1 = k >> 1, k2 = k - k1; /* both in [-75, 64] */
    uint32_t b1 = (uint32_t)(k1 + 127) << 23, b2 = (uint32_t)(k2 + 127) << 23;
    float s1, s2;
    memcpy(&s1, &b1, 4);
    memcpy(&s2, &b2, 4);
    return (p * s1) * s2;
}

/* SwiGLU of moe_layer.c:146-148 (sig = 1/(1+exp(-g)), silu = g*sig,
 * s = silu*u), evaluated in fp32 with jto_expf. */
float jto_swiglu(float g, float u) {
    const float e = jto_expf(-g);
    const float den = 1.0f + e;
    const float sig = 1.0f / den;
    const float silu = g * sig;
    return silu * u;
}

/* ------------------------------------------------------------ low-bit GEMV */

static inline int signed_code(int li, int bits) { return 2 * li - ((1 << bits) - 1); }

void jto_lowbit_partials(const int8_t *a, const uint8_t *packed, int N, int K, int bits,
                         int32_t *P) {
    const int ng = K / 64;
    for (int n = 0; n < N; n++)
        for (int g = 0; g < ng; g++) {
            int32_t s = 0;
            for (int i = 0; i < 64; i++) {
                const int k = g * 64 + i;
                s += (int32_t)a[k] * signed_code(jto_code_at(packed, K, bits, n, k), bits);
            }
            P[(size_t)n * ng + g] = s;
        }
}

void jto_lowbit_gemv(const int8_t *a, float sa, const uint8_t *packed, const uint16_t *scales,
                     int N, int K, int bits, float *y) {
    const int ng = K / 64;
    int32_t *P = (int32_t *)malloc((size_t)ng * sizeof(int32_t));
    for (int n = 0; n < N; n++) {
        jto_lowbit_partials(a, packed + (size_t)n * (size_t)(K * bits / 8), 1, K, bits, P);
        float r = 0.0f;
        for (int g = 0; g < ng; g++)
            r = fmaf((float)P[g], jto_half_to_float(scales[(size_t)n * ng + g]), r);
        y[n] = r * sa;
    }
    free(P);
}

/* ------------------------------------------------------------ MoE layer */

/* The gate/up weight of code c (in {-3, -1, 1, 3}) in a group with fp16
 * scale s: fp16_rn(c * s) (c * s is exact in fp32; +-s needs no rounding). */
static float gu_weight16(int c, uint16_t s) {
    return jto_half_to_float(jto_float_to_half((float)c * jto_half_to_float(s)));
}

/* sum_k x[k] * w16[k] of one packed INT2 row in double (every product and
 * partial sum exact up to the final rounding: 18-bit products, |sum| < 2^40),
 * rounded once to fp32: the value the tensor core's fp32 accumulation
 * approximates. */
static float gu_dot16(const int8_t *xq, const uint8_t *row, const uint16_t *s_col, int d, int f) {
    double acc = 0.0;
    for (int g = 0; g < d / 64; g++) {
        const uint16_t sg = s_col[(size_t)g * f];
        float wv[4];
        for (int li = 0; li < 4; li++) wv[li] = gu_weight16(2 * li - 3, sg);
        for (int i = 0; i < 64; i++) {
            const int k = g * 64 + i;
            const int li = (row[k / 4] >> (2 * (k % 4))) & 3;
            acc += (double)xq[k] * (double)wv[li];
        }
    }
    return (float)acc;
}

/* The down weight of INT4 code li (c = 2 li - 15) in a group with fp16
 * scale s: bf16_rn(c * bf16_rn(s)) (the product is exact in fp32). */
static float dn_weight16(int li, uint16_t s) {
    const float sb = jto_bf16_to_float(jto_float_to_bf16(jto_half_to_float(s)));
    return jto_bf16_to_float(jto_float_to_bf16((float)(2 * li - 15) * sb));
}

/* Routed expert e on one quantized token row:
 *   gate/up: g = fl32(dot16 * sa) with dot16 = sum_k x[k] * fp16_rn(c_k * s_g(k))
 *     (gu_dot16; the CUDA path accumulates the same products in fp32 on the
 *     tensor cores, so it agrees to rounding, not bit for bit)
 *   h = bf16_rn(SwiGLU(gate, up))  (hb: bf16 bits [f])
 *   down: y[o] = fl32(sum_k h[k] * bf16_rn(c_ok * bf16_rn(s_g(k)[o]))) accumulated in
 *     double (bf16 x bf16 products are exact), the value the tensor core's
 *     fp32 accumulation approximates. */
static void routed_expert(const jto_moe_dims *dm, const jto_moe_weights *w, int e,
                          const int8_t *xq, float xs, uint16_t *hb, float *yout,
                          float *gbuf, float *ubuf, float *hbuf) {
    const int d = dm->d, f = dm->f, gd = d / 64, gf = f / 64;
    const uint8_t *wg = w->wg + (size_t)e * f * (d / 4);
    const uint8_t *wu = w->wu + (size_t)e * f * (d / 4);
    const uint16_t *sg = w->sg + (size_t)e * gd * f; /* [g][c] */
    const uint16_t *su = w->su + (size_t)e * gd * f;
    const uint8_t *wd = w->wd + (size_t)e * d * (f / 2);
    const uint16_t *sd = w->sd + (size_t)e * gf * d; /* [g][o] */
    for (int c = 0; c < f; c++) {
        gbuf[c] = gu_dot16(xq, wg + (size_t)c * (d / 4), sg + c, d, f) * xs;
        ubuf[c] = gu_dot16(xq, wu + (size_t)c * (d / 4), su + c, d, f) * xs;
        hb[c] = jto_float_to_bf16(jto_swiglu(gbuf[c], ubuf[c]));
        hbuf[c] = jto_bf16_to_float(hb[c]);
    }
    for (int o = 0; o < d; o++) {
        const uint8_t *row = wd + (size_t)o * (f / 2);
        double acc = 0.0;
        for (int g = 0; g < gf; g++) {
            float wv[16];
            for (int li = 0; li < 16; li++) wv[li] = dn_weight16(li, sd[(size_t)g * d + o]);
            for (int i = 0; i < 64; i++) {
                const int k = g * 64 + i;
                const int li = (row[k / 2] >> (4 * (k % 2))) & 15;
                acc += (double)hbuf[k] * (double)wv[li];
            }
        }
        yout[o] = (float)acc;
    }
}

/* Shared expert s on token t:
 *   gate = ((float)acc * xs) * ssg[c]; up likewise; h = bf16_rn(SwiGLU);
 *   h requantized per token row (one scale over all fs channels,
 *   w8a8.c:688-747 on the row); down: y = ((float)acc * hs) * ssd[o] with
 *   acc = sum_k hq[k] * wsd[o][k] (int32, exact) - the per-token x
 *   per-channel W8A8 of w8a8.c:1021-1072. */
static void shared_expert(const jto_moe_dims *dm, const jto_moe_weights *w, int s,
                          const int8_t *xq, float xs, float *yout, float *hbuf, int8_t *hq,
                          float *hs) {
    const int d = dm->d, fs = dm->fs;
    const int8_t *wsg = w->wsg + (size_t)s * fs * d;
    const int8_t *wsu = w->wsu + (size_t)s * fs * d;
    const int8_t *wsd = w->wsd + (size_t)s * d * fs;
    for (int c = 0; c < fs; c++) {
        int32_t ag = 0, au = 0;
        for (int k = 0; k < d; k++) {
            ag += (int32_t)xq[k] * (int32_t)wsg[(size_t)c * d + k];
            au += (int32_t)xq[k] * (int32_t)wsu[(size_t)c * d + k];
        }
        float g = ((float)ag * xs) * w->ssg[(size_t)s * fs + c];
        float u = ((float)au * xs) * w->ssu[(size_t)s * fs + c];
        hbuf[c] = jto_bf16_to_float(jto_float_to_bf16(jto_swiglu(g, u)));
    }
    jto_quant_blocks(hbuf, 1, fs, fs, hq, hs);
    for (int o = 0; o < d; o++) {
        int32_t acc = 0;
        for (int k = 0; k < fs; k++) acc += (int32_t)hq[k] * (int32_t)wsd[(size_t)o * fs + k];
        yout[o] = ((float)acc * hs[0]) * w->ssd[(size_t)s * d + o];
    }
}

int jto_moe_forward(const jto_moe_dims *dm, const jto_moe_weights *w, const float *x,
                    const float *logits, const float *bias, float *y, jto_moe_trace *tr) {
    const int T = dm->T, d = dm->d, f = dm->f, E = dm->E, k = dm->k, S = dm->S, fs = dm->fs;
    if (T <= 0 || d <= 0 || f <= 0 || E <= 0 || k <= 0 || k > E || S < 0) return 2;
    if (d % 128 || f % 128 || (S > 0 && fs % 128)) return 2;
    const size_t Tk = (size_t)T * k;
    int rc = 2;
    int32_t *ids = malloc(Tk * sizeof(int32_t));
    float *wt = malloc(Tk * sizeof(float));
    int32_t *perm = malloc(Tk * sizeof(int32_t));
    int32_t *off = malloc(((size_t)E + 1) * sizeof(int32_t));
    uint8_t *drop = malloc(Tk);
    int8_t *xq = malloc((size_t)T * d);
    float *xs = malloc((size_t)T * sizeof(float));
    int fmax_ = f > fs ? f : fs;
    float *gbuf = malloc((size_t)fmax_ * sizeof(float));
    float *ubuf = malloc((size_t)fmax_ * sizeof(float));
    float *hbuf = malloc((size_t)fmax_ * sizeof(float));
    int8_t *hqtmp = malloc((size_t)fmax_);
    float *hstmp = malloc((size_t)(fmax_ / 64 + 1) * sizeof(float));
    uint16_t *hbtmp = malloc((size_t)fmax_ * sizeof(uint16_t));
    float *ypair = malloc(Tk * (size_t)d * sizeof(float));
    float *ys = malloc((size_t)(S > 0 ? S : 1) * T * (size_t)d * sizeof(float));
    double *yacc = calloc((size_t)T * d, sizeof(double));
    int kept = 0;
    if (!ids || !wt || !perm || !off || !drop || !xq || !xs || !gbuf || !ubuf || !hbuf ||
        !hqtmp || !hstmp || !hbtmp || !ypair || !ys || !yacc) {
        rc = 1;
        goto out;
    }
    if (jto_route_topk(logits, bias, T, E, k, ids, wt)) goto out;
    if (jto_batch_sort(ids, T, k, E, dm->cap_factor, perm, off, drop, &kept)) goto out;
    if (jto_renorm(wt, drop, T, k)) goto out;
    if (jto_quant_blocks(x, T, d, d, xq, xs)) goto out;
    for (int i = 0; i < kept; i++) {
        const int q = perm[i], t = q / k, e = ids[q];
        routed_expert(dm, w, e, xq + (size_t)t * d, xs[t], hbtmp, ypair + (size_t)i * d, gbuf, ubuf,
                      hbuf);
        if (tr && tr->h) memcpy(tr->h + (size_t)i * f, hbtmp, (size_t)f * sizeof(uint16_t));
    }
    for (int s = 0; s < S; s++)
        for (int t = 0; t < T; t++)
            shared_expert(dm, w, s, xq + (size_t)t * d, xs[t], ys + ((size_t)s * T + t) * d,
                          hbuf, hqtmp, hstmp);
    /* combine: moe_layer.c:1443-1463 (slots ascending, dropped skipped) then
     * shared experts in s order (moe_layer.c:1549-1559), commit (:1568-1574). */
    {
        int32_t *pos = malloc(Tk * sizeof(int32_t)); /* q -> perm index */
        if (!pos) {
            rc = 1;
            goto out;
        }
        for (int i = 0; i < kept; i++) pos[perm[i]] = i;
        for (int t = 0; t < T; t++) {
            double *ya = yacc + (size_t)t * d;
            for (int p = 0; p < k; p++) {
                const size_t q = (size_t)t * k + p;
                if (drop[q]) continue;
                const float *yp = ypair + (size_t)pos[q] * d;
                for (int o = 0; o < d; o++) ya[o] += (double)wt[q] * (double)yp[o];
            }
            for (int s = 0; s < S; s++) {
                const float *yp = ys + ((size_t)s * T + t) * d;
                for (int o = 0; o < d; o++) ya[o] += (double)yp[o];
            }
        }
        free(pos);
    }
    for (size_t i = 0; i < (size_t)T * d; i++) y[i] = (float)yacc[i];
    if (tr) {
        if (tr->ids) memcpy(tr->ids, ids, Tk * sizeof(int32_t));
        if (tr->w) memcpy(tr->w, wt, Tk * sizeof(float));
        if (tr->perm) memcpy(tr->perm, perm, (size_t)kept * sizeof(int32_t));
        if (tr->off) memcpy(tr->off, off, ((size_t)E + 1) * sizeof(int32_t));
        if (tr->drop) memcpy(tr->drop, drop, Tk);
        if (tr->xq) memcpy(tr->xq, xq, (size_t)T * d);
        if (tr->xs) memcpy(tr->xs, xs, (size_t)T * sizeof(float));
        if (tr->ypair) memcpy(tr->ypair, ypair, (size_t)kept * d * sizeof(float));
        if (tr->yshared) {
            for (size_t i = 0; i < (size_t)T * d; i++) {
                float acc = 0.0f;
                for (int s = 0; s < S; s++) acc += ys[(size_t)s * T * d + i];
                tr->yshared[i] = acc;
            }
        }
        tr->kept = kept;
    }
    rc = 0;
out:
    free(ids);
    free(wt);
    free(perm);
    free(off);
    free(drop);
    free(xq);
    free(xs);
    free(gbuf);
    free(ubuf);
    free(hbuf);
    free(hqtmp);
    free(hstmp);
    free(hbtmp);
    free(ypair);
    free(ys);
    free(yacc);
    return rc;
}

/* Sampled form of jto_moe_forward for layer shapes whose full restatement
 * takes too long on one core (the benchmarked configurations).  Routing
 * (routing.c:16-76), the capacity sort (moe_layer.c:895-978), the
 * renormalization (moe_layer.c:1171-1201) and the token quantization run in
 * full and go to `tr` (ids, w, perm, off, drop, xq, xs, kept).  The routed
 * expert chain runs only for the kept rows rows[i] % kept (perm indices;
 * the index used is written back to rows[i]) -> hq_rows [n_rows][f],
 * hs_rows [n_rows][f/64].  The layer output, combined as in
 * moe_layer.c:1443-1574 (double, slots ascending, then the shared experts
 * in order), is formed only for the tokens toks[i] -> y_tok [n_tok][d].
 * Every computed value is the one jto_moe_forward gives for the same row or
 * token. */
int jto_moe_forward_sampled(const jto_moe_dims *dm, const jto_moe_weights *w, const float *x,
                            const float *logits, const float *bias, int32_t *rows, int n_rows,
                            uint16_t *h_rows, const int32_t *toks, int n_tok, float *y_tok,
                            jto_moe_trace *tr) {
    const int T = dm->T, d = dm->d, f = dm->f, E = dm->E, k = dm->k, S = dm->S, fs = dm->fs;
    if (T <= 0 || d <= 0 || f <= 0 || E <= 0 || k <= 0 || k > E || S < 0) return 2;
    if (d % 128 || f % 128 || (S > 0 && fs % 128)) return 2;
    if (n_rows < 0 || n_tok < 0) return 2;
    for (int i = 0; i < n_tok; i++)
        if (toks[i] < 0 || toks[i] >= T) return 2;
    const size_t Tk = (size_t)T * k;
    int rc = 2, kept = 0;
    int32_t *ids = malloc(Tk * sizeof(int32_t));
    float *wt = malloc(Tk * sizeof(float));
    int32_t *perm = malloc(Tk * sizeof(int32_t));
    int32_t *off = malloc(((size_t)E + 1) * sizeof(int32_t));
    uint8_t *drop = malloc(Tk);
    int8_t *xq = malloc((size_t)T * d);
    float *xs = malloc((size_t)T * sizeof(float));
    const int fmax_ = f > fs ? f : fs;
    float *gbuf = malloc((size_t)fmax_ * sizeof(float));
    float *ubuf = malloc((size_t)fmax_ * sizeof(float));
    float *hbuf = malloc((size_t)fmax_ * sizeof(float));
    int8_t *hqtmp = malloc((size_t)fmax_);
    float *hstmp = malloc((size_t)(fmax_ / 64 + 1) * sizeof(float));
    uint16_t *hbtmp = malloc((size_t)fmax_ * sizeof(uint16_t));
    float *yrow = malloc((size_t)d * sizeof(float));
    double *yacc = malloc((size_t)d * sizeof(double));
    if (!ids || !wt || !perm || !off || !drop || !xq || !xs || !gbuf || !ubuf || !hbuf ||
        !hqtmp || !hstmp || !hbtmp || !yrow || !yacc) {
        rc = 1;
        goto out;
    }
    if (jto_route_topk(logits, bias, T, E, k, ids, wt)) goto out;
    if (jto_batch_sort(ids, T, k, E, dm->cap_factor, perm, off, drop, &kept)) goto out;
    if (jto_renorm(wt, drop, T, k)) goto out;
    if (jto_quant_blocks(x, T, d, d, xq, xs)) goto out;
    for (int i = 0; i < n_rows && kept > 0; i++) {
        const int r = (int)((uint32_t)rows[i] % (uint32_t)kept);
        rows[i] = r;
        const int q = perm[r], t = q / k, e = ids[q];
        routed_expert(dm, w, e, xq + (size_t)t * d, xs[t], h_rows + (size_t)i * f, yrow, gbuf, ubuf, hbuf);
    }
    for (int i = 0; i < n_tok; i++) {
        const int t = toks[i];
        for (int o = 0; o < d; o++) yacc[o] = 0.0;
        for (int p = 0; p < k; p++) {
            const size_t q = (size_t)t * k + p;
            if (drop[q]) continue;
            routed_expert(dm, w, ids[q], xq + (size_t)t * d, xs[t], hbtmp, yrow, gbuf, ubuf, hbuf);
            for (int o = 0; o < d; o++) yacc[o] += (double)wt[q] * (double)yrow[o];
        }
        for (int s = 0; s < S; s++) {
            shared_expert(dm, w, s, xq + (size_t)t * d, xs[t], yrow, hbuf, hqtmp, hstmp);
            for (int o = 0; o < d; o++) yacc[o] += (double)yrow[o];
        }
        for (int o = 0; o < d; o++) y_tok[(size_t)i * d + o] = (float)yacc[o];
    }
    if (tr) {
        if (tr->ids) memcpy(tr->ids, ids, Tk * sizeof(int32_t));
        if (tr->w) memcpy(tr->w, wt, Tk * sizeof(float));
        if (tr->perm) memcpy(tr->perm, perm, (size_t)kept * sizeof(int32_t));
        if (tr->off) memcpy(tr->off, off, ((size_t)E + 1) * sizeof(int32_t));
        if (tr->drop) memcpy(tr->drop, drop, Tk);
        if (tr->xq) memcpy(tr->xq, xq, (size_t)T * d);
        if (tr->xs) memcpy(tr->xs, xs, (size_t)T * sizeof(float));
        tr->kept = kept;
    }
    rc = 0;
out:
    free(ids);
    free(wt);
    free(perm);
    free(off);
    free(drop);
    free(xq);
    free(xs);
    free(gbuf);
    free(ubuf);
    free(hbuf);
    free(hqtmp);
    free(hstmp);
    free(hbtmp);
    free(yrow);
    free(yacc);
    return rc;
}
