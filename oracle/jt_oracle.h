/* jt_oracle.h - CPU restatement of the JIMOTONO quantized MoE / W8A8 hot
 * path, used ONLY as the parity checker by tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline leg.  Nothing in the shipped library links
 * or calls it.
 *
 * Parity status: every function that the reference defines is pinned
 * against the reference itself (oracle/_ref/libjtref.so compiled from the
 * reference sources) and against the reference's own known-answer tests
 * (tests/test_oracle_pins.py).  The group-64 INT2/INT4 format, per-token
 * activation scales and the SwiGLU requantization are formats the
 * reference does not define; for those this restatement IS the
 * specification (built from the reference's per-column rules applied per
 * group) and is pinned to the reference only where the two coincide
 * (group = K, one token). */
#ifndef JT_ORACLE_H
#define JT_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Symmetric int8 quantization of each `blk`-long block of each row, the
 * arithmetic of w8a8.c:688-747.  scales[row * (cols/blk) + b]. 0 ok, 2 inval. */
int jto_quant_blocks(const float *x, int rows, int cols, int blk, int8_t *q, float *scales);

/* acc[m][n] = sum_k A[m][k] * W[n][k] (int32), w8a8.c:654-686 with B = W^T. */
void jto_gemm_s8(const int8_t *A, const int8_t *W, int32_t *acc, int M, int N, int K);

/* C[m][n] = ((float)acc[m][n] * sx[m]) * sw[n] (fp32, two roundings). */
void jto_w8a8_token_channel(const int32_t *acc, const float *sx, const float *sw, float *C,
                            int M, int N);

/* Router logits of moe_layer.c:1114-1137: logits[t][e] = (float) of the
 * double dot product of x[t] and wgate[e] in the 4-lane order of the
 * reference's AVX2 build (moe_layer.c:67-86: lane l sums the products of
 * j = l mod 4 in ascending j, then (l0 + l1) + (l2 + l3), then the tail
 * j >= d & ~3 in order).  x [T][d], wgate [E][d], logits [T][E].  2 on a
 * non-finite dot or logit (moe_layer.c:1128-1135). */
int jto_router_logits(const float *x, const float *wgate, int T, int d, int E, float *logits);

/* Top-k + softmax of routing.c:16-76 on logits[t] (+ bias, added in float
 * before selection) for T tokens.  ids int32 [T][k], w float [T][k]. */
int jto_route_topk(const float *logits, const float *bias, int T, int E, int k, int32_t *ids,
                   float *w);

/* Stable capacity sort of moe_layer.c:895-978.  perm int32 [T*k] (kept
 * entries first), off int32 [E+1], drop uint8 [T*k]. */
int jto_batch_sort(const int32_t *ids, int T, int k, int E, float cap_factor, int32_t *perm,
                   int32_t *off, uint8_t *drop, int *out_kept);

/* Renormalization of moe_layer.c:1171-1201, in place on w [T][k]. */
int jto_renorm(float *w, const uint8_t *drop, int T, int k);

/* fp16 <-> fp32 (IEEE binary16, round to nearest even). */
float jto_half_to_float(uint16_t h);
uint16_t jto_float_to_half(float f);
/* bf16 <-> fp32 (round to nearest even; NaN stays NaN). */
float jto_bf16_to_float(uint16_t h);
uint16_t jto_float_to_bf16(float f);

/* Pack fp32 weights W [rows][K] into odd-symmetric `bits`-bit codes with
 * one fp16 scale per `group` elements: per group maxa = max|w|, level rule
 * of lowbit.c:78-88 (li = floor(t*(n-1)/2 + (n-1)/2 + 0.5), t = w/maxa,
 * clamped), scale = maxa/(2^bits - 1).  Codes little-endian along K:
 * INT2 element k at bits 2*(k%4) of byte k/4, INT4 element k in the low
 * nibble (k even) / high nibble (k odd) of byte k/2. */
int jto_pack_lowbit(const float *W, int rows, int K, int bits, int group, uint8_t *packed,
                    uint16_t *scales);
/* Unsigned code li of element (r, k) of a packed matrix with K columns. */
int jto_code_at(const uint8_t *packed, int K, int bits, int r, int k);

/* Deterministic fp32 exp / SwiGLU shared bit-for-bit with the CUDA path. */
float jto_expf(float x);
float jto_swiglu(float g, float u);

/* Low-bit GEMV / per-token grouped dot:
 *   P[g] = sum_{k in group g} a[k] * c[n][k]   (int32, c = 2li - (2^bits-1))
 *   r = 0; for g ascending: r = fmaf((float)P[g], s[n][g], r);  y[n] = r * sa
 * a int8 [K], packed [N][...], scales fp16 [N][K/64]. */
void jto_lowbit_gemv(const int8_t *a, float sa, const uint8_t *packed, const uint16_t *scales,
                     int N, int K, int bits, float *y);
/* Same with the int32 group partials written to P [N][K/64]. */
void jto_lowbit_partials(const int8_t *a, const uint8_t *packed, int N, int K, int bits,
                         int32_t *P);

/* Prepared quantized MoE layer (the B200 path's specification). */
typedef struct jto_moe_dims {
    int T, d, f, E, k, S, fs;
    float cap_factor;
} jto_moe_dims;

typedef struct jto_moe_weights {
    const uint8_t *wg, *wu;   /* INT2 [E][f][d/4] */
    const uint16_t *sg, *su;  /* fp16 [E][d/64][f] (group-major) */
    const uint8_t *wd;        /* INT4 [E][d][f/2] */
    const uint16_t *sd;       /* fp16 [E][f/64][d] (group-major) */
    const int8_t *wsg, *wsu;  /* int8 [S][fs][d] */
    const float *ssg, *ssu;   /* fp32 [S][fs] */
    const int8_t *wsd;        /* int8 [S][d][fs] */
    const float *ssd;         /* fp32 [S][d] */
} jto_moe_weights;

typedef struct jto_moe_trace {
    int32_t *ids;     /* [T][k] */
    float *w;         /* [T][k] after renorm */
    int32_t *perm;    /* [T*k] */
    int32_t *off;     /* [E+1] */
    uint8_t *drop;    /* [T*k] */
    int8_t *xq;       /* [T][d] */
    float *xs;        /* [T] */
    uint16_t *h;      /* [kept][f] routed SwiGLU output, bf16 bits (perm order) */
    float *ypair;     /* [kept][d]  expert output before weighting */
    float *yshared;   /* [T][d]     sum of shared experts */
    int kept;
} jto_moe_trace;

/* Y [T][d] fp32.  trace fields may be NULL. 0 ok, 2 inval. */
int jto_moe_forward(const jto_moe_dims *dm, const jto_moe_weights *w, const float *x,
                    const float *logits, const float *bias, float *y, jto_moe_trace *trace);

/* Sampled form for the benchmarked shapes: routing, sort, renormalization
 * and token quantization in full (trace ids/w/perm/off/drop/xq/xs/kept);
 * the routed h (bf16) only for the kept rows rows[i] % kept (index written
 * back) -> h_rows [n_rows][f], the output only for the tokens toks[i]
 * (y_tok [n_tok][d]).  Same values as jto_moe_forward for those rows and
 * tokens. */
int jto_moe_forward_sampled(const jto_moe_dims *dm, const jto_moe_weights *w, const float *x,
                            const float *logits, const float *bias, int32_t *rows, int n_rows,
                            uint16_t *h_rows, const int32_t *toks, int n_tok, float *y_tok,
                            jto_moe_trace *trace);

#ifdef __cplusplus
}
#endif

#endif
