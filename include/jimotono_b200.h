/* jimotono_b200.h - C ABI of libjimotono_b200.so, the B200 (sm_100a)
 * implementation of JIMOTONO's quantized matrix-multiply hot path.
 *
 * Two groups of entry points:
 *
 *  1. Reference-compatible symbols.  Same names, prototypes, argument
 *     meaning, validation order and error behaviour as the reference C
 *     library, so a program linked against the reference core library can
 *     link this one instead.  They take HOST pointers, stage to the GPU,
 *     run the CUDA kernels and copy results back (synchronous, like the
 *     reference).  Each cites the reference declaration it replaces.
 *
 *  2. jt_b200_* device entry points.  DEVICE pointers, caller-owned
 *     buffers, asynchronous on the given stream (a cudaStream_t passed as
 *     void*; NULL = legacy default stream).  These are the timed path.
 *
 * Return codes are the reference's jt_err_t values (include/jimotono/
 * common.h:21-28): JT_OK 0, JT_ERR_NOMEM 1, JT_ERR_INVAL 2; plus
 * JT_ERR_CUDA 6 for a CUDA runtime failure or a kernel-reported fault
 * (the reference has no device, so it never returns 6).
 */
#ifndef JIMOTONO_B200_H
#define JIMOTONO_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- error codes and limits (reference: common.h:21-28, w8a8.h:54-55,
 *      train_bwd.h:35, moe_layer.h:52-54, moe_gemm.h:53-54) ---- */
#ifndef JIMOTONO_COMMON_H
typedef enum jt_err {
    JT_OK = 0,
    JT_ERR_NOMEM = 1,
    JT_ERR_INVAL = 2,
    JT_ERR_IO = 3,
    JT_ERR_ALIGN = 4,
    JT_ERR_NOSUP = 5,
} jt_err_t;
#endif
#define JT_ERR_CUDA 6
#define JT_W8A8_QMAX 127
#define JT_W8A8_QMIN (-127)
#define JT_BWD_MAX_WIDE 4096

/* ======================================================================
 * 1. Reference-compatible W8A8 API (reference include/jimotono/w8a8.h)
 * ====================================================================== */

/* Process-global mode flag, 0/1 else INVAL.  Replaces w8a8.h:100-104
 * (w8a8.c:53-73). */
int jt_w8a8_set_enabled(int enabled);
int jt_w8a8_get_enabled(int *out_enabled);
int jt_w8a8_is_enabled(void);

/* Symmetric per-tensor quantization, scale = max|x|/127 (double), round
 * half away from zero, clamp to [-127,127]; zero tensor -> scale 1, q 0.
 * Replaces w8a8.h:110-112 (w8a8.c:688-747). */
int jt_w8a8_quant_per_tensor(const float *src, size_t n, int8_t *dst, float *out_scale);
/* dst[i] = (float)((double)src[i] * scale).  Replaces w8a8.h:115-116
 * (w8a8.c:749-785). */
int jt_w8a8_dequant_per_tensor(const int8_t *src, float scale, size_t n, float *dst);
/* Per-row quantization.  Replaces w8a8.h:122-124 (w8a8.c:787-855). */
int jt_w8a8_quant_per_channel(const float *src, size_t rows, size_t cols, int8_t *dst,
                              float *scales);
/* Replaces w8a8.h:127-129 (w8a8.c:857-907). */
int jt_w8a8_dequant_per_channel(const int8_t *src, const float *scales, size_t rows,
                                size_t cols, float *dst);
/* C[M][N] = (float)((double)acc * ((double)sA*(double)sB)), Aq [M][K],
 * Bq [K][N] row-major, M,N,K <= 4096, M == 0 is a no-op.  Replaces
 * w8a8.h:140-142 (w8a8.c:955-1019). */
int jt_w8a8_gemm_per_tensor(const int8_t *Aq, const int8_t *Bq, float sA, float sB, float *C,
                            int M, int N, int K);
/* Same with a per-column sB_col[N].  Replaces w8a8.h:147-150
 * (w8a8.c:1021-1072). */
int jt_w8a8_gemm_per_channel(const int8_t *Aq, const int8_t *Bq, float sA, const float *sB_col,
                             float *C, int M, int N, int K);
/* dequant(quant(x)).  Replaces w8a8.h:156-159 (w8a8.c:1074-1200). */
int jt_w8a8_fakequant_per_tensor(const float *src, size_t n, float *dst);
int jt_w8a8_fakequant_per_channel(const float *src, size_t rows, size_t cols, float *dst);

/* ---- reference-compatible routing / sort / fp32 GEMM / low-bit helpers ---- */

/* Top-k of one token's logits with ties to the lowest index, NaN -> INVAL,
 * softmax over the selected logits in double (w = (float)e * (float)(1/sum)),
 * non-finite softmax -> INVAL.  Replaces routing.h:56-57 (routing.c:16-76). */
int jt_routing_topk(const float *logits, size_t n, size_t k, size_t *out_ids, float *out_weights);
/* Stable capacity sort: cap = ceil(cap_factor*T*k/E), the first cap pairs of
 * each expert in q = t*k + p order kept (perm [kept], off [E+1]), the rest
 * dropped.  Replaces moe_layer.h:194-198 (moe_layer.c:895-978). */
int jt_moe_batch_sort(const size_t *ids, int T, int k, int E, float cap_factor, size_t *perm,
                      size_t *off, unsigned char *drop, size_t *out_kept, size_t *out_dropped);
/* C[M][N] = A[M][K] B[K][N], fp32, products and sums rounded one by one in
 * ascending k (no fused multiply-add); M == 0 no-op; non-finite C -> INVAL
 * (C written).  Replaces moe_gemm.h:59-61 (moe_gemm.c:92-170). */
int jt_gemm_mat_f32(const float *A, const float *B, float *C, int M, int N, int K);
/* dst[c][r] = src[r][c].  Replaces moe_gemm.h:65-66 (moe_gemm.c:17-42). */
int jt_transpose_f32(const float *src, float *dst, int rows, int cols);
/* Low-bit mode flag 0/1/2 and bit widths (gate/up 2, down 4).  Replace
 * lowbit.h:30-34 (lowbit.c:16-39). */
int jt_lowbit_set_mode(int mode);
int jt_lowbit_get_mode(void);
int jt_lowbit_bits_for(int is_down, int *out_bits);
/* Odd-symmetric fake quantization over the whole array (one max-abs):
 * li = floor(t(n-1)/2 + (n-1)/2 + 0.5), t = w/maxa (double), value
 * ((2li - (n-1))/(n-1)) * maxa.  Replaces lowbit.h:38-39 (lowbit.c:47-91). */
int jt_lowbit_fakequant(const float *w, float *fq, size_t n, int bits);
/* The same codes as bit planes idx[b*(k/4) + g] (bit j = bit b of code
 * 4g+j), *w_scale = maxa.  Replaces lowbit.h:43-44 (lowbit.c:93-141). */
int jt_lowbit_col_to_idx(const float *col, size_t k, int bits, uint8_t *idx, float *w_scale);
/* The whole MoE layer on the reference's fp32 weights: X [T][n], Wgate
 * [E][n], Wg/Wu/Wd [E][h][n], shared [S][h][n]; gate logits (4-lane double
 * dot), top-k + softmax, capacity sort (cap_factor 1.0-1.5) and
 * renormalization, routed experts in the mode jt_w8a8_set_enabled /
 * jt_lowbit_set_mode select (fp32, W8A8, low-bit fake-quant, LUT), SwiGLU
 * in double, double combine in slot order plus the shared experts.
 * out_ids/out_weights [T][k]; optional caches [T][k*h], [T][k*n],
 * [T][S*h]; optional perm/off/drop/kept/dropped.  Y is written only on
 * success.  _unchecked skips the finiteness scan of the inputs.  Replaces
 * moe_layer.h:230-275 (moe_layer.c:980-1663). */
int jt_moe_fwd_batch(const float *X, const float *Wgate, const float *Wg, const float *Wu, const float *Wd,
                     const float *Wg_s, const float *Wu_s, const float *Wd_s, float *Y, int T, int n, int h,
                     int n_experts, int topk, int n_shared, size_t *out_ids, float *out_weights, float *cache_Gsel,
                     float *cache_Usel, float *cache_Ysel, float *cache_Gs, float *cache_Us, float cap_factor,
                     size_t *out_perm, size_t *out_off, unsigned char *out_drop, size_t *out_kept,
                     size_t *out_dropped);
int jt_moe_fwd_batch_unchecked(const float *X, const float *Wgate, const float *Wg, const float *Wu,
                               const float *Wd, const float *Wg_s, const float *Wu_s, const float *Wd_s, float *Y,
                               int T, int n, int h, int n_experts, int topk, int n_shared, size_t *out_ids,
                               float *out_weights, float *cache_Gsel, float *cache_Usel, float *cache_Ysel,
                               float *cache_Gs, float *cache_Us, float cap_factor, size_t *out_perm,
                               size_t *out_off, unsigned char *out_drop, size_t *out_kept, size_t *out_dropped);
/* Single-token layer, always fp32: double dots for the logits and the
 * expert gate/up rows, SwiGLU and down sum in double.  out_logits [E],
 * caches [k][h], [k][n], [S][h] optional.  Replaces moe_layer.h:73-117
 * (moe_layer.c:304-545). */
int jt_moe_fwd(const float *X, const float *Wgate, const float *Wg, const float *Wu, const float *Wd,
               const float *Wg_s, const float *Wu_s, const float *Wd_s, float *Y, int n, int h, int n_experts,
               int topk, int n_shared, size_t *out_ids, float *out_weights, float *out_logits, float *cache_Gsel,
               float *cache_Usel, float *cache_Ysel, float *cache_Gs, float *cache_Us);
int jt_moe_fwd_unchecked(const float *X, const float *Wgate, const float *Wg, const float *Wu, const float *Wd,
                         const float *Wg_s, const float *Wu_s, const float *Wd_s, float *Y, int n, int h,
                         int n_experts, int topk, int n_shared, size_t *out_ids, float *out_weights,
                         float *out_logits, float *cache_Gsel, float *cache_Usel, float *cache_Ysel,
                         float *cache_Gs, float *cache_Us);
/* Exact fp32 product through the T-MAC tables: activation LUT of X, bit
 * planes of every column of W [k][h] (row-major), lookups, and the sign
 * correction Y = (float)((2o - (n-1)*ws*rowsum)/(n-1)); k % 32 != 0 takes
 * the double-accumulated fallback; me == 0 is a no-op.  Y is unchanged on
 * failure.  Replaces lowbit.h:52-53 (lowbit.c:158-267). */
int jt_lowbit_gemm_lut(const float *X, const float *W, float *Y, int me, int h, int k, int bits);

/* ---- reference-compatible T-MAC LUT (tmac.h) ---- */
#define JT_TMAC_G 4          /* tmac.h:44 */
#define JT_TMAC_LUT_HALF 8   /* tmac.h:45 */
#define JT_TMAC_LUT_FULL 16  /* tmac.h:46 */
#define JT_TMAC_ACT_GROUP 32 /* tmac.h:47 */
#define JT_TMAC_ALIGN 64     /* tmac.h:48 */
/* n*(k/4)*8 and n*(k/32)*sizeof(float) bytes (k % 4, k % 32; overflow ->
 * JT_ERR_NOMEM).  Replace tmac.h:53-54 (tmac.c:168-228). */
int jt_tmac_qlut_bytes(size_t n, size_t k, size_t *out);
int jt_tmac_param_bytes(size_t n, size_t k, size_t *out);
/* Per 32-activation block: 8 groups x patterns p = 8..15 of F(p) = sum_j
 * +-a_j (double), scale = max|F|/127, bias = sum a, q = clamp(round(F /
 * scale), -128, 127); all-zero block -> q 0, scale 1.  Non-finite input ->
 * INVAL (EINVAL), bias overflow -> INVAL (ERANGE); outputs unchanged on
 * failure.  Replaces tmac.h:59-60 (tmac.c:230-385). */
int jt_tmac_lut_ctor(const float *act, size_t n, size_t k, int8_t *qlut, float *scales, float *biases);
/* One dot product: per block and plane the int32 sum of 8 mirrored
 * lookups, total += ((sc*acc + bi)*0.5)*2^b in double (ascending block,
 * then plane), *out = (float)(total*w_scale).  Replaces tmac.h:69-72
 * (tmac.c:387-506). */
int jt_tmac_lookup_accum(const int8_t *qlut, const uint8_t *idx, const float *scales, const float *biases,
                         size_t ngroups, size_t nblocks, int bits, float w_scale, float *out);

/* ======================================================================
 * 2. B200 device entry points
 * ====================================================================== */

/* Per-token x per-channel W8A8 GEMM on device buffers (the shared-expert /
 * attention projection form of w8a8.c:1021-1072 with a per-row sA):
 *   C[m][n] = ((float)acc[m][n] * sx[m]) * sw[n],
 *   acc[m][n] = sum_k X[m][k] * W[n][k]   (int32, exact).
 * X int8 [M][K] (row stride ldx bytes), W int8 [N][K] (row stride ldw
 * bytes, i.e. the reference's Bq transposed), C fp32 [M][ldc].
 * K, ldx, ldw multiples of 16; X, W 16-byte aligned. */
int jt_b200_w8a8_gemm(const int8_t *X, int ldx, const float *sx, const int8_t *W, int ldw,
                      const float *sw, float *C, int ldc, int M, int N, int K, void *stream);

/* Same operands, writes the raw int32 accumulators C32[m][n] = acc[m][n]. */
int jt_b200_w8a8_gemm_i32(const int8_t *X, int ldx, const int8_t *W, int ldw, int32_t *C32,
                          int ldc, int M, int N, int K, void *stream);

/* y = W8A8 linear layer on fp32 activations, in one call that allocates
 * no memory.  Each row of x [M][K] is quantized to int8 codes with its own
 * fp32 scale (max|x_row| / 127, round half away from zero), then
 * C[m][n] = ((float)acc[m][n] * scale[m]) * sw[n] as jt_b200_w8a8_gemm
 * computes it.  The codes and row scales live in a fixed device array
 * inside the library.  No counterpart in the reference.
 *
 * For callers that must not allocate device memory at all - a runtime
 * with a fixed memory budget, or one that enqueues work where an
 * allocation would synchronize the device.  Limits: M <= 4096 and
 * M * K <= 2 MiB of codes (larger shapes return JT_ERR_INVAL, errno
 * E2BIG); K and ldw multiples of 16; W 16-byte aligned (else
 * JT_ERR_INVAL).  The scratch is one per device and keeps the last call's
 * contents, so calls on one device must not overlap: issue them on one
 * stream or order them.  The first call on a device looks up the scratch
 * address (a host-side, synchronous step); make it before any stream
 * capture.  A row of x holding a non-finite value comes out as NaN in every
 * column of C and jt_b200_sync reports JT_ERR_CUDA; the other rows are
 * valid. */
#define JT_B200_LINEAR_NOALLOC_MAX_ROWS 4096
#define JT_B200_LINEAR_NOALLOC_MAX_CODES (2 * 1024 * 1024)
int jt_b200_w8a8_linear_noalloc(const float *x, int M, int K, const int8_t *W, int ldw,
                                const float *sw, float *C, int ldc, int N, void *stream);

/* Batch-1 low-bit GEMV, the decode replacement of the LUT path
 * (jt_lowbit_gemm_lut, lowbit.h:52 / lowbit.c:158-267, and
 * jt_tmac_lookup_accum, tmac.h:69 / tmac.c:387-506), on the packed
 * group-64 format:
 *   P[n][g] = sum_{k in group g} a[k] * c[n][k]   (int32, c = 2li - (2^b-1))
 *   r = 0; for g ascending: r = fmaf((float)P[n][g], s[n][g], r); y[n] = r * sa
 * y[0..n2) from INT2 rows w2 [n2][K/4], y[n2..n2+n4) from INT4 rows
 * w4 [n4][K/2] (both little-endian along K), fp16 scales s2 [n2][K/64],
 * s4 [n4][K/64].  a int8 [K]; K % 64 == 0, K <= 4096; a, w2, w4 16-byte
 * aligned.  Device pointers, asynchronous on stream.  The kernel starts
 * streaming w2/w4/s2/s4 before the previous work of the stream has
 * finished (programmatic dependent launch); a and y are ordered normally.
 * The weight buffers must not be written by work still pending in the
 * same stream. */
int jt_b200_lowbit_gemv(const int8_t *a, float sa, const uint8_t *w2, const uint16_t *s2, int n2,
                        const uint8_t *w4, const uint16_t *s4, int n4, int K, float *y,
                        void *stream);

/* Weight packer: fp32 masters W [rows][K] (device) -> the packed format
 * read by jt_b200_lowbit_gemv and the prepared MoE layer.  Replaces the
 * per-call weight preparation of the reference's low-bit path
 * (jt_lowbit_col_to_idx, lowbit.h:45 / lowbit.c:93-141, rebuilt for every
 * column on every call by jt_lowbit_gemm_lut, lowbit.c:228-237) with a
 * one-time pack.  Its level rule is applied per 64-element K group:
 * maxa = max |w| of the group, li = floor(w/maxa * (n-1)/2 + (n-1)/2 + 0.5)
 * clamped to [0, n-1] (double, n = 2^bits), scale = (half)(float)(maxa/(n-1)).
 * bits 2 or 4; K % 64 == 0; W 8-byte aligned.  packed [rows][K*bits/8];
 * scales fp16: n_ch == 0 -> [rows][K/64] (GEMV layout); n_ch > 0 -> rows
 * are blocks of n_ch output channels (one expert each) and the scales are
 * group-major per block, [rows/n_ch][K/64][n_ch] (jt_b200_moe_weights
 * layout).  A non-finite weight is reported by jt_b200_sync.  Device
 * pointers, asynchronous on stream. */
int jt_b200_lowbit_pack(const float *W, int rows, int K, int bits, int n_ch, uint8_t *packed,
                        uint16_t *scales, void *stream);

/* Converter from the reference's bit-plane index (jt_lowbit_col_to_idx,
 * lowbit.h:45 / lowbit.c:117-139) to packed rows: idx holds `cols`
 * consecutive columns of bits*K/4 bytes each; byte b*K/4 + q of a column
 * carries, in bit i, bit b of the code of element 4q + i.  packed
 * [cols][K*bits/8] receives the same codes li.  With w_scale [cols] (the
 * reference's whole-column max-abs) every group of column j gets the scale
 * (half)(float)(w_scale[j]/(n-1)), in the layout chosen by n_ch as above;
 * w_scale and scales are both NULL or both given.  bits 2 or 4, K % 64 == 0.
 * Device pointers, asynchronous on stream. */
int jt_b200_lowbit_planes_to_packed(const uint8_t *idx, const float *w_scale, int cols, int K,
                                    int bits, int n_ch, uint8_t *packed, uint16_t *scales,
                                    void *stream);

/* ---- quantized MoE layer (prepared weights) ----
 *
 * The layer of jt_moe_fwd_batch (moe_layer.c:980-1614; moe_layer.h:230-246)
 * with the B200 precision policy: int8 per-token activations, routed
 * gate/up INT2 and down INT4 with one fp16 scale per 64 K (group 64),
 * shared experts int8 with per-channel scales, SwiGLU between the
 * projections and h requantized to int8 per (row, 64 channels).  Routing
 * (top-k, softmax, capacity sort, drop, renormalization) follows the
 * reference bit for bit.  Dimension names follow the reference: d = n
 * (model dim), f = h (expert ffn); the shared ffn fs may differ from f.
 * Packed weights are little-endian along K: INT2 element k at bits
 * 2*(k%4) of byte k/4, INT4 element k in the low (k even) or high (k odd)
 * nibble of byte k/2; code li maps to (2*li - (2^bits-1)) * scale, the
 * odd-symmetric levels of lowbit.c:41-45. */
typedef struct jt_b200_moe_dims {
    int T;            /* largest token count a forward call may pass */
    int d;            /* model dim, multiple of 128 */
    int f;            /* routed expert ffn, multiple of 128 */
    int E;            /* routed experts, 1..4096 */
    int k;            /* top-k, 1..min(E, 64) */
    int S;            /* shared experts, 0..8 */
    int fs;           /* shared expert ffn, multiple of 128 when S > 0 */
    float cap_factor; /* capacity factor in [1.0, 1.5] (moe_layer.c:913-917) */
} jt_b200_moe_dims;

typedef struct jt_b200_moe_weights { /* device pointers */
    const uint8_t *wg, *wu;  /* INT2 [E][f][d/4] */
    const uint16_t *sg, *su; /* fp16 [E][d/64][f] (group-major) */
    const uint8_t *wd;       /* INT4 [E][d][f/2] */
    const uint16_t *sd;      /* fp16 [E][f/64][d] (group-major) */
    const int8_t *wsg, *wsu; /* int8 [S][fs][d] */
    const float *ssg, *ssu;  /* fp32 [S][fs] per-channel scales */
    const int8_t *wsd;       /* int8 [S][d][fs] */
    const float *ssd;        /* fp32 [S][d] */
} jt_b200_moe_weights;

typedef struct jt_b200_moe_plan jt_b200_moe_plan;

/* Allocate the device workspace for one layer shape (the only allocation;
 * forward calls allocate nothing). */
int jt_b200_moe_plan_create(const jt_b200_moe_dims *dims, jt_b200_moe_plan **out);
int jt_b200_moe_plan_destroy(jt_b200_moe_plan *plan);
size_t jt_b200_moe_plan_bytes(const jt_b200_moe_plan *plan);

/* On-disk form of the prepared weights (written once, loaded at start-up,
 * instead of re-deriving the quantized weights from fp32 masters on every
 * call as the reference layer does, moe_layer.c:185-274, lowbit.c:228-237).
 * Format: a 4096-byte little-endian header (magic "JTB2MOE1", version 1,
 * d, f, E, S, fs, and per array its offset, size and FNV-1a 64 checksum),
 * then the twelve arrays of jt_b200_moe_weights in field order, each at a
 * 4096-byte aligned offset.  A reader rejects a header that does not match
 * `dims` (JT_ERR_INVAL) and data that does not match its checksums
 * (JT_ERR_IO); it checks every checksum before it writes any destination,
 * so a rejected file leaves the arrays untouched (a file modified while it
 * is being read is reported as JT_ERR_IO too, with the arrays then partly
 * overwritten).  _sizes gives each array's byte size for `dims` (T, k and
 * cap_factor are not part of the weights).  _write_host / _read_host take
 * host arrays in field order; _save / _load take device buffers (the
 * pointers in `w`; _load writes into them), wait for all work on the
 * device to finish (cudaDeviceSynchronize) and copy through a pinned host
 * buffer, synchronously. */
int jt_b200_moe_weights_sizes(const jt_b200_moe_dims *dims, size_t sizes[12]);
int jt_b200_moe_weights_write_host(const char *path, const jt_b200_moe_dims *dims,
                                   const void *const arrays[12]);
int jt_b200_moe_weights_read_host(const char *path, const jt_b200_moe_dims *dims,
                                  void *const arrays[12]);
int jt_b200_moe_weights_save(const char *path, const jt_b200_moe_dims *dims,
                             const jt_b200_moe_weights *w);
int jt_b200_moe_weights_load(const char *path, const jt_b200_moe_dims *dims,
                             const jt_b200_moe_weights *w);

/* Router logits, the gate projection in front of the layer
 * (moe_layer.c:1114-1137, inside jt_moe_fwd_batch): logits[t][e] =
 * (float) of the double dot product of x[t] and wgate[e], accumulated in
 * the order of the reference's AVX2 build (moe_layer.c:67-86: four lanes
 * over j mod 4, combined as (l0 + l1) + (l2 + l3)), so the logits - and the
 * experts the top-k picks from them - are bit-identical to the reference's.
 * x fp32 [T][d], wgate fp32 [E][d] (row-major, 16-byte aligned), logits
 * fp32 [T][E]; d % 32 == 0, T <= 2097120.  A non-finite dot or logit (an
 * EINVAL in the reference) is reported by jt_b200_sync.  Device pointers,
 * asynchronous on stream; feed logits to jt_b200_moe_forward. */
int jt_b200_moe_router_logits(const float *x, const float *wgate, int T, int d, int E,
                              float *logits, void *stream);

/* Y[T][d] = sum over kept slots of w * expert(x) + sum of shared experts.
 * x fp32 [T][d], logits fp32 [T][E] (router output), bias fp32 [E] or NULL
 * (added to the logits before selection), y fp32 [T][d] or bf16 when
 * y_bf16 != 0.  T <= dims.T; no 4096 cap on T.  Asynchronous on stream. */
int jt_b200_moe_forward(jt_b200_moe_plan *plan, const jt_b200_moe_weights *w, const float *x,
                        const float *logits, const float *bias, int T, void *y, int y_bf16,
                        void *stream);

/* Per-stage device timing of forward calls (CUDA events recorded on the
 * forward's stream around each stage): begin() arms it for up to max_steps
 * calls, end() waits for them and returns the summed milliseconds per
 * stage (stage_ms[JT_B200_MOE_NSTAGE]) and the number of timed calls. */
enum {
    JT_B200_STAGE_ROUTE = 0,    /* top-k + softmax */
    JT_B200_STAGE_SORT = 1,     /* capacity sort, drop, renormalization */
    JT_B200_STAGE_DISPATCH = 2, /* per-token quantization + dispatch */
    JT_B200_STAGE_SHARED = 3,   /* shared experts */
    JT_B200_STAGE_GATEUP = 4,   /* routed gate/up + SwiGLU + requant */
    JT_B200_STAGE_DOWN = 5,     /* routed down + weighted combine */
    JT_B200_STAGE_OUTPUT = 6,   /* bf16 conversion */
    JT_B200_MOE_NSTAGE = 7
};
int jt_b200_moe_profile_begin(jt_b200_moe_plan *plan, int max_steps);
int jt_b200_moe_profile_end(jt_b200_moe_plan *plan, float *stage_ms, int nstage, int *steps);

/* Copy an intermediate of the last forward to host memory (synchronizes). */
enum {
    JT_B200_DBG_IDS = 0,     /* int32 [T][k] selected experts */
    JT_B200_DBG_WEIGHTS = 1, /* fp32 [T][k] weights after renormalization */
    JT_B200_DBG_PERM = 2,    /* int32 [kept] flattened (t*k+p) indices in expert order */
    JT_B200_DBG_OFF = 3,     /* int32 [E+1] expert boundaries in perm */
    JT_B200_DBG_DROP = 4,    /* uint8 [T][k] dropped flags */
    JT_B200_DBG_XQ = 5,      /* int8 [T][d] per-token codes */
    JT_B200_DBG_XS = 6,      /* fp32 [T] per-token scales */
    JT_B200_DBG_H = 7,       /* bf16 [kept][f] routed SwiGLU output, perm order */
    JT_B200_DBG_META = 9     /* int32 [4]: kept, token tiles, max kept per expert */
};
int jt_b200_moe_debug_copy(jt_b200_moe_plan *plan, int what, void *host_dst, size_t bytes);

/* ---- expert-parallel layer (one process per GPU, NCCL over NVLink) ----
 *
 * Rank r of N holds tokens [r*T, (r+1)*T) of the global batch (dims.T = T
 * tokens per rank, the same on every rank) and routed experts
 * [r*E/N, (r+1)*E/N) (dims.E = E, the global count; the weights passed to
 * the forward hold only the rank's E/N experts); shared experts are
 * replicated.  Routing, capacity and drop follow the reference over the
 * whole batch: a pair of expert e is kept when fewer than cap pairs of e
 * precede it in the global q = t*k + p order (moe_layer.c:931-970).
 * Dispatch and combine are NCCL send/recv; each forward waits once on the
 * host for the gathered expert counts (to size the exchange).  That wait is
 * bounded (jt_b200_ep_comm_set_timeout, default 60 s, or the environment
 * variable JT_B200_EP_TIMEOUT_MS): when a peer reports an error or the
 * deadline passes, the communicator is aborted (its in-flight NCCL work
 * ends) and the forward returns JT_ERR_CUDA with jt_b200_last_error naming
 * the cause; the communicator then stays dead (later forwards fail at
 * once) and is freed by jt_b200_ep_comm_destroy.
 * NCCL is loaded at run time (libnccl.so.2); without it the calls return
 * JT_ERR_NOSUP. */
typedef struct jt_b200_ep_comm jt_b200_ep_comm;
typedef struct jt_b200_moe_ep_plan jt_b200_moe_ep_plan;
/* 128-byte NCCL unique id, created on one rank and given to all. */
int jt_b200_ep_unique_id(void *id128);
/* Communicator of the current CUDA device (collective over the N ranks). */
int jt_b200_ep_comm_create(const void *id128, int nranks, int rank, jt_b200_ep_comm **out);
int jt_b200_ep_comm_destroy(jt_b200_ep_comm *comm);
/* Deadline of the forward's host wait, in milliseconds (> 0). */
int jt_b200_ep_comm_set_timeout(jt_b200_ep_comm *comm, int timeout_ms);
/* 1 when the communicator was aborted by the watchdog, else 0. */
int jt_b200_ep_comm_failed(const jt_b200_ep_comm *comm);
/* The watchdog's polling loop against fake operations, without a GPU:
 * scenario 0 completes after a few polls, 1 reports an asynchronous error,
 * 2 never completes (the deadline timeout_ms runs out).  Returns 0
 * (completed), 1 (error) or 2 (timeout); *out_aborted = whether it aborted. */
int jt_b200_watchdog_selftest(int scenario, int timeout_ms, int *out_aborted);
int jt_b200_moe_ep_plan_create(const jt_b200_moe_dims *dims, jt_b200_ep_comm *comm,
                               jt_b200_moe_ep_plan **out);
int jt_b200_moe_ep_plan_destroy(jt_b200_moe_ep_plan *plan);
/* x [T][d], logits [T][E] of the local tokens; y [T][d] (fp32, or bf16). */
int jt_b200_moe_ep_forward(jt_b200_moe_ep_plan *plan, const jt_b200_moe_weights *w, const float *x,
                           const float *logits, const float *bias, void *y, int y_bf16,
                           void *stream);
/* Intermediates of the last forward (synchronizes): local JT_B200_DBG_IDS,
 * _WEIGHTS, _DROP, _XQ, _XS, _PERM (kept local pairs in send order); _H
 * the bf16 SwiGLU rows of the owned experts (expert-contiguous);
 * _META int32 [4] {kept local pairs, owned rows, owned token tiles, cap}. */
int jt_b200_moe_ep_debug_copy(jt_b200_moe_ep_plan *plan, int what, void *host_dst, size_t bytes);
/* cap = ceil(cap_factor * T_global * k / E) in double (moe_layer.c:931-943);
 * -1 when out of range. */
int jt_b200_ep_capacity(long long T_global, int k, int E, float cap_factor);
/* Exchange layout of rank `rank` from the per-rank expert counts cnt [N][E]:
 * gbase [E] pairs of each expert on lower ranks; send_cnt [N] rows to each
 * owner; recv_cnt [N] rows from each source; own_off [E/N+1] and
 * own_tile_off [E/N+1] row and token-tile offsets of the owned experts;
 * gather [N][E/N][4] {first received row, first owned row, rows, 0}.  Host
 * memory; used by the forward and exposed for tests. */
int jt_b200_ep_layout(const int32_t *cnt, int N, int E, int rank, int cap, int32_t *gbase,
                      int32_t *send_cnt, int32_t *recv_cnt, int32_t *own_off,
                      int32_t *own_tile_off, int32_t *gather);

/* Synchronize the current device and fold any kernel-reported fault into
 * the return code (JT_OK or JT_ERR_CUDA). */
int jt_b200_sync(void);

/* jt_b200_sync, with the code a kernel reported (0 when none) written to
 * *kernel_code: JT_B200_KERR_TIMEOUT (a bounded wait of a kernel ran out;
 * the kernel drained and returned), JT_B200_KERR_SHAPE, JT_B200_KERR_NONFINITE,
 * JT_B200_KERR_RANGE, or 0x81-0x85 (routing: NaN logit, bad softmax sum,
 * expert id out of range, -, non-finite activation). */
#define JT_B200_KERR_TIMEOUT 0x71
#define JT_B200_KERR_SHAPE 0x72
#define JT_B200_KERR_NONFINITE 0x73
#define JT_B200_KERR_RANGE 0x74
int jt_b200_sync_code(int *kernel_code);

/* Diagnostic of the failure-detection path: one kernel waits, with the same
 * bounded wait every kernel of the library uses, on a barrier that nothing
 * completes, for budget_cycles SM clock cycles (1 .. 4e9), then raises
 * JT_B200_KERR_TIMEOUT and returns.  jt_b200_sync_code then reports it and
 * the context stays usable.  No counterpart in the reference (which has no
 * device). */
int jt_b200_selftest_bounded_wait(long long budget_cycles, void *stream);

/* Human-readable description of the last failed launch on this thread. */
const char *jt_b200_last_error(void);

/* Library version string. */
const char *jt_b200_version(void);

#ifdef __cplusplus
}
#endif

#endif /* JIMOTONO_B200_H */
