/* jt_internal.h - launcher prototypes shared between the C11 host layer
 * (jt_api.c, jt_moe.c) and the CUDA translation units.  Everything here
 * takes device pointers and a cudaStream_t and only enqueues work; the
 * host layer owns validation, staging and error mapping. */
#ifndef JT_INTERNAL_H
#define JT_INTERNAL_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Token rows per tile of the expert GEMMs (the routed-expert tile table and
 * the shared-expert tiles are cut to this size). */
#define JT_TILE_ROWS 256
/* Token rows of the routed gate/up GEMM's tiles (jtk_split_tiles). */
#define JT_SUB_ROWS 128

/* Epilogue modes of the dense int8 tensor-core GEMM. */
enum jtk_w8a8_epi {
    JTK_EPI_TOKEN_CHANNEL_F32 = 0, /* C = ((float)acc * sx[m]) * sw[n] */
    JTK_EPI_TENSOR_CHANNEL_F64 = 1, /* C = (float)((double)acc * ((double)sA * sw[n])) */
    JTK_EPI_RAW_I32 = 2,           /* C = acc (int32) */
    JTK_EPI_TOKEN_CHANNEL_F32_ACC = 3 /* C += ((float)acc * sx[m]) * sw[n] (one writer per element) */
};

/* C[M][N] from X int8 [M][K] (row stride ldx bytes) and W int8 [N][K]
 * (row stride ldw bytes).  K % 16 == 0, ldx/ldw % 16 == 0, pointers 16-byte
 * aligned.  out row stride is ldo elements.  sx may be NULL for the F64 and
 * raw epilogues; sw may be NULL for raw. */
int jtk_w8a8_gemm(const int8_t *X, int ldx, const int8_t *W, int ldw, int M, int N, int K,
                  const float *sx, const float *sw, double sA, void *out, int ldo, int epi,
                  cudaStream_t stream);

/* Utility kernels (jt_util.cu).  `bad` is a device int set to 1 on a hit. */
int jtk_transpose_s8(const int8_t *src, int K, int N, int8_t *dst, int Kp, int *bad,
                     cudaStream_t stream);
int jtk_pad_rows_s8(const int8_t *src, int M, int K, int8_t *dst, int Kp, int *bad,
                    cudaStream_t stream);
int jtk_check_s8(const int8_t *p, size_t n, int *bad, cudaStream_t stream);
int jtk_check_finite_f32(const float *p, size_t n, int *bad, cudaStream_t stream);

/* Quantization kernels (jt_quant.cu).  mode 0 = int8 codes + scales,
 * mode 1 = fake-quantized floats into fq.  `bad`: 1 non-finite input or
 * -128 code, 2 scale underflow / non-finite result. */
int jtk_quant_blocks(const float *x, int rows, int cols, int blk, int mode, int8_t *q,
                     float *scales, float *fq, int *bad, cudaStream_t stream);
int jtk_quant_tensor(const float *x, size_t n, int mode, int8_t *q, float *scale, float *fq,
                     unsigned *maxbits_scratch, int *bad, cudaStream_t stream);
int jtk_dequant_rows(const int8_t *src, const float *scales, size_t rows, size_t cols,
                     float *dst, int *bad, cudaStream_t stream);

/* fp32 -> bf16 (round to nearest even). */
int jtk_f32_to_bf16(const float *src, uint16_t *dst, size_t n, cudaStream_t stream);

/* Router logits (jt_router.cu): logits[t][e] = (float) 4-lane double dot of
 * x[t] and wgate[e]; d % 32 == 0, x and wgate 16-byte aligned. */
int jtk_router_logits(const float *x, const float *wgate, int T, int d, int E, float *logits,
                      cudaStream_t stream);

/* MoE routing (jt_route.cu). */
int jtk_route_topk(const float *logits, const float *bias, int T, int E, int k, int32_t *ids,
                   float *w, cudaStream_t stream);
int jtk_sort_chunks(int T);

/* Capacity sort.  tile_off [E+1]: JT_TILE_ROWS-row token tiles per expert (scan);
 * tiles: table of {expert, row0, row_end, 0} per token tile; meta[0] kept,
 * meta[1] token tiles (= tile_off[E]), meta[2] max kept per expert. */
/* gbase [E] (may be NULL): pairs of each expert that precede this token
 * range in the global q order (expert-parallel ranks); capacity left for
 * expert e is cap - gbase[e]. */
int jtk_moe_sort(const int32_t *ids, const float *w_in, int T, int k, int E, int cap,
                 const int32_t *gbase,
                 int32_t *hist, int32_t *off, int32_t *tile_off, int4 *tiles, int32_t *meta,
                 int32_t *perm, int32_t *pos, uint8_t *drop, float *w_out, cudaStream_t stream);
/* Token-tile table from per-expert row offsets off [E+1] and tile offsets
 * tile_off [E+1] (one CTA list entry {e, row0, row_end, 0} per tile). */
/* The JT_SUB_ROWS-row tile table of the JT_TILE_ROWS-row one (ntiles
 * entries, read on the device): out [ntiles * JT_TILE_ROWS / JT_SUB_ROWS]
 * in the same order, each entry {e, first row, expert's end row, 0}; nout
 * its entry count.  One CTA. */
int jtk_split_tiles(const int4 *tiles, const int32_t *ntiles, int4 *out, int32_t *nout, cudaStream_t stream);
int jtk_build_tiles(const int32_t *off, const int32_t *tile_off, int E, int4 *tiles,
                    cudaStream_t stream);

/* Shared gate/up of one shared expert on CTA-pair tiles (jt_shared_pair.cu):
 * hb [T][fs] bf16 SwiGLU output, rowmax [T] its row maxima (atomic max on
 * the bits: zero before the call).  -1: shape outside the kernel. */
int jtk_shared_gu_pair(const int8_t *wsg, const int8_t *wsu, const float *ssg, const float *ssu, int fs,
                       int d, const int8_t *xq, const float4 *sh_meta, int T, uint16_t *hb, float *rowmax,
                       cudaStream_t stream);
/* The S shared experts on T token rows into y (jt_shared.cu): stored by the
 * first expert, added by the others.  Scratch hb [T][fs] bf16, hq [T][fs],
 * hs [T]; g32 / u32 [T][fs] fp32 used only when T < 256. */
int jtk_moe_shared(const int8_t *wsg, const int8_t *wsu, const float *ssg, const float *ssu,
                   const int8_t *wsd, const float *ssd, int S, int fs, int d, const int8_t *xq,
                   const float *xs, const float4 *sh_meta, int T, uint16_t *hb, int8_t *hq, float *hs,
                   float *g32, float *u32, float *y, cudaStream_t stream);

/* Expert-parallel exchange kernels (jt_ep.cu). */
int jtk_ep_count(const int32_t *ids, int n, int E, int32_t *cnt, cudaStream_t stream);
int jtk_ep_tokens(const int32_t *ids, int T, int k, int El, int N, int32_t *trow, int32_t *ntok,
                  cudaStream_t stream);
int jtk_ep_pack(const int8_t *xq, const float *xs, int T, int d, int k, int El, int N, const int32_t *ids,
                const int32_t *pos, const float *wfin, const int32_t *trow, const int32_t *tsoff,
                int8_t *send_tok, float4 *row_meta, cudaStream_t stream);
/* dst_x: the owner's expert-ordered token rows as fp16 in the routed gate/up
 * GEMM's K order (as jtk_quant_dispatch's xd). */
int jtk_ep_gather(const int4 *ent, int n_ent, const int8_t *rtok, const float4 *src_meta, int d,
                  uint16_t *dst_x, float4 *dst_meta, cudaStream_t stream);
int jtk_ep_combine(const int32_t *trow, const int32_t *tsoff, int T, int N, const float *back, int d,
                   float *y, cudaStream_t stream);

/* Per-token quantization + dispatch; row_meta[row] = {scale, weight, token bits, 0}
 * for every kept row, sh_meta[t] = {scale, 1, t bits, 0} (may be NULL).
 * xq [T][d] int8; xd [kept rows][d] the same codes as exact fp16 values, in
 * expert order and in the K order of the routed gate/up GEMM (jt::kX16Order
 * inside every 16-element block). */
int jtk_quant_dispatch(const float *x, int T, int d, int k, const int32_t *pos,
                       const float *wfin, int8_t *xq, float *xs, uint16_t *xd, float4 *row_meta,
                       float4 *sh_meta, cudaStream_t stream);

/* Expert GEMMs, JT_TILE_ROWS-row token tiles.  tiles / ntiles: tile table
 * and its length (device).  row_meta [rows]: float4 records above.  Group
 * scales fp16 [E][K/64][n_ch].  Routed gate/up (jt_moe_gu16.cu) writes the
 * bf16 SwiGLU output h [rows][f]; the routed down (jt_moe_dn16.cu) reads it. */
int jtk_moe_gateup_routed(const uint8_t *wg, const uint8_t *wu, const void *gs, const void *us,
                          int E, int f, int d, const uint16_t *xd, int rows_cap,
                          const float4 *row_meta, const int4 *tiles, const int32_t *ntiles,
                          uint16_t *h, int max_tiles_hint, cudaStream_t stream);
/* Routed down projection (jt_moe_dn16.cu) of the bf16 h rows [rows][f].
 * y_accumulate 1: y[token][:] += w * row (combine into the layer output);
 * 0: y[row_meta.z][:] = w * row (one output row per routed row). */
int jtk_moe_down_routed(const uint8_t *wd, const void *ds, int E, int d, int f, const uint16_t *h,
                        int rows_cap, const float4 *row_meta, const int4 *tiles,
                        const int32_t *ntiles, float *y, int y_accumulate, int max_tiles_hint,
                        cudaStream_t stream);

/* Batch-1 low-bit GEMV (jt_gemv.cu): y[0..n2) from INT2 rows w2 [n2][K/4],
 * y[n2..n2+n4) from INT4 rows w4 [n4][K/2]; fp16 scales s [rows][K/64]. */
int jtk_lowbit_gemv(const int8_t *a, float sa, const uint8_t *w2, const uint16_t *s2, int n2,
                    const uint8_t *w4, const uint16_t *s4, int n4, int K, float *y,
                    cudaStream_t stream);

/* Weight preparation (jt_pack.cu).  W fp32 [rows][K] -> packed codes
 * [rows][K*bits/8] + fp16 group-64 scales, row-major [rows][K/64] for
 * n_ch == 0, group-major per block of n_ch rows otherwise.  The planes
 * form converts the reference's per-column bit planes (w_scale / scales
 * both NULL or both given). */
int jtk_pack_lowbit(const float *W, int rows, int K, int bits, int n_ch, uint8_t *packed,
                    uint16_t *scales, cudaStream_t stream);
int jtk_planes_to_packed(const uint8_t *idx, const float *w_scale, int cols, int K, int bits,
                         int n_ch, uint8_t *packed, uint16_t *scales, cudaStream_t stream);

/* T-MAC LUT kernels (jt_compat.cu).  Weight column j of expert e has k
 * elements at W + e*ws + t*st + j*sj.  Error keys (atomicMin, all ones =
 * none): position << 1 | kind (0 EINVAL, 1 ERANGE). */
int jtk_tmac_ctor(const float *act, size_t n, size_t k, int8_t *qlut, float *scales, float *biases,
                  unsigned long long *err, cudaStream_t stream);
int jtk_lut_gemm(const float *X, const float *W, int E, long long ws, long long st, long long sj,
                 const int32_t *rexp, const int8_t *qlut, const float *scales, const float *biases,
                 double *maxa, void *idx_planes, double *rowsum, float *Y, int me, int h, int k, int bits,
                 unsigned long long *err, cudaStream_t stream);
int jtk_gemm_f64acc(const float *X, const float *W, long long ws, long long st, long long sj,
                    const int32_t *rexp, float *Y, int me, int h, int k, cudaStream_t stream);
/* Top-k + softmax of routing.c:16-76 for T tokens of n logits (one CTA per
 * token); taken [T][ceil(n/32)] scratch; flag[0] = 1 on a bad softmax. */
int jtk_topk_any(const float *logits, int T, int n, int k, uint32_t *taken, int32_t *ids, float *w, int *flag,
                 cudaStream_t stream);

/* Batch-1 layer (jt_decode.cu): router, gate/up + SwiGLU + requant, and
 * down + combine as two matrix-vector kernels; also writes the router
 * output (ids, w) and the per-token results of the sort (perm, pos, off, tile_off, meta, drop,
 * w_fin, xq, xs, hq, hs).  acc_s [S][2][fs] and cnt_s [S][fs/64] are int32
 * scratch that must be zero before the first call (each call leaves them
 * zero).  -1: shape not handled (use the batched chain). */
int jtk_moe_decode(const float *x, const float *logits, const float *bias, int32_t *ids, float *w,
                   const uint8_t *wg, const uint8_t *wu,
                   const void *sg, const void *su, const uint8_t *wd, const void *sd, const int8_t *wsg,
                   const int8_t *wsu, const float *ssg, const float *ssu, const int8_t *wsd, const float *ssd,
                   int d, int f, int E, int k, int S, int fs, int8_t *xq, float *xs, uint16_t *h,
                   uint16_t *hb_s, int32_t *acc_s, int32_t *cnt_s,
                   int32_t *perm, int32_t *pos, int32_t *off, int32_t *tile_off, int32_t *meta,
                   uint8_t *drop, float *w_fin, float *y, uint16_t *y_bf16, cudaStream_t stream);

/* Bounded host wait (jt_watchdog.c): polls done() (> 0 done, < 0 failed)
 * and async_error() (!= 0: the communicator reported an error) until done
 * or timeout_ms; on an error or the deadline calls abort_comm().  Returns
 * JT_WD_DONE, JT_WD_ERROR or JT_WD_TIMEOUT; *polls (may be NULL) = polls made. */
typedef struct {
    int (*done)(void *ctx);
    int (*async_error)(void *ctx);
    void (*abort_comm)(void *ctx);
    void *ctx;
} jt_watchdog_ops;
enum { JT_WD_DONE = 0, JT_WD_ERROR = 1, JT_WD_TIMEOUT = 2 };
int jt_watchdog_wait(const jt_watchdog_ops *ops, int timeout_ms, int *polls);

/* Device error word shared by all kernels of the library (0 = clean). */
int jtk_read_and_clear_error(int *out_code);
int *jtk_error_word(void);

/* Number of SMs of the current device (cached). */
int jtk_num_sms(void);

#ifdef __cplusplus
}
#endif

#endif
