/* jt_api_layer.c - the reference's MoE layer entry points with its fp32
 * weight API: jt_moe_fwd_batch / _unchecked (moe_layer.h:230-275,
 * moe_layer.c:980-1663) and jt_moe_fwd / _unchecked (moe_layer.c:304-545).
 *
 * Same prototypes, validation order, modes and fail-closed behaviour (Y is
 * written only after every step succeeded); the computation runs on the
 * GPU through the staging area with the reference's arithmetic:
 *   - gate logits: 4-lane double dot, (float) (k_logits);
 *   - top-k + softmax, capacity sort, renormalization: jt_compat.cu /
 *     jt_route.cu, bit-exact;
 *   - routed experts in the mode the flags select (moe_layer.c:1280-1390):
 *     fp32 GEMM (one rounding per multiply and add, ascending k), W8A8
 *     (per-tensor activations x per-channel gate/up, per-tensor down; the
 *     tensor-core GEMM with the fp64 epilogue), low-bit fake-quant + fp32
 *     GEMM (mode 1), or the T-MAC LUT GEMM (mode 2);
 *   - SwiGLU in double, combine in double in slot order, shared experts.
 * The single-token form keeps its own arithmetic (double dots for gate/up,
 * s kept in double for the down sum) and always runs fp32.
 */
#include <errno.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "../../include/jimotono_b200.h"
#include "jt_internal.h"
#include "jt_stage.h"

#define MOE_MAX_EXPERTS 4096 /* moe_layer.h:52 */
#define MOE_MAX_TOPK 64      /* moe_layer.h:53 */
#define MOE_MAX_SHARED 8     /* moe_layer.h:54 */
#define BWD_MAX_WIDE 4096    /* train_bwd.h:35 */

int jtk_ref_logits(const float *X, const float *Wgate, int T, int n, int E, float *logits, int *flags,
                   cudaStream_t st);
int jtk_ref_gather(const float *X, const int32_t *perm, int k, int R, int n, float *Xe, cudaStream_t st);
int jtk_ref_row_expert(const int32_t *off, int E, int32_t *rexp, cudaStream_t st);
int jtk_ref_gemm_f32(const float *A, int lda, const float *W, long long ws, int wt, const int4 *tiles, int ntiles,
                     float *C, int ldc, int N, int K, cudaStream_t st);
int jtk_ref_silu(const float *G, const float *U, float *S, size_t count, int *flags, cudaStream_t st);
int jtk_ref_fq_rows(const float *W, int rows, int cols, int bits, float *out, int *flags, cudaStream_t st);
int jtk_ref_fq_cols(const float *W, int E, int h, int n, int bits, float *out, int *flags, cudaStream_t st);
int jtk_ref_fill_rows(const float *src, int E, int n, float *dst, cudaStream_t st);
int jtk_ref_combine(const float *Ye, const int32_t *pos, const float *w, const uint8_t *drop, int T, int k, int n,
                    const float *Ys, int S, float *Y, int *flags, cudaStream_t st);
int jtk_ref_scatter_rows(const float *src, const int32_t *pos, const uint8_t *drop, size_t Tk, int cols, float *dst,
                         cudaStream_t st);
int jtk_ref_tok_gateup(const float *x, const float *Wg, const float *Wu, const int32_t *ids, int P, int n, int h,
                       double *s, float *G, float *U, int *flags, cudaStream_t st);
int jtk_ref_tok_down(const double *s, const float *Wd, const int32_t *ids, int P, int n, int h, float *y,
                     int *flags, cudaStream_t st);
int jtk_ref_tok_combine(const float *Yr, const float *w, int P, const float *Ys, int S, int n, float *Y, int *flags,
                        cudaStream_t st);

/* Staging slots of this file. */
enum {
    S_X = JT_SLOT_L0, S_WGATE, S_WG, S_WU, S_WD, S_WGS, S_WUS, S_WDS,
    S_LOGITS, S_TAKEN, S_IDS, S_W, S_WR, S_HIST, S_OFF, S_TOFF, S_TILES, S_META,
    S_PERM, S_POS, S_DROP, S_REXP, S_GT, S_GTS,
    S_XE, S_GE, S_UE, S_SE, S_YE, S_GS, S_US, S_SS, S_YS, S_Y, S_FLAGS,
    S_C1, S_C2, S_C3,
    S_Q1, S_Q2, S_Q3, S_Q4, S_SC1, S_SC2, S_SC3, S_FILL, S_MAXB,
    S_PL, S_MX, S_RS, S_QL, S_QS, S_QB, S_WQ, S_TS, S_TG, S_TU, S_TY, S_TYS
};

/* Flag words: 0 logits / SwiGLU / combine (EINVAL), 1 finiteness scan,
 * 2 top-k softmax, 3 quantization / check flags (1 EINVAL, 2 ERANGE),
 * 4 W8A8 output range (ERANGE); LUT error keys live after them. */
#define F_MAIN 0
#define F_SCAN 1
#define F_TOPK 2
#define F_QUANT 3
#define F_RANGE 4
#define F_WORDS 16

static int moe_valid_dims(int n, int h, int e, int k, int s) { /* moe_layer.c:278-295 */
    if (n <= 0 || h <= 0 || n > BWD_MAX_WIDE || h > BWD_MAX_WIDE) return 0;
    if (e <= 0 || e > MOE_MAX_EXPERTS) return 0;
    if (k <= 0 || k > e || k > MOE_MAX_TOPK) return 0;
    if (s < 0 || s > MOE_MAX_SHARED) return 0;
    return 1;
}

static int host_all_finite(const float *x, size_t n) { /* moe_layer.c:297-303 */
    for (size_t i = 0; i < n; i++)
        if (!isfinite((double)x[i])) return 0;
    return 1;
}

#define NEED(ptr)            \
    do {                     \
        if ((ptr) == NULL) { \
            rc = JT_ERR_NOMEM; \
            errno = ENOMEM;  \
            goto out;        \
        }                    \
    } while (0)
#define CU(expr)                \
    do {                        \
        if ((expr) != 0) {      \
            rc = JT_ERR_CUDA;   \
            errno = EIO;        \
            goto out;           \
        }                       \
    } while (0)
#define FAIL(code)          \
    do {                    \
        errno = (code);     \
        rc = JT_ERR_INVAL;  \
        goto out;           \
    } while (0)

/* 32-row tiles {expert, row0, row_end, 0} over each expert's sorted rows. */
static int4 *row_tiles(const int32_t *off, int E, int *nt) {
    int n = 0;
    for (int e = 0; e < E; e++) n += (off[e + 1] - off[e] + 31) / 32;
    int4 *t = (int4 *)malloc(((size_t)n + 1) * sizeof(int4));
    if (!t) return NULL;
    int i = 0;
    for (int e = 0; e < E; e++)
        for (int r = off[e]; r < off[e + 1]; r += 32) {
            t[i].x = e;
            t[i].y = r;
            t[i].z = r + 32 < off[e + 1] ? r + 32 : off[e + 1];
            t[i].w = 0;
            i++;
        }
    *nt = n;
    return t;
}

/* ====================================================================== */
/* Batched layer                                                          */
/* ====================================================================== */

/* W8A8 gate/up of moe_layer.c:228-274 for every expert with rows: Xe
 * segments quantized per tensor, W [E][N][K] per channel, C = (float)(acc *
 * (sA * sB[n])).  xs_host receives the per-expert activation scales. */
static int w8a8_pc_all(const float *Xe, const int32_t *off, int E, const float *W, int N, int K, float *C,
                       int *dflags, cudaStream_t st) {
    const int Kp = (K + 15) & ~15;
    const size_t R = (size_t)off[E];
    int8_t *q1 = (int8_t *)jt_stage_buf(S_Q1, R * (size_t)K);
    int8_t *q2 = (int8_t *)jt_stage_buf(S_Q2, R * (size_t)Kp);
    int8_t *w1 = (int8_t *)jt_stage_buf(S_Q3, (size_t)E * N * K);
    int8_t *w2 = (int8_t *)jt_stage_buf(S_Q4, (size_t)E * N * Kp);
    float *xs = (float *)jt_stage_buf(S_SC1, (size_t)E * sizeof(float));
    float *sw = (float *)jt_stage_buf(S_SC2, (size_t)E * N * sizeof(float));
    unsigned *mb = (unsigned *)jt_stage_buf(S_MAXB, 64);
    float *hxs = (float *)malloc((size_t)E * sizeof(float));
    int rc = JT_ERR_CUDA;
    if (!q1 || !q2 || !w1 || !w2 || !xs || !sw || !mb || !hxs) {
        free(hxs);
        errno = ENOMEM;
        return JT_ERR_NOMEM;
    }
    for (int e = 0; e < E; e++) {
        const int me = off[e + 1] - off[e];
        if (me == 0) continue;
        if (jtk_quant_tensor(Xe + (size_t)off[e] * K, (size_t)me * K, 0, q1 + (size_t)off[e] * K, xs + e, NULL, mb,
                             dflags + F_QUANT, st))
            goto done;
    }
    if (jtk_quant_blocks(W, E * N, K, K, 0, w1, sw, NULL, dflags + F_QUANT, st)) goto done;
    const int8_t *X8 = q1, *W8 = w1;
    if (Kp != K) {
        if (jtk_pad_rows_s8(q1, (int)R, K, q2, Kp, dflags + F_QUANT, st) ||
            jtk_pad_rows_s8(w1, E * N, K, w2, Kp, dflags + F_QUANT, st))
            goto done;
        X8 = q2;
        W8 = w2;
    }
    if (jt_stage_d2h(hxs, xs, (size_t)E * sizeof(float)) || jt_stage_sync()) goto done;
    for (int e = 0; e < E; e++) {
        const int me = off[e + 1] - off[e];
        if (me == 0) continue;
        if (jtk_w8a8_gemm(X8 + (size_t)off[e] * Kp, Kp, W8 + (size_t)e * N * Kp, Kp, me, N, Kp, NULL,
                          sw + (size_t)e * N, (double)hxs[e], C + (size_t)off[e] * N, N,
                          JTK_EPI_TENSOR_CHANNEL_F64, st))
            goto done;
    }
    if (jtk_check_finite_f32(C, R * (size_t)N, dflags + F_RANGE, st)) goto done;
    rc = JT_OK;
done:
    free(hxs);
    return rc;
}

/* W8A8 down of moe_layer.c:185-223: Se segments and each expert's
 * W [K][N] quantized per tensor, W transposed to [N][Kp]. */
static int w8a8_pt_all(const float *Se, const int32_t *off, int E, const float *W, int N, int K, float *C,
                       int *dflags, cudaStream_t st) {
    const int Kp = (K + 15) & ~15;
    const size_t R = (size_t)off[E];
    int8_t *q1 = (int8_t *)jt_stage_buf(S_Q1, R * (size_t)K);
    int8_t *q2 = (int8_t *)jt_stage_buf(S_Q2, R * (size_t)Kp);
    int8_t *w1 = (int8_t *)jt_stage_buf(S_Q3, (size_t)E * N * K);
    int8_t *w2 = (int8_t *)jt_stage_buf(S_Q4, (size_t)E * N * Kp);
    float *xs = (float *)jt_stage_buf(S_SC1, (size_t)E * sizeof(float));
    float *sb = (float *)jt_stage_buf(S_SC3, (size_t)E * sizeof(float));
    float *fill = (float *)jt_stage_buf(S_FILL, (size_t)E * N * sizeof(float));
    unsigned *mb = (unsigned *)jt_stage_buf(S_MAXB, 64);
    float *hxs = (float *)malloc((size_t)E * sizeof(float));
    int rc = JT_ERR_CUDA;
    if (!q1 || !q2 || !w1 || !w2 || !xs || !sb || !fill || !mb || !hxs) {
        free(hxs);
        errno = ENOMEM;
        return JT_ERR_NOMEM;
    }
    for (int e = 0; e < E; e++) {
        const int me = off[e + 1] - off[e];
        if (me == 0) continue;
        if (jtk_quant_tensor(Se + (size_t)off[e] * K, (size_t)me * K, 0, q1 + (size_t)off[e] * K, xs + e, NULL, mb,
                             dflags + F_QUANT, st))
            goto done;
    }
    if (jtk_quant_blocks(W, E, K * N, K * N, 0, w1, sb, NULL, dflags + F_QUANT, st)) goto done;
    for (int e = 0; e < E; e++) {
        if (off[e + 1] == off[e]) continue;
        if (jtk_transpose_s8(w1 + (size_t)e * K * N, K, N, w2 + (size_t)e * N * Kp, Kp, dflags + F_QUANT, st))
            goto done;
    }
    if (jtk_ref_fill_rows(sb, E, N, fill, st)) goto done;
    const int8_t *X8 = q1;
    if (Kp != K) {
        if (jtk_pad_rows_s8(q1, (int)R, K, q2, Kp, dflags + F_QUANT, st)) goto done;
        X8 = q2;
    }
    if (jt_stage_d2h(hxs, xs, (size_t)E * sizeof(float)) || jt_stage_sync()) goto done;
    for (int e = 0; e < E; e++) {
        const int me = off[e + 1] - off[e];
        if (me == 0) continue;
        if (jtk_w8a8_gemm(X8 + (size_t)off[e] * Kp, Kp, w2 + (size_t)e * N * Kp, Kp, me, N, Kp, NULL,
                          fill + (size_t)e * N, (double)hxs[e], C + (size_t)off[e] * N, N,
                          JTK_EPI_TENSOR_CHANNEL_F64, st))
            goto done;
    }
    if (jtk_check_finite_f32(C, R * (size_t)N, dflags + F_RANGE, st)) goto done;
    rc = JT_OK;
done:
    free(hxs);
    return rc;
}

/* LUT product of lowbit.c:158-267 for every sorted row: the row tables of
 * A [R][K], the columns of its expert's weights (WCols layout), the sign
 * correction; K % 32 != 0 takes the double fallback.  Errors go to keys[0]
 * (table) and keys[1] (columns / lookups). */
static int lut_all(const float *A, int R, int K, const float *W, int E, long long ws, long long st_, long long sj,
                   const int32_t *rexp, float *C, int N, int bits, unsigned long long *keys, cudaStream_t st) {
    if (K % 32 != 0) return jtk_gemm_f64acc(A, W, ws, st_, sj, rexp, C, R, N, K, st) ? JT_ERR_CUDA : JT_OK;
    const size_t nb = (size_t)K / 32;
    int8_t *ql = (int8_t *)jt_stage_buf(S_QL, (size_t)R * nb * 64);
    float *qs = (float *)jt_stage_buf(S_QS, (size_t)R * nb * sizeof(float));
    float *qb = (float *)jt_stage_buf(S_QB, (size_t)R * nb * sizeof(float));
    double *mx = (double *)jt_stage_buf(S_MX, (size_t)E * N * sizeof(double));
    void *pl = jt_stage_buf(S_PL, (size_t)E * bits * nb * N * 8);
    double *rs = (double *)jt_stage_buf(S_RS, (size_t)R * sizeof(double));
    if (!ql || !qs || !qb || !mx || !pl || !rs) {
        errno = ENOMEM;
        return JT_ERR_NOMEM;
    }
    if (jtk_tmac_ctor(A, (size_t)R, (size_t)K, ql, qs, qb, keys, st) ||
        jtk_lut_gemm(A, W, E, ws, st_, sj, rexp, ql, qs, qb, mx, pl, rs, C, R, N, K, bits, keys + 1, st))
        return JT_ERR_CUDA;
    return JT_OK;
}

static int layer_batch(const float *X, const float *Wgate, const float *Wg, const float *Wu, const float *Wd,
                       const float *Wg_s, const float *Wu_s, const float *Wd_s, float *Y, int T, int n, int h,
                       int E, int topk, int S, size_t *out_ids, float *out_weights, float *cache_Gsel,
                       float *cache_Usel, float *cache_Ysel, float *cache_Gs, float *cache_Us, float cap_factor,
                       size_t *out_perm, size_t *out_off, unsigned char *out_drop, size_t *out_kept,
                       size_t *out_dropped, int validate) {
    /* moe_layer.c:1024-1069 */
    if (X == NULL || Wgate == NULL || Wg == NULL || Wu == NULL || Wd == NULL || Y == NULL || out_ids == NULL ||
        out_weights == NULL || T <= 0 || !moe_valid_dims(n, h, E, topk, S)) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    if (S > 0 && (Wg_s == NULL || Wu_s == NULL || Wd_s == NULL)) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    if (!(cap_factor >= 1.0f) || !(cap_factor <= 1.5f) || !isfinite((double)cap_factor)) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    const size_t Tk = (size_t)T * (size_t)topk;
    if (Tk > (size_t)INT32_MAX / 2) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    const int w8 = jt_w8a8_is_enabled();
    const int lb = jt_lowbit_get_mode();
    const size_t nX = (size_t)T * n, nG = (size_t)E * n, nE = (size_t)E * h * n, nS = (size_t)S * h * n;
    const double capd = ceil((double)cap_factor * (double)Tk / (double)E); /* moe_layer.c:931-943 */
    const int cap = (int)capd;

    int rc = JT_ERR_CUDA;
    int flags[F_WORDS];
    unsigned long long keys[6];
    int32_t meta[4] = {0, 0, 0, 0};
    int32_t *hoff = NULL, *hperm = NULL, *hids = NULL;
    int4 *htiles = NULL, *hstiles = NULL;
    float *hw = NULL;
    jt_stage_lock();
    cudaStream_t st = jt_stage_stream();
    float *dX = (float *)jt_stage_buf(S_X, nX * 4);
    float *dGate = (float *)jt_stage_buf(S_WGATE, nG * 4);
    float *dWg = (float *)jt_stage_buf(S_WG, nE * 4);
    float *dWu = (float *)jt_stage_buf(S_WU, nE * 4);
    float *dWd = (float *)jt_stage_buf(S_WD, nE * 4);
    float *dWgs = S ? (float *)jt_stage_buf(S_WGS, nS * 4) : NULL;
    float *dWus = S ? (float *)jt_stage_buf(S_WUS, nS * 4) : NULL;
    float *dWds = S ? (float *)jt_stage_buf(S_WDS, nS * 4) : NULL;
    float *dlog = (float *)jt_stage_buf(S_LOGITS, (size_t)T * E * 4);
    uint32_t *dtaken = (uint32_t *)jt_stage_buf(S_TAKEN, (size_t)T * ((E + 31) / 32) * 4);
    int32_t *dids = (int32_t *)jt_stage_buf(S_IDS, Tk * 4);
    float *dw = (float *)jt_stage_buf(S_W, Tk * 4);
    float *dwr = (float *)jt_stage_buf(S_WR, Tk * 4);
    int32_t *dhist = (int32_t *)jt_stage_buf(S_HIST, (size_t)jtk_sort_chunks(T) * E * 4);
    int32_t *doff = (int32_t *)jt_stage_buf(S_OFF, ((size_t)E + 1) * 4);
    int32_t *dtoff = (int32_t *)jt_stage_buf(S_TOFF, ((size_t)E + 1) * 4);
    int4 *dtl = (int4 *)jt_stage_buf(S_TILES, (Tk / JT_TILE_ROWS + (size_t)E + 1) * 16);
    int32_t *dmeta = (int32_t *)jt_stage_buf(S_META, 64);
    int32_t *dperm = (int32_t *)jt_stage_buf(S_PERM, Tk * 4);
    int32_t *dpos = (int32_t *)jt_stage_buf(S_POS, Tk * 4);
    uint8_t *ddrop = (uint8_t *)jt_stage_buf(S_DROP, Tk);
    float *dY = (float *)jt_stage_buf(S_Y, nX * 4);
    int *dflags = (int *)jt_stage_buf(S_FLAGS, F_WORDS * 4 + 6 * 8);
    NEED(dX);
    NEED(dGate);
    NEED(dWg);
    NEED(dWu);
    NEED(dWd);
    NEED(dlog);
    NEED(dtaken);
    NEED(dids);
    NEED(dw);
    NEED(dwr);
    NEED(dhist);
    NEED(doff);
    NEED(dtoff);
    NEED(dtl);
    NEED(dmeta);
    NEED(dperm);
    NEED(dpos);
    NEED(ddrop);
    NEED(dY);
    NEED(dflags);
    if (S) {
        NEED(dWgs);
        NEED(dWus);
        NEED(dWds);
    }
    unsigned long long *dkeys = (unsigned long long *)(dflags + F_WORDS);
    CU(cudaMemsetAsync(dflags, 0, F_WORDS * 4, st) != cudaSuccess);
    CU(cudaMemsetAsync(dkeys, 0xff, 6 * 8, st) != cudaSuccess);
    CU(jt_stage_h2d(dX, X, nX * 4) || jt_stage_h2d(dGate, Wgate, nG * 4) || jt_stage_h2d(dWg, Wg, nE * 4) ||
       jt_stage_h2d(dWu, Wu, nE * 4) || jt_stage_h2d(dWd, Wd, nE * 4));
    if (S) CU(jt_stage_h2d(dWgs, Wg_s, nS * 4) || jt_stage_h2d(dWus, Wu_s, nS * 4) || jt_stage_h2d(dWds, Wd_s, nS * 4));
    if (validate) { /* moe_layer.c:1072-1096 */
        int *fs = dflags + F_SCAN;
        CU(jtk_check_finite_f32(dX, nX, fs, st) || jtk_check_finite_f32(dGate, nG, fs, st) ||
           jtk_check_finite_f32(dWg, nE, fs, st) || jtk_check_finite_f32(dWu, nE, fs, st) ||
           jtk_check_finite_f32(dWd, nE, fs, st));
        if (S)
            CU(jtk_check_finite_f32(dWgs, nS, fs, st) || jtk_check_finite_f32(dWus, nS, fs, st) ||
               jtk_check_finite_f32(dWds, nS, fs, st));
    }
    /* logits, top-k, capacity sort + renormalization (moe_layer.c:1114-1201) */
    CU(jtk_ref_logits(dX, dGate, T, n, E, dlog, dflags + F_MAIN, st));
    CU(jtk_topk_any(dlog, T, E, topk, dtaken, dids, dw, dflags + F_TOPK, st));
    CU(jtk_moe_sort(dids, dw, T, topk, E, cap, NULL, dhist, doff, dtoff, dtl, dmeta, dperm, dpos, ddrop, dwr, st));
    hoff = (int32_t *)malloc(((size_t)E + 1) * 4);
    NEED(hoff);
    CU(jt_stage_d2h(flags, dflags, sizeof flags) || jt_stage_d2h(meta, dmeta, sizeof meta) ||
       jt_stage_d2h(hoff, doff, ((size_t)E + 1) * 4) || jt_stage_sync());
    if (flags[F_SCAN] || flags[F_MAIN] || flags[F_TOPK]) FAIL(EINVAL);
    const int R = meta[0];
    int ntiles = 0;
    htiles = row_tiles(hoff, E, &ntiles);
    NEED(htiles);

    float *dGe = NULL, *dUe = NULL, *dSe = NULL, *dYe = NULL;
    if (R > 0) {
        float *dXe = (float *)jt_stage_buf(S_XE, (size_t)R * n * 4);
        int32_t *drexp = (int32_t *)jt_stage_buf(S_REXP, (size_t)R * 4);
        int4 *dgt = (int4 *)jt_stage_buf(S_GT, ((size_t)ntiles + 1) * 16);
        dGe = (float *)jt_stage_buf(S_GE, (size_t)R * h * 4);
        dUe = (float *)jt_stage_buf(S_UE, (size_t)R * h * 4);
        dSe = (float *)jt_stage_buf(S_SE, (size_t)R * h * 4);
        dYe = (float *)jt_stage_buf(S_YE, (size_t)R * n * 4);
        NEED(dXe);
        NEED(drexp);
        NEED(dgt);
        NEED(dGe);
        NEED(dUe);
        NEED(dSe);
        NEED(dYe);
        CU(jtk_ref_gather(dX, dperm, topk, R, n, dXe, st) || jtk_ref_row_expert(doff, E, drexp, st) ||
           jt_stage_h2d(dgt, htiles, (size_t)ntiles * 16));
        const long long ws = (long long)h * n;
        if (lb == 2) { /* true LUT (moe_layer.c:1325-1332, :1382-1387) */
            int r = lut_all(dXe, R, n, dWg, E, ws, 1, n, drexp, dGe, h, 2, dkeys, st);
            if (r == JT_OK) r = lut_all(dXe, R, n, dWu, E, ws, 1, n, drexp, dUe, h, 2, dkeys + 2, st);
            if (r != JT_OK) {
                rc = r;
                goto out;
            }
        } else if (lb == 1) { /* fake-quant + fp32 GEMM (moe_layer.c:1308-1324) */
            float *dwq = (float *)jt_stage_buf(S_WQ, nE * 4);
            NEED(dwq);
            CU(jtk_ref_fq_rows(dWg, E * h, n, 2, dwq, dflags + F_MAIN, st) ||
               jtk_ref_gemm_f32(dXe, n, dwq, ws, 1, dgt, ntiles, dGe, h, h, n, st) ||
               jtk_ref_fq_rows(dWu, E * h, n, 2, dwq, dflags + F_MAIN, st) ||
               jtk_ref_gemm_f32(dXe, n, dwq, ws, 1, dgt, ntiles, dUe, h, h, n, st));
        } else if (w8) { /* W8A8 (moe_layer.c:1333-1341) */
            for (int e = 0; e < E; e++)
                if (hoff[e + 1] - hoff[e] > BWD_MAX_WIDE) FAIL(EINVAL); /* w8a8.c:910-953 M cap */
            int r = w8a8_pc_all(dXe, hoff, E, dWg, h, n, dGe, dflags, st);
            if (r == JT_OK) r = w8a8_pc_all(dXe, hoff, E, dWu, h, n, dUe, dflags, st);
            if (r != JT_OK) {
                rc = r;
                goto out;
            }
        } else { /* fp32 (moe_layer.c:1342-1359) */
            CU(jtk_ref_gemm_f32(dXe, n, dWg, ws, 1, dgt, ntiles, dGe, h, h, n, st) ||
               jtk_ref_gemm_f32(dXe, n, dWu, ws, 1, dgt, ntiles, dUe, h, h, n, st));
        }
        CU(jtk_ref_silu(dGe, dUe, dSe, (size_t)R * h, dflags + F_MAIN, st));
        if (lb == 2) {
            int r = lut_all(dSe, R, h, dWd, E, ws, n, 1, drexp, dYe, n, 4, dkeys + 4, st);
            if (r != JT_OK) {
                rc = r;
                goto out;
            }
        } else if (lb == 1) {
            float *dwq = (float *)jt_stage_buf(S_WQ, nE * 4);
            NEED(dwq);
            CU(jtk_ref_fq_cols(dWd, E, h, n, 4, dwq, dflags + F_MAIN, st) ||
               jtk_ref_gemm_f32(dSe, h, dwq, ws, 0, dgt, ntiles, dYe, n, n, h, st));
        } else if (w8) {
            int r = w8a8_pt_all(dSe, hoff, E, dWd, n, h, dYe, dflags, st);
            if (r != JT_OK) {
                rc = r;
                goto out;
            }
        } else {
            CU(jtk_ref_gemm_f32(dSe, h, dWd, ws, 0, dgt, ntiles, dYe, n, n, h, st));
        }
    }
    /* shared experts (moe_layer.c:1466-1553) */
    float *dGs = NULL, *dUs = NULL, *dYs = NULL;
    if (S > 0) {
        dGs = (float *)jt_stage_buf(S_GS, (size_t)S * T * h * 4);
        dUs = (float *)jt_stage_buf(S_US, (size_t)S * T * h * 4);
        float *dSs = (float *)jt_stage_buf(S_SS, (size_t)T * h * 4);
        dYs = (float *)jt_stage_buf(S_YS, (size_t)S * T * n * 4);
        NEED(dGs);
        NEED(dUs);
        NEED(dSs);
        NEED(dYs);
        int32_t toff[2] = {0, T};
        int nst = 0;
        hstiles = row_tiles(toff, 1, &nst);
        NEED(hstiles);
        int4 *dst_ = (int4 *)jt_stage_buf(S_GTS, ((size_t)nst + 1) * 16);
        NEED(dst_);
        CU(jt_stage_h2d(dst_, hstiles, (size_t)nst * 16));
        if (w8 && T > BWD_MAX_WIDE) FAIL(EINVAL);
        for (int s = 0; s < S; s++) {
            const size_t so = (size_t)s * h * n;
            float *gs = dGs + (size_t)s * T * h, *us = dUs + (size_t)s * T * h, *ys = dYs + (size_t)s * T * n;
            if (w8) {
                int r = w8a8_pc_all(dX, toff, 1, dWgs + so, h, n, gs, dflags, st);
                if (r == JT_OK) r = w8a8_pc_all(dX, toff, 1, dWus + so, h, n, us, dflags, st);
                if (r != JT_OK) {
                    rc = r;
                    goto out;
                }
            } else {
                CU(jtk_ref_gemm_f32(dX, n, dWgs + so, 0, 1, dst_, nst, gs, h, h, n, st) ||
                   jtk_ref_gemm_f32(dX, n, dWus + so, 0, 1, dst_, nst, us, h, h, n, st));
            }
            CU(jtk_ref_silu(gs, us, dSs, (size_t)T * h, dflags + F_MAIN, st));
            if (w8) {
                int r = w8a8_pt_all(dSs, toff, 1, dWds + so, n, h, ys, dflags, st);
                if (r != JT_OK) {
                    rc = r;
                    goto out;
                }
            } else {
                CU(jtk_ref_gemm_f32(dSs, h, dWds + so, 0, 0, dst_, nst, ys, n, n, h, st));
            }
        }
    }
    CU(jtk_ref_combine(dYe, dpos, dwr, ddrop, T, topk, n, dYs, S, dY, dflags + F_MAIN, st));
    CU(jt_stage_d2h(flags, dflags, sizeof flags) || jt_stage_d2h(keys, dkeys, sizeof keys) || jt_stage_sync());
    for (int i = 0; i < 6; i++)
        if (keys[i] != ~0ull) FAIL((keys[i] & 1ull) ? ERANGE : EINVAL);
    if (flags[F_QUANT] == 1) FAIL(EINVAL);
    if (flags[F_QUANT] == 2 || flags[F_RANGE]) FAIL(ERANGE);
    if (flags[F_MAIN]) FAIL(EINVAL);

    /* commit (moe_layer.c:1561-1598) */
    hids = (int32_t *)malloc(Tk * 4);
    hw = (float *)malloc(Tk * 4);
    hperm = (int32_t *)malloc(((size_t)R + 1) * 4);
    NEED(hids);
    NEED(hw);
    NEED(hperm);
    CU(jt_stage_d2h(Y, dY, nX * 4) || jt_stage_d2h(hids, dids, Tk * 4) || jt_stage_d2h(hw, dwr, Tk * 4) ||
       jt_stage_d2h(hperm, dperm, (size_t)R * 4));
    if (out_drop != NULL) CU(jt_stage_d2h(out_drop, ddrop, Tk));
    if (cache_Gsel || cache_Usel || cache_Ysel) {
        float *dc1 = (float *)jt_stage_buf(S_C1, Tk * (size_t)(h > n ? h : n) * 4);
        NEED(dc1);
        if (cache_Gsel)
            CU(jtk_ref_scatter_rows(dGe, dpos, ddrop, Tk, h, dc1, st) || jt_stage_d2h(cache_Gsel, dc1, Tk * h * 4) ||
               jt_stage_sync());
        if (cache_Usel)
            CU(jtk_ref_scatter_rows(dUe, dpos, ddrop, Tk, h, dc1, st) || jt_stage_d2h(cache_Usel, dc1, Tk * h * 4) ||
               jt_stage_sync());
        if (cache_Ysel)
            CU(jtk_ref_scatter_rows(dYe, dpos, ddrop, Tk, n, dc1, st) || jt_stage_d2h(cache_Ysel, dc1, Tk * n * 4) ||
               jt_stage_sync());
    }
    for (int s = 0; s < S; s++) { /* cache_Gs/Us [T][S][h] (moe_layer.c:1503-1521) */
        if (cache_Gs)
            CU(cudaMemcpy2DAsync(cache_Gs + (size_t)s * h, (size_t)S * h * 4, dGs + (size_t)s * T * h,
                                 (size_t)h * 4, (size_t)h * 4, (size_t)T, cudaMemcpyDeviceToHost, st) != cudaSuccess);
        if (cache_Us)
            CU(cudaMemcpy2DAsync(cache_Us + (size_t)s * h, (size_t)S * h * 4, dUs + (size_t)s * T * h,
                                 (size_t)h * 4, (size_t)h * 4, (size_t)T, cudaMemcpyDeviceToHost, st) != cudaSuccess);
    }
    CU(jt_stage_sync());
    for (size_t q = 0; q < Tk; q++) {
        out_ids[q] = (size_t)hids[q];
        out_weights[q] = hw[q];
    }
    if (out_perm)
        for (int i = 0; i < R; i++) out_perm[i] = (size_t)hperm[i];
    if (out_off)
        for (int e = 0; e <= E; e++) out_off[e] = (size_t)hoff[e];
    if (out_kept) *out_kept = (size_t)R;
    if (out_dropped) *out_dropped = Tk - (size_t)R;
    rc = JT_OK;
out:
    if (rc == JT_ERR_CUDA) cudaStreamSynchronize(st);
    free(hoff);
    free(hperm);
    free(hids);
    free(hw);
    free(htiles);
    free(hstiles);
    jt_stage_unlock();
    return rc;
}

int jt_moe_fwd_batch(const float *X, const float *Wgate, const float *Wg, const float *Wu, const float *Wd,
                     const float *Wg_s, const float *Wu_s, const float *Wd_s, float *Y, int T, int n, int h,
                     int n_experts, int topk, int n_shared, size_t *out_ids, float *out_weights, float *cache_Gsel,
                     float *cache_Usel, float *cache_Ysel, float *cache_Gs, float *cache_Us, float cap_factor,
                     size_t *out_perm, size_t *out_off, unsigned char *out_drop, size_t *out_kept,
                     size_t *out_dropped) {
    return layer_batch(X, Wgate, Wg, Wu, Wd, Wg_s, Wu_s, Wd_s, Y, T, n, h, n_experts, topk, n_shared, out_ids,
                       out_weights, cache_Gsel, cache_Usel, cache_Ysel, cache_Gs, cache_Us, cap_factor, out_perm,
                       out_off, out_drop, out_kept, out_dropped, 1);
}

int jt_moe_fwd_batch_unchecked(const float *X, const float *Wgate, const float *Wg, const float *Wu,
                               const float *Wd, const float *Wg_s, const float *Wu_s, const float *Wd_s, float *Y,
                               int T, int n, int h, int n_experts, int topk, int n_shared, size_t *out_ids,
                               float *out_weights, float *cache_Gsel, float *cache_Usel, float *cache_Ysel,
                               float *cache_Gs, float *cache_Us, float cap_factor, size_t *out_perm,
                               size_t *out_off, unsigned char *out_drop, size_t *out_kept, size_t *out_dropped) {
    return layer_batch(X, Wgate, Wg, Wu, Wd, Wg_s, Wu_s, Wd_s, Y, T, n, h, n_experts, topk, n_shared, out_ids,
                       out_weights, cache_Gsel, cache_Usel, cache_Ysel, cache_Gs, cache_Us, cap_factor, out_perm,
                       out_off, out_drop, out_kept, out_dropped, 0);
}

/* ====================================================================== */
/* Single-token layer (moe_layer.c:304-545)                               */
/* ====================================================================== */

static int layer_tok(const float *X, const float *Wgate, const float *Wg, const float *Wu, const float *Wd,
                     const float *Wg_s, const float *Wu_s, const float *Wd_s, float *Y, int n, int h, int E,
                     int topk, int S, size_t *out_ids, float *out_weights, float *out_logits, float *cache_Gsel,
                     float *cache_Usel, float *cache_Ysel, float *cache_Gs, float *cache_Us, int validate) {
    if (X == NULL || Wgate == NULL || Wg == NULL || Wu == NULL || Wd == NULL || Y == NULL || out_ids == NULL ||
        out_weights == NULL || !moe_valid_dims(n, h, E, topk, S)) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    if (S > 0 && (Wg_s == NULL || Wu_s == NULL || Wd_s == NULL)) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    const size_t hn = (size_t)h * n;
    if (validate) { /* the reference's own host scan (moe_layer.c:340-360) */
        if (!host_all_finite(X, (size_t)n) || !host_all_finite(Wgate, (size_t)E * n) ||
            !host_all_finite(Wg, (size_t)E * hn) || !host_all_finite(Wu, (size_t)E * hn) ||
            !host_all_finite(Wd, (size_t)E * hn)) {
            errno = EINVAL;
            return JT_ERR_INVAL;
        }
        if (S > 0 && (!host_all_finite(Wg_s, (size_t)S * hn) || !host_all_finite(Wu_s, (size_t)S * hn) ||
                      !host_all_finite(Wd_s, (size_t)S * hn))) {
            errno = EINVAL;
            return JT_ERR_INVAL;
        }
    }
    int rc = JT_ERR_CUDA;
    int flags[F_WORDS];
    int32_t hids[MOE_MAX_TOPK];
    float hw[MOE_MAX_TOPK];
    jt_stage_lock();
    cudaStream_t st = jt_stage_stream();
    const int P = topk + S;
    float *dX = (float *)jt_stage_buf(S_X, (size_t)n * 4);
    float *dGate = (float *)jt_stage_buf(S_WGATE, (size_t)E * n * 4);
    float *dlog = (float *)jt_stage_buf(S_LOGITS, (size_t)E * 4);
    uint32_t *dtaken = (uint32_t *)jt_stage_buf(S_TAKEN, (size_t)((E + 31) / 32) * 4);
    int32_t *dids = (int32_t *)jt_stage_buf(S_IDS, (size_t)topk * 4);
    float *dw = (float *)jt_stage_buf(S_W, (size_t)topk * 4);
    float *dWg = (float *)jt_stage_buf(S_WG, (size_t)P * hn * 4);
    float *dWu = (float *)jt_stage_buf(S_WU, (size_t)P * hn * 4);
    float *dWd = (float *)jt_stage_buf(S_WD, (size_t)P * hn * 4);
    double *ds = (double *)jt_stage_buf(S_TS, (size_t)P * h * 8);
    float *dG = (float *)jt_stage_buf(S_TG, (size_t)P * h * 4);
    float *dU = (float *)jt_stage_buf(S_TU, (size_t)P * h * 4);
    float *dYp = (float *)jt_stage_buf(S_TY, (size_t)P * n * 4);
    float *dY = (float *)jt_stage_buf(S_Y, (size_t)n * 4);
    int *dflags = (int *)jt_stage_buf(S_FLAGS, F_WORDS * 4 + 6 * 8);
    NEED(dX);
    NEED(dGate);
    NEED(dlog);
    NEED(dtaken);
    NEED(dids);
    NEED(dw);
    NEED(dWg);
    NEED(dWu);
    NEED(dWd);
    NEED(ds);
    NEED(dG);
    NEED(dU);
    NEED(dYp);
    NEED(dY);
    NEED(dflags);
    CU(cudaMemsetAsync(dflags, 0, F_WORDS * 4, st) != cudaSuccess);
    CU(jt_stage_h2d(dX, X, (size_t)n * 4) || jt_stage_h2d(dGate, Wgate, (size_t)E * n * 4));
    CU(jtk_ref_logits(dX, dGate, 1, n, E, dlog, dflags + F_MAIN, st));
    CU(jtk_topk_any(dlog, 1, E, topk, dtaken, dids, dw, dflags + F_TOPK, st));
    CU(jt_stage_d2h(flags, dflags, sizeof flags) || jt_stage_d2h(hids, dids, (size_t)topk * 4) ||
       jt_stage_d2h(hw, dw, (size_t)topk * 4) || jt_stage_sync());
    if (flags[F_MAIN] || flags[F_TOPK]) FAIL(EINVAL);
    /* the selected experts' weights, then the shared ones, as P packed experts */
    for (int p = 0; p < topk; p++) {
        const size_t e = (size_t)hids[p];
        CU(jt_stage_h2d(dWg + (size_t)p * hn, Wg + e * hn, hn * 4) ||
           jt_stage_h2d(dWu + (size_t)p * hn, Wu + e * hn, hn * 4) ||
           jt_stage_h2d(dWd + (size_t)p * hn, Wd + e * hn, hn * 4));
    }
    if (S > 0)
        CU(jt_stage_h2d(dWg + (size_t)topk * hn, Wg_s, (size_t)S * hn * 4) ||
           jt_stage_h2d(dWu + (size_t)topk * hn, Wu_s, (size_t)S * hn * 4) ||
           jt_stage_h2d(dWd + (size_t)topk * hn, Wd_s, (size_t)S * hn * 4));
    CU(jtk_ref_tok_gateup(dX, dWg, dWu, NULL, P, n, h, ds, dG, dU, dflags + F_MAIN, st) ||
       jtk_ref_tok_down(ds, dWd, NULL, P, n, h, dYp, dflags + F_MAIN, st) ||
       jtk_ref_tok_combine(dYp, dw, topk, S ? dYp + (size_t)topk * n : NULL, S, n, dY, dflags + F_MAIN, st));
    CU(jt_stage_d2h(flags, dflags, sizeof flags) || jt_stage_sync());
    if (flags[F_MAIN]) FAIL(EINVAL);
    CU(jt_stage_d2h(Y, dY, (size_t)n * 4));
    if (out_logits) CU(jt_stage_d2h(out_logits, dlog, (size_t)E * 4));
    if (cache_Gsel) CU(jt_stage_d2h(cache_Gsel, dG, (size_t)topk * h * 4));
    if (cache_Usel) CU(jt_stage_d2h(cache_Usel, dU, (size_t)topk * h * 4));
    if (cache_Ysel) CU(jt_stage_d2h(cache_Ysel, dYp, (size_t)topk * n * 4));
    if (cache_Gs && S) CU(jt_stage_d2h(cache_Gs, dG + (size_t)topk * h, (size_t)S * h * 4));
    if (cache_Us && S) CU(jt_stage_d2h(cache_Us, dU + (size_t)topk * h, (size_t)S * h * 4));
    CU(jt_stage_sync());
    for (int p = 0; p < topk; p++) {
        out_ids[p] = (size_t)hids[p];
        out_weights[p] = hw[p];
    }
    rc = JT_OK;
out:
    if (rc == JT_ERR_CUDA) cudaStreamSynchronize(st);
    jt_stage_unlock();
    return rc;
}

int jt_moe_fwd(const float *X, const float *Wgate, const float *Wg, const float *Wu, const float *Wd,
               const float *Wg_s, const float *Wu_s, const float *Wd_s, float *Y, int n, int h, int n_experts,
               int topk, int n_shared, size_t *out_ids, float *out_weights, float *out_logits, float *cache_Gsel,
               float *cache_Usel, float *cache_Ysel, float *cache_Gs, float *cache_Us) {
    return layer_tok(X, Wgate, Wg, Wu, Wd, Wg_s, Wu_s, Wd_s, Y, n, h, n_experts, topk, n_shared, out_ids,
                     out_weights, out_logits, cache_Gsel, cache_Usel, cache_Ysel, cache_Gs, cache_Us, 1);
}

int jt_moe_fwd_unchecked(const float *X, const float *Wgate, const float *Wg, const float *Wu, const float *Wd,
                         const float *Wg_s, const float *Wu_s, const float *Wd_s, float *Y, int n, int h,
                         int n_experts, int topk, int n_shared, size_t *out_ids, float *out_weights,
                         float *out_logits, float *cache_Gsel, float *cache_Usel, float *cache_Ysel,
                         float *cache_Gs, float *cache_Us) {
    return layer_tok(X, Wgate, Wg, Wu, Wd, Wg_s, Wu_s, Wd_s, Y, n, h, n_experts, topk, n_shared, out_ids,
                     out_weights, out_logits, cache_Gsel, cache_Usel, cache_Ysel, cache_Gs, cache_Us, 0);
}
