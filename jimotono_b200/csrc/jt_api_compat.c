/* jt_api_compat.c - the reference's routing, batch-sort, fp32 GEMM and
 * low-bit host entry points (routing.h:56, moe_layer.h:194, moe_gemm.h:59-66,
 * lowbit.h:30-43) with their validation order, errno values and fail-closed
 * behaviour; the computation runs on the GPU through the staging area.
 */
#include <errno.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "../../include/jimotono_b200.h"
#include "jt_internal.h"
#include "jt_stage.h"

int jtk_topk_any(const float *logits, int n, int k, uint32_t *taken, int32_t *ids, float *w, int *flag,
                 cudaStream_t stream);
int jtk_gemm_f32_seq(const float *A, const float *B, float *C, int M, int N, int K, cudaStream_t stream);
int jtk_transpose_f32(const float *src, float *dst, int rows, int cols, cudaStream_t stream);
int jtk_lowbit_absmax(const float *w, size_t n, unsigned long long *maxbits, int *bad, cudaStream_t stream);
int jtk_lowbit_fq(const float *w, size_t n, int bits, const unsigned long long *maxbits, float *fq,
                  cudaStream_t stream);
int jtk_lowbit_idx(const float *col, size_t k, int bits, const unsigned long long *maxbits, uint8_t *idx,
                   cudaStream_t stream);

#define MOE_MAX_EXPERTS 4096 /* moe_layer.h:52 */
#define MOE_MAX_TOPK 64      /* moe_layer.h:53 */

static int cuda_fail(void) {
    errno = EIO;
    return JT_ERR_CUDA;
}

/* ---------------------------------------------------------------- routing.c:16-76 */
int jt_routing_topk(const float *logits, size_t n, size_t k, size_t *out_ids, float *out_weights) {
    if (logits == NULL || out_ids == NULL || out_weights == NULL) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    if (n == 0 || k == 0 || k > n) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    for (size_t i = 0; i < n; i++) {
        if (isnan(logits[i])) {
            errno = EINVAL;
            return JT_ERR_INVAL;
        }
    }
    if (n > (size_t)INT32_MAX) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    int rc = JT_ERR_CUDA;
    jt_stage_lock();
    float *dl = (float *)jt_stage_buf(JT_SLOT_X, n * sizeof(float));
    uint32_t *taken = (uint32_t *)jt_stage_buf(JT_SLOT_AUX1, ((n + 31) / 32) * sizeof(uint32_t));
    int32_t *dids = (int32_t *)jt_stage_buf(JT_SLOT_AUX2, k * sizeof(int32_t));
    float *dw = (float *)jt_stage_buf(JT_SLOT_Y, k * sizeof(float));
    int *dflag = (int *)jt_stage_buf(JT_SLOT_FLAGS, 64);
    int32_t *hids = (int32_t *)malloc(k * sizeof(int32_t));
    float *hw = (float *)malloc(k * sizeof(float));
    int flag = 0;
    cudaStream_t st = jt_stage_stream();
    if (!dl || !taken || !dids || !dw || !dflag || !hids || !hw) {
        errno = ENOMEM;
        rc = JT_ERR_NOMEM;
        goto out;
    }
    if (cudaMemsetAsync(dflag, 0, 64, st) != cudaSuccess || jt_stage_h2d(dl, logits, n * sizeof(float)) ||
        jtk_topk_any(dl, (int)n, (int)k, taken, dids, dw, dflag, st) != 0 ||
        jt_stage_d2h(&flag, dflag, sizeof(int)) || jt_stage_d2h(hids, dids, k * sizeof(int32_t)) ||
        jt_stage_d2h(hw, dw, k * sizeof(float)) || jt_stage_sync()) {
        rc = cuda_fail();
        goto out;
    }
    if (flag) { /* non-finite softmax (all -inf, +inf) */
        errno = EINVAL;
        rc = JT_ERR_INVAL;
        goto out;
    }
    for (size_t p = 0; p < k; p++) {
        out_ids[p] = (size_t)hids[p];
        out_weights[p] = hw[p];
    }
    rc = JT_OK;
out:
    free(hids);
    free(hw);
    jt_stage_unlock();
    return rc;
}

/* ---------------------------------------------------------------- moe_layer.c:895-978 */
int jt_moe_batch_sort(const size_t *ids, int T, int k, int E, float cap_factor, size_t *perm,
                      size_t *off, unsigned char *drop, size_t *out_kept, size_t *out_dropped) {
    if (ids == NULL || perm == NULL || off == NULL || drop == NULL) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    if (T <= 0 || k <= 0 || E <= 0 || E > MOE_MAX_EXPERTS || k > E || k > MOE_MAX_TOPK) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    if (!(cap_factor >= 1.0f) || !(cap_factor <= 1.5f) || !isfinite((double)cap_factor)) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    if ((size_t)k > SIZE_MAX / (size_t)T || (size_t)T * (size_t)k > (size_t)INT32_MAX) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    const size_t Tk = (size_t)T * (size_t)k;
    for (size_t q = 0; q < Tk; q++) {
        if (ids[q] >= (size_t)E) {
            errno = EINVAL;
            return JT_ERR_INVAL;
        }
    }
    const double capd = ceil((double)cap_factor * (double)Tk / (double)E);
    if (!isfinite(capd) || capd < 1.0 || capd > 2147483647.0) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    const int cap = (int)capd;
    int rc = JT_ERR_CUDA;
    const size_t nch = (size_t)jtk_sort_chunks(T);
    jt_stage_lock();
    int32_t *hid = (int32_t *)malloc(Tk * sizeof(int32_t));
    int32_t *hperm = (int32_t *)malloc(Tk * sizeof(int32_t));
    int32_t *hoff = (int32_t *)malloc(((size_t)E + 1) * sizeof(int32_t));
    int32_t *dids = (int32_t *)jt_stage_buf(JT_SLOT_A, Tk * 4);
    float *dw = (float *)jt_stage_buf(JT_SLOT_W1, Tk * 4);
    float *dwo = (float *)jt_stage_buf(JT_SLOT_W2, Tk * 4);
    int32_t *dhist = (int32_t *)jt_stage_buf(JT_SLOT_AUX1, nch * (size_t)E * 4);
    int32_t *doff = (int32_t *)jt_stage_buf(JT_SLOT_AUX2, ((size_t)E + 1) * 4);
    int32_t *dtoff = (int32_t *)jt_stage_buf(JT_SLOT_AUX3, ((size_t)E + 1) * 4);
    int4 *dtiles = (int4 *)jt_stage_buf(JT_SLOT_C, (Tk / JT_TILE_ROWS + (size_t)E + 1) * 16);
    int32_t *dmeta = (int32_t *)jt_stage_buf(JT_SLOT_FLAGS, 64);
    int32_t *dperm = (int32_t *)jt_stage_buf(JT_SLOT_B, Tk * 4);
    int32_t *dpos = (int32_t *)jt_stage_buf(JT_SLOT_B2, Tk * 4);
    uint8_t *ddrop = (uint8_t *)jt_stage_buf(JT_SLOT_AUX4, Tk);
    cudaStream_t st = jt_stage_stream();
    if (!hid || !hperm || !hoff || !dids || !dw || !dwo || !dhist || !doff || !dtoff || !dtiles || !dmeta ||
        !dperm || !dpos || !ddrop) {
        errno = ENOMEM;
        rc = JT_ERR_NOMEM;
        goto out;
    }
    for (size_t q = 0; q < Tk; q++) hid[q] = (int32_t)ids[q];
    int32_t meta[4] = {0, 0, 0, 0};
    if (jt_stage_h2d(dids, hid, Tk * 4) || cudaMemsetAsync(dw, 0, Tk * 4, st) != cudaSuccess ||
        jtk_moe_sort(dids, dw, T, k, E, cap, NULL, dhist, doff, dtoff, dtiles, dmeta, dperm, dpos, ddrop,
                     dwo, st) != 0 ||
        jt_stage_d2h(meta, dmeta, sizeof meta) || jt_stage_d2h(hoff, doff, ((size_t)E + 1) * 4) ||
        jt_stage_sync()) {
        rc = cuda_fail();
        goto out;
    }
    const size_t kept = (size_t)meta[0];
    if (jt_stage_d2h(hperm, dperm, kept * 4) || jt_stage_d2h(drop, ddrop, Tk) || jt_stage_sync()) {
        rc = cuda_fail();
        goto out;
    }
    for (size_t i = 0; i < kept; i++) perm[i] = (size_t)hperm[i];
    for (int e = 0; e <= E; e++) off[e] = (size_t)hoff[e];
    if (out_kept != NULL) *out_kept = kept;
    if (out_dropped != NULL) *out_dropped = Tk - kept;
    rc = JT_OK;
out:
    free(hid);
    free(hperm);
    free(hoff);
    jt_stage_unlock();
    return rc;
}

/* ---------------------------------------------------------------- moe_gemm.c:17-170 */
int jt_transpose_f32(const float *src, float *dst, int rows, int cols) {
    if (src == NULL || dst == NULL || rows <= 0 || cols <= 0 ||
        (size_t)rows > SIZE_MAX / (size_t)cols) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    const size_t n = (size_t)rows * (size_t)cols;
    int rc = JT_ERR_CUDA;
    jt_stage_lock();
    float *ds = (float *)jt_stage_buf(JT_SLOT_X, n * 4);
    float *dd = (float *)jt_stage_buf(JT_SLOT_Y, n * 4);
    if (!ds || !dd) {
        errno = ENOMEM;
        rc = JT_ERR_NOMEM;
        goto out;
    }
    if (jt_stage_h2d(ds, src, n * 4) || jtk_transpose_f32(ds, dd, rows, cols, jt_stage_stream()) != 0 ||
        jt_stage_d2h(dst, dd, n * 4) || jt_stage_sync()) {
        rc = cuda_fail();
        goto out;
    }
    rc = JT_OK;
out:
    jt_stage_unlock();
    return rc;
}

int jt_gemm_mat_f32(const float *A, const float *B, float *C, int M, int N, int K) {
    if (A == NULL || B == NULL || C == NULL) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    if (M == 0) {
        if (N <= 0 || K <= 0) {
            errno = EINVAL;
            return JT_ERR_INVAL;
        }
        return JT_OK;
    }
    if (M < 0 || N <= 0 || K <= 0 || (size_t)M > SIZE_MAX / (size_t)K ||
        (size_t)M > SIZE_MAX / (size_t)N || (size_t)K > SIZE_MAX / (size_t)N) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    int rc = JT_ERR_CUDA;
    jt_stage_lock();
    float *dA = (float *)jt_stage_buf(JT_SLOT_A, (size_t)M * K * 4);
    float *dB = (float *)jt_stage_buf(JT_SLOT_B, (size_t)K * N * 4);
    float *dC = (float *)jt_stage_buf(JT_SLOT_C, (size_t)M * N * 4);
    if (!dA || !dB || !dC) {
        errno = ENOMEM;
        rc = JT_ERR_NOMEM;
        goto out;
    }
    if (jt_stage_h2d(dA, A, (size_t)M * K * 4) || jt_stage_h2d(dB, B, (size_t)K * N * 4) ||
        jtk_gemm_f32_seq(dA, dB, dC, M, N, K, jt_stage_stream()) != 0 ||
        jt_stage_d2h(C, dC, (size_t)M * N * 4) || jt_stage_sync()) {
        rc = cuda_fail();
        goto out;
    }
    /* like the reference: C is written, then a non-finite value is INVAL */
    rc = JT_OK;
    for (size_t i = 0; i < (size_t)M * N; i++) {
        if (!isfinite((double)C[i])) {
            errno = EINVAL;
            rc = JT_ERR_INVAL;
            break;
        }
    }
out:
    jt_stage_unlock();
    return rc;
}

/* ---------------------------------------------------------------- lowbit.c:16-141 */
static int g_lowbit_mode = 0; /* lowbit.c:16 */

int jt_lowbit_set_mode(int mode) {
    if (mode < 0 || mode > 2) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    g_lowbit_mode = mode;
    return JT_OK;
}

int jt_lowbit_get_mode(void) { return g_lowbit_mode; }

int jt_lowbit_bits_for(int is_down, int *out_bits) {
    if (out_bits == NULL) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    *out_bits = (is_down != 0) ? 4 : 2;
    return JT_OK;
}

/* maxabs in double on the GPU; returns 0, JT_ERR_INVAL (non-finite input) or
 * a CUDA failure; *maxa_dev points at the staged result. */
static int lowbit_prepare(const float *w, size_t n, float **dw, unsigned long long **maxbits,
                          double *maxa) {
    *dw = (float *)jt_stage_buf(JT_SLOT_X, n * 4);
    *maxbits = (unsigned long long *)jt_stage_buf(JT_SLOT_AUX1, 16);
    int *dbad = (int *)jt_stage_buf(JT_SLOT_FLAGS, 64);
    if (!*dw || !*maxbits || !dbad) {
        errno = ENOMEM;
        return JT_ERR_NOMEM;
    }
    cudaStream_t st = jt_stage_stream();
    int bad = 0;
    unsigned long long mb = 0;
    if (cudaMemsetAsync(dbad, 0, 64, st) != cudaSuccess || jt_stage_h2d(*dw, w, n * 4) ||
        jtk_lowbit_absmax(*dw, n, *maxbits, dbad, st) != 0 || jt_stage_d2h(&bad, dbad, sizeof bad) ||
        jt_stage_d2h(&mb, *maxbits, sizeof mb) || jt_stage_sync())
        return cuda_fail();
    if (bad) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    memcpy(maxa, &mb, sizeof mb);
    return JT_OK;
}

int jt_lowbit_fakequant(const float *w, float *fq, size_t n, int bits) {
    if (w == NULL || fq == NULL || n == 0 || (bits != 2 && bits != 4)) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    jt_stage_lock();
    float *dw = NULL;
    unsigned long long *maxbits = NULL;
    double maxa = 0.0;
    int rc = lowbit_prepare(w, n, &dw, &maxbits, &maxa);
    if (rc == JT_OK) {
        float *dfq = (float *)jt_stage_buf(JT_SLOT_Y, n * 4);
        if (!dfq) {
            errno = ENOMEM;
            rc = JT_ERR_NOMEM;
        } else if (jtk_lowbit_fq(dw, n, bits, maxbits, dfq, jt_stage_stream()) != 0 ||
                   jt_stage_d2h(fq, dfq, n * 4) || jt_stage_sync()) {
            rc = cuda_fail();
        }
    }
    jt_stage_unlock();
    return rc;
}

int jt_lowbit_col_to_idx(const float *col, size_t k, int bits, uint8_t *idx, float *w_scale) {
    if (col == NULL || idx == NULL || w_scale == NULL || k == 0) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    if ((bits != 2 && bits != 4) || (k % 4u) != 0u) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    jt_stage_lock();
    float *dw = NULL;
    unsigned long long *maxbits = NULL;
    double maxa = 0.0;
    int rc = lowbit_prepare(col, k, &dw, &maxbits, &maxa);
    if (rc == JT_OK) {
        const size_t nb = (size_t)bits * (k / 4);
        uint8_t *didx = (uint8_t *)jt_stage_buf(JT_SLOT_Y, nb);
        if (!didx) {
            errno = ENOMEM;
            rc = JT_ERR_NOMEM;
        } else if (jtk_lowbit_idx(dw, k, bits, maxbits, didx, jt_stage_stream()) != 0 ||
                   jt_stage_d2h(idx, didx, nb) || jt_stage_sync()) {
            rc = cuda_fail();
        } else {
            *w_scale = (float)maxa;
        }
    }
    jt_stage_unlock();
    return rc;
}
