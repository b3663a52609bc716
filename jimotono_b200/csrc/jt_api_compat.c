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
        jtk_topk_any(dl, 1, (int)n, (int)k, taken, dids, dw, dflag, st) != 0 ||
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

/* ---------------------------------------------------------------- tmac.c / lowbit.c:158-267 */
int jtk_tmac_lookup_one(const int8_t *qlut, const uint8_t *idx, const float *scales, const float *biases,
                        size_t ngroups, size_t nblocks, int bits, float w_scale, float *out, int *flag,
                        cudaStream_t stream);

#define TMAC_G 4          /* tmac.h:44 */
#define TMAC_LUT_HALF 8   /* tmac.h:45 */
#define TMAC_ACT_GROUP 32 /* tmac.h:47 */

static int size_mul_ov(size_t a, size_t b, size_t *out) {
    if (a == 0 || b == 0) {
        *out = 0;
        return 0;
    }
    if (a > SIZE_MAX / b) return 1;
    *out = a * b;
    return 0;
}

/* tmac.c:168-197 */
int jt_tmac_qlut_bytes(size_t n, size_t k, size_t *out) {
    if (out == NULL) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    *out = 0;
    if (n == 0 || k == 0 || k % TMAC_G != 0) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    size_t t = 0, bytes = 0;
    if (size_mul_ov(n, k / TMAC_G, &t) || size_mul_ov(t, TMAC_LUT_HALF, &bytes)) {
        errno = ENOMEM;
        return JT_ERR_NOMEM;
    }
    *out = bytes;
    return JT_OK;
}

/* tmac.c:199-228 */
int jt_tmac_param_bytes(size_t n, size_t k, size_t *out) {
    if (out == NULL) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    *out = 0;
    if (n == 0 || k == 0 || k % TMAC_ACT_GROUP != 0) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    size_t t = 0, bytes = 0;
    if (size_mul_ov(n, k / TMAC_ACT_GROUP, &t) || size_mul_ov(t, sizeof(float), &bytes)) {
        errno = ENOMEM;
        return JT_ERR_NOMEM;
    }
    *out = bytes;
    return JT_OK;
}

/* Arguments of tmac.c:230-272: 0, or the error to return. */
static int tmac_ctor_check(const float *act, size_t n, size_t k, const void *qlut, const void *scales,
                           const void *biases) {
    if (act == NULL || qlut == NULL || scales == NULL || biases == NULL || n == 0 || k == 0 ||
        k % TMAC_G != 0 || k % TMAC_ACT_GROUP != 0) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    size_t t = 0, u = 0;
    if (size_mul_ov(n, k, &t) || size_mul_ov(n, k / TMAC_G, &t) || size_mul_ov(t, TMAC_LUT_HALF, &u) ||
        size_mul_ov(n, k / TMAC_ACT_GROUP, &t) || size_mul_ov(n * k, sizeof(float), &t)) {
        errno = ENOMEM;
        return JT_ERR_NOMEM;
    }
    return JT_OK;
}

/* A ctor error key posted by the kernel: block index << 1 | (1 = ERANGE). */
static int tmac_err(unsigned long long key) {
    errno = (key & 1ull) ? ERANGE : EINVAL;
    return JT_ERR_INVAL;
}

/* tmac.c:230-385.  On failure the outputs are left unchanged (the
 * reference has written the blocks before the failing one). */
int jt_tmac_lut_ctor(const float *act, size_t n, size_t k, int8_t *qlut, float *scales, float *biases) {
    int rc = tmac_ctor_check(act, n, k, qlut, scales, biases);
    if (rc != JT_OK) return rc;
    const size_t nb = k / TMAC_ACT_GROUP, qn = n * (k / TMAC_G) * TMAC_LUT_HALF;
    jt_stage_lock();
    float *da = (float *)jt_stage_buf(JT_SLOT_X, n * k * sizeof(float));
    int8_t *dq = (int8_t *)jt_stage_buf(JT_SLOT_A, qn);
    float *ds = (float *)jt_stage_buf(JT_SLOT_SCALE, n * nb * sizeof(float));
    float *dbi = (float *)jt_stage_buf(JT_SLOT_AUX1, n * nb * sizeof(float));
    unsigned long long *derr = (unsigned long long *)jt_stage_buf(JT_SLOT_FLAGS, 64);
    unsigned long long key = 0;
    cudaStream_t st = jt_stage_stream();
    if (!da || !dq || !ds || !dbi || !derr) {
        errno = ENOMEM;
        rc = JT_ERR_NOMEM;
        goto out;
    }
    if (jt_stage_h2d(da, act, n * k * sizeof(float)) ||
        jtk_tmac_ctor(da, n, k, dq, ds, dbi, derr, st) != 0 || jt_stage_d2h(&key, derr, sizeof key) ||
        jt_stage_sync()) {
        rc = cuda_fail();
        goto out;
    }
    if (key != ~0ull) {
        rc = tmac_err(key);
        goto out;
    }
    if (jt_stage_d2h(qlut, dq, qn) || jt_stage_d2h(scales, ds, n * nb * sizeof(float)) ||
        jt_stage_d2h(biases, dbi, n * nb * sizeof(float)) || jt_stage_sync()) {
        rc = cuda_fail();
        goto out;
    }
    rc = JT_OK;
out:
    jt_stage_unlock();
    return rc;
}

/* tmac.c:387-506 */
int jt_tmac_lookup_accum(const int8_t *qlut, const uint8_t *idx, const float *scales, const float *biases,
                         size_t ngroups, size_t nblocks, int bits, float w_scale, float *out) {
    if (qlut == NULL || idx == NULL || scales == NULL || biases == NULL || out == NULL ||
        ngroups == 0 || nblocks == 0) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    if (nblocks > SIZE_MAX / 8u) {
        errno = ENOMEM;
        return JT_ERR_NOMEM;
    }
    if (ngroups != nblocks * 8u || bits < 1 || bits > 4) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    if (ngroups > SIZE_MAX / TMAC_LUT_HALF || ngroups > SIZE_MAX / (size_t)bits) {
        errno = ENOMEM;
        return JT_ERR_NOMEM;
    }
    if (!isfinite((double)w_scale)) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    int rc = JT_ERR_CUDA;
    jt_stage_lock();
    int8_t *dq = (int8_t *)jt_stage_buf(JT_SLOT_A, ngroups * TMAC_LUT_HALF);
    uint8_t *di = (uint8_t *)jt_stage_buf(JT_SLOT_B, ngroups * (size_t)bits);
    float *ds = (float *)jt_stage_buf(JT_SLOT_SCALE, nblocks * sizeof(float));
    float *dbi = (float *)jt_stage_buf(JT_SLOT_AUX1, nblocks * sizeof(float));
    float *dout = (float *)jt_stage_buf(JT_SLOT_Y, 16);
    int *dflag = (int *)jt_stage_buf(JT_SLOT_FLAGS, 64);
    int flag = 0;
    float o = 0.0f;
    cudaStream_t st = jt_stage_stream();
    if (!dq || !di || !ds || !dbi || !dout || !dflag) {
        errno = ENOMEM;
        rc = JT_ERR_NOMEM;
        goto out;
    }
    if (cudaMemsetAsync(dflag, 0, 64, st) != cudaSuccess || jt_stage_h2d(dq, qlut, ngroups * TMAC_LUT_HALF) ||
        jt_stage_h2d(di, idx, ngroups * (size_t)bits) || jt_stage_h2d(ds, scales, nblocks * sizeof(float)) ||
        jt_stage_h2d(dbi, biases, nblocks * sizeof(float)) ||
        jtk_tmac_lookup_one(dq, di, ds, dbi, ngroups, nblocks, bits, w_scale, dout, dflag, st) != 0 ||
        jt_stage_d2h(&flag, dflag, sizeof flag) || jt_stage_d2h(&o, dout, sizeof o) || jt_stage_sync()) {
        rc = cuda_fail();
        goto out;
    }
    if (flag) {
        errno = flag == 1 ? EINVAL : ERANGE;
        rc = JT_ERR_INVAL;
        goto out;
    }
    *out = o;
    rc = JT_OK;
out:
    jt_stage_unlock();
    return rc;
}

/* lowbit.c:158-267: Y[me][h] = X[me][k] . W[k][h] through the activation
 * LUT and per-column bit planes, with the sign correction; k % 32 != 0
 * takes the double-accumulated fallback.  Y is left unchanged on failure. */
int jt_lowbit_gemm_lut(const float *X, const float *W, float *Y, int me, int h, int k, int bits) {
    if (X == NULL || W == NULL || Y == NULL || me < 0 || h <= 0 || k <= 0) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    if (bits != 2 && bits != 4) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    if (me == 0) return JT_OK;
    const size_t nx = (size_t)me * (size_t)k, nw = (size_t)k * (size_t)h, ny = (size_t)me * (size_t)h;
    int rc = JT_ERR_CUDA;
    jt_stage_lock();
    cudaStream_t st = jt_stage_stream();
    float *dx = (float *)jt_stage_buf(JT_SLOT_X, nx * sizeof(float));
    float *dw = (float *)jt_stage_buf(JT_SLOT_W1, nw * sizeof(float));
    float *dy = (float *)jt_stage_buf(JT_SLOT_Y, ny * sizeof(float));
    unsigned long long *derr = (unsigned long long *)jt_stage_buf(JT_SLOT_FLAGS, 64);
    unsigned long long keys[2] = {~0ull, ~0ull};
    if (!dx || !dw || !dy || !derr) {
        errno = ENOMEM;
        rc = JT_ERR_NOMEM;
        goto out;
    }
    if (k % TMAC_ACT_GROUP != 0) {
        if (jt_stage_h2d(dx, X, nx * sizeof(float)) || jt_stage_h2d(dw, W, nw * sizeof(float)) ||
            jtk_gemm_f64acc(dx, dw, 0, h, 1, NULL, dy, me, h, k, st) != 0 || jt_stage_d2h(Y, dy, ny * sizeof(float)) ||
            jt_stage_sync()) {
            rc = cuda_fail();
            goto out;
        }
        rc = JT_OK;
        goto out;
    }
    {
        const size_t nb = (size_t)k / TMAC_ACT_GROUP;
        int8_t *dq = (int8_t *)jt_stage_buf(JT_SLOT_A, (size_t)me * nb * 64);
        float *ds = (float *)jt_stage_buf(JT_SLOT_SCALE, (size_t)me * nb * sizeof(float));
        float *dbi = (float *)jt_stage_buf(JT_SLOT_AUX1, (size_t)me * nb * sizeof(float));
        double *drs = (double *)jt_stage_buf(JT_SLOT_AUX2, (size_t)me * sizeof(double));
        double *dmx = (double *)jt_stage_buf(JT_SLOT_AUX3, (size_t)h * sizeof(double));
        void *didx = jt_stage_buf(JT_SLOT_B, (size_t)bits * nb * (size_t)h * 8);
        if (!dq || !ds || !dbi || !drs || !dmx || !didx) {
            errno = ENOMEM;
            rc = JT_ERR_NOMEM;
            goto out;
        }
        if (jt_stage_h2d(dx, X, nx * sizeof(float)) || jt_stage_h2d(dw, W, nw * sizeof(float)) ||
            jtk_tmac_ctor(dx, (size_t)me, (size_t)k, dq, ds, dbi, derr, st) != 0 ||
            jtk_lut_gemm(dx, dw, 1, 0, h, 1, NULL, dq, ds, dbi, dmx, didx, drs, dy, me, h, k, bits, derr + 1, st) != 0 ||
            jt_stage_d2h(keys, derr, sizeof keys) || jt_stage_sync()) {
            rc = cuda_fail();
            goto out;
        }
        if (keys[0] != ~0ull) { /* the activation table failed first */
            rc = tmac_err(keys[0]);
            goto out;
        }
        if (keys[1] != ~0ull) { /* column check (EINVAL) or a lookup total (ERANGE) */
            rc = tmac_err(keys[1]);
            goto out;
        }
        if (jt_stage_d2h(Y, dy, ny * sizeof(float)) || jt_stage_sync()) {
            rc = cuda_fail();
            goto out;
        }
        rc = JT_OK;
    }
out:
    jt_stage_unlock();
    return rc;
}
