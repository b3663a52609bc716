/* jt_api_w8a8.c - reference-compatible W8A8 entry points (host pointers)
 * and the jt_b200_* device W8A8 entry points.
 *
 * Validation mirrors the reference step by step so the same inputs give
 * the same return code and errno; compute always runs on the GPU; outputs
 * are written to the caller's buffer only after the device result has been
 * checked (fail-closed: an INVAL return leaves every output untouched). */
#include <errno.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "../../include/jimotono_b200.h"
#include "jt_internal.h"
#include "jt_stage.h"

static int g_w8a8_enabled = 0; /* w8a8.c:53 */

int jt_w8a8_set_enabled(int enabled) {
    if (enabled != 0 && enabled != 1) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    g_w8a8_enabled = enabled;
    return JT_OK;
}

int jt_w8a8_get_enabled(int *out_enabled) {
    if (out_enabled == NULL) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    *out_enabled = g_w8a8_enabled;
    return JT_OK;
}

int jt_w8a8_is_enabled(void) { return g_w8a8_enabled; }

/* ---------------------------------------------------------------- quant */

/* Shared body of quant / fake-quant per-tensor (one row) and per-channel
 * (rows x cols).  mode 0 writes codes + scales, mode 1 fake-quant floats. */
static int quant_common(const float *src, size_t rows, size_t cols, int per_tensor, int mode,
                        int8_t *dst_q, float *dst_scales, float *dst_fq) {
    const size_t n = rows * cols;
    int rc = JT_ERR_INVAL;
    jt_stage_lock();
    float *dx = (float *)jt_stage_buf(JT_SLOT_X, n * sizeof(float));
    int8_t *dq = (int8_t *)jt_stage_buf(JT_SLOT_A, mode == 0 ? n : 16);
    float *dfq = (float *)jt_stage_buf(JT_SLOT_Y, mode == 1 ? n * sizeof(float) : 16);
    float *ds = (float *)jt_stage_buf(JT_SLOT_SCALE, rows * sizeof(float) + 16);
    int *dflag = (int *)jt_stage_buf(JT_SLOT_FLAGS, 64);
    cudaStream_t st = jt_stage_stream();
    if (!dx || !dq || !dfq || !ds || !dflag) {
        errno = ENOMEM;
        rc = JT_ERR_NOMEM;
        goto out;
    }
    if (cudaMemsetAsync(dflag, 0, 64, st) != cudaSuccess || jt_stage_h2d(dx, src, n * sizeof(float)))
        goto cuda_fail;
    if (per_tensor && n > 65536) {
        if (jtk_quant_tensor(dx, n, mode, dq, ds, dfq, (unsigned *)(dflag + 4), dflag, st) != 0)
            goto cuda_fail;
    } else {
        if (jtk_quant_blocks(dx, (int)rows, (int)cols, (int)cols, mode, dq, ds, dfq, dflag, st) != 0)
            goto cuda_fail;
    }
    int flag = 0;
    if (jt_stage_d2h(&flag, dflag, sizeof(int)) || jt_stage_sync()) goto cuda_fail;
    if (flag == 1) {
        errno = EINVAL; /* non-finite input (w8a8.c:703-709) */
        goto out;
    }
    if (flag == 2) {
        errno = ERANGE; /* scale out of float range (w8a8.c:725-733) */
        goto out;
    }
    if (mode == 0) {
        if (jt_stage_d2h(dst_q, dq, n) || jt_stage_d2h(dst_scales, ds, rows * sizeof(float)))
            goto cuda_fail;
    } else {
        if (jt_stage_d2h(dst_fq, dfq, n * sizeof(float))) goto cuda_fail;
    }
    if (jt_stage_sync()) goto cuda_fail;
    rc = JT_OK;
    goto out;
cuda_fail:
    errno = EIO;
    rc = JT_ERR_CUDA;
out:
    jt_stage_unlock();
    return rc;
}

int jt_w8a8_quant_per_tensor(const float *src, size_t n, int8_t *dst, float *out_scale) {
    if (src == NULL || dst == NULL || out_scale == NULL || n == 0) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    return quant_common(src, 1, n, 1, 0, dst, out_scale, NULL);
}

int jt_w8a8_quant_per_channel(const float *src, size_t rows, size_t cols, int8_t *dst,
                              float *scales) {
    if (src == NULL || dst == NULL || scales == NULL || rows == 0 || cols == 0 ||
        rows > SIZE_MAX / cols || cols > 0x7fffffffu || rows > 0x7fffffffu) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    return quant_common(src, rows, cols, 0, 0, dst, scales, NULL);
}

int jt_w8a8_fakequant_per_tensor(const float *src, size_t n, float *dst) {
    if (src == NULL || dst == NULL || n == 0) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    return quant_common(src, 1, n, 1, 1, NULL, NULL, dst);
}

int jt_w8a8_fakequant_per_channel(const float *src, size_t rows, size_t cols, float *dst) {
    if (src == NULL || dst == NULL || rows == 0 || cols == 0 || rows > SIZE_MAX / cols ||
        cols > 0x7fffffffu || rows > 0x7fffffffu) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    return quant_common(src, rows, cols, 0, 1, NULL, NULL, dst);
}

/* ---------------------------------------------------------------- dequant */

static int dequant_common(const int8_t *src, const float *scales, size_t rows, size_t cols,
                          float *dst) {
    const size_t n = rows * cols;
    int rc = JT_ERR_INVAL;
    jt_stage_lock();
    int8_t *dq = (int8_t *)jt_stage_buf(JT_SLOT_A, n);
    float *ds = (float *)jt_stage_buf(JT_SLOT_SCALE, rows * sizeof(float));
    float *dy = (float *)jt_stage_buf(JT_SLOT_Y, n * sizeof(float));
    int *dflag = (int *)jt_stage_buf(JT_SLOT_FLAGS, 64);
    cudaStream_t st = jt_stage_stream();
    int flag = 0;
    if (!dq || !ds || !dy || !dflag) {
        errno = ENOMEM;
        rc = JT_ERR_NOMEM;
        goto out;
    }
    if (cudaMemsetAsync(dflag, 0, 64, st) != cudaSuccess || jt_stage_h2d(dq, src, n) ||
        jt_stage_h2d(ds, scales, rows * sizeof(float)))
        goto cuda_fail;
    if (jtk_dequant_rows(dq, ds, rows, cols, dy, dflag, st) != 0) goto cuda_fail;
    if (jt_stage_d2h(&flag, dflag, sizeof(int)) || jt_stage_sync()) goto cuda_fail;
    if (flag == 1) {
        errno = EINVAL; /* q == -128 (w8a8.c:765-772) */
        goto out;
    }
    if (flag == 2) {
        errno = ERANGE; /* non-finite result (w8a8.c:776-780) */
        goto out;
    }
    if (jt_stage_d2h(dst, dy, n * sizeof(float)) || jt_stage_sync()) goto cuda_fail;
    rc = JT_OK;
    goto out;
cuda_fail:
    errno = EIO;
    rc = JT_ERR_CUDA;
out:
    jt_stage_unlock();
    return rc;
}

int jt_w8a8_dequant_per_tensor(const int8_t *src, float scale, size_t n, float *dst) {
    if (src == NULL || dst == NULL || n == 0) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    if (!isfinite((double)scale) || (double)scale <= 0.0) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    return dequant_common(src, &scale, 1, n, dst);
}

int jt_w8a8_dequant_per_channel(const int8_t *src, const float *scales, size_t rows,
                                size_t cols, float *dst) {
    if (src == NULL || scales == NULL || dst == NULL || rows == 0 || cols == 0 ||
        rows > SIZE_MAX / cols) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    for (size_t r = 0; r < rows; r++) {
        if (!isfinite((double)scales[r]) || (double)scales[r] <= 0.0) {
            errno = EINVAL;
            return JT_ERR_INVAL;
        }
    }
    return dequant_common(src, scales, rows, cols, dst);
}

/* ---------------------------------------------------------------- GEMM */

/* Validation of w8a8.c:910-953 (NULL, dims, 4096 cap, sA, sB_col). */
static int gemm_validate(const int8_t *Aq, const int8_t *Bq, float sA, const float *sB_col,
                         const float *C, int M, int N, int K, int need_col) {
    if (Aq == NULL || Bq == NULL || C == NULL) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    if (M < 0 || N <= 0 || K <= 0) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    if (M > JT_BWD_MAX_WIDE || N > JT_BWD_MAX_WIDE || K > JT_BWD_MAX_WIDE) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    if (!isfinite((double)sA) || sA <= 0.0f) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    if (need_col) {
        if (sB_col == NULL) {
            errno = EINVAL;
            return JT_ERR_INVAL;
        }
        for (int n = 0; n < N; n++) {
            if (!isfinite((double)sB_col[n]) || sB_col[n] <= 0.0f) {
                errno = EINVAL;
                return JT_ERR_INVAL;
            }
        }
    }
    return JT_OK;
}

/* Stage Aq [M][K] and Bq [K][N] to the device, transpose B to [N][Kp],
 * run the fp64-epilogue tensor-core GEMM, check the -128 range and the
 * finiteness of the result on the device, then commit C. */
static int gemm_run(const int8_t *Aq, const int8_t *Bq, float sA, const float *sB_col,
                    float sB_single, float *C, int M, int N, int K) {
    const int Kp = (K + 15) & ~15;
    int rc = JT_ERR_INVAL;
    jt_stage_lock();
    cudaStream_t st = jt_stage_stream();
    int8_t *dA = (int8_t *)jt_stage_buf(JT_SLOT_A, (size_t)M * K);
    int8_t *dAp = (int8_t *)jt_stage_buf(JT_SLOT_A2, (size_t)M * Kp);
    int8_t *dB = (int8_t *)jt_stage_buf(JT_SLOT_B, (size_t)K * N);
    int8_t *dW = (int8_t *)jt_stage_buf(JT_SLOT_B2, (size_t)N * Kp);
    float *dS = (float *)jt_stage_buf(JT_SLOT_SCALE, (size_t)N * sizeof(float));
    float *dC = (float *)jt_stage_buf(JT_SLOT_C, (size_t)M * N * sizeof(float));
    int *dflag = (int *)jt_stage_buf(JT_SLOT_FLAGS, 64);
    int flags[2] = {0, 0};
    if (!dA || !dAp || !dB || !dW || !dS || !dC || !dflag) {
        errno = ENOMEM;
        rc = JT_ERR_NOMEM;
        goto out;
    }
    if (cudaMemsetAsync(dflag, 0, 64, st) != cudaSuccess) goto cuda_fail;
    if (jt_stage_h2d(dA, Aq, (size_t)M * K) || jt_stage_h2d(dB, Bq, (size_t)K * N)) goto cuda_fail;
    if (sB_col) {
        if (jt_stage_h2d(dS, sB_col, (size_t)N * sizeof(float))) goto cuda_fail;
    } else {
        /* per-tensor: every column carries sB (w8a8.c:1007 ss = sA*sB) */
        static float fill[JT_BWD_MAX_WIDE];
        for (int n = 0; n < N; n++) fill[n] = sB_single;
        if (jt_stage_h2d(dS, fill, (size_t)N * sizeof(float)) || jt_stage_sync()) goto cuda_fail;
    }
    const int8_t *dX = dA;
    if (Kp != K) {
        if (jtk_pad_rows_s8(dA, M, K, dAp, Kp, dflag, st)) goto cuda_fail;
        dX = dAp;
    } else {
        if (jtk_check_s8(dA, (size_t)M * K, dflag, st)) goto cuda_fail;
    }
    if (jtk_transpose_s8(dB, K, N, dW, Kp, dflag, st)) goto cuda_fail;
    if (jtk_w8a8_gemm(dX, Kp, dW, Kp, M, N, Kp, NULL, dS, (double)sA, dC, N,
                      JTK_EPI_TENSOR_CHANNEL_F64, st))
        goto cuda_fail;
    if (jtk_check_finite_f32(dC, (size_t)M * N, dflag + 1, st)) goto cuda_fail;
    if (jt_stage_d2h(flags, dflag, sizeof(flags)) || jt_stage_sync()) goto cuda_fail;
    if (flags[0]) {
        errno = EINVAL; /* q == -128 (w8a8.c:1041-1060) */
        goto out;
    }
    if (flags[1]) {
        errno = ERANGE; /* non-finite output (w8a8.c:676-681) */
        goto out;
    }
    if (jt_stage_d2h(C, dC, (size_t)M * N * sizeof(float)) || jt_stage_sync()) goto cuda_fail;
    rc = JT_OK;
    goto out;
cuda_fail:
    errno = EIO;
    rc = JT_ERR_CUDA;
out:
    jt_stage_unlock();
    return rc;
}

int jt_w8a8_gemm_per_tensor(const int8_t *Aq, const int8_t *Bq, float sA, float sB, float *C,
                            int M, int N, int K) {
    if (M == 0) { /* w8a8.c:959-971 */
        if (Aq == NULL || Bq == NULL || C == NULL || N <= 0 || K <= 0) {
            errno = EINVAL;
            return JT_ERR_INVAL;
        }
        return JT_OK;
    }
    if (gemm_validate(Aq, Bq, sA, NULL, C, M, N, K, 0) != JT_OK) return JT_ERR_INVAL;
    if (!isfinite((double)sB) || sB <= 0.0f) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    {
        double ss = (double)sA * (double)sB;
        if (!isfinite(ss) || ss <= 0.0) {
            errno = ERANGE;
            return JT_ERR_INVAL;
        }
    }
    return gemm_run(Aq, Bq, sA, NULL, sB, C, M, N, K);
}

int jt_w8a8_gemm_per_channel(const int8_t *Aq, const int8_t *Bq, float sA, const float *sB_col,
                             float *C, int M, int N, int K) {
    if (M == 0) { /* w8a8.c:1025-1037 */
        if (Aq == NULL || Bq == NULL || C == NULL || N <= 0 || K <= 0) {
            errno = EINVAL;
            return JT_ERR_INVAL;
        }
        return JT_OK;
    }
    if (gemm_validate(Aq, Bq, sA, sB_col, C, M, N, K, 1) != JT_OK) return JT_ERR_INVAL;
    for (int n = 0; n < N; n++) { /* per-column ss check (w8a8.c:664-669) */
        double ss = (double)sA * (double)sB_col[n];
        if (!isfinite(ss) || ss <= 0.0) {
            errno = ERANGE;
            return JT_ERR_INVAL;
        }
    }
    return gemm_run(Aq, Bq, sA, sB_col, 1.0f, C, M, N, K);
}

/* ---------------------------------------------------------------- device API */

static int map_launch(int r) {
    if (r == 0) return JT_OK;
    if (r == -1) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    errno = EIO;
    return JT_ERR_CUDA;
}

int jt_b200_w8a8_gemm(const int8_t *X, int ldx, const float *sx, const int8_t *W, int ldw,
                      const float *sw, float *C, int ldc, int M, int N, int K, void *stream) {
    if (M == 0) return JT_OK;
    if (X == NULL || sx == NULL || W == NULL || sw == NULL || C == NULL) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    return map_launch(jtk_w8a8_gemm(X, ldx, W, ldw, M, N, K, sx, sw, 0.0, C, ldc,
                                    JTK_EPI_TOKEN_CHANNEL_F32, (cudaStream_t)stream));
}

int jt_b200_w8a8_gemm_i32(const int8_t *X, int ldx, const int8_t *W, int ldw, int32_t *C32,
                          int ldc, int M, int N, int K, void *stream) {
    if (M == 0) return JT_OK;
    if (X == NULL || W == NULL || C32 == NULL) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    return map_launch(jtk_w8a8_gemm(X, ldx, W, ldw, M, N, K, NULL, NULL, 0.0, C32, ldc,
                                    JTK_EPI_RAW_I32, (cudaStream_t)stream));
}

int jt_b200_lowbit_gemv(const int8_t *a, float sa, const uint8_t *w2, const uint16_t *s2, int n2,
                        const uint8_t *w4, const uint16_t *s4, int n4, int K, float *y,
                        void *stream) {
    if (a == NULL || y == NULL || n2 < 0 || n4 < 0 || K <= 0 || K % 64 != 0 || K > 4096 ||
        !isfinite(sa) || (n2 > 0 && (w2 == NULL || s2 == NULL)) ||
        (n4 > 0 && (w4 == NULL || s4 == NULL)) || ((uintptr_t)w2 & 15u) != 0 ||
        ((uintptr_t)w4 & 15u) != 0 || ((uintptr_t)a & 15u) != 0) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    if (n2 + n4 == 0) return JT_OK;
    return map_launch(jtk_lowbit_gemv(a, sa, w2, s2, n2, w4, s4, n4, K, y, (cudaStream_t)stream));
}

int jt_b200_lowbit_pack(const float *W, int rows, int K, int bits, int n_ch, uint8_t *packed,
                        uint16_t *scales, void *stream) {
    if (W == NULL || packed == NULL || scales == NULL || rows <= 0 || K <= 0 || K % 64 != 0 ||
        (bits != 2 && bits != 4) || n_ch < 0 || (n_ch > 0 && rows % n_ch != 0) ||
        ((uintptr_t)W & 7u) != 0) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    return map_launch(jtk_pack_lowbit(W, rows, K, bits, n_ch, packed, scales, (cudaStream_t)stream));
}

int jt_b200_lowbit_planes_to_packed(const uint8_t *idx, const float *w_scale, int cols, int K,
                                    int bits, int n_ch, uint8_t *packed, uint16_t *scales,
                                    void *stream) {
    if (idx == NULL || packed == NULL || cols <= 0 || K <= 0 || K % 64 != 0 ||
        (bits != 2 && bits != 4) || n_ch < 0 || (n_ch > 0 && cols % n_ch != 0) ||
        ((w_scale == NULL) != (scales == NULL))) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    return map_launch(jtk_planes_to_packed(idx, w_scale, cols, K, bits, n_ch, packed, scales,
                                           (cudaStream_t)stream));
}

int jt_b200_sync(void) {
    if (cudaDeviceSynchronize() != cudaSuccess) {
        errno = EIO;
        return JT_ERR_CUDA;
    }
    int code = 0;
    if (jtk_read_and_clear_error(&code) != 0 || code != 0) {
        errno = EIO;
        return JT_ERR_CUDA;
    }
    return JT_OK;
}

const char *jt_b200_version(void) { return "jimotono_b200 0.1.0 (sm_100a)"; }
