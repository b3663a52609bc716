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

/* Synchronize the current device and fold any kernel-reported fault into
 * the return code (JT_OK or JT_ERR_CUDA). */
int jt_b200_sync(void);

/* Library version string. */
const char *jt_b200_version(void);

#ifdef __cplusplus
}
#endif

#endif /* JIMOTONO_B200_H */
