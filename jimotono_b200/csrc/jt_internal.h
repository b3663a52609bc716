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

/* Epilogue modes of the dense int8 tensor-core GEMM. */
enum jtk_w8a8_epi {
    JTK_EPI_TOKEN_CHANNEL_F32 = 0, /* C = ((float)acc * sx[m]) * sw[n] */
    JTK_EPI_TENSOR_CHANNEL_F64 = 1, /* C = (float)((double)acc * ((double)sA * sw[n])) */
    JTK_EPI_RAW_I32 = 2            /* C = acc (int32) */
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

/* Device error word shared by all kernels of the library (0 = clean). */
int jtk_read_and_clear_error(int *out_code);
int *jtk_error_word(void);

/* Number of SMs of the current device (cached). */
int jtk_num_sms(void);

#ifdef __cplusplus
}
#endif

#endif
