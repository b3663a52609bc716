// jt_noalloc.cu - jt_b200_w8a8_linear_noalloc: per-token int8 quantization
// of fp32 activations followed by the W8A8 tensor-core GEMM, with the
// intermediate codes and scales held in a fixed file-scope device array
// instead of caller- or library-allocated memory.  Nothing on this path
// calls cudaMalloc, cudaFree or any allocating library routine.
//
// Arithmetic is exactly that of jt_w8a8_quant_per_channel (w8a8.c:787-855
// per row) feeding jt_b200_w8a8_gemm, so the output is bit-identical to
// those two calls made in sequence.
#include <cuda_runtime.h>
#include <errno.h>
#include <stdint.h>

#include <mutex>

#include "../../include/jimotono_b200.h"
#include "jt_internal.h"
#include "jt_ptx.cuh"

// Scratch: codes [M][K] int8 (row stride K), one fp32 scale per row, and a
// fault flag.  The flag must read zero when a call starts; it is zero at
// module load and the fold kernel below clears it after reporting.
static __device__ __align__(256) int8_t g_nl_codes[JT_B200_LINEAR_NOALLOC_MAX_CODES];
static __device__ __align__(256) float g_nl_scales[JT_B200_LINEAR_NOALLOC_MAX_ROWS];
static __device__ __align__(256) int g_nl_bad;

namespace {

struct Scratch {
    int8_t *codes;
    float *scales;
    int *bad;
};

std::mutex g_mu;
Scratch g_cache[64];

// Device addresses of the scratch symbols for the current device, looked
// up once per device with that device current.
int scratch_for_current_device(Scratch *out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
    std::lock_guard<std::mutex> lk(g_mu);
    Scratch &s = g_cache[dev];
    if (s.codes == nullptr) {
        void *c = nullptr, *sc = nullptr, *b = nullptr;
        if (cudaGetSymbolAddress(&c, g_nl_codes) != cudaSuccess ||
            cudaGetSymbolAddress(&sc, g_nl_scales) != cudaSuccess ||
            cudaGetSymbolAddress(&b, g_nl_bad) != cudaSuccess)
            return -1;
        s.codes = static_cast<int8_t *>(c);
        s.scales = static_cast<float *>(sc);
        s.bad = static_cast<int *>(b);
    }
    *out = s;
    return 0;
}

// Row scales start every call as NaN: the quantizer overwrites the scale of
// each row it accepts and leaves a row with a non-finite activation (or a
// scale that underflows) alone, so that row of C comes out NaN in every
// column instead of carrying an earlier call's codes.
__global__ void k_nl_begin(float *scales, int M) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < M) scales[i] = __int_as_float(0x7fc00000);
}

// A non-finite activation or a scale underflow found by the quantizer is
// moved into the library's error word (reported by jt_b200_sync) and the
// flag is reset for the next call.
__global__ void k_nl_fold(int *bad, int *err_word) {
    const int v = *bad;
    if (v != 0) {
        if (err_word) atomicExch(err_word, JT_KERR_NONFINITE);
        *bad = 0;
    }
}

}  // namespace

extern "C" int jt_b200_w8a8_linear_noalloc(const float *x, int M, int K, const int8_t *W,
                                           int ldw, const float *sw, float *C, int ldc, int N,
                                           void *stream) {
    if (M == 0) return JT_OK;
    if (x == nullptr || W == nullptr || sw == nullptr || C == nullptr || M < 0 || N <= 0 ||
        K <= 0 || K % 16 != 0 || ldw < K || ldw % 16 != 0 || ldc < N) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    if (M > JT_B200_LINEAR_NOALLOC_MAX_ROWS ||
        (long long)M * K > (long long)JT_B200_LINEAR_NOALLOC_MAX_CODES) {
        errno = E2BIG;
        return JT_ERR_INVAL;
    }
    // The tensor map of W needs a 16-byte aligned base; the fp32 operands
    // are read and written as whole floats.
    if ((reinterpret_cast<uintptr_t>(W) & 15u) != 0 || (reinterpret_cast<uintptr_t>(x) & 3u) != 0 ||
        (reinterpret_cast<uintptr_t>(sw) & 3u) != 0 || (reinterpret_cast<uintptr_t>(C) & 3u) != 0) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    Scratch s;
    if (scratch_for_current_device(&s) != 0) {
        errno = EIO;
        return JT_ERR_CUDA;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    k_nl_begin<<<(M + 255) / 256, 256, 0, st>>>(s.scales, M);
    if (cudaGetLastError() != cudaSuccess) {
        errno = EIO;
        return JT_ERR_CUDA;
    }
    int r = jtk_quant_blocks(x, M, K, K, 0, s.codes, s.scales, nullptr, s.bad, st);
    if (r == 0) {
        r = jtk_w8a8_gemm(s.codes, K, W, ldw, M, N, K, s.scales, sw, 0.0, C, ldc,
                          JTK_EPI_TOKEN_CHANNEL_F32, st);
        // The quantizer ran: whatever happened to the GEMM, its fault flag
        // is folded into the error word and cleared for the next call.
        k_nl_fold<<<1, 1, 0, st>>>(s.bad, jtk_error_word());
        if (cudaGetLastError() != cudaSuccess && r == 0) r = -4;
    }
    if (r == -1) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    if (r != 0) {
        errno = EIO;
        return JT_ERR_CUDA;
    }
    return JT_OK;
}
