// jt_runtime.cu - process-wide device helpers: the library's device error
// word, the SM count cache and TMA tensor-map encoding through the driver
// entry point (so the library does not link libcuda at build time).
#include <cuda.h>
#include <cuda_runtime.h>
#include <mutex>

#include "jt_internal.h"
#include "jt_runtime.cuh"

// One error word per device for every kernel in the library.  Kernels only
// ever write a non-zero code into it (atomicExch); the host reads and clears.
__device__ int g_jt_err_word;

namespace {
typedef CUresult (*PFN_encodeTiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                    const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                    const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
PFN_encodeTiled g_encode = nullptr;
std::once_flag g_encode_once;

void load_encode() {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
        g_encode = reinterpret_cast<PFN_encodeTiled>(fn);
    }
}
}  // namespace

namespace jt {

bool make_tmap_2d_u8(CUtensorMap *map, const void *base, uint64_t inner, uint64_t rows,
                     uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows,
                     bool swizzle128) {
    std::call_once(g_encode_once, load_encode);
    if (!g_encode) return false;
    if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (row_stride_bytes & 15u) != 0)
        return false;
    cuuint64_t gdim[2] = {inner, rows};
    cuuint64_t gstride[1] = {row_stride_bytes};
    cuuint32_t box[2] = {box_inner, box_rows};
    cuuint32_t estride[2] = {1, 1};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), gdim,
                          gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

}  // namespace jt

// Device address of the error word, looked up once per device (the host
// symbol g_jt_err_word is not a device address; cudaGetSymbolAddress is).
extern "C" int *jtk_error_word(void) {
    static int *cache[64] = {nullptr};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return nullptr;
    if (dev < 64 && cache[dev]) return cache[dev];
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_jt_err_word) != cudaSuccess) return nullptr;
    if (dev < 64) cache[dev] = static_cast<int *>(p);
    return static_cast<int *>(p);
}

extern "C" int jtk_read_and_clear_error(int *out_code) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_jt_err_word, sizeof(int)) != cudaSuccess) return -1;
    if (v != 0) {
        int z = 0;
        if (cudaMemcpyToSymbol(g_jt_err_word, &z, sizeof(int)) != cudaSuccess) return -1;
    }
    if (out_code) *out_code = v;
    return 0;
}

extern "C" int jtk_num_sms(void) {
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (dev >= 0 && dev < 64 && cache[dev]) return cache[dev];
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
        return 148;
    if (dev >= 0 && dev < 64) cache[dev] = n;
    return n;
}
