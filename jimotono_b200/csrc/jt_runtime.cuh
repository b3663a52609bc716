// jt_runtime.cuh - C++-side helpers shared by the CUDA translation units.
#pragma once
#include <cuda.h>
#include <cstdint>

// Kernels receive the device error word as a pointer argument (obtained with
// jtk_error_word()), so no translation unit needs relocatable device code.

namespace jt {

// Encode a 2-D uint8 tiled tensor map: `inner` bytes per row (innermost),
// `rows` rows, row stride in bytes, box of box_inner x box_rows.  Returns
// false when the driver entry point is missing or the encode is rejected.
bool make_tmap_2d_u8(CUtensorMap *map, const void *base, uint64_t inner, uint64_t rows,
                     uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows,
                     bool swizzle128);

}  // namespace jt
