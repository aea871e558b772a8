// tmap.cuh -- host-side creation of TMA tensor maps (CUtensorMap) without linking libcuda:
// the driver's cuTensorMapEncodeTiled is fetched once through the runtime's entry-point
// query.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace k3 {

// 2-D row-major tensor [outer][inner] of `elem_bytes` elements with `row_bytes` between
// rows; box [box_outer][box_inner]; 128-byte swizzle when box_inner * elem_bytes == 128.
// Returns K3CUDA_OK or an error code with the message set.
int make_tmap_2d(CUtensorMap *map, const void *base, CUtensorMapDataType dtype,
                 uint32_t elem_bytes, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                 uint32_t box_inner, uint32_t box_outer);

// 3-D tensor [d2][d1][d0] with byte strides s1 (between d1 rows) and s2 (between d2 planes);
// box [b2][b1][b0], 128-byte swizzle.
int make_tmap_3d(CUtensorMap *map, const void *base, CUtensorMapDataType dtype,
                 uint32_t elem_bytes, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1,
                 uint64_t s2, uint32_t b0, uint32_t b1, uint32_t b2);

}  // namespace k3
