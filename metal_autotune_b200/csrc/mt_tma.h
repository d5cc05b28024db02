// Host-side TMA tensor-map construction.
#pragma once
#include <cuda.h>
#include <stdint.h>

namespace mt {

// 2-D tiled tensor map over a row-major matrix of `outer` rows x `inner`
// elements, rows `row_stride_bytes` apart, box of box_outer x box_inner
// elements. Out-of-range box elements read as zero.
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes,
                 uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                 uint32_t box_outer, CUtensorMapSwizzle swizzle);

// Tiled tensor map of `rank` (2..5) dimensions, innermost first: dims[rank],
// byte strides of dimensions 1..rank-1 in strides[rank-1] (any order, each a
// multiple of 16), box[rank] elements. Out-of-range box elements read as zero.
int make_tmap(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes, int rank,
              const uint64_t* dims, const uint64_t* strides, const uint32_t* box, CUtensorMapSwizzle swizzle);

}  // namespace mt
