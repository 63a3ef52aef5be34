// tmap.h -- TMA tensor maps (CUtensorMap) for the tensor-core kernels, encoded
// through the driver entry point so that libcuda is not a link dependency.
#pragma once
#include <cuda.h>
#include <cstdint>

namespace mlpg {

// 2-D row-major map, 128-byte swizzle: `inner` elements per row (contiguous),
// `outer` rows, `row_bytes` between rows, boxes of box_inner x box_outer.
bool make_map(CUtensorMap* m, const void* base, CUtensorMapDataType ty, uint64_t inner, uint64_t outer,
              uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer);

// The same for bytes, without swizzle.
bool make_map_plain(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                    uint32_t box_inner, uint32_t box_outer);

// Packed scale-factor blocks: `rows` rows of 128 x 32-bit, boxes of `cells` rows.
bool make_map_sf(CUtensorMap* m, const void* base, uint64_t rows, uint32_t cells);

}  // namespace mlpg
