// rk_tma.h — host-side TMA tensor maps (cuTensorMapEncodeTiled through the
// runtime's driver entry point, so the library does not link libcuda).
#pragma once
#include <cstdint>
#include <cuda.h>

namespace rk {

// A row-major 2-D array of `outer` rows of `inner` elements, `row_bytes`
// apart, read in (box_inner × box_outer) tiles; elements outside the array
// read as zero. swizzle128: the 128-byte swizzle (rows of the box must then
// be 128 bytes). Returns false when the driver refuses the map or has no
// encoder.
bool tmap_2d(CUtensorMap *map, CUtensorMapDataType dtype, const void *ptr, uint64_t inner, uint64_t outer,
             uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, bool swizzle128);

// Whether the driver exposes the tensor-map encoder.
bool tmap_available();

}  // namespace rk
