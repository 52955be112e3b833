// hakm_tmap.h — host-side tensor maps for the tiled bulk copies
// (cp.async.bulk.tensor) of the batched matmuls.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdint>

namespace hakm {

// 2-D tiled tensor map: d0 elements of `type` per row (innermost), d1 rows
// stride1 bytes apart, boxes of b0 x b1; out-of-range elements read as zero.
// False when the driver's encoder is unavailable or rejects the shape
// (e.g. a base or stride that is not 16-byte aligned).
bool encode_tmap_2d(CUtensorMap* m, CUtensorMapDataType type, const void* base, uint64_t d0, uint64_t d1,
                    uint64_t stride1, uint32_t b0, uint32_t b1,
                    CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_NONE);

}  // namespace hakm
