// Host-side TMA descriptor encoding (cuTensorMapEncodeTiled, reached through
// the runtime's driver entry point so the library needs no libcuda link).
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace ddpm {

// Tiled descriptor over `base`: `dims` and `box` innermost first, `strides`
// in bytes for dimensions 1 .. rank-1, unit element strides, zero fill out of
// bounds. Returns DDPM_OK, or an error code with a message when the driver
// rejects the description (callers fall back to their non-TMA path).
int encode_tmap(CUtensorMap* map, CUtensorMapDataType type, int rank, const void* base,
                const uint64_t* dims, const uint64_t* strides, const uint32_t* box,
                CUtensorMapSwizzle swizzle);

}  // namespace ddpm
