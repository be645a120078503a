// Host-side TMA tensor-map encoding through the driver entry point (no link
// against libcuda; the runtime hands out cuTensorMapEncodeTiled).
#pragma once

#include <cuda.h>

#include "opl_common.cuh"

namespace opl {

// Encodes a tiled tensor map of `rank` (2 or 3) dimensions.  dims[0] is the
// innermost (contiguous) extent; strides_bytes[i] is the byte stride of
// dimension i+1 (must be a multiple of 16).  Out-of-bounds elements read as
// zero.  Returns cudaErrorInvalidValue when the driver rejects the map.
cudaError_t encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank,
                        const void* base, const uint64_t* dims,
                        const uint64_t* strides_bytes, const uint32_t* box,
                        CUtensorMapSwizzle swizzle);

}  // namespace opl
