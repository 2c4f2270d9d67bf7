// Tensor-map encoding shared by the TMA kernels (host side).
#pragma once

#include <cuda.h>

namespace m3b {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled from the driver the runtime is bound to (null when unavailable).
EncodeTiledFn encode_tiled();

}  // namespace m3b
