// Tensor-map encoding for the TMA kernels (host side): cuTensorMapEncodeTiled, looked up once through the runtime's
// driver entry point so that the library links the CUDA runtime only.
#pragma once
#include <cudaTypedefs.h>

#include "common.h"

namespace evie {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
// The driver's cuTensorMapEncodeTiled, or nullptr when the driver does not provide it (errors.cpp).
EncodeTiledFn encode_tiled();

}  // namespace evie
