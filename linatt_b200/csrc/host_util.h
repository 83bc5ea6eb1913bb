// host_util.h -- host-side helpers shared by the C-ABI entry points: TMA tensor-map encoding
// through the driver entry point (no link-time dependency on libcuda), and error plumbing.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kata_b200.h"

namespace kata {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// Resolved once per process; returns null when the driver does not expose the symbol.
EncodeTiledFn get_encode_tiled();

inline CUtensorMapSwizzle swizzle_enum(int bytes) {
  return bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
         : bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
         : bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                       : CU_TENSOR_MAP_SWIZZLE_NONE;
}

// Encode a tiled map for a 16-bit tensor of rank <= 5.  dims/strides are innermost first;
// strides are in bytes for dims 1..rank-1.  Returns a KATA_ERR_* code.
int encode_tmap_16bit(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                      const uint64_t* strides_bytes, const uint32_t* box, int swizzle_bytes);

inline int from_cuda(cudaError_t e) { return e == cudaSuccess ? KATA_OK : KATA_ERR_CUDA; }

}  // namespace kata
