// host_util.cu -- tensor-map encoding through the driver entry point, error strings.
#include <mutex>

#include "host_util.h"

namespace kata {

EncodeTiledFn get_encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  });
  return fn;
}

int encode_tmap_16bit(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                      const uint64_t* strides_bytes, const uint32_t* box, int swizzle_bytes) {
  EncodeTiledFn enc = get_encode_tiled();
  if (!enc) return KATA_ERR_DRIVER;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return KATA_ERR_ALIGN;
  // The encoder is a driver-API call and needs a current context on this thread.  A thread that
  // has made no CUDA runtime call yet (e.g. a framework's autograd worker whose buffers came from
  // a cache) has none, and the encoder then fails with CUDA_ERROR_INVALID_CONTEXT; setting the
  // current device binds that device's primary context to the thread.
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaSetDevice(dev) != cudaSuccess) return KATA_ERR_CUDA;
  cuuint64_t gdim[5];
  cuuint64_t gstr[4];
  cuuint32_t bdim[5];
  cuuint32_t estr[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estr[i] = 1;
    if (i > 0) {
      if (strides_bytes[i - 1] % 16 != 0) return KATA_ERR_ALIGN;
      gstr[i - 1] = strides_bytes[i - 1];
    }
  }
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, static_cast<cuuint32_t>(rank), const_cast<void*>(base),
                   gdim, gstr, bdim, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_enum(swizzle_bytes),
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? KATA_OK : KATA_ERR_SHAPE;
}

}  // namespace kata

extern "C" const char* kata_strerror(int code) {
  switch (code) {
    case KATA_OK: return "ok";
    case KATA_ERR_INVALID: return "invalid argument (null pointer or inconsistent sizes)";
    case KATA_ERR_DTYPE: return "unsupported dtype";
    case KATA_ERR_SHAPE: return "unsupported or inconsistent shape";
    case KATA_ERR_ALIGN: return "pointer or stride not 16-byte aligned";
    case KATA_ERR_WORKSPACE: return "workspace missing or too small";
    case KATA_ERR_CUDA: return "CUDA runtime error";
    case KATA_ERR_DRIVER: return "driver entry point cuTensorMapEncodeTiled unavailable";
    case KATA_ERR_UNSUPPORTED: return "algorithm not available for this configuration";
    case KATA_ERR_SCRATCH_LIMIT: return "problem needs more scratch than the library's fixed 16 MiB array";
    default: return "unknown error";
  }
}

extern "C" int kata_abi_version(void) { return KATA_ABI_VERSION; }
