// capi_noalloc.cu -- backward entry point that needs no caller-provided workspace.
//
// kata_attn_bwd needs a few MB of device scratch (per-query delta = <o, dO>, 1/den and
// delta/den), which its caller normally allocates and passes in.  Some callers cannot allocate:
// host code running under a fixed, pre-reserved device-memory budget that forbids any further
// cudaMalloc once the model is loaded, or a plugin host whose operator interface hands the
// kernel only its input and output buffers and offers no workspace.  For them this file holds
// the scratch in a file-scope device array, sized once for every GPU that loads the library,
// and kata_attn_bwd_noalloc runs the same backward on it.
//
// Properties a caller must know:
//  * capacity: kNoAllocScratchBytes (16 MiB) per device; larger problems are rejected with
//    KATA_ERR_SCRATCH_LIMIT (kata_attn_bwd_workspace_bytes() with algo TC or SIMT tells the
//    requirement; with AUTO, the Gram form of the sum score runs when its larger workspace fits);
//  * the array lives until the process exits, on every device that loads this library;
//  * set-up: the first call on a device resolves the array's device address for that device
//    (cudaGetSymbolAddress, with that device current); make that first call outside any stream
//    capture;
//  * all calls on a device share one array: two calls whose kernels overlap on the GPU (e.g. on
//    different streams without ordering) race on it.  Nothing in it has to start at zero: the
//    dq pass writes every entry the dk/dv pass later reads, and the array keeps whatever the
//    last call left there;
//  * only the full backward (phases == 0) is accepted.  A dk/dv-only call (phases == 2) would
//    read what the last call on the device left in the shared array, possibly another
//    problem's, so it is rejected with KATA_ERR_INVALID, as is the dq-only pass (phases == 1)
//    that would exist only to feed it;
//  * the address is resolved once per device ordinal and kept for the life of the process: a
//    caller that resets the device (cudaDeviceReset) or switches that ordinal to another
//    context must not call this entry point afterwards;
//  * no cudaMalloc, cudaFree or any other allocating routine is called on this path.
#include <mutex>

#include "attn_common.cuh"
#include "attn_internal.h"
#include "host_util.h"

namespace kata {

// 16 MiB of fp32 scratch, 256-byte aligned.  Enough for B*T*HQ up to ~1.3 M query rows, e.g.
// config 3 (B=16, T=4096, HQ=8) needs 6.3 MB.
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
static __device__ __align__(256) float g_bwd_scratch[kNoAllocScratchBytes / sizeof(float)];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_bwd_scratch on the current device (resolved once per device).
int scratch_address(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return KATA_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return KATA_ERR_INVALID;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_bwd_scratch) != cudaSuccess || !p) return KATA_ERR_CUDA;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return KATA_OK;
}

}  // namespace
}  // namespace kata

extern "C" int kata_attn_bwd_noalloc(const kata_attn_bwd_args* args, kata_stream_t stream) {
  if (!args) return KATA_ERR_INVALID;
  if (args->phases != 0) return KATA_ERR_INVALID;
  // AUTO runs the Gram form of the sum score only when it fits in the array, the parts form otherwise
  const size_t need = kata::attn_bwd_min_workspace_bytes(args);
  if (need > kata::kNoAllocScratchBytes) return KATA_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  const int e = kata::scratch_address(&scratch);
  if (e) return e;
  kata_attn_bwd_args a = *args;
  a.workspace = scratch;
  a.workspace_bytes = kata::kNoAllocScratchBytes;
  return kata_attn_bwd(&a, stream);
}
