// attn_common.cuh -- parameter blocks and small helpers shared by the attention kernels.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace kata {

template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <>
__device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

// Forward problem description (time-major contiguous tensors).
struct AttnFwdParams {
  const void* q;
  const void* k;
  const void* v;
  const float* c;
  void* o;
  float* den;
  int* status;
  int B, T, H, HQ, D, Dv, M;
  int G;  // HQ / H
  float scale;
  // packed documents (tensor-core kernels only): nseq + 1 offsets into T (B == 1), or null
  const int* cu;
  int nseq;
};

struct AttnBwdParams {
  const void* q;
  const void* k;
  const void* v;
  const void* o;
  const float* den;
  const void* dout;
  const float* c;
  void* dq;
  void* dk;
  void* dv;
  float* dc;
  float* delta;  // workspace (B,T,HQ)
  int* status;
  int B, T, H, HQ, D, Dv, M;
  int G;
  float scale;
  int phases;  // 0 both passes, 1 dq pass, 2 dk/dv pass
  // Internal callers only (not in the C ABI): per-row delta_t given instead of <o_t, dO_t>
  // (o is then not read and may be null).  (B,T,HQ) fp32.
  const float* delta_in;
  // packed documents (tensor-core kernels only): nseq + 1 offsets into T (B == 1), or null
  const int* cu;
  int nseq;
};

}  // namespace kata
