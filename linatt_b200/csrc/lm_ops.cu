// lm_ops.cu -- the two elementwise-heavy steps of the KATA LM around the mixer (kata/modeling.py's
// fla GatedMLP and fused cross-entropy loss): SwiGLU and the next-token cross entropy.
//
//   swiglu     y = silu(g) * u over a (rows, 2I) tensor [g | u]  (the fused gate/up GEMM output);
//              backward dg = dy u silu'(g), du = dy silu(g) into one (rows, 2I) gradient: one pass each
//   cross      per row of V logits: lse = log sum exp, loss_row = lse - logit[target] (0 for ignored
//   entropy    rows, target < 0); backward dlogit = (exp(logit - lse) - onehot) * scale, scale = the
//              upstream gradient times 1 / (valid rows), both read from device scalars (no host sync)
//
// HBM-bound: 16-byte vectors, fp32 arithmetic, one read of the logits forward and one read + one write
// backward (no fp32 copy of the logits is ever formed).
#include <algorithm>
#include <cfloat>

#include "attn_common.cuh"
#include "host_util.h"

namespace kata {
namespace {

template <typename T>
struct V16 {
  static constexpr int N = 16 / static_cast<int>(sizeof(T));
};

template <typename T>
__device__ __forceinline__ void ld16v(const T* p, float (&v)[V16<T>::N]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int i = 0; i < V16<T>::N; ++i) v[i] = to_f32<T>(e[i]);
}
template <typename T>
__device__ __forceinline__ void st16v(T* p, const float (&v)[V16<T>::N]) {
  uint4 u;
  T* e = reinterpret_cast<T*>(&u);
#pragma unroll
  for (int i = 0; i < V16<T>::N; ++i) e[i] = from_f32<T>(v[i]);
  *reinterpret_cast<uint4*>(p) = u;
}

__device__ __forceinline__ float sigm(float a) { return __fdividef(1.f, 1.f + __expf(-a)); }

// grid-stride over (row, vector of the I columns)
template <typename T>
__global__ void __launch_bounds__(256) swiglu_fwd_kernel(const T* __restrict__ gu, T* __restrict__ y, long long rows,
                                                         int I) {
  constexpr int V = V16<T>::N;
  const int nv = I / V;
  const long long total = rows * nv;
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i < total; i += static_cast<long long>(gridDim.x) * 256) {
    const long long r = i / nv;
    const int c = static_cast<int>(i - r * nv) * V;
    float g[V], u[V], o[V];
    ld16v<T>(gu + r * 2 * I + c, g);
    ld16v<T>(gu + r * 2 * I + I + c, u);
#pragma unroll
    for (int j = 0; j < V; ++j) o[j] = g[j] * sigm(g[j]) * u[j];
    st16v<T>(y + r * I + c, o);
  }
}

template <typename T>
__global__ void __launch_bounds__(256) swiglu_bwd_kernel(const T* __restrict__ gu, const T* __restrict__ dy,
                                                         T* __restrict__ dgu, long long rows, int I) {
  constexpr int V = V16<T>::N;
  const int nv = I / V;
  const long long total = rows * nv;
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i < total; i += static_cast<long long>(gridDim.x) * 256) {
    const long long r = i / nv;
    const int c = static_cast<int>(i - r * nv) * V;
    float g[V], u[V], d[V], dg[V], du[V];
    ld16v<T>(gu + r * 2 * I + c, g);
    ld16v<T>(gu + r * 2 * I + I + c, u);
    ld16v<T>(dy + r * I + c, d);
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const float s = sigm(g[j]);
      du[j] = d[j] * g[j] * s;
      dg[j] = d[j] * u[j] * s * (1.f + g[j] * (1.f - s));
    }
    st16v<T>(dgu + r * 2 * I + c, dg);
    st16v<T>(dgu + r * 2 * I + I + c, du);
  }
}

// One CTA of 256 threads per row: online max / sum of exponentials over the row's vectors, then a
// block reduction of (max, sum) pairs.
constexpr int kCeThreads = 256;

__device__ __forceinline__ void lse_merge(float& m, float& s, float m2, float s2) {
  const float mm = fmaxf(m, m2);
  s = (m == -FLT_MAX ? 0.f : s * __expf(m - mm)) + (m2 == -FLT_MAX ? 0.f : s2 * __expf(m2 - mm));
  m = mm;
}

template <typename T>
__global__ void __launch_bounds__(kCeThreads) ce_fwd_kernel(const T* __restrict__ logits,
                                                            const long long* __restrict__ tgt, float* __restrict__ lse,
                                                            float* __restrict__ loss, int V) {
  constexpr int VN = V16<T>::N;
  __shared__ float sm_m[kCeThreads / 32], sm_s[kCeThreads / 32];
  const long long r = blockIdx.x;
  const T* x = logits + r * V;
  float m = -FLT_MAX, s = 0.f;
  for (int c = threadIdx.x * VN; c < V; c += kCeThreads * VN) {
    float v[VN];
    ld16v<T>(x + c, v);
    float vm = v[0];
#pragma unroll
    for (int j = 1; j < VN; ++j) vm = fmaxf(vm, v[j]);
    float vs = 0.f;
#pragma unroll
    for (int j = 0; j < VN; ++j) vs += __expf(v[j] - vm);
    lse_merge(m, s, vm, vs);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    lse_merge(m, s, m2, s2);
  }
  if ((threadIdx.x & 31) == 0) {
    sm_m[threadIdx.x >> 5] = m;
    sm_s[threadIdx.x >> 5] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float mm = sm_m[0], ss = sm_s[0];
    for (int w = 1; w < kCeThreads / 32; ++w) lse_merge(mm, ss, sm_m[w], sm_s[w]);
    const float l = mm + __logf(ss);
    lse[r] = l;
    const long long t = tgt[r];
    loss[r] = (t >= 0 && t < V) ? l - to_f32<T>(x[t]) : 0.f;
  }
}

template <typename T>
__global__ void __launch_bounds__(kCeThreads) ce_bwd_kernel(const T* __restrict__ logits,
                                                            const long long* __restrict__ tgt,
                                                            const float* __restrict__ lse,
                                                            const float* __restrict__ gscale,
                                                            const float* __restrict__ inv_n, T* __restrict__ dlogits,
                                                            int V) {
  constexpr int VN = V16<T>::N;
  const long long r = blockIdx.x;
  const long long t = tgt[r];
  const bool valid = t >= 0 && t < V;
  const float sc = valid ? gscale[0] * inv_n[0] : 0.f, l = lse[r];
  const T* x = logits + r * V;
  T* dx = dlogits + r * V;
  for (int c = threadIdx.x * VN; c < V; c += kCeThreads * VN) {
    float v[VN];
    ld16v<T>(x + c, v);
#pragma unroll
    for (int j = 0; j < VN; ++j) v[j] = (__expf(v[j] - l) - (c + j == t ? 1.f : 0.f)) * sc;
    st16v<T>(dx + c, v);
  }
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
int vec_of(int dtype) { return dtype == KATA_DTYPE_F32 ? 4 : 8; }
int grid_for(long long n) { return static_cast<int>(std::min<long long>(148 * 16, (n + 255) / 256)); }

}  // namespace
}  // namespace kata

using namespace kata;

#define KATA_DISPATCH_T(dtype, ...)                                 \
  switch (dtype) {                                                  \
    case KATA_DTYPE_BF16: { using T = __nv_bfloat16; __VA_ARGS__; } \
    case KATA_DTYPE_F16: { using T = __half; __VA_ARGS__; }          \
    case KATA_DTYPE_F32: { using T = float; __VA_ARGS__; }           \
    default: return KATA_ERR_DTYPE;                                 \
  }

extern "C" int kata_swiglu_fwd(const void* gu, void* y, long long rows, int I, int dtype, kata_stream_t stream) {
  if (!gu || !y || rows < 0 || I < 1) return KATA_ERR_INVALID;
  if (I % vec_of(dtype)) return KATA_ERR_SHAPE;
  if (!al16(gu) || !al16(y)) return KATA_ERR_ALIGN;
  if (rows == 0) return KATA_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int g = grid_for(rows * (I / vec_of(dtype)));
  KATA_DISPATCH_T(dtype, swiglu_fwd_kernel<T><<<g, 256, 0, st>>>(static_cast<const T*>(gu), static_cast<T*>(y), rows, I);
                  return from_cuda(cudaGetLastError()))
}

extern "C" int kata_swiglu_bwd(const void* gu, const void* dy, void* dgu, long long rows, int I, int dtype,
                               kata_stream_t stream) {
  if (!gu || !dy || !dgu || rows < 0 || I < 1) return KATA_ERR_INVALID;
  if (I % vec_of(dtype)) return KATA_ERR_SHAPE;
  if (!al16(gu) || !al16(dy) || !al16(dgu)) return KATA_ERR_ALIGN;
  if (rows == 0) return KATA_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int g = grid_for(rows * (I / vec_of(dtype)));
  KATA_DISPATCH_T(dtype, swiglu_bwd_kernel<T><<<g, 256, 0, st>>>(static_cast<const T*>(gu), static_cast<const T*>(dy),
                                                                 static_cast<T*>(dgu), rows, I);
                  return from_cuda(cudaGetLastError()))
}

extern "C" int kata_cross_entropy_fwd(const void* logits, const int64_t* targets, float* lse, float* loss_rows,
                                      long long rows, int V, int dtype, kata_stream_t stream) {
  if (!logits || !targets || !lse || !loss_rows || rows < 0 || V < 1) return KATA_ERR_INVALID;
  if (V % vec_of(dtype)) return KATA_ERR_SHAPE;
  if (!al16(logits)) return KATA_ERR_ALIGN;
  if (rows == 0) return KATA_OK;
  if (rows > 0x7fffffffll) return KATA_ERR_SHAPE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  KATA_DISPATCH_T(dtype, ce_fwd_kernel<T><<<static_cast<unsigned>(rows), kCeThreads, 0, st>>>(
                             static_cast<const T*>(logits), reinterpret_cast<const long long*>(targets), lse, loss_rows, V);
                  return from_cuda(cudaGetLastError()))
}

extern "C" int kata_cross_entropy_bwd(const void* logits, const int64_t* targets, const float* lse,
                                      const float* grad_loss, const float* inv_count, void* dlogits, long long rows,
                                      int V, int dtype, kata_stream_t stream) {
  if (!logits || !targets || !lse || !grad_loss || !inv_count || !dlogits || rows < 0 || V < 1)
    return KATA_ERR_INVALID;
  if (V % vec_of(dtype)) return KATA_ERR_SHAPE;
  if (!al16(logits) || !al16(dlogits)) return KATA_ERR_ALIGN;
  if (rows == 0) return KATA_OK;
  if (rows > 0x7fffffffll) return KATA_ERR_SHAPE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  KATA_DISPATCH_T(dtype, ce_bwd_kernel<T><<<static_cast<unsigned>(rows), kCeThreads, 0, st>>>(
                             static_cast<const T*>(logits), reinterpret_cast<const long long*>(targets), lse, grad_loss,
                             inv_count, static_cast<T*>(dlogits), V);
                  return from_cuda(cudaGetLastError()))
}
