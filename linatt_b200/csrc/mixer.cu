// mixer.cu -- the KATA mixer's prologue and epilogue around the attention op, forward and backward:
//
//   short convolution  y[t,c] = act(sum_i w[c,i] x[t-K+1+i, c] + bias[c]), causal, depthwise, act =
//                      SiLU or none (fla ShortConvolution as used on q, k, v by kata/layer.py:305-319)
//   row normalisation  per row of N values (a (token, head) slice): l2 (x / sqrt(sum x^2 + eps),
//                      fla l2norm) or RMS (x rsqrt(mean x^2 + eps) w, fla RMSNorm), then optionally
//                      RoPE (kata/layer.py:344-372: interleaved pairs over the whole head, or the
//                      half-rotation inside every group of R values for rope_group); with no rotation
//                      it is the output RMSNorm over head_v_dim (kata/layer.py:199-209, :539)
//
// All of them are HBM-bound passes.  Every thread moves 16-byte vectors (8 bf16/fp16 or 4 fp32
// values), computes in fp32 and reads every input element once per pass: the convolution keeps a
// sliding window of the last K inputs (and, backward, the last K gradients) in registers over a run
// of kConvRun time steps, the row kernels reduce a row over the few lanes that hold it with shuffles.
// Weight gradients are per-CTA partial sums reduced by a second kernel in a fixed order, so every
// result is deterministic (no atomics).
#include <algorithm>

#include "attn_common.cuh"
#include "host_util.h"
#include "tc64.cuh"

namespace kata {
namespace {

template <typename T>
struct VecN {
  static constexpr int N = 16 / static_cast<int>(sizeof(T));
};

template <typename T>
__device__ __forceinline__ void load_vec(const T* p, float (&v)[VecN<T>::N]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int i = 0; i < VecN<T>::N; ++i) v[i] = to_f32<T>(e[i]);
}
template <typename T>
__device__ __forceinline__ void store_vec(T* p, const float (&v)[VecN<T>::N]) {
  uint4 u;
  T* e = reinterpret_cast<T*>(&u);
#pragma unroll
  for (int i = 0; i < VecN<T>::N; ++i) e[i] = from_f32<T>(v[i]);
  *reinterpret_cast<uint4*>(p) = u;
}

__device__ __forceinline__ float sigmoidf_(float a) { return __fdividef(1.f, 1.f + __expf(-a)); }

// VB-byte vectors (VB = 8 or 16) of the convolution's channel slices
template <int VB>
struct VecRaw;
template <>
struct VecRaw<16> {
  using type = uint4;
};
template <>
struct VecRaw<8> {
  using type = uint2;
};
template <typename T, int VB>
__device__ __forceinline__ void unpack_raw(const typename VecRaw<VB>::type& u, float* v) {
  const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int i = 0; i < VB / static_cast<int>(sizeof(T)); ++i) v[i] = to_f32<T>(e[i]);
}
template <typename T, int VB>
__device__ __forceinline__ void store_raw(T* p, const float* v) {
  typename VecRaw<VB>::type u;
  T* e = reinterpret_cast<T*>(&u);
#pragma unroll
  for (int i = 0; i < VB / static_cast<int>(sizeof(T)); ++i) e[i] = from_f32<T>(v[i]);
  *reinterpret_cast<typename VecRaw<VB>::type*>(p) = u;
}
template <int VB>
__device__ __forceinline__ void cp_async_vec(uint32_t dst, const void* src) {
  if constexpr (VB == 16)
    tc64::cp_async16(dst, src, true);
  else
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(dst), "l"(src) : "memory");
}

// ------------------------------------------------------------------------------------------------
// short convolution
// ------------------------------------------------------------------------------------------------
constexpr int kConvRun = 32;  // time steps per thread (short runs: enough warps per SM to cover HBM latency)
constexpr int kConvU = 8;      // time steps whose loads are issued together (memory-level parallelism)

struct ConvParams {
  const void* x;
  const float* w;
  const float* bias;
  void* y;
  const void* dy;
  void* dx;
  float* part;  // backward: (B * nrun, C, K + 1) partial sums of dw and dbias
  int T, C;
  long long ldx, ldy, lddx;
  int act;
  int nrun;
};

// Per-thread input ring in shared memory: [buffer][step of the batch][thread] 16-byte slots, filled by
// cp.async and read back only by the thread that issued the copies (its own commit groups order
// them, so no barrier is needed).  Two batches of kConvU steps are in flight while one is consumed,
// and the raw vectors no longer occupy registers.
template <typename R>
__device__ __forceinline__ R* conv_slot(R* ring, int bf, int u) {
  return ring + (bf * kConvU + u) * blockDim.x + threadIdx.x;
}

// grid (ceil(channel vectors / blockDim), runs of kConvRun steps, B); a thread owns one 16-byte
// channel vector over one run.  Steps go in batches of kConvU, double-buffered through the
// thread's cp.async ring.
template <typename T, int K, int VB>
__global__ void __launch_bounds__(128) conv_fwd_kernel(ConvParams p) {
  using R = typename VecRaw<VB>::type;
  extern __shared__ __align__(16) uint8_t conv_smem[];
  R* conv_ring = reinterpret_cast<R*>(conv_smem);  // [2][kConvU][blockDim.x]
  constexpr int V = VB / static_cast<int>(sizeof(T));
  const int c0 = (blockIdx.x * blockDim.x + threadIdx.x) * V;
  if (c0 >= p.C) return;
  const int b = blockIdx.z, t0 = blockIdx.y * kConvRun;
  const int t1 = min(t0 + kConvRun, p.T);
  float wr[K][V], br[V];
#pragma unroll
  for (int j = 0; j < V; ++j) {
#pragma unroll
    for (int i = 0; i < K; ++i) wr[i][j] = p.w[(c0 + j) * K + i];
    br[j] = p.bias ? p.bias[c0 + j] : 0.f;
  }
  const T* xb = static_cast<const T*>(p.x) + static_cast<size_t>(b) * p.T * p.ldx + c0;
  T* yb = static_cast<T*>(p.y) + static_cast<size_t>(b) * p.T * p.ldy + c0;
  float win[K][V];  // win[i] = x[t - K + 1 + i]
#pragma unroll
  for (int i = 0; i < K - 1; ++i) {
    const int t = t0 - (K - 1) + i;
    if (t >= 0) unpack_raw<T, VB>(*reinterpret_cast<const R*>(xb + static_cast<size_t>(t) * p.ldx), win[i]);
    else {
#pragma unroll
      for (int j = 0; j < V; ++j) win[i][j] = 0.f;
    }
  }
  const auto issue = [&](int tb, int bf) {
#pragma unroll
    for (int u = 0; u < kConvU; ++u)
      if (tb + u < t1) cp_async_vec<VB>(smem_u32(conv_slot(conv_ring, bf, u)), xb + static_cast<size_t>(tb + u) * p.ldx);
    tc64::cp_async_commit();
  };
  issue(t0, 0);
  for (int tb = t0, it = 0; tb < t1; tb += kConvU, ++it) {
    const int bf = it & 1;
    if (tb + kConvU < t1) {
      issue(tb + kConvU, bf ^ 1);
      tc64::cp_async_wait<1>();
    } else {
      tc64::cp_async_wait<0>();
    }
#pragma unroll
    for (int u = 0; u < kConvU; ++u) {
      if (tb + u < t1) {  // (a guard, not a break: the batch stays fully unrolled)
      unpack_raw<T, VB>(*conv_slot(conv_ring, bf, u), win[K - 1]);
      float out[V];
#pragma unroll
      for (int j = 0; j < V; ++j) {
        float a = br[j];
#pragma unroll
        for (int i = 0; i < K; ++i) a = fmaf(wr[i][j], win[i][j], a);
        out[j] = p.act ? a * sigmoidf_(a) : a;
      }
      store_raw<T, VB>(yb + static_cast<size_t>(tb + u) * p.ldy, out);
#pragma unroll
      for (int i = 0; i < K - 1; ++i)
#pragma unroll
        for (int j = 0; j < V; ++j) win[i][j] = win[i + 1][j];
      }
    }
  }
}

// out[o] = sum over nparts rows of part (nparts x n, row-major) of column o, in row order
// (deterministic).  Block: 32 columns x 8 row lanes; lane r sums rows r, r + 8, ...; the eight lane
// sums are added in lane order.  Reads are 128-byte rows per warp.
__global__ void __launch_bounds__(256) column_sum_kernel(const float* part, int nparts, int n, float* out) {
  __shared__ float red[8][33];
  const int col = blockIdx.x * 32 + (threadIdx.x & 31), r = threadIdx.x >> 5;
  float s = 0.f;
  if (col < n)
    for (int k = r; k < nparts; k += 8) s += part[static_cast<size_t>(k) * n + col];
  red[r][threadIdx.x & 31] = s;
  __syncthreads();
  if (r == 0 && col < n) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += red[k][threadIdx.x & 31];
    out[col] = t;
  }
}

// (C, K + 1) sums -> dw (C, K) and dbias (C).
__global__ void conv_split_kernel(const float* sums, int C, int K, float* dw, float* dbias) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= C * (K + 1)) return;
  const int c = idx / (K + 1), i = idx % (K + 1);
  if (i < K) dw[c * K + i] = sums[idx];
  else if (dbias) dbias[c] = sums[idx];
}

// Backward: g = dy * act'(a) (a recomputed from x), dx[s] = sum_i w[i] g[s + K - 1 - i],
// dw[c,i] = sum_t g[t] x[t - K + 1 + i], dbias[c] = sum_t g[t].  A thread walks its run plus K - 1
// steps of look-ahead (the g values its last dx outputs need), keeping the last K x and g values;
// loads go in batches of kConvU steps as in the forward.
template <typename T, int K, int VB>
__global__ void __launch_bounds__(128) conv_bwd_kernel(ConvParams p) {
  using R = typename VecRaw<VB>::type;
  extern __shared__ __align__(16) uint8_t conv_smem[];
  R* conv_ring = reinterpret_cast<R*>(conv_smem);  // x: [2][kConvU][blockDim.x], then dy: the same
  constexpr int V = VB / static_cast<int>(sizeof(T));
  const int c0 = (blockIdx.x * blockDim.x + threadIdx.x) * V;
  if (c0 >= p.C) return;
  const int b = blockIdx.z, t0 = blockIdx.y * kConvRun;
  const int t1 = min(t0 + kConvRun, p.T);
  float wr[K][V], br[V];
#pragma unroll
  for (int j = 0; j < V; ++j) {
#pragma unroll
    for (int i = 0; i < K; ++i) wr[i][j] = p.w[(c0 + j) * K + i];
    br[j] = p.bias ? p.bias[c0 + j] : 0.f;
  }
  const T* xb = static_cast<const T*>(p.x) + static_cast<size_t>(b) * p.T * p.ldx + c0;
  const T* dyb = static_cast<const T*>(p.dy) + static_cast<size_t>(b) * p.T * p.ldy + c0;
  T* dxb = static_cast<T*>(p.dx) + static_cast<size_t>(b) * p.T * p.lddx + c0;
  float win[K][V], gq[K][V], dwa[K][V], dba[V];
#pragma unroll
  for (int i = 0; i < K; ++i)
#pragma unroll
    for (int j = 0; j < V; ++j) gq[i][j] = dwa[i][j] = 0.f;
#pragma unroll
  for (int j = 0; j < V; ++j) dba[j] = 0.f;
#pragma unroll
  for (int i = 0; i < K - 1; ++i) {
    const int t = t0 - (K - 1) + i;
    if (t >= 0) unpack_raw<T, VB>(*reinterpret_cast<const R*>(xb + static_cast<size_t>(t) * p.ldx), win[i]);
    else {
#pragma unroll
      for (int j = 0; j < V; ++j) win[i][j] = 0.f;
    }
  }
  const int tend = t1 + K - 1;  // exclusive
  const int tload = min(tend, p.T);
  R* ring_d = conv_ring + 2 * kConvU * blockDim.x;
  const auto issue = [&](int tb, int bf) {
#pragma unroll
    for (int u = 0; u < kConvU; ++u) {
      if (tb + u < tload) {
        cp_async_vec<VB>(smem_u32(conv_slot(conv_ring, bf, u)), xb + static_cast<size_t>(tb + u) * p.ldx);
        cp_async_vec<VB>(smem_u32(conv_slot(ring_d, bf, u)), dyb + static_cast<size_t>(tb + u) * p.ldy);
      }
    }
    tc64::cp_async_commit();
  };
  issue(t0, 0);
  for (int tb = t0, it = 0; tb < tend; tb += kConvU, ++it) {
    const int bf = it & 1;
    if (tb + kConvU < tend) {
      issue(tb + kConvU, bf ^ 1);
      tc64::cp_async_wait<1>();
    } else {
      tc64::cp_async_wait<0>();
    }
#pragma unroll
    for (int u = 0; u < kConvU; ++u) {
      const int t = tb + u;
      if (t < tend) {  // (a guard, not a break: the batch stays fully unrolled)
      if (t < p.T) {
        float gin[V];
        unpack_raw<T, VB>(*conv_slot(conv_ring, bf, u), win[K - 1]);
        unpack_raw<T, VB>(*conv_slot(ring_d, bf, u), gin);
#pragma unroll
        for (int j = 0; j < V; ++j) {
          float g = gin[j];
          if (p.act) {
            float a = br[j];
#pragma unroll
            for (int i = 0; i < K; ++i) a = fmaf(wr[i][j], win[i][j], a);
            const float sg = sigmoidf_(a);
            g *= sg * (1.f + a * (1.f - sg));
          }
          gq[K - 1][j] = g;
        }
        if (t < t1) {
#pragma unroll
          for (int j = 0; j < V; ++j) {
#pragma unroll
            for (int i = 0; i < K; ++i) dwa[i][j] = fmaf(gq[K - 1][j], win[i][j], dwa[i][j]);
            dba[j] += gq[K - 1][j];
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < V; ++j) gq[K - 1][j] = 0.f;
      }
      const int s0 = t - (K - 1);  // gq[i] = g[s0 + i]
      if (s0 >= t0) {
        float out[V];
#pragma unroll
        for (int j = 0; j < V; ++j) {
          float acc = 0.f;
#pragma unroll
          for (int i = 0; i < K; ++i) acc = fmaf(wr[i][j], gq[K - 1 - i][j], acc);
          out[j] = acc;
        }
        store_raw<T, VB>(dxb + static_cast<size_t>(s0) * p.lddx, out);
      }
#pragma unroll
      for (int i = 0; i < K - 1; ++i)
#pragma unroll
        for (int j = 0; j < V; ++j) {
          win[i][j] = win[i + 1][j];
          gq[i][j] = gq[i + 1][j];
        }
      }
    }
  }
  float* pr = p.part + (static_cast<size_t>(b) * p.nrun + blockIdx.y) * p.C * (K + 1);
#pragma unroll
  for (int j = 0; j < V; ++j) {
#pragma unroll
    for (int i = 0; i < K; ++i) pr[(c0 + j) * (K + 1) + i] = dwa[i][j];
    pr[(c0 + j) * (K + 1) + K] = dba[j];
  }
}

// ------------------------------------------------------------------------------------------------
// row normalisation + RoPE
// ------------------------------------------------------------------------------------------------
constexpr int kRowThreads = 256;
constexpr int kRowGrid = 148 * 8;  // grid-stride; the weight-gradient partials are one per CTA

struct RowParams {
  const void* x;
  const float* w;
  const float* cos;
  const float* sin;
  void* y;
  float* rstd;
  const void* dy;
  void* dx;
  float* part;  // backward: (gridDim.x, N) partials of dw
  long long rows;
  int N, T, heads;
  int norm, rope, R;
  float eps;
};

// Rotation of the values this thread holds (elements e0 .. e0 + V - 1 of row `row`), by +theta
// (forward) or -theta (backward, the transpose).  rope 1: pairs (2f, 2f + 1) over the row, angle
// index f; rope 2: inside every group of R values, element r < R/2 pairs with r + R/2, angle index
// r % (R/2); the partner lives in lane ^ (R/2/V) of the row's lanes (R/2 a multiple of V).
template <int V>
__device__ __forceinline__ void rotate(float (&v)[V], int e0, int t, const RowParams& p, bool inverse) {
  const float sg = inverse ? -1.f : 1.f;
  if (p.rope == 1) {
#pragma unroll
    for (int j = 0; j < V; j += 2) {
      const int f = (e0 + j) >> 1;
      const float c = p.cos[static_cast<size_t>(t) * (p.R / 2) + f], s = sg * p.sin[static_cast<size_t>(t) * (p.R / 2) + f];
      const float a = v[j], b = v[j + 1];
      v[j] = a * c - b * s;
      v[j + 1] = a * s + b * c;
    }
  } else if (p.rope == 2) {
    const int half = p.R / 2;
    const int r0 = e0 % p.R;
    const bool lo = r0 < half;
    float o[V];
#pragma unroll
    for (int j = 0; j < V; ++j) o[j] = __shfl_xor_sync(0xffffffffu, v[j], half / V);
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const int f = (r0 + j) % half;
      const float c = p.cos[static_cast<size_t>(t) * half + f], s = sg * p.sin[static_cast<size_t>(t) * half + f];
      v[j] = lo ? v[j] * c - o[j] * s : v[j] * c + o[j] * s;
    }
  }
}

// Sum over the TPR lanes that hold one row (TPR a power of two, <= 32, lane groups aligned).
template <int TPR>
__device__ __forceinline__ float row_sum(float s) {
#pragma unroll
  for (int o = TPR / 2; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  return s;
}

template <typename T, int TPR>
__global__ void __launch_bounds__(kRowThreads) row_fwd_kernel(RowParams p) {
  constexpr int V = VecN<T>::N;
  constexpr int RPC = kRowThreads / TPR;  // rows per CTA per iteration
  const int sub = threadIdx.x % TPR, e0 = sub * V;
  for (long long row = static_cast<long long>(blockIdx.x) * RPC + threadIdx.x / TPR; row - threadIdx.x / TPR < p.rows;
       row += static_cast<long long>(gridDim.x) * RPC) {
    const bool live = row < p.rows;
    float v[V];
    if (live) load_vec<T>(static_cast<const T*>(p.x) + row * p.N + e0, v);
    else {
#pragma unroll
      for (int j = 0; j < V; ++j) v[j] = 0.f;
    }
    if (p.norm) {
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < V; ++j) ss = fmaf(v[j], v[j], ss);
      ss = row_sum<TPR>(ss);
      const float r = rsqrtf((p.norm == 2 ? ss / p.N : ss) + p.eps);
#pragma unroll
      for (int j = 0; j < V; ++j) v[j] *= (p.norm == 2 && p.w) ? r * p.w[e0 + j] : r;
      if (live && p.rstd && sub == 0) p.rstd[row] = r;
    }
    if (p.rope) rotate<V>(v, e0, static_cast<int>((row / p.heads) % p.T), p, false);
    if (live) store_vec<T>(static_cast<T*>(p.y) + row * p.N + e0, v);
  }
}

// Backward: dy0 = R^T dy, then l2: dx = r (dy0 - xh sum(dy0 xh)); RMS: g = dy0 w,
// dx = r (g - xh mean(g xh)), dw += dy0 xh; no norm: dx = dy0.  xh = x r with the saved r.
template <typename T, int TPR>
__global__ void __launch_bounds__(kRowThreads) row_bwd_kernel(RowParams p) {
  constexpr int V = VecN<T>::N;
  constexpr int RPC = kRowThreads / TPR;
  const int sub = threadIdx.x % TPR, e0 = sub * V;
  float dwa[V];
#pragma unroll
  for (int j = 0; j < V; ++j) dwa[j] = 0.f;
  for (long long row = static_cast<long long>(blockIdx.x) * RPC + threadIdx.x / TPR; row - threadIdx.x / TPR < p.rows;
       row += static_cast<long long>(gridDim.x) * RPC) {
    const bool live = row < p.rows;
    float g[V], x[V];
    if (live) {
      load_vec<T>(static_cast<const T*>(p.dy) + row * p.N + e0, g);
      load_vec<T>(static_cast<const T*>(p.x) + row * p.N + e0, x);
    } else {
#pragma unroll
      for (int j = 0; j < V; ++j) g[j] = x[j] = 0.f;
    }
    if (p.rope) rotate<V>(g, e0, static_cast<int>((row / p.heads) % p.T), p, true);
    if (p.norm) {
      const float r = live ? p.rstd[row] : 0.f;
      float gw[V], dot = 0.f;
#pragma unroll
      for (int j = 0; j < V; ++j) {
        const float xh = x[j] * r;
        x[j] = xh;
        gw[j] = (p.norm == 2 && p.w) ? g[j] * p.w[e0 + j] : g[j];
        if (p.norm == 2 && p.w) dwa[j] = fmaf(g[j], xh, dwa[j]);
        dot = fmaf(gw[j], xh, dot);
      }
      dot = row_sum<TPR>(dot);
      if (p.norm == 2) dot /= p.N;
#pragma unroll
      for (int j = 0; j < V; ++j) g[j] = r * (gw[j] - x[j] * dot);
    }
    if (live) store_vec<T>(static_cast<T*>(p.dx) + row * p.N + e0, g);
  }
  if (p.part) {
    // CTA partial of dw: lanes with the same `sub` hold the same columns; sum them in shared memory
    __shared__ float red[kRowThreads][V + 1];
#pragma unroll
    for (int j = 0; j < V; ++j) red[threadIdx.x][j] = dwa[j];
    __syncthreads();
    if (threadIdx.x < TPR) {
      float s[V];
#pragma unroll
      for (int j = 0; j < V; ++j) s[j] = 0.f;
      for (int k = threadIdx.x; k < kRowThreads; k += TPR)
#pragma unroll
        for (int j = 0; j < V; ++j) s[j] += red[k][j];
#pragma unroll
      for (int j = 0; j < V; ++j) p.part[static_cast<size_t>(blockIdx.x) * p.N + e0 + j] = s[j];
    }
  }
}

// Rows wider than 32 vectors (e.g. the model's 768-wide hidden RMSNorm): one warp per row, lane l
// holding the NV vectors l, l + 32, ... (each warp load is 512 contiguous bytes).  Normalisation
// only (no rotation).
template <typename T, int NV>
__global__ void __launch_bounds__(kRowThreads) wide_row_fwd_kernel(RowParams p) {
  constexpr int V = VecN<T>::N;
  constexpr int RPC = kRowThreads / 32;
  const int lane = threadIdx.x & 31;
  for (long long row = static_cast<long long>(blockIdx.x) * RPC + threadIdx.x / 32; row - threadIdx.x / 32 < p.rows;
       row += static_cast<long long>(gridDim.x) * RPC) {
    if (row >= p.rows) continue;  // warp-uniform
    const T* xr = static_cast<const T*>(p.x) + row * p.N;
    float v[NV][V];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      load_vec<T>(xr + (lane + 32 * k) * V, v[k]);
#pragma unroll
      for (int j = 0; j < V; ++j) ss = fmaf(v[k][j], v[k][j], ss);
    }
    ss = row_sum<32>(ss);
    const float r = rsqrtf((p.norm == 2 ? ss / p.N : ss) + p.eps);
    if (p.rstd && lane == 0) p.rstd[row] = r;
    T* yr = static_cast<T*>(p.y) + row * p.N;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int e0 = (lane + 32 * k) * V;
#pragma unroll
      for (int j = 0; j < V; ++j) v[k][j] *= (p.norm == 2 && p.w) ? r * p.w[e0 + j] : r;
      store_vec<T>(yr + e0, v[k]);
    }
  }
}

template <typename T, int NV>
__global__ void __launch_bounds__(kRowThreads) wide_row_bwd_kernel(RowParams p) {
  constexpr int V = VecN<T>::N;
  constexpr int RPC = kRowThreads / 32;
  const int lane = threadIdx.x & 31;
  float dwa[NV][V];
#pragma unroll
  for (int k = 0; k < NV; ++k)
#pragma unroll
    for (int j = 0; j < V; ++j) dwa[k][j] = 0.f;
  const bool has_w = p.norm == 2 && p.w;
  for (long long row = static_cast<long long>(blockIdx.x) * RPC + threadIdx.x / 32; row - threadIdx.x / 32 < p.rows;
       row += static_cast<long long>(gridDim.x) * RPC) {
    if (row >= p.rows) continue;  // warp-uniform
    const float r = p.rstd[row];
    float g[NV][V], x[NV][V];
    float dot = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int e0 = (lane + 32 * k) * V;
      load_vec<T>(static_cast<const T*>(p.dy) + row * p.N + e0, g[k]);
      load_vec<T>(static_cast<const T*>(p.x) + row * p.N + e0, x[k]);
#pragma unroll
      for (int j = 0; j < V; ++j) {
        x[k][j] *= r;
        if (has_w) {
          dwa[k][j] = fmaf(g[k][j], x[k][j], dwa[k][j]);
          g[k][j] *= p.w[e0 + j];
        }
        dot = fmaf(g[k][j], x[k][j], dot);
      }
    }
    dot = row_sum<32>(dot);
    if (p.norm == 2) dot /= p.N;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
#pragma unroll
      for (int j = 0; j < V; ++j) g[k][j] = r * (g[k][j] - x[k][j] * dot);
      store_vec<T>(static_cast<T*>(p.dx) + row * p.N + (lane + 32 * k) * V, g[k]);
    }
  }
  if (p.part) {  // CTA partial of dw: the RPC warps' lanes hold the same columns; sum in lane order
    __shared__ float red[RPC][32 * NV * V];
#pragma unroll
    for (int k = 0; k < NV; ++k)
#pragma unroll
      for (int j = 0; j < V; ++j) red[threadIdx.x / 32][(lane + 32 * k) * V + j] = dwa[k][j];
    __syncthreads();
    for (int e = threadIdx.x; e < p.N; e += kRowThreads) {
      float acc = 0.f;
#pragma unroll
      for (int w = 0; w < RPC; ++w) acc += red[w][e];
      p.part[static_cast<size_t>(blockIdx.x) * p.N + e] = acc;
    }
  }
}

// ------------------------------------------------------------------------------------------------
// residual add + RMSNorm of the LM's hidden stream (fla's fused add-norm around every mixer / MLP):
//   h_out = h + x (fp32),  y = h_out * rsqrt(mean h_out^2 + eps) * w (in x's 16-bit type)
// backward: dh = dh_in + r (w g - xhat <w g, xhat> / N), g = dy, xhat = r h_out; dx = dh in x's type
// One warp per row, eight values per lane and vector (two float4 of h, one 16-byte vector of x / y);
// N a multiple of 256.  One pass over each operand in each direction (the unfused form reads and
// writes the fp32 stream twice more per add).
// ------------------------------------------------------------------------------------------------
struct AddNormParams {
  const float* h;
  const void* x;
  const float* w;
  float* h_out;
  void* y;
  float* rstd;
  const void* dy;
  const float* dh_in;
  float* dh;
  void* dx;
  float* part;
  long long rows;
  int N;
  float eps;
};

template <typename T>
__device__ __forceinline__ void ld8(const T* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = to_f32<T>(e[i]);
}
template <typename T>
__device__ __forceinline__ void st8(T* p, const float (&v)[8]) {
  uint4 u;
  T* e = reinterpret_cast<T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) e[i] = from_f32<T>(v[i]);
  *reinterpret_cast<uint4*>(p) = u;
}
__device__ __forceinline__ void ld8f(const float* p, float (&v)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void st8f(float* p, const float (&v)[8]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}

template <typename T, int NV>
__global__ void __launch_bounds__(kRowThreads) add_rmsnorm_fwd_kernel(AddNormParams p) {
  constexpr int RPC = kRowThreads / 32;
  const int lane = threadIdx.x & 31;
  for (long long row = static_cast<long long>(blockIdx.x) * RPC + threadIdx.x / 32; row - threadIdx.x / 32 < p.rows;
       row += static_cast<long long>(gridDim.x) * RPC) {
    if (row >= p.rows) continue;  // warp-uniform
    const size_t base = static_cast<size_t>(row) * p.N;
    float v[NV][8];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int e0 = (lane + 32 * k) * 8;
      float xv[8];
      ld8f(p.h + base + e0, v[k]);
      ld8<T>(static_cast<const T*>(p.x) + base + e0, xv);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[k][j] += xv[j];
        ss = fmaf(v[k][j], v[k][j], ss);
      }
      st8f(p.h_out + base + e0, v[k]);
    }
    ss = row_sum<32>(ss);
    const float r = rsqrtf(ss / p.N + p.eps);
    if (lane == 0) p.rstd[row] = r;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int e0 = (lane + 32 * k) * 8;
      float wv[8];
      ld8f(p.w + e0, wv);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[k][j] *= r * wv[j];
      st8<T>(static_cast<T*>(p.y) + base + e0, v[k]);
    }
  }
}

template <typename T, int NV>
__global__ void __launch_bounds__(kRowThreads) add_rmsnorm_bwd_kernel(AddNormParams p) {
  constexpr int RPC = kRowThreads / 32;
  const int lane = threadIdx.x & 31;
  float dwa[NV][8];
#pragma unroll
  for (int k = 0; k < NV; ++k)
#pragma unroll
    for (int j = 0; j < 8; ++j) dwa[k][j] = 0.f;
  for (long long row = static_cast<long long>(blockIdx.x) * RPC + threadIdx.x / 32; row - threadIdx.x / 32 < p.rows;
       row += static_cast<long long>(gridDim.x) * RPC) {
    if (row >= p.rows) continue;  // warp-uniform
    const size_t base = static_cast<size_t>(row) * p.N;
    const float r = p.rstd[row];
    float g[NV][8], xh[NV][8];
    float dot = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int e0 = (lane + 32 * k) * 8;
      float wv[8];
      ld8<T>(static_cast<const T*>(p.dy) + base + e0, g[k]);
      ld8f(p.h_out + base + e0, xh[k]);
      ld8f(p.w + e0, wv);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        xh[k][j] *= r;
        dwa[k][j] = fmaf(g[k][j], xh[k][j], dwa[k][j]);
        g[k][j] *= wv[j];
        dot = fmaf(g[k][j], xh[k][j], dot);
      }
    }
    dot = row_sum<32>(dot) / p.N;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int e0 = (lane + 32 * k) * 8;
      float din[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (p.dh_in) ld8f(p.dh_in + base + e0, din);
#pragma unroll
      for (int j = 0; j < 8; ++j) g[k][j] = r * (g[k][j] - xh[k][j] * dot) + din[j];
      if (p.dh) st8f(p.dh + base + e0, g[k]);
      if (p.dx) st8<T>(static_cast<T*>(p.dx) + base + e0, g[k]);
    }
  }
  // CTA partial of dw: the RPC warps' lanes hold the same columns; summed in warp order
  __shared__ float red[RPC][32 * NV * 8];
#pragma unroll
  for (int k = 0; k < NV; ++k)
#pragma unroll
    for (int j = 0; j < 8; ++j) red[threadIdx.x / 32][(lane + 32 * k) * 8 + j] = dwa[k][j];
  __syncthreads();
  for (int e = threadIdx.x; e < p.N; e += kRowThreads) {
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < RPC; ++w) acc += red[w][e];
    p.part[static_cast<size_t>(blockIdx.x) * p.N + e] = acc;
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
size_t esize(int dtype) { return dtype == KATA_DTYPE_F32 ? 4 : 2; }

int conv_check(const kata_conv_args* a, bool bwd) {
  if (!a) return KATA_ERR_INVALID;
  if (a->dtype != KATA_DTYPE_F32 && a->dtype != KATA_DTYPE_BF16 && a->dtype != KATA_DTYPE_F16) return KATA_ERR_DTYPE;
  if (a->B < 0 || a->T < 0 || a->C < 1 || a->K < 1 || a->K > 4) return KATA_ERR_SHAPE;
  const int V = static_cast<int>(16 / esize(a->dtype));
  if (a->C % V || a->ldx < a->C || a->ldy < a->C || a->ldx % V || a->ldy % V) return KATA_ERR_SHAPE;
  if (a->activation != 0 && a->activation != 1) return KATA_ERR_INVALID;
  if (!a->x || !a->w) return KATA_ERR_INVALID;
  if (!aligned16(a->x)) return KATA_ERR_ALIGN;
  if (!bwd) {
    if (!a->y) return KATA_ERR_INVALID;
    if (!aligned16(a->y)) return KATA_ERR_ALIGN;
  } else {
    if (!a->dy || !a->dx || !a->dw) return KATA_ERR_INVALID;
    if (a->lddx < a->C || a->lddx % V) return KATA_ERR_SHAPE;
    if (!aligned16(a->dy) || !aligned16(a->dx)) return KATA_ERR_ALIGN;
  }
  return KATA_OK;
}

template <typename T>
int conv_launch(const kata_conv_args* a, bool bwd, cudaStream_t st) {
  // 8-byte channel vectors: with 16-byte ones the backward's per-thread window, gradient window
  // and weight-gradient sums held the registers of only two CTAs per SM
  const int VB = 8;
  const int V = VB / static_cast<int>(sizeof(T));
  const int nrun = (a->T + kConvRun - 1) / kConvRun;
  ConvParams p{a->x, a->w, a->bias, a->y, a->dy, a->dx, static_cast<float*>(a->workspace), a->T, a->C, a->ldx,
               a->ldy, a->lddx, a->activation, nrun};
  // as many threads as channel vectors (up to 128, whole warps): no idle lanes at C = 768
  const int nvec = a->C / V;
  const int threads = std::min(128, (nvec + 31) / 32 * 32);
  const dim3 grid((nvec + threads - 1) / threads, nrun, a->B);
  const size_t ring = static_cast<size_t>(VB) * 2 * kConvU * threads * (bwd ? 2 : 1);  // per-thread cp.async rings
  const auto go = [&](auto kern) -> int {
    if (ring > 48 * 1024 &&
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(ring)) != cudaSuccess)
      return KATA_ERR_CUDA;
    kern<<<grid, threads, ring, st>>>(p);
    return KATA_OK;
  };
#define KATA_CONV_CASE(KK)                                                                            \
  case KK:                                                                                            \
    if (const int e = bwd ? go(conv_bwd_kernel<T, KK, 8>) : go(conv_fwd_kernel<T, KK, 8>)) return e;  \
    break;
  switch (a->K) {
    KATA_CONV_CASE(1)
    KATA_CONV_CASE(2)
    KATA_CONV_CASE(3)
    KATA_CONV_CASE(4)
    default: return KATA_ERR_SHAPE;
  }
#undef KATA_CONV_CASE
  if (cudaGetLastError() != cudaSuccess) return KATA_ERR_CUDA;
  if (bwd) {
    const int per = a->C * (a->K + 1);
    float* sums = p.part + static_cast<size_t>(a->B) * nrun * per;  // after the partials
    column_sum_kernel<<<(per + 31) / 32, 256, 0, st>>>(p.part, a->B * nrun, per, sums);
    conv_split_kernel<<<(per + 255) / 256, 256, 0, st>>>(sums, a->C, a->K, a->dw, a->dbias);
    if (cudaGetLastError() != cudaSuccess) return KATA_ERR_CUDA;
  }
  return KATA_OK;
}

int row_check(const kata_rownorm_args* a, bool bwd) {
  if (!a) return KATA_ERR_INVALID;
  if (a->dtype != KATA_DTYPE_F32 && a->dtype != KATA_DTYPE_BF16 && a->dtype != KATA_DTYPE_F16) return KATA_ERR_DTYPE;
  const int V = static_cast<int>(16 / esize(a->dtype));
  const int tpr = a->N / V;
  if (a->rows < 0 || a->N < V || a->N % V) return KATA_ERR_SHAPE;
  if (tpr > 32) {  // wide rows: 2, 3, 4 or 6 vectors per lane of one warp, no rotation
    if (tpr % 32 || tpr > 192 || tpr == 160 || a->rope) return KATA_ERR_SHAPE;
  } else if (tpr & (tpr - 1)) {
    return KATA_ERR_SHAPE;
  }
  if (a->norm < 0 || a->norm > 2 || a->rope < 0 || a->rope > 2) return KATA_ERR_INVALID;
  if (a->rope) {
    if (!a->cos || !a->sin || a->T < 1 || a->heads < 1) return KATA_ERR_INVALID;
    if (a->rope == 1 && a->R != a->N) return KATA_ERR_SHAPE;
    if (a->rope == 2 && (a->R < 2 || a->N % a->R || (a->R / 2) % V)) return KATA_ERR_SHAPE;
  }
  if (a->norm && !a->rstd) return KATA_ERR_INVALID;
  if (!a->x) return KATA_ERR_INVALID;
  if (!aligned16(a->x)) return KATA_ERR_ALIGN;
  if (!bwd) {
    if (!a->y) return KATA_ERR_INVALID;
    if (!aligned16(a->y)) return KATA_ERR_ALIGN;
  } else {
    if (!a->dy || !a->dx) return KATA_ERR_INVALID;
    if (!aligned16(a->dy) || !aligned16(a->dx)) return KATA_ERR_ALIGN;
    if (a->norm == 2 && a->w && !a->dw) return KATA_ERR_INVALID;
  }
  return KATA_OK;
}

template <typename T>
int row_launch(const kata_rownorm_args* a, bool bwd, cudaStream_t st) {
  constexpr int V = VecN<T>::N;
  const int tpr = a->N / V;
  const bool want_dw = bwd && a->norm == 2 && a->w;
  RowParams p{a->x, a->w, a->cos, a->sin, a->y, a->rstd, a->dy, a->dx,
              want_dw ? static_cast<float*>(a->workspace) : nullptr, a->rows, a->N, a->T, a->heads, a->norm,
              a->rope, a->R, a->eps};
  const long long rpc = kRowThreads / std::min(tpr, 32);
  const int grid = static_cast<int>(std::min<long long>(kRowGrid, (a->rows + rpc - 1) / rpc));
  if (grid == 0) {
    if (want_dw) return from_cuda(cudaMemsetAsync(a->dw, 0, sizeof(float) * a->N, st));
    return KATA_OK;
  }
#define KATA_ROW_CASE(TP)                                                               \
  case TP:                                                                              \
    if (bwd) row_bwd_kernel<T, TP><<<grid, kRowThreads, 0, st>>>(p);                    \
    else row_fwd_kernel<T, TP><<<grid, kRowThreads, 0, st>>>(p);                        \
    break;
#define KATA_WIDE_CASE(NVV)                                                             \
  case 32 * NVV:                                                                        \
    if (bwd) wide_row_bwd_kernel<T, NVV><<<grid, kRowThreads, 0, st>>>(p);              \
    else wide_row_fwd_kernel<T, NVV><<<grid, kRowThreads, 0, st>>>(p);                  \
    break;
  switch (tpr) {
    KATA_WIDE_CASE(2)
    KATA_WIDE_CASE(3)
    KATA_WIDE_CASE(4)
    KATA_WIDE_CASE(6)
    KATA_ROW_CASE(1)
    KATA_ROW_CASE(2)
    KATA_ROW_CASE(4)
    KATA_ROW_CASE(8)
    KATA_ROW_CASE(16)
    KATA_ROW_CASE(32)
    default: return KATA_ERR_SHAPE;
  }
#undef KATA_ROW_CASE
#undef KATA_WIDE_CASE
  if (cudaGetLastError() != cudaSuccess) return KATA_ERR_CUDA;
  if (want_dw) {
    column_sum_kernel<<<(a->N + 31) / 32, 256, 0, st>>>(p.part, grid, a->N, a->dw);
    if (cudaGetLastError() != cudaSuccess) return KATA_ERR_CUDA;
  }
  return KATA_OK;
}

int row_grid(const kata_rownorm_args* a) {
  const int V = static_cast<int>(16 / esize(a->dtype));
  const long long rpc = kRowThreads / std::min(a->N / V, 32);
  return static_cast<int>(std::min<long long>(kRowGrid, (a->rows + rpc - 1) / rpc));
}

}  // namespace
}  // namespace kata

using namespace kata;

extern "C" int kata_short_conv_fwd(const kata_conv_args* a, kata_stream_t stream) {
  int e = conv_check(a, false);
  if (e) return e;
  if (a->B == 0 || a->T == 0) return KATA_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (a->dtype) {
    case KATA_DTYPE_BF16: return conv_launch<__nv_bfloat16>(a, false, st);
    case KATA_DTYPE_F16: return conv_launch<__half>(a, false, st);
    default: return conv_launch<float>(a, false, st);
  }
}

extern "C" size_t kata_short_conv_bwd_workspace_bytes(const kata_conv_args* a) {
  if (!a || a->B < 0 || a->T < 0 || a->C < 1 || a->K < 1) return 0;
  const size_t nrun = (static_cast<size_t>(a->T) + kConvRun - 1) / kConvRun;
  return sizeof(float) * (static_cast<size_t>(a->B) * nrun + 1) * a->C * (a->K + 1);  // partials + sums
}

extern "C" int kata_short_conv_bwd(const kata_conv_args* a, kata_stream_t stream) {
  int e = conv_check(a, true);
  if (e) return e;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (a->B == 0 || a->T == 0) {
    if (cudaMemsetAsync(a->dw, 0, sizeof(float) * a->C * a->K, st) != cudaSuccess) return KATA_ERR_CUDA;
    if (a->dbias && cudaMemsetAsync(a->dbias, 0, sizeof(float) * a->C, st) != cudaSuccess) return KATA_ERR_CUDA;
    return KATA_OK;
  }
  if (!a->workspace || a->workspace_bytes < kata_short_conv_bwd_workspace_bytes(a)) return KATA_ERR_WORKSPACE;
  switch (a->dtype) {
    case KATA_DTYPE_BF16: return conv_launch<__nv_bfloat16>(a, true, st);
    case KATA_DTYPE_F16: return conv_launch<__half>(a, true, st);
    default: return conv_launch<float>(a, true, st);
  }
}

extern "C" int kata_rownorm_fwd(const kata_rownorm_args* a, kata_stream_t stream) {
  int e = row_check(a, false);
  if (e) return e;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (a->dtype) {
    case KATA_DTYPE_BF16: return row_launch<__nv_bfloat16>(a, false, st);
    case KATA_DTYPE_F16: return row_launch<__half>(a, false, st);
    default: return row_launch<float>(a, false, st);
  }
}

extern "C" size_t kata_rownorm_bwd_workspace_bytes(const kata_rownorm_args* a) {
  if (!a || row_check(a, true) == KATA_ERR_SHAPE || a->N < 1) return 0;
  if (!(a->norm == 2 && a->w)) return 0;
  return sizeof(float) * static_cast<size_t>(row_grid(a)) * a->N;
}

extern "C" int kata_rownorm_bwd(const kata_rownorm_args* a, kata_stream_t stream) {
  int e = row_check(a, true);
  if (e) return e;
  if (a->norm == 2 && a->w && a->rows > 0 &&
      (!a->workspace || a->workspace_bytes < kata_rownorm_bwd_workspace_bytes(a)))
    return KATA_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (a->dtype) {
    case KATA_DTYPE_BF16: return row_launch<__nv_bfloat16>(a, true, st);
    case KATA_DTYPE_F16: return row_launch<__half>(a, true, st);
    default: return row_launch<float>(a, true, st);
  }
}

// ------------------------------------------------------------------------------------------------
// residual add + RMSNorm
// ------------------------------------------------------------------------------------------------
namespace {
int addnorm_check(const kata_add_rmsnorm_args* a, bool bwd) {
  if (!a) return KATA_ERR_INVALID;
  if (a->dtype != KATA_DTYPE_BF16 && a->dtype != KATA_DTYPE_F16) return KATA_ERR_DTYPE;
  if (a->rows < 0 || a->N < 256 || a->N % 256 || a->N > 1024) return KATA_ERR_SHAPE;
  if (!a->w || !a->h_out || !a->rstd) return KATA_ERR_INVALID;
  if (!bwd && (!a->h || !a->x || !a->y)) return KATA_ERR_INVALID;
  if (bwd && (!a->dy || !a->dw || (!a->dh && !a->dx))) return KATA_ERR_INVALID;
  const void* ptrs[] = {a->h, a->x, a->w, a->h_out, a->y, a->dy, a->dh_in, a->dh, a->dx};
  for (const void* q : ptrs)
    if (q && !aligned16(q)) return KATA_ERR_ALIGN;
  return KATA_OK;
}

template <typename T>
int addnorm_launch(const kata_add_rmsnorm_args* a, bool bwd, cudaStream_t st) {
  const long long need = (a->rows + kRowThreads / 32 - 1) / (kRowThreads / 32);
  const int grid = static_cast<int>(std::min<long long>(kRowGrid, std::max<long long>(need, 1)));
  AddNormParams p{a->h, a->x, a->w, a->h_out, a->y, a->rstd, a->dy, a->dh_in, a->dh, a->dx,
                  static_cast<float*>(a->workspace), a->rows, a->N, a->eps};
#define KATA_ADDNORM_CASE(NVV)                                                         \
  case NVV:                                                                            \
    if (bwd) add_rmsnorm_bwd_kernel<T, NVV><<<grid, kRowThreads, 0, st>>>(p);          \
    else add_rmsnorm_fwd_kernel<T, NVV><<<grid, kRowThreads, 0, st>>>(p);              \
    break;
  switch (a->N / 256) {
    KATA_ADDNORM_CASE(1)
    KATA_ADDNORM_CASE(2)
    KATA_ADDNORM_CASE(3)
    KATA_ADDNORM_CASE(4)
    default: return KATA_ERR_SHAPE;
  }
#undef KATA_ADDNORM_CASE
  if (cudaGetLastError() != cudaSuccess) return KATA_ERR_CUDA;
  if (bwd) {
    column_sum_kernel<<<(a->N + 31) / 32, 256, 0, st>>>(p.part, grid, a->N, a->dw);
    if (cudaGetLastError() != cudaSuccess) return KATA_ERR_CUDA;
  }
  return KATA_OK;
}
}  // namespace

extern "C" int kata_add_rmsnorm_fwd(const kata_add_rmsnorm_args* a, kata_stream_t stream) {
  int e = addnorm_check(a, false);
  if (e) return e;
  if (a->rows == 0) return KATA_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return a->dtype == KATA_DTYPE_BF16 ? addnorm_launch<__nv_bfloat16>(a, false, st) : addnorm_launch<__half>(a, false, st);
}

extern "C" size_t kata_add_rmsnorm_bwd_workspace_bytes(const kata_add_rmsnorm_args* a) {
  if (!a || a->rows <= 0 || a->N < 1) return 0;
  const long long need = (a->rows + kRowThreads / 32 - 1) / (kRowThreads / 32);
  return sizeof(float) * static_cast<size_t>(std::min<long long>(kRowGrid, need)) * a->N;
}

extern "C" int kata_add_rmsnorm_bwd(const kata_add_rmsnorm_args* a, kata_stream_t stream) {
  int e = addnorm_check(a, true);
  if (e) return e;
  if (a->rows == 0) return KATA_OK;
  if (!a->workspace || a->workspace_bytes < kata_add_rmsnorm_bwd_workspace_bytes(a)) return KATA_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return a->dtype == KATA_DTYPE_BF16 ? addnorm_launch<__nv_bfloat16>(a, true, st) : addnorm_launch<__half>(a, true, st);
}
