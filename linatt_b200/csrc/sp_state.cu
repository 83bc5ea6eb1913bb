// sp_state.cu -- per-token kernels of the sequence-parallel KATA-SPD path.
//
// With the concat score A[t,s] = sum_g (scale q_g[t].k_g[s])^2 and the quadratic feature map
//   psi(x)[g,a,b] = scale * (x_{g,a} x_{g,b})           (F = M E^2 features, E = D/M)
// A[t,s] = psi(q_t).psi(k_s), so the keys of earlier sequence shards enter a shard's queries only
// through the state P = sum_s psi(k_s) [v_s | 1] (F x (Dv+1)).  These kernels expand features,
// contract feature gradients back to q/k, and combine the shard-local attention with the prefix
// term; the F-contractions themselves are plain GEMMs.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "attn_common.cuh"
#include "host_util.h"
#include "kata_b200.h"

namespace kata {
namespace {

constexpr int NT = 256;
constexpr int TOK = 16;  // tokens per CTA of the feature kernel

// R (B,H,T,F) bf16, R[.., g E^2 + a E + b] = scale * (x_a * x_b)  (product first: exactly symmetric).
// HBM-bound on the writes (F bf16 per token and head).  A thread owns fixed 8-feature chunks, so the
// chunk's (g, a, b0) offsets are computed once, and streams over the CTA's tokens: two 16-byte
// shared loads and one 16-byte coalesced store per chunk and token.  With fewer chunks than
// threads, the threads split the tokens instead.  SUM: the sum score's features
// psi[a,b] = scale * sum_g x_{g,a} x_{g,b} (F = E^2), summed in group order with fused multiply-adds.
template <typename T, bool SUM>
__global__ void __launch_bounds__(NT) sp_features_kernel(const T* __restrict__ x, __nv_bfloat16* __restrict__ R,
                                                         int B, int Tn, int H, int D, int M, float scale) {
  extern __shared__ float xs[];  // TOK x D
  const int E = D / M, EE = E * E, F = SUM ? EE : M * EE, bh = blockIdx.y, b = bh / H, h = bh % H;
  const int t0 = blockIdx.x * TOK, tid = threadIdx.x;
  for (int i = tid; i < TOK * D; i += NT) {
    const int j = i / D, d = i % D, t = t0 + j;
    xs[i] = t < Tn ? to_f32<T>(x[((static_cast<size_t>(b) * Tn + t) * H + h) * D + d]) : 0.f;
  }
  __syncthreads();
  const int chunks = F / 8;
  const bool wide = chunks >= NT;
  const int js = wide ? 1 : NT / chunks;  // token stride
  if (!wide && tid >= js * chunks) return;
  const int j0 = wide ? 0 : tid / chunks;
  for (int ci = wide ? tid : tid % chunks; ci < chunks; ci += NT) {
    const int f0 = ci * 8, g = SUM ? 0 : f0 / EE, a = (f0 - g * EE) / E, b0 = f0 % E;
    const int oa = g * E + a, ob = g * E + b0;  // ob is a multiple of 8: 32-byte aligned rows of xs
    __nv_bfloat16* out = R + (static_cast<size_t>(bh) * Tn + t0) * F + f0;
    for (int j = j0; j < TOK && t0 + j < Tn; j += js) {
      const float* xr = xs + j * D;
      if constexpr (SUM) {
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int gg = 0; gg < M; ++gg) {
          const float xa = xr[gg * E + a];
          const float4 lo = *reinterpret_cast<const float4*>(xr + gg * E + b0);
          const float4 hi = *reinterpret_cast<const float4*>(xr + gg * E + b0 + 4);
          const float xb[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[i] = fmaf(xa, xb[i], acc[i]);
        }
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const __nv_bfloat162 v = __floats2bfloat162_rn(scale * acc[2 * i], scale * acc[2 * i + 1]);
          w[i] = *reinterpret_cast<const uint32_t*>(&v);
        }
        *reinterpret_cast<uint4*>(out + static_cast<size_t>(j) * F) = make_uint4(w[0], w[1], w[2], w[3]);
        continue;
      }
      const float xa = xr[oa];
      const float4 lo = *reinterpret_cast<const float4*>(xr + ob);
      const float4 hi = *reinterpret_cast<const float4*>(xr + ob + 4);
      const float xb[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
      uint32_t w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const __nv_bfloat162 v = __floats2bfloat162_rn(scale * (xa * xb[2 * i]), scale * (xa * xb[2 * i + 1]));
        w[i] = *reinterpret_cast<const uint32_t*>(&v);
      }
      *reinterpret_cast<uint4*>(out + static_cast<size_t>(j) * F) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

// dx_{g,a} (+)= factor * sum_b G[g,b,a] x_{g,b}, G = dR of one (token, head), symmetric in (a,b).
// One warp per (token, head): lanes walk a, the warp walks b (coalesced rows of G).
template <typename T>
__global__ void __launch_bounds__(NT) sp_contract_kernel(const __nv_bfloat16* __restrict__ G, const T* __restrict__ x,
                                                         float* __restrict__ dx, int B, int Tn, int H, int D, int M,
                                                         float factor, int accumulate) {
  const int warp = (blockIdx.x * NT + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const long total = static_cast<long>(B) * H * Tn;
  if (warp >= total) return;
  const int bh = warp / Tn, t = warp % Tn, b = bh / H, h = bh % H;
  const int E = D / M, F = M * E * E;
  const size_t xo = ((static_cast<size_t>(b) * Tn + t) * H + h) * D;
  const __nv_bfloat16* g = G + (static_cast<size_t>(bh) * Tn + t) * F;
  for (int gi = 0; gi < M; ++gi) {
    for (int a0 = 0; a0 < E; a0 += 32) {
      const int a = a0 + lane;
      float acc = 0.f;
      for (int bb = 0; bb < E; ++bb) {
        const float xb = to_f32<T>(x[xo + gi * E + bb]);
        if (a < E) acc = fmaf(__bfloat162float(g[gi * E * E + bb * E + a]), xb, acc);
      }
      if (a < E) {
        float* o = dx + xo + gi * E + a;
        *o = accumulate ? *o + factor * acc : factor * acc;
      }
    }
  }
}

// The same contraction with 16-byte loads, for E/8 dividing 32 (E = 16, 32, ..., 256).  One warp
// per (token, head); LPR = E/8 lanes cover one row b of G_g (8 consecutive a each), so a warp load
// reads 32/LPR whole rows = 512 contiguous bytes.  Each lane accumulates its 8 a's over the rows
// b = lane/LPR + i*(32/LPR); the lanes sharing the same a's then combine by shuffles.
template <typename T, int LPR>
__global__ void __launch_bounds__(NT) sp_contract_vec_kernel(const __nv_bfloat16* __restrict__ G,
                                                             const T* __restrict__ x, float* __restrict__ dx, int B,
                                                             int Tn, int H, int D, int M, float factor,
                                                             int accumulate) {
  constexpr int E = LPR * 8, RPP = 32 / LPR;  // rows per pass
  const int warp = (blockIdx.x * NT + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const long total = static_cast<long>(B) * H * Tn;
  if (warp >= total) return;
  const int bh = warp / Tn, t = warp % Tn, b = bh / H, h = bh % H;
  const size_t xo = ((static_cast<size_t>(b) * Tn + t) * H + h) * D;
  const __nv_bfloat16* g = G + (static_cast<size_t>(bh) * Tn + t) * static_cast<size_t>(M) * E * E;
  const int a0 = (lane % LPR) * 8, r0 = lane / LPR;
  for (int gi = 0; gi < M; ++gi) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    const __nv_bfloat16* gg = g + static_cast<size_t>(gi) * E * E;
#pragma unroll 4
    for (int bb = r0; bb < E; bb += RPP) {
      const uint4 w = *reinterpret_cast<const uint4*>(gg + bb * E + a0);
      const float xb = to_f32<T>(x[xo + gi * E + bb]);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ws[i]));
        acc[2 * i] = fmaf(f.x, xb, acc[2 * i]);
        acc[2 * i + 1] = fmaf(f.y, xb, acc[2 * i + 1]);
      }
    }
#pragma unroll
    for (int off = LPR; off < 32; off <<= 1)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], off);
    if (r0 == 0) {
      float* o = dx + xo + gi * E + a0;
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = accumulate ? o[i] + factor * acc[i] : factor * acc[i];
    }
  }
}

// o = (o_loc * den_loc' + X) / D',  D = den_loc + y   (x' = x if x > 0 else 1);  XY (B*H, T, ldxy)
template <typename T>
__global__ void __launch_bounds__(NT) sp_combine_kernel(const T* __restrict__ oloc, const float* __restrict__ den,
                                                        const float* __restrict__ XY, T* __restrict__ o,
                                                        float* __restrict__ Dout, int B, int Tn, int H, int Dv,
                                                        int ldxy) {
  const int warp = (blockIdx.x * NT + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const long total = static_cast<long>(B) * Tn * H;
  if (warp >= total) return;
  const int h = warp % H, t = (warp / H) % Tn, b = warp / (H * Tn);
  const size_t row = (static_cast<size_t>(b) * Tn + t) * H + h;
  const float* xy = XY + ((static_cast<size_t>(b) * H + h) * Tn + t) * ldxy;
  const float dl = den[row];
  const float Dt = dl + xy[Dv];
  const float nl = dl > 0.f ? dl : 1.f;
  const float inv = 1.f / (Dt > 0.f ? Dt : 1.f);
  for (int c = lane; c < Dv; c += 32) o[row * Dv + c] = from_f32<T>((to_f32<T>(oloc[row * Dv + c]) * nl + xy[c]) * inv);
  if (lane == 0) Dout[row] = Dt;
}

// W1 (B*H, T, ldw) bf16 = [dO / D' | -delta / D' | 0...],  delta = <dO, o>
template <typename T>
__global__ void __launch_bounds__(NT) sp_bwd_prep_kernel(const T* __restrict__ o, const T* __restrict__ dout,
                                                         const float* __restrict__ Dn, __nv_bfloat16* __restrict__ W1,
                                                         int B, int Tn, int H, int Dv, int ldw) {
  const int warp = (blockIdx.x * NT + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const long total = static_cast<long>(B) * Tn * H;
  if (warp >= total) return;
  const int h = warp % H, t = (warp / H) % Tn, b = warp / (H * Tn);
  const size_t row = (static_cast<size_t>(b) * Tn + t) * H + h;
  __nv_bfloat16* w = W1 + ((static_cast<size_t>(b) * H + h) * Tn + t) * ldw;
  const float Dt = Dn[row];
  const float inv = 1.f / (Dt > 0.f ? Dt : 1.f);
  float delta = 0.f;
  for (int c = lane; c < Dv; c += 32) {
    const float g = to_f32<T>(dout[row * Dv + c]);
    delta = fmaf(g, to_f32<T>(o[row * Dv + c]), delta);
    w[c] = __float2bfloat16_rn(g * inv);
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) delta += __shfl_xor_sync(0xffffffffu, delta, off);
  for (int c = Dv + lane; c < ldw; c += 32) w[c] = __float2bfloat16_rn(c == Dv ? -delta * inv : 0.f);
}

template <typename T>
void launch_contract_vec(int E, unsigned blocks, cudaStream_t st, const __nv_bfloat16* g, const T* x, float* dx, int B,
                         int Tn, int H, int D, int M, float factor, int accumulate) {
  switch (E) {
    case 16: sp_contract_vec_kernel<T, 2><<<blocks, NT, 0, st>>>(g, x, dx, B, Tn, H, D, M, factor, accumulate); break;
    case 32: sp_contract_vec_kernel<T, 4><<<blocks, NT, 0, st>>>(g, x, dx, B, Tn, H, D, M, factor, accumulate); break;
    case 64: sp_contract_vec_kernel<T, 8><<<blocks, NT, 0, st>>>(g, x, dx, B, Tn, H, D, M, factor, accumulate); break;
    case 128: sp_contract_vec_kernel<T, 16><<<blocks, NT, 0, st>>>(g, x, dx, B, Tn, H, D, M, factor, accumulate); break;
    default: sp_contract_vec_kernel<T, 32><<<blocks, NT, 0, st>>>(g, x, dx, B, Tn, H, D, M, factor, accumulate); break;
  }
}

int check(int dtype, int B, int T, int H, int D, int M) {
  if (dtype != KATA_DTYPE_F32 && dtype != KATA_DTYPE_BF16 && dtype != KATA_DTYPE_F16) return KATA_ERR_DTYPE;
  if (B < 1 || T < 1 || H < 1 || D < 1 || M < 1 || D % M) return KATA_ERR_SHAPE;
  if ((D / M) % 8) return KATA_ERR_UNSUPPORTED;
  return KATA_OK;
}

unsigned warp_blocks(long warps) { return static_cast<unsigned>((warps * 32 + NT - 1) / NT); }

}  // namespace
}  // namespace kata

using namespace kata;

namespace kata {
namespace {
template <bool SUM>
int launch_features(const void* x, void* R, int dtype, int B, int T, int H, int D, int M, float scale,
                    kata_stream_t stream) {
  int e = check(dtype, B, T, H, D, M);
  if (e) return e;
  if (!x || !R) return KATA_ERR_INVALID;
  if (reinterpret_cast<uintptr_t>(R) % 16) return KATA_ERR_ALIGN;
  if (sizeof(float) * TOK * D > 48 * 1024) return KATA_ERR_UNSUPPORTED;  // the CTA's rows of x in shared memory
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const dim3 grid((T + TOK - 1) / TOK, B * H);
  const size_t smem = sizeof(float) * TOK * D;
  auto* r = static_cast<__nv_bfloat16*>(R);
  switch (dtype) {
    case KATA_DTYPE_F32: sp_features_kernel<float, SUM><<<grid, NT, smem, st>>>(static_cast<const float*>(x), r, B, T, H, D, M, scale); break;
    case KATA_DTYPE_BF16: sp_features_kernel<__nv_bfloat16, SUM><<<grid, NT, smem, st>>>(static_cast<const __nv_bfloat16*>(x), r, B, T, H, D, M, scale); break;
    default: sp_features_kernel<__half, SUM><<<grid, NT, smem, st>>>(static_cast<const __half*>(x), r, B, T, H, D, M, scale); break;
  }
  return from_cuda(cudaGetLastError());
}
}  // namespace
}  // namespace kata

extern "C" int kata_sp_features(const void* x, void* R, int dtype, int B, int T, int H, int D, int M, float scale,
                                kata_stream_t stream) {
  return launch_features<false>(x, R, dtype, B, T, H, D, M, scale, stream);
}

extern "C" int kata_sum_features(const void* x, void* R, int dtype, int B, int T, int H, int D, int M, float scale,
                                 kata_stream_t stream) {
  return launch_features<true>(x, R, dtype, B, T, H, D, M, scale, stream);
}

extern "C" int kata_sp_contract(const void* G, const void* x, float* dx, int dtype, int B, int T, int H, int D, int M,
                                float factor, int accumulate, kata_stream_t stream) {
  int e = check(dtype, B, T, H, D, M);
  if (e) return e;
  if (!G || !x || !dx) return KATA_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const unsigned blocks = warp_blocks(static_cast<long>(B) * H * T);
  const auto* g = static_cast<const __nv_bfloat16*>(G);
  const int E = D / M;
  if (E == 16 || E == 32 || E == 64 || E == 128 || E == 256) {
    if (reinterpret_cast<uintptr_t>(G) % 16) return KATA_ERR_ALIGN;
    switch (dtype) {
      case KATA_DTYPE_F32: launch_contract_vec<float>(E, blocks, st, g, static_cast<const float*>(x), dx, B, T, H, D, M, factor, accumulate); break;
      case KATA_DTYPE_BF16: launch_contract_vec<__nv_bfloat16>(E, blocks, st, g, static_cast<const __nv_bfloat16*>(x), dx, B, T, H, D, M, factor, accumulate); break;
      default: launch_contract_vec<__half>(E, blocks, st, g, static_cast<const __half*>(x), dx, B, T, H, D, M, factor, accumulate); break;
    }
    return from_cuda(cudaGetLastError());
  }
  switch (dtype) {
    case KATA_DTYPE_F32: sp_contract_kernel<float><<<blocks, NT, 0, st>>>(g, static_cast<const float*>(x), dx, B, T, H, D, M, factor, accumulate); break;
    case KATA_DTYPE_BF16: sp_contract_kernel<__nv_bfloat16><<<blocks, NT, 0, st>>>(g, static_cast<const __nv_bfloat16*>(x), dx, B, T, H, D, M, factor, accumulate); break;
    default: sp_contract_kernel<__half><<<blocks, NT, 0, st>>>(g, static_cast<const __half*>(x), dx, B, T, H, D, M, factor, accumulate); break;
  }
  return from_cuda(cudaGetLastError());
}

extern "C" int kata_sp_combine(const void* o_local, const float* den_local, const float* XY, void* o, float* D_out,
                               int dtype, int B, int T, int H, int Dv, int ldxy, kata_stream_t stream) {
  if (dtype != KATA_DTYPE_F32 && dtype != KATA_DTYPE_BF16 && dtype != KATA_DTYPE_F16) return KATA_ERR_DTYPE;
  if (B < 1 || T < 1 || H < 1 || Dv < 1 || ldxy < Dv + 1) return KATA_ERR_SHAPE;
  if (!o_local || !den_local || !XY || !o || !D_out) return KATA_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const unsigned blocks = warp_blocks(static_cast<long>(B) * H * T);
  switch (dtype) {
    case KATA_DTYPE_F32: sp_combine_kernel<float><<<blocks, NT, 0, st>>>(static_cast<const float*>(o_local), den_local, XY, static_cast<float*>(o), D_out, B, T, H, Dv, ldxy); break;
    case KATA_DTYPE_BF16: sp_combine_kernel<__nv_bfloat16><<<blocks, NT, 0, st>>>(static_cast<const __nv_bfloat16*>(o_local), den_local, XY, static_cast<__nv_bfloat16*>(o), D_out, B, T, H, Dv, ldxy); break;
    default: sp_combine_kernel<__half><<<blocks, NT, 0, st>>>(static_cast<const __half*>(o_local), den_local, XY, static_cast<__half*>(o), D_out, B, T, H, Dv, ldxy); break;
  }
  return from_cuda(cudaGetLastError());
}

extern "C" int kata_sp_bwd_prep(const void* o, const void* dout, const float* D_in, void* W1, int dtype, int B, int T,
                                int H, int Dv, int ldw, kata_stream_t stream) {
  if (dtype != KATA_DTYPE_F32 && dtype != KATA_DTYPE_BF16 && dtype != KATA_DTYPE_F16) return KATA_ERR_DTYPE;
  if (B < 1 || T < 1 || H < 1 || Dv < 1 || ldw < Dv + 1) return KATA_ERR_SHAPE;
  if (!o || !dout || !D_in || !W1) return KATA_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const unsigned blocks = warp_blocks(static_cast<long>(B) * H * T);
  auto* w = static_cast<__nv_bfloat16*>(W1);
  switch (dtype) {
    case KATA_DTYPE_F32: sp_bwd_prep_kernel<float><<<blocks, NT, 0, st>>>(static_cast<const float*>(o), static_cast<const float*>(dout), D_in, w, B, T, H, Dv, ldw); break;
    case KATA_DTYPE_BF16: sp_bwd_prep_kernel<__nv_bfloat16><<<blocks, NT, 0, st>>>(static_cast<const __nv_bfloat16*>(o), static_cast<const __nv_bfloat16*>(dout), D_in, w, B, T, H, Dv, ldw); break;
    default: sp_bwd_prep_kernel<__half><<<blocks, NT, 0, st>>>(static_cast<const __half*>(o), static_cast<const __half*>(dout), D_in, w, B, T, H, Dv, ldw); break;
  }
  return from_cuda(cudaGetLastError());
}
