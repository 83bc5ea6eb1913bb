// decode.cu -- one-token decode step of causal KATA-SPD attention (concat score) on the
// feature state.
//
// With psi(x)[g,a,b] = scale * x_{g,a} x_{g,b} (F = M E^2 features, E = D/M), A[t,s] =
// psi(q_t).psi(k_s), so every prefix of keys is summarised by the state
//   S = sum_s psi(k_s) [v_s | 1]          (F x lds fp32 per (batch, head); columns >= Dv+1 zero)
// and the token that follows it has  o = X / y',  [X | y] = psi(q)^T (S + psi(k) [v | 1]),
// y' = y if y > 0 else 1 -- the row of the full causal attention for that token.
//
// The step is one pass over the state, HBM-bound at 2 * F * lds * 4 bytes per (batch, head):
// every CTA owns a chunk of rows of one head, reads each 16-byte column group once, adds the
// rank-1 update, writes it back and accumulates psi(q)^T S_new for its columns.  The chunk
// partials go to a workspace; the last CTA of a head (an atomic ticket, no waiting) adds them in
// chunk order -- so the result does not depend on CTA scheduling -- and writes o and y.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "attn_common.cuh"
#include "host_util.h"
#include "kata_b200.h"

namespace kata {
namespace {

constexpr int DNT = 256;     // threads per CTA
constexpr int DUNROLL = 4;   // row groups per thread per iteration; the next group's loads are in flight meanwhile

struct DecodeGeom {
  int F, cols4, rpi, chunk_rows, nchunk;
};

// Rows per CTA.  A state above 128 MB streams from HBM: ~16 CTAs per SM over the whole grid
// (several waves, so the last partial wave costs little), at least 32 rows each.  A smaller one is
// latency-bound: one wave of 4 CTAs per SM (the kernel's occupancy at 256 threads), at least 64
// rows each.  Measured on B200 against coarser and finer grids and deeper unrolling.
inline DecodeGeom decode_geom(int B, int H, int D, int M, int lds) {
  DecodeGeom g;
  const int E = D / M;
  g.F = M * E * E;
  g.cols4 = lds / 4;
  g.rpi = DNT / g.cols4;
  const long rows = static_cast<long>(B) * H * g.F;
  const bool big = rows * lds * 4 > (128L << 20);
  long cr;
  if (big) {
    cr = (rows + 148L * 16 - 1) / (148L * 16);
    if (cr < 32) cr = 32;
  } else {
    long n = 592L / (static_cast<long>(B) * H);
    if (n < 1) n = 1;
    cr = (g.F + n - 1) / n;
    if (cr < 64) cr = 64;
  }
  if (cr > g.F) cr = g.F;
  g.chunk_rows = static_cast<int>(cr);
  g.nchunk = (g.F + g.chunk_rows - 1) / g.chunk_rows;
  return g;
}

// work: tickets (B*H) int32, then (16-byte aligned) partials (B*H, nchunk, lds) fp32.
template <typename T>
__global__ void __launch_bounds__(DNT) decode_step_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                          const T* __restrict__ v, float* __restrict__ S,
                                                          T* __restrict__ o, float* __restrict__ den,
                                                          float* __restrict__ part, int* __restrict__ ticket, int H,
                                                          int D, int Dv, int M, int lds, float scale,
                                                          DecodeGeom geo) {
  extern __shared__ float sm[];
  float* qs = sm;              // D
  float* ks = qs + D;          // D
  float* red = ks + D;         // rpi x lds
  __shared__ int last;
  const int bh = blockIdx.y, chunk = blockIdx.x, tid = threadIdx.x;
  const int E = D / M, EE = E * E;
  const size_t xo = static_cast<size_t>(bh) * D;
  for (int i = tid; i < D; i += DNT) {
    qs[i] = to_f32<T>(q[xo + i]);
    ks[i] = to_f32<T>(k[xo + i]);
  }
  const int c4 = tid % geo.cols4, r = tid / geo.cols4;
  const bool active = r < geo.rpi;
  // this thread's 4 columns of [v | 1 | 0 ...]
  float v1[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int c = 4 * c4 + j;
    v1[j] = c < Dv ? to_f32<T>(v[static_cast<size_t>(bh) * Dv + c]) : (c == Dv ? 1.f : 0.f);
  }
  __syncthreads();

  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  const int f0 = chunk * geo.chunk_rows;
  const int f1 = min(f0 + geo.chunk_rows, geo.F);
  float* Sh = S + static_cast<size_t>(bh) * geo.F * lds;
  if (active) {
    const int step = DUNROLL * geo.rpi;
    float4 s[DUNROLL], nx[DUNROLL];
#pragma unroll
    for (int u = 0; u < DUNROLL; ++u) {
      const int f = f0 + r + u * geo.rpi;
      if (f < f1) s[u] = *reinterpret_cast<const float4*>(Sh + static_cast<size_t>(f) * lds + 4 * c4);
    }
    for (int fb = f0 + r; fb < f1; fb += step) {
#pragma unroll
      for (int u = 0; u < DUNROLL; ++u) {
        const int f = fb + step + u * geo.rpi;
        if (f < f1) nx[u] = *reinterpret_cast<const float4*>(Sh + static_cast<size_t>(f) * lds + 4 * c4);
      }
#pragma unroll
      for (int u = 0; u < DUNROLL; ++u) {
        const int f = fb + u * geo.rpi;
        if (f < f1) {
          const int g = f / EE, rem = f - g * EE, a = rem / E, b = rem - a * E;
          const int ia = g * E + a, ib = g * E + b;
          const float pk = scale * (ks[ia] * ks[ib]);
          const float pq = scale * (qs[ia] * qs[ib]);
          s[u].x = fmaf(pk, v1[0], s[u].x);
          s[u].y = fmaf(pk, v1[1], s[u].y);
          s[u].z = fmaf(pk, v1[2], s[u].z);
          s[u].w = fmaf(pk, v1[3], s[u].w);
          *reinterpret_cast<float4*>(Sh + static_cast<size_t>(f) * lds + 4 * c4) = s[u];
          acc[0] = fmaf(pq, s[u].x, acc[0]);
          acc[1] = fmaf(pq, s[u].y, acc[1]);
          acc[2] = fmaf(pq, s[u].z, acc[2]);
          acc[3] = fmaf(pq, s[u].w, acc[3]);
        }
        s[u] = nx[u];
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) red[r * lds + 4 * c4 + j] = acc[j];
  }
  __syncthreads();
  float* pp = part + (static_cast<size_t>(bh) * geo.nchunk + chunk) * lds;
  for (int c = tid; c < lds; c += DNT) {
    float t = 0.f;
    for (int i = 0; i < geo.rpi; ++i) t += red[i * lds + c];
    pp[c] = t;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int prev = atomicAdd(ticket + bh, 1);
    last = prev == geo.nchunk - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  const float* ph = part + static_cast<size_t>(bh) * geo.nchunk * lds;
  // y first (every thread needs it), then X / y'
  float y = 0.f;
  for (int i = 0; i < geo.nchunk; ++i) y += __ldcg(ph + static_cast<size_t>(i) * lds + Dv);
  const float inv = 1.f / (y > 0.f ? y : 1.f);
  for (int c = tid; c < Dv; c += DNT) {
    float x = 0.f;
    for (int i = 0; i < geo.nchunk; ++i) x += __ldcg(ph + static_cast<size_t>(i) * lds + c);
    o[static_cast<size_t>(bh) * Dv + c] = from_f32<T>(x * inv);
  }
  if (tid == 0) {
    if (den) den[bh] = y;
    ticket[bh] = 0;  // ready for the next step on this workspace
  }
}

inline size_t decode_ticket_bytes(int B, int H) { return (static_cast<size_t>(B) * H * sizeof(int) + 15) / 16 * 16; }

int decode_check(int dtype, int B, int H, int D, int Dv, int M, int lds) {
  if (dtype != KATA_DTYPE_F32 && dtype != KATA_DTYPE_BF16 && dtype != KATA_DTYPE_F16) return KATA_ERR_DTYPE;
  if (B < 1 || H < 1 || D < 1 || Dv < 1 || M < 1 || D % M) return KATA_ERR_SHAPE;
  if (lds < Dv + 1 || lds % 4 || lds / 4 > DNT) return KATA_ERR_SHAPE;
  if (D > 2048) return KATA_ERR_UNSUPPORTED;  // q and k rows are staged in shared memory
  if (static_cast<long>(B) * H > 65535) return KATA_ERR_UNSUPPORTED;  // (batch, head) is the grid's y
  return KATA_OK;
}

}  // namespace
}  // namespace kata

using namespace kata;

extern "C" size_t kata_decode_workspace_bytes(int B, int H, int D, int Dv, int M, int lds) {
  if (decode_check(KATA_DTYPE_F32, B, H, D, Dv, M, lds)) return 0;
  const DecodeGeom g = decode_geom(B, H, D, M, lds);
  const size_t bh = static_cast<size_t>(B) * H;
  return decode_ticket_bytes(B, H) + bh * g.nchunk * lds * sizeof(float);
}

extern "C" int kata_decode_step(const void* q, const void* k, const void* v, float* state, void* o, float* den,
                                void* work, int dtype, int B, int H, int D, int Dv, int M, int lds, float scale,
                                kata_stream_t stream) {
  int e = decode_check(dtype, B, H, D, Dv, M, lds);
  if (e) return e;
  if (!q || !k || !v || !state || !o || !work) return KATA_ERR_INVALID;
  if (reinterpret_cast<uintptr_t>(state) % 16 || reinterpret_cast<uintptr_t>(work) % 16) return KATA_ERR_ALIGN;
  const DecodeGeom g = decode_geom(B, H, D, M, lds);
  int* ticket = static_cast<int*>(work);
  float* part = reinterpret_cast<float*>(static_cast<char*>(work) + decode_ticket_bytes(B, H));
  const dim3 grid(g.nchunk, B * H);
  const size_t smem = sizeof(float) * (2 * D + g.rpi * lds);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case KATA_DTYPE_F32:
      decode_step_kernel<float><<<grid, DNT, smem, st>>>(static_cast<const float*>(q), static_cast<const float*>(k),
                                                          static_cast<const float*>(v), state, static_cast<float*>(o),
                                                          den, part, ticket, H, D, Dv, M, lds, scale, g);
      break;
    case KATA_DTYPE_BF16:
      decode_step_kernel<__nv_bfloat16><<<grid, DNT, smem, st>>>(
          static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
          static_cast<const __nv_bfloat16*>(v), state, static_cast<__nv_bfloat16*>(o), den, part, ticket, H, D, Dv, M,
          lds, scale, g);
      break;
    default:
      decode_step_kernel<__half><<<grid, DNT, smem, st>>>(static_cast<const __half*>(q), static_cast<const __half*>(k),
                                                           static_cast<const __half*>(v), state, static_cast<__half*>(o),
                                                           den, part, ticket, H, D, Dv, M, lds, scale, g);
      break;
  }
  return from_cuda(cudaGetLastError());
}
