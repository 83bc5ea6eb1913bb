// decode.cu -- one-token decode step of causal KATA-SPD attention on the feature state.
//
// Both scores are inner products of quadratic features, A[t,s] = psi(q_t).psi(k_s):
//   concat  A = sum_g (scale q_g.k_g)^2      psi(x)[g,a,b] = scale x_{g,a} x_{g,b}      F = M E^2
//   sum     A = sum_{g,h} (scale q_g.k_h)^2  psi(x)[a,b]   = scale sum_g x_{g,a} x_{g,b}  F = E^2
// (E = D/M), so every prefix of keys is summarised by the state
//   S = sum_s w_s psi(k_s) [v_s | 1]          (F x lds fp32; columns >= Dv+1 zero)
// with w_s = 1, or w_s = exp(c_t - c_s) under a per-token log-decay g_t = c_t - c_{t-1} <= 0, and
// the token that follows has  o = X / y',  [X | y] = psi(q)^T S_t,  S_t = exp(g_t) S + psi(k)[v|1],
// y' = y if y > 0 else 1 -- its row of the full causal attention.
//
// Without decay one state serves the G = HQ/H query heads of a key/value head; with decay the
// state is per query head (its decay differs).  The step is one pass over the state, HBM-bound at
// 2 * F * lds * 4 bytes per state: every CTA owns a chunk of rows of one state, reads each 16-byte
// column group once, applies the update, writes it back and accumulates psi(q_j)^T S_t for its
// columns and each of its query heads j.  The loads of the next group of rows are in flight while
// the current group is stored.  Chunk partials go to a workspace; the last CTA of a state (an
// atomic ticket, no waiting) adds them in chunk order -- the result does not depend on CTA
// scheduling -- and writes o and y.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "attn_common.cuh"
#include "host_util.h"
#include "kata_b200.h"

namespace kata {
namespace {

constexpr int DNT = 256;    // threads per CTA
constexpr int DUNROLL = 4;  // row groups per thread per iteration; the next group's loads are in flight meanwhile

struct DecodeGeom {
  int F, cols4, rpi, chunk_rows, nchunk;
};

// Rows per CTA.  A state above 128 MB streams from HBM: ~16 CTAs per SM over the whole grid
// (several waves, so the last partial wave costs little), at least 32 rows each.  A smaller one is
// latency-bound: one wave of 4 CTAs per SM, at least 64 rows each.  Measured on B200 against
// coarser and finer grids and deeper unrolling.
inline DecodeGeom decode_geom(long nstate, int F, int lds) {
  DecodeGeom g;
  g.F = F;
  g.cols4 = lds / 4;
  g.rpi = DNT / g.cols4;
  const long rows = nstate * F;
  const bool big = rows * lds * 4 > (128L << 20);
  long cr;
  if (big) {
    cr = (rows + 148L * 16 - 1) / (148L * 16);
    if (cr < 32) cr = 32;
  } else {
    long n = 592L / nstate;
    if (n < 1) n = 1;
    cr = (F + n - 1) / n;
    if (cr < 64) cr = 64;
  }
  if (cr > F) cr = F;
  g.chunk_rows = static_cast<int>(cr);
  g.nchunk = (F + g.chunk_rows - 1) / g.chunk_rows;
  return g;
}

template <bool SUM>
__device__ __forceinline__ float feature(const float* x, int f, int E, int M, float scale) {
  if constexpr (SUM) {
    const int a = f / E, b = f - a * E;
    float t = 0.f;
    for (int g = 0; g < M; ++g) t = fmaf(x[g * E + a], x[g * E + b], t);
    return scale * t;
  } else {
    const int EE = E * E, g = f / EE, rem = f - g * EE, a = rem / E, b = rem - a * E;
    return scale * (x[g * E + a] * x[g * E + b]);
  }
}

struct DecodeParams {
  const float* gate;  // (B, HQ) log-decay or nullptr
  float* S;
  float* den;
  float* part;
  int* ticket;
  int HQ, H, HS, D, Dv, M, lds;
  float scale;
};

// work: tickets (B*HS) int32, then (16-byte aligned) partials (B*HS, nchunk, G, lds) fp32.
// One or two query heads per state: capped at 64 registers, so 4 CTAs fit on an SM.
template <typename T, bool SUM, int G>
__global__ void __launch_bounds__(DNT, G <= 2 ? 4 : 2) decode_step_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                          const T* __restrict__ v, T* __restrict__ o, DecodeParams p,
                                                          DecodeGeom geo) {
  extern __shared__ float sm[];
  float* qs = sm;            // G x D
  float* ks = qs + G * p.D;  // D
  float* red = ks + p.D;     // G x rpi x lds
  __shared__ int last;
  const int bs = blockIdx.y, chunk = blockIdx.x, tid = threadIdx.x;
  const int b = bs / p.HS, hs = bs - b * p.HS;
  // decay: one query head per state; otherwise the G query heads of key/value head hs
  const int kh = p.gate ? hs / (p.HQ / p.H) : hs;
  const int qh0 = p.gate ? hs : hs * G;
  const int E = p.D / p.M;
  for (int i = tid; i < p.D; i += DNT) {
#pragma unroll
    for (int j = 0; j < G; ++j) qs[j * p.D + i] = to_f32<T>(q[(static_cast<size_t>(b) * p.HQ + qh0 + j) * p.D + i]);
    ks[i] = to_f32<T>(k[(static_cast<size_t>(b) * p.H + kh) * p.D + i]);
  }
  const int c4 = tid % geo.cols4, r = tid / geo.cols4;
  const bool active = r < geo.rpi;
  float v1[4];  // this thread's 4 columns of [v | 1 | 0 ...]
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int c = 4 * c4 + j;
    v1[j] = c < p.Dv ? to_f32<T>(v[(static_cast<size_t>(b) * p.H + kh) * p.Dv + c]) : (c == p.Dv ? 1.f : 0.f);
  }
  const float a = p.gate ? expf(p.gate[static_cast<size_t>(b) * p.HQ + hs]) : 1.f;
  __syncthreads();

  float acc[G][4];
#pragma unroll
  for (int j = 0; j < G; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
  const int f0 = chunk * geo.chunk_rows;
  const int f1 = min(f0 + geo.chunk_rows, geo.F);
  float* Sh = p.S + static_cast<size_t>(bs) * geo.F * p.lds;
  if (active) {
    const int step = DUNROLL * geo.rpi;
    float4 s[DUNROLL], nx[DUNROLL];
#pragma unroll
    for (int u = 0; u < DUNROLL; ++u) {
      const int f = f0 + r + u * geo.rpi;
      if (f < f1) s[u] = *reinterpret_cast<const float4*>(Sh + static_cast<size_t>(f) * p.lds + 4 * c4);
    }
    for (int fb = f0 + r; fb < f1; fb += step) {
#pragma unroll
      for (int u = 0; u < DUNROLL; ++u) {
        const int f = fb + step + u * geo.rpi;
        if (f < f1) nx[u] = *reinterpret_cast<const float4*>(Sh + static_cast<size_t>(f) * p.lds + 4 * c4);
      }
#pragma unroll
      for (int u = 0; u < DUNROLL; ++u) {
        const int f = fb + u * geo.rpi;
        if (f < f1) {
          const float pk = feature<SUM>(ks, f, E, p.M, p.scale);
          s[u].x = fmaf(pk, v1[0], a * s[u].x);
          s[u].y = fmaf(pk, v1[1], a * s[u].y);
          s[u].z = fmaf(pk, v1[2], a * s[u].z);
          s[u].w = fmaf(pk, v1[3], a * s[u].w);
          *reinterpret_cast<float4*>(Sh + static_cast<size_t>(f) * p.lds + 4 * c4) = s[u];
#pragma unroll
          for (int j = 0; j < G; ++j) {
            const float pq = feature<SUM>(qs + j * p.D, f, E, p.M, p.scale);
            acc[j][0] = fmaf(pq, s[u].x, acc[j][0]);
            acc[j][1] = fmaf(pq, s[u].y, acc[j][1]);
            acc[j][2] = fmaf(pq, s[u].z, acc[j][2]);
            acc[j][3] = fmaf(pq, s[u].w, acc[j][3]);
          }
        }
        s[u] = nx[u];
      }
    }
#pragma unroll
    for (int j = 0; j < G; ++j)
#pragma unroll
      for (int i = 0; i < 4; ++i) red[(j * geo.rpi + r) * p.lds + 4 * c4 + i] = acc[j][i];
  }
  __syncthreads();
  float* pp = p.part + (static_cast<size_t>(bs) * geo.nchunk + chunk) * G * p.lds;
  for (int c = tid; c < G * p.lds; c += DNT) {
    const int j = c / p.lds, cc = c - j * p.lds;
    float t = 0.f;
    for (int i = 0; i < geo.rpi; ++i) t += red[(j * geo.rpi + i) * p.lds + cc];
    pp[c] = t;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int prev = atomicAdd(p.ticket + bs, 1);
    last = prev == geo.nchunk - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  const float* ph = p.part + static_cast<size_t>(bs) * geo.nchunk * G * p.lds;
  const size_t cstride = static_cast<size_t>(G) * p.lds;
#pragma unroll
  for (int j = 0; j < G; ++j) {
    float y = 0.f;  // every thread needs y; then X / y'
    for (int i = 0; i < geo.nchunk; ++i) y += __ldcg(ph + i * cstride + j * p.lds + p.Dv);
    const float inv = 1.f / (y > 0.f ? y : 1.f);
    const size_t orow = static_cast<size_t>(b) * p.HQ + qh0 + j;
    for (int c = tid; c < p.Dv; c += DNT) {
      float x = 0.f;
      for (int i = 0; i < geo.nchunk; ++i) x += __ldcg(ph + i * cstride + j * p.lds + c);
      o[orow * p.Dv + c] = from_f32<T>(x * inv);
    }
    if (tid == 0 && p.den) p.den[orow] = y;
  }
  if (tid == 0) p.ticket[bs] = 0;  // ready for the next step on this workspace
}

inline size_t decode_ticket_bytes(long nstate) { return (static_cast<size_t>(nstate) * sizeof(int) + 15) / 16 * 16; }

struct DecodeShape {
  int G, HS, F;
  long nstate;
};

int decode_check(const kata_decode_args* a, DecodeShape* sh) {
  if (!a) return KATA_ERR_INVALID;
  if (a->dtype != KATA_DTYPE_F32 && a->dtype != KATA_DTYPE_BF16 && a->dtype != KATA_DTYPE_F16) return KATA_ERR_DTYPE;
  if (a->score != KATA_SCORE_CONCAT && a->score != KATA_SCORE_SUM) return KATA_ERR_INVALID;
  if (a->B < 1 || a->H < 1 || a->HQ < a->H || a->HQ % a->H || a->D < 1 || a->Dv < 1 || a->M < 1 || a->D % a->M)
    return KATA_ERR_SHAPE;
  if (a->lds < a->Dv + 1 || a->lds % 4 || a->lds / 4 > DNT) return KATA_ERR_SHAPE;
  if (a->D > 256) return KATA_ERR_UNSUPPORTED;  // q and k rows are staged in shared memory
  const int G = a->g ? 1 : a->HQ / a->H;
  if (G != 1 && G != 2 && G != 4 && G != 8) return KATA_ERR_UNSUPPORTED;
  const int E = a->D / a->M;
  sh->G = G;
  sh->HS = a->g ? a->HQ : a->H;
  sh->F = a->score == KATA_SCORE_SUM ? E * E : a->M * E * E;
  sh->nstate = static_cast<long>(a->B) * sh->HS;
  if (sh->nstate > 65535) return KATA_ERR_UNSUPPORTED;  // the states are the grid's y
  return KATA_OK;
}

template <typename T, bool SUM, int G>
void launch(const kata_decode_args* a, const DecodeShape& sh, const DecodeGeom& geo, cudaStream_t st) {
  DecodeParams p;
  p.gate = a->g;
  p.S = a->state;
  p.den = a->den;
  p.ticket = static_cast<int*>(a->work);
  p.part = reinterpret_cast<float*>(static_cast<char*>(a->work) + decode_ticket_bytes(sh.nstate));
  p.HQ = a->HQ;
  p.H = a->H;
  p.HS = sh.HS;
  p.D = a->D;
  p.Dv = a->Dv;
  p.M = a->M;
  p.lds = a->lds;
  p.scale = a->scale;
  const dim3 grid(geo.nchunk, static_cast<unsigned>(sh.nstate));
  const size_t smem = sizeof(float) * ((G + 1) * a->D + G * geo.rpi * a->lds);
  decode_step_kernel<T, SUM, G><<<grid, DNT, smem, st>>>(static_cast<const T*>(a->q), static_cast<const T*>(a->k),
                                                         static_cast<const T*>(a->v), static_cast<T*>(a->o), p, geo);
}

template <typename T, bool SUM>
void launch_g(const kata_decode_args* a, const DecodeShape& sh, const DecodeGeom& geo, cudaStream_t st) {
  switch (sh.G) {
    case 1: launch<T, SUM, 1>(a, sh, geo, st); break;
    case 2: launch<T, SUM, 2>(a, sh, geo, st); break;
    case 4: launch<T, SUM, 4>(a, sh, geo, st); break;
    default: launch<T, SUM, 8>(a, sh, geo, st); break;
  }
}

template <typename T>
void launch_t(const kata_decode_args* a, const DecodeShape& sh, const DecodeGeom& geo, cudaStream_t st) {
  if (a->score == KATA_SCORE_SUM)
    launch_g<T, true>(a, sh, geo, st);
  else
    launch_g<T, false>(a, sh, geo, st);
}

}  // namespace
}  // namespace kata

using namespace kata;

extern "C" size_t kata_decode_workspace_bytes(const kata_decode_args* a) {
  DecodeShape sh;
  if (decode_check(a, &sh)) return 0;
  const DecodeGeom g = decode_geom(sh.nstate, sh.F, a->lds);
  return decode_ticket_bytes(sh.nstate) + static_cast<size_t>(sh.nstate) * g.nchunk * sh.G * a->lds * sizeof(float);
}

extern "C" int kata_decode_step(const kata_decode_args* a, kata_stream_t stream) {
  DecodeShape sh;
  int e = decode_check(a, &sh);
  if (e) return e;
  if (!a->q || !a->k || !a->v || !a->state || !a->o || !a->work) return KATA_ERR_INVALID;
  if (reinterpret_cast<uintptr_t>(a->state) % 16 || reinterpret_cast<uintptr_t>(a->work) % 16) return KATA_ERR_ALIGN;
  const DecodeGeom g = decode_geom(sh.nstate, sh.F, a->lds);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (a->dtype) {
    case KATA_DTYPE_F32: launch_t<float>(a, sh, g, st); break;
    case KATA_DTYPE_BF16: launch_t<__nv_bfloat16>(a, sh, g, st); break;
    default: launch_t<__half>(a, sh, g, st); break;
  }
  return from_cuda(cudaGetLastError());
}
