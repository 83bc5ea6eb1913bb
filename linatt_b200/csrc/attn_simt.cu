// attn_simt.cu -- fp32-exact CUDA-core kernels for causal KATA-SPD attention (all variants).
//
// These kernels are the fp32-accurate mode (fp32 inputs, rel-L2 <= 1e-5 against the reference)
// and cover every shape the tensor-core kernels do not: any D, Dv <= 256, concat or sum score,
// optional decay, GQA.  Math follows kata/kernels/parallel_kata.py (K1 :10-197, K2 :202-345)
// for the forward and kata/parallel_kata_attn.py:49-146 / :579-653 / :291-347 for the backward,
// computed in fp32 throughout (inputs of any float dtype are widened on load).
#include "attn_common.cuh"
#include "host_util.h"

namespace kata {
namespace {

constexpr int BQ = 32;    // query rows per CTA
constexpr int BS = 32;    // keys per inner tile
constexpr int NTH = 256;  // threads per CTA
constexpr int MAXP = 16;  // max score parts (M for concat, M*M for sum)

// ---------------------------------------------------------------------------------------------
// Shared helpers
// ---------------------------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ void load_rows(float* dst, int ld, const T* src, size_t row_stride, int row0, int nrows,
                                          int ncols, int T_) {
  for (int i = threadIdx.x; i < nrows * ncols; i += NTH) {
    const int r = i / ncols, c = i - r * ncols;
    const int t = row0 + r;
    dst[r * ld + c] = (t < T_) ? to_f32<T>(src[static_cast<size_t>(t) * row_stride + c]) : 0.f;
  }
}

// Score parts of one (query row, key row) pair.  qk[p] = scale * <q_a, k_b> for part p=(a,b):
// concat parts are (g,g); sum parts are (a,b) for all a,b (p = a*M + b).
template <bool SUM>
__device__ __forceinline__ void score_parts(const float* qr, const float* kr, int M, int E, float scale,
                                            float* qk) {
  if (!SUM) {
    for (int g = 0; g < M; ++g) {
      float d = 0.f;
      for (int e = 0; e < E; ++e) d = fmaf(qr[g * E + e], kr[g * E + e], d);
      qk[g] = d * scale;
    }
  } else {
    for (int a = 0; a < M; ++a)
      for (int b = 0; b < M; ++b) {
        float d = 0.f;
        for (int e = 0; e < E; ++e) d = fmaf(qr[a * E + e], kr[b * E + e], d);
        qk[a * M + b] = d * scale;
      }
  }
}

// ---------------------------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------------------------
template <typename T, bool SUM, bool DECAY>
__global__ void __launch_bounds__(NTH) attn_fwd_simt(AttnFwdParams p) {
  extern __shared__ float sm[];
  const int D = p.D, Dv = p.Dv, M = p.M, E = D / M, T_ = p.T;
  const int ldq = D + 1, ldv = Dv + 1, lda = BS + 1;
  float* sQ = sm;
  float* sK = sQ + BQ * ldq;
  float* sV = sK + BS * ldq;
  float* sA = sV + BS * ldv;
  float* sCq = sA + BQ * lda;
  float* sCk = sCq + BQ;

  const int nqt = (T_ + BQ - 1) / BQ;
  const int qt = nqt - 1 - blockIdx.x;  // heaviest query tiles first
  const int bh = blockIdx.y, b = bh / p.HQ, hq = bh % p.HQ, h = hq / p.G;
  const int t0 = qt * BQ;
  const T* q = static_cast<const T*>(p.q) + (static_cast<size_t>(b) * T_ * p.HQ + hq) * D;
  const T* k = static_cast<const T*>(p.k) + (static_cast<size_t>(b) * T_ * p.H + h) * D;
  const T* v = static_cast<const T*>(p.v) + (static_cast<size_t>(b) * T_ * p.H + h) * Dv;
  const float* c = DECAY ? p.c + static_cast<size_t>(b) * T_ * p.HQ + hq : nullptr;
  const size_t sq = static_cast<size_t>(p.HQ) * D, sk = static_cast<size_t>(p.H) * D,
               sv = static_cast<size_t>(p.H) * Dv;

  load_rows<T>(sQ, ldq, q, sq, t0, BQ, D, T_);
  if (DECAY)
    for (int i = threadIdx.x; i < BQ; i += NTH) sCq[i] = (t0 + i < T_) ? c[static_cast<size_t>(t0 + i) * p.HQ] : 0.f;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int orow = tid >> 3, ocol = tid & 7;  // output ownership: row, column phase
  const int nu = Dv / 8;
  float oacc[32];
#pragma unroll
  for (int u = 0; u < 32; ++u) oacc[u] = 0.f;
  float den = 0.f;

  const int s_end = min(t0 + BQ, T_);
  for (int s0 = 0; s0 < s_end; s0 += BS) {
    __syncthreads();
    load_rows<T>(sK, ldq, k, sk, s0, BS, D, T_);
    load_rows<T>(sV, ldv, v, sv, s0, BS, Dv, T_);
    if (DECAY)
      for (int i = threadIdx.x; i < BS; i += NTH) sCk[i] = (s0 + i < T_) ? c[static_cast<size_t>(s0 + i) * p.HQ] : 0.f;
    __syncthreads();
    // scores: warp w handles rows w, w+8, w+16, w+24; lane = key
    for (int i = 0; i < BQ / 8; ++i) {
      const int r = warp + 8 * i, s = lane;
      float qk[MAXP];
      score_parts<SUM>(sQ + r * ldq, sK + s * ldq, M, E, p.scale, qk);
      const int np = SUM ? M * M : M;
      float a = 0.f;
      for (int j = 0; j < np; ++j) a = fmaf(qk[j], qk[j], a);
      const int t = t0 + r, sg = s0 + s;
      if (sg > t || sg >= T_) a = 0.f;
      if (DECAY) a *= __expf(fminf(sCq[r] - sCk[s], 0.f));
      sA[r * lda + s] = a;
    }
    __syncthreads();
    for (int s = 0; s < BS; ++s) {
      const float a = sA[orow * lda + s];
      den += a;
#pragma unroll
      for (int u = 0; u < 32; ++u)
        if (u < nu) oacc[u] = fmaf(a, sV[s * ldv + ocol + 8 * u], oacc[u]);
    }
  }
  const int t = t0 + orow;
  if (t < T_) {
    const float inv = 1.f / (den > 0.f ? den : 1.f);
    T* o = static_cast<T*>(p.o) + ((static_cast<size_t>(b) * T_ + t) * p.HQ + hq) * Dv;
#pragma unroll
    for (int u = 0; u < 32; ++u)
      if (u < nu) o[ocol + 8 * u] = from_f32<T>(oacc[u] * inv);
    if (ocol == 0) p.den[(static_cast<size_t>(b) * T_ + t) * p.HQ + hq] = den;
  }
}

// ---------------------------------------------------------------------------------------------
// Backward, pass 1: delta = <o, dO>, dq, and the row part of dc.
// W_p[t,s] = 2 * scale * qk_p * dec * dA   so that   dq_a[t] = sum_s sum_b W_(a,b)[t,s] k_b[s].
// ---------------------------------------------------------------------------------------------
template <typename T, bool SUM, bool DECAY>
__global__ void __launch_bounds__(NTH) attn_bwd_dq_simt(AttnBwdParams p) {
  extern __shared__ float sm[];
  const int D = p.D, Dv = p.Dv, M = p.M, E = D / M, T_ = p.T;
  const int NP = SUM ? M * M : M;
  const int ldq = D + 1, ldv = Dv + 1, lda = BS + 1;
  float* sQ = sm;
  float* sDO = sQ + BQ * ldq;
  float* sK = sDO + BQ * ldv;
  float* sV = sK + BS * ldq;
  float* sW = sV + BS * ldv;  // NP x BQ x lda
  float* sDelta = sW + NP * BQ * lda;
  float* sRden = sDelta + BQ;
  float* sCq = sRden + BQ;
  float* sCk = sCq + BQ;

  const int nqt = (T_ + BQ - 1) / BQ;
  const int qt = nqt - 1 - blockIdx.x;
  const int bh = blockIdx.y, b = bh / p.HQ, hq = bh % p.HQ, h = hq / p.G;
  const int t0 = qt * BQ;
  const size_t rowq = (static_cast<size_t>(b) * T_) * p.HQ + hq;  // + t*HQ
  const T* q = static_cast<const T*>(p.q) + rowq * D;
  const T* o = static_cast<const T*>(p.o) + rowq * Dv;
  const T* dO = static_cast<const T*>(p.dout) + rowq * Dv;
  const T* k = static_cast<const T*>(p.k) + (static_cast<size_t>(b) * T_ * p.H + h) * D;
  const T* v = static_cast<const T*>(p.v) + (static_cast<size_t>(b) * T_ * p.H + h) * Dv;
  const size_t sq = static_cast<size_t>(p.HQ) * D, sqv = static_cast<size_t>(p.HQ) * Dv,
               sk = static_cast<size_t>(p.H) * D, sv = static_cast<size_t>(p.H) * Dv;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  load_rows<T>(sQ, ldq, q, sq, t0, BQ, D, T_);
  load_rows<T>(sDO, ldv, dO, sqv, t0, BQ, Dv, T_);
  // delta_t = <o_t, dO_t>: warp w reduces rows w, w+8, ...
  for (int r = warp; r < BQ; r += 8) {
    const int t = t0 + r;
    float acc = 0.f;
    if (t < T_ && !p.delta_in)
      for (int j = lane; j < Dv; j += 32)
        acc = fmaf(to_f32<T>(o[static_cast<size_t>(t) * sqv + j]), to_f32<T>(dO[static_cast<size_t>(t) * sqv + j]), acc);
    for (int off = 16; off; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (t < T_ && p.delta_in) acc = p.delta_in[rowq + static_cast<size_t>(t) * p.HQ];
    if (lane == 0) {
      sDelta[r] = acc;
      float dn = (t < T_) ? p.den[rowq + static_cast<size_t>(t) * p.HQ] : 1.f;
      sRden[r] = 1.f / (dn > 0.f ? dn : 1.f);
      if (t < T_) p.delta[rowq + static_cast<size_t>(t) * p.HQ] = acc;
      if (DECAY) sCq[r] = (t < T_) ? p.c[rowq + static_cast<size_t>(t) * p.HQ] : 0.f;
    }
  }

  const int orow = tid >> 3, ocol = tid & 7, nu = D / 8;
  float dq[32];
#pragma unroll
  for (int u = 0; u < 32; ++u) dq[u] = 0.f;
  float rsum[BQ / 8];
#pragma unroll
  for (int i = 0; i < BQ / 8; ++i) rsum[i] = 0.f;

  const int s_end = min(t0 + BQ, T_);
  for (int s0 = 0; s0 < s_end; s0 += BS) {
    __syncthreads();
    load_rows<T>(sK, ldq, k, sk, s0, BS, D, T_);
    load_rows<T>(sV, ldv, v, sv, s0, BS, Dv, T_);
    if (DECAY)
      for (int i = threadIdx.x; i < BS; i += NTH)
        sCk[i] = (s0 + i < T_) ? p.c[rowq + static_cast<size_t>(s0 + i) * p.HQ] : 0.f;
    __syncthreads();
    for (int i = 0; i < BQ / 8; ++i) {
      const int r = warp + 8 * i, s = lane;
      const int t = t0 + r, sg = s0 + s;
      const bool valid = (sg <= t) && (sg < T_) && (t < T_);
      float qk[MAXP];
      score_parts<SUM>(sQ + r * ldq, sK + s * ldq, M, E, p.scale, qk);
      float dn = 0.f;
      for (int j = 0; j < Dv; ++j) dn = fmaf(sDO[r * ldv + j], sV[s * ldv + j], dn);
      float dA = valid ? (dn - sDelta[r]) * sRden[r] : 0.f;
      float dec = 1.f;
      if (DECAY) {
        const float x = sCq[r] - sCk[s];
        dec = __expf(fminf(x, 0.f));
        float a = 0.f;
        for (int j = 0; j < NP; ++j) a = fmaf(qk[j], qk[j], a);
        // G = dA * A over pairs whose clamp is inactive (c_t - c_s <= 0)
        if (valid && x <= 0.f) rsum[i] += dA * a * dec;
      }
      const float w = 2.f * p.scale * dec * dA;
      for (int j = 0; j < NP; ++j) sW[(j * BQ + r) * lda + s] = w * qk[j];
    }
    __syncthreads();
    // dq accumulation: thread owns row orow, columns ocol + 8u
    if (!SUM) {
      for (int s = 0; s < BS; ++s) {
#pragma unroll
        for (int u = 0; u < 32; ++u) {
          if (u < nu) {
            const int d = ocol + 8 * u;
            dq[u] = fmaf(sW[((d / E) * BQ + orow) * lda + s], sK[s * ldq + d], dq[u]);
          }
        }
      }
    } else {
      for (int s = 0; s < BS; ++s) {
        for (int bb = 0; bb < M; ++bb) {
#pragma unroll
          for (int u = 0; u < 32; ++u) {
            if (u < nu) {
              const int d = ocol + 8 * u, a = d / E, e = d - a * E;
              dq[u] = fmaf(sW[((a * M + bb) * BQ + orow) * lda + s], sK[s * ldq + bb * E + e], dq[u]);
            }
          }
        }
      }
    }
  }
  const int t = t0 + orow;
  if (t < T_) {
    T* dqp = static_cast<T*>(p.dq) + (rowq + static_cast<size_t>(t) * p.HQ) * D;
#pragma unroll
    for (int u = 0; u < 32; ++u)
      if (u < nu) dqp[ocol + 8 * u] = from_f32<T>(dq[u]);
  }
  if (DECAY) {
    // row sums: the 32 lanes of warp w hold partial sums of rows w+8i over 32 keys each
    for (int i = 0; i < BQ / 8; ++i) {
      float x = rsum[i];
      for (int off = 16; off; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
      const int tt = t0 + warp + 8 * i;
      if (lane == 0 && tt < T_) p.dc[rowq + static_cast<size_t>(tt) * p.HQ] = x;
    }
  }
}

// ---------------------------------------------------------------------------------------------
// Backward, pass 2: dk, dv (summed over the G query heads of a key/value head) and the column
// part of dc (dc_s -= sum_t G[t,s]).
// ---------------------------------------------------------------------------------------------
template <typename T, bool SUM, bool DECAY>
__global__ void __launch_bounds__(NTH) attn_bwd_dkdv_simt(AttnBwdParams p) {
  extern __shared__ float sm[];
  const int D = p.D, Dv = p.Dv, M = p.M, E = D / M, T_ = p.T;
  const int NP = SUM ? M * M : M;
  const int ldq = D + 1, ldv = Dv + 1, lda = BS + 1;
  float* sK = sm;
  float* sV = sK + BS * ldq;
  float* sQ = sV + BS * ldv;
  float* sDO = sQ + BQ * ldq;
  float* sW = sDO + BQ * ldv;  // NP x BQ x lda
  float* sP = sW + NP * BQ * lda;
  float* sDelta = sP + BQ * lda;
  float* sRden = sDelta + BQ;
  float* sCq = sRden + BQ;
  float* sCk = sCq + BQ;
  float* sCol = sCk + BS;  // 8 x BS partial column sums

  const int nkt = (T_ + BS - 1) / BS;
  const int kt = blockIdx.x;
  const int bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const int s0 = kt * BS;
  const T* k = static_cast<const T*>(p.k) + (static_cast<size_t>(b) * T_ * p.H + h) * D;
  const T* v = static_cast<const T*>(p.v) + (static_cast<size_t>(b) * T_ * p.H + h) * Dv;
  const size_t sk = static_cast<size_t>(p.H) * D, sv = static_cast<size_t>(p.H) * Dv;
  const size_t sq = static_cast<size_t>(p.HQ) * D, sqv = static_cast<size_t>(p.HQ) * Dv;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  (void)nkt;

  load_rows<T>(sK, ldq, k, sk, s0, BS, D, T_);
  load_rows<T>(sV, ldv, v, sv, s0, BS, Dv, T_);

  const int orow = tid >> 3, ocol = tid & 7, nuk = D / 8, nuv = Dv / 8;
  float dk[32], dv[32];
#pragma unroll
  for (int u = 0; u < 32; ++u) dk[u] = dv[u] = 0.f;

  for (int gq = 0; gq < p.G; ++gq) {
    const int hq = h * p.G + gq;
    const size_t rowq = (static_cast<size_t>(b) * T_) * p.HQ + hq;
    const T* q = static_cast<const T*>(p.q) + rowq * D;
    const T* dO = static_cast<const T*>(p.dout) + rowq * Dv;
    float csum = 0.f;  // this thread's column (lane) partial of sum_t G[t, s0+lane]
    if (DECAY) {
      __syncthreads();
      for (int i = threadIdx.x; i < BS; i += NTH) sCk[i] = (s0 + i < T_) ? p.c[rowq + static_cast<size_t>(s0 + i) * p.HQ] : 0.f;
    }
    for (int t0 = (s0 / BQ) * BQ; t0 < T_; t0 += BQ) {
      __syncthreads();
      load_rows<T>(sQ, ldq, q, sq, t0, BQ, D, T_);
      load_rows<T>(sDO, ldv, dO, sqv, t0, BQ, Dv, T_);
      for (int r = threadIdx.x; r < BQ; r += NTH) {
        const int t = t0 + r;
        sDelta[r] = (t < T_) ? p.delta[rowq + static_cast<size_t>(t) * p.HQ] : 0.f;
        const float dn = (t < T_) ? p.den[rowq + static_cast<size_t>(t) * p.HQ] : 1.f;
        sRden[r] = 1.f / (dn > 0.f ? dn : 1.f);
        if (DECAY) sCq[r] = (t < T_) ? p.c[rowq + static_cast<size_t>(t) * p.HQ] : 0.f;
      }
      __syncthreads();
      for (int i = 0; i < BQ / 8; ++i) {
        const int r = warp + 8 * i, s = lane;
        const int t = t0 + r, sg = s0 + s;
        const bool valid = (sg <= t) && (sg < T_) && (t < T_);
        float qk[MAXP];
        score_parts<SUM>(sQ + r * ldq, sK + s * ldq, M, E, p.scale, qk);
        float a = 0.f;
        for (int j = 0; j < NP; ++j) a = fmaf(qk[j], qk[j], a);
        float dn = 0.f;
        for (int j = 0; j < Dv; ++j) dn = fmaf(sDO[r * ldv + j], sV[s * ldv + j], dn);
        const float dA = valid ? (dn - sDelta[r]) * sRden[r] : 0.f;
        float dec = 1.f;
        if (DECAY) {
          const float x = sCq[r] - sCk[s];
          dec = __expf(fminf(x, 0.f));
          if (valid && x <= 0.f) csum += dA * a * dec;
        }
        sP[r * lda + s] = valid ? a * dec * sRden[r] : 0.f;
        const float w = 2.f * p.scale * dec * dA;
        for (int j = 0; j < NP; ++j) sW[(j * BQ + r) * lda + s] = w * qk[j];
      }
      __syncthreads();
      // thread owns key row orow (0..31) with columns ocol + 8u
      const int s = orow;
      for (int r = 0; r < BQ; ++r) {
        const float pr = sP[r * lda + s];
#pragma unroll
        for (int u = 0; u < 32; ++u)
          if (u < nuv) dv[u] = fmaf(pr, sDO[r * ldv + ocol + 8 * u], dv[u]);
        if (!SUM) {
#pragma unroll
          for (int u = 0; u < 32; ++u) {
            if (u < nuk) {
              const int d = ocol + 8 * u;
              dk[u] = fmaf(sW[((d / E) * BQ + r) * lda + s], sQ[r * ldq + d], dk[u]);
            }
          }
        } else {
          for (int a = 0; a < M; ++a) {
#pragma unroll
            for (int u = 0; u < 32; ++u) {
              if (u < nuk) {
                const int d = ocol + 8 * u, bb = d / E, e = d - bb * E;
                dk[u] = fmaf(sW[((a * M + bb) * BQ + r) * lda + s], sQ[r * ldq + a * E + e], dk[u]);
              }
            }
          }
        }
      }
    }
    if (DECAY) {
      __syncthreads();
      sCol[warp * BS + lane] = csum;
      __syncthreads();
      if (tid < BS) {
        float x = 0.f;
        for (int w = 0; w < 8; ++w) x += sCol[w * BS + tid];
        const int sg = s0 + tid;
        if (sg < T_) p.dc[rowq + static_cast<size_t>(sg) * p.HQ] -= x;
      }
    }
  }
  const int sg = s0 + orow;
  if (sg < T_) {
    T* dkp = static_cast<T*>(p.dk) + ((static_cast<size_t>(b) * T_ + sg) * p.H + h) * D;
    T* dvp = static_cast<T*>(p.dv) + ((static_cast<size_t>(b) * T_ + sg) * p.H + h) * Dv;
#pragma unroll
    for (int u = 0; u < 32; ++u) {
      if (u < nuk) dkp[ocol + 8 * u] = from_f32<T>(dk[u]);
      if (u < nuv) dvp[ocol + 8 * u] = from_f32<T>(dv[u]);
    }
  }
}

size_t fwd_smem(int D, int Dv) {
  return sizeof(float) * (BQ * (D + 1) + BS * (D + 1) + BS * (Dv + 1) + BQ * (BS + 1) + BQ + BS);
}
size_t dq_smem(int D, int Dv, int NP) {
  return sizeof(float) * (BQ * (D + 1) + BQ * (Dv + 1) + BS * (D + 1) + BS * (Dv + 1) + NP * BQ * (BS + 1) + 3 * BQ + BS);
}
size_t dkdv_smem(int D, int Dv, int NP) {
  return sizeof(float) * (BS * (D + 1) + BS * (Dv + 1) + BQ * (D + 1) + BQ * (Dv + 1) + NP * BQ * (BS + 1) +
                          BQ * (BS + 1) + 3 * BQ + BS + 8 * BS);
}

template <typename K, typename P>
int launch(K kernel, dim3 grid, size_t smem, cudaStream_t st, const P& p) {
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
      cudaSuccess)
    return KATA_ERR_CUDA;
  kernel<<<grid, NTH, smem, st>>>(p);
  return from_cuda(cudaGetLastError());
}

template <typename T>
int fwd_typed(const AttnFwdParams& p, bool sum, cudaStream_t st) {
  const dim3 grid((p.T + BQ - 1) / BQ, p.B * p.HQ);
  const size_t smem = fwd_smem(p.D, p.Dv);
  const bool dec = p.c != nullptr;
  if (!sum && !dec) return launch(attn_fwd_simt<T, false, false>, grid, smem, st, p);
  if (!sum && dec) return launch(attn_fwd_simt<T, false, true>, grid, smem, st, p);
  if (sum && !dec) return launch(attn_fwd_simt<T, true, false>, grid, smem, st, p);
  return launch(attn_fwd_simt<T, true, true>, grid, smem, st, p);
}

template <typename T, bool SUM, bool DEC>
int bwd_typed2(const AttnBwdParams& p, cudaStream_t st) {
  const int NP = SUM ? p.M * p.M : p.M;
  if (p.phases != 2) {
    int e = launch(attn_bwd_dq_simt<T, SUM, DEC>, dim3((p.T + BQ - 1) / BQ, p.B * p.HQ), dq_smem(p.D, p.Dv, NP), st,
                   p);
    if (e) return e;
  }
  if (p.phases == 1) return KATA_OK;
  return launch(attn_bwd_dkdv_simt<T, SUM, DEC>, dim3((p.T + BS - 1) / BS, p.B * p.H), dkdv_smem(p.D, p.Dv, NP), st,
                p);
}

template <typename T>
int bwd_typed(const AttnBwdParams& p, bool sum, cudaStream_t st) {
  const bool dec = p.c != nullptr;
  if (!sum && !dec) return bwd_typed2<T, false, false>(p, st);
  if (!sum && dec) return bwd_typed2<T, false, true>(p, st);
  if (sum && !dec) return bwd_typed2<T, true, false>(p, st);
  return bwd_typed2<T, true, true>(p, st);
}

}  // namespace

bool simt_supported(int D, int Dv, int M, bool sum) {
  if (D < 1 || Dv < 1 || D > 256 || Dv > 256 || D % 8 || Dv % 8 || M < 1 || D % M) return false;
  const int np = sum ? M * M : M;
  if (np > MAXP) return false;
  return dkdv_smem(D, Dv, np) <= 227 * 1024;
}

int simt_attn_fwd(const AttnFwdParams& p, int dtype, bool sum, cudaStream_t st) {
  switch (dtype) {
    case KATA_DTYPE_F32: return fwd_typed<float>(p, sum, st);
    case KATA_DTYPE_BF16: return fwd_typed<__nv_bfloat16>(p, sum, st);
    case KATA_DTYPE_F16: return fwd_typed<__half>(p, sum, st);
    default: return KATA_ERR_DTYPE;
  }
}

int simt_attn_bwd(const AttnBwdParams& p, int dtype, bool sum, cudaStream_t st) {
  switch (dtype) {
    case KATA_DTYPE_F32: return bwd_typed<float>(p, sum, st);
    case KATA_DTYPE_BF16: return bwd_typed<__nv_bfloat16>(p, sum, st);
    case KATA_DTYPE_F16: return bwd_typed<__half>(p, sum, st);
    default: return KATA_ERR_DTYPE;
  }
}

}  // namespace kata
