// delta_simt.cu -- SPD delta rule ("flash_delta", kata/spd/flash_delta.py) on CUDA cores, fp32.
//
// Per (batch, head), with kappa(x,y) = sum_{g,h} (scale x_g.y_h)^2 (all group pairs):
//   L = tril(kappa(k,k), -1),  P = tril(kappa(q,k))  (diagonal included)
//   U = (I + diag(beta) L)^{-1} diag(beta) V          (chunk-sequential forward substitution)
//   E = L U                                           (erase term, saved for d beta)
//   num = P U,  den = rowsum(P),  o = num / (den + eps) if normalize else num
// Backward (dO given, dnum = dO/(den+eps) or dO, z_t = <dO_t, o_t>/(den_t+eps) or 0):
//   dU = P^T dnum
//   Y  = (I + diag(beta) L)^{-T} dU                    (chunk-sequential backward substitution)
//   dV = beta * Y,  dbeta_t = Y_t . (V_t - E_t)
//   dA_qk[t,s] = dnum_t . U_s - z_t          (s <= t)
//   dA_kk[t,s] = -beta_t (Y_t . U_s)          (s <  t)
//   dq_t = sum_s dA_qk[t,s] d kappa(q_t,k_s)/d q_t
//   dk_s = sum_t dA_qk[t,s] d kappa(q_t,k_s)/d k_s + sum_j Dkk[s,j] d kappa(k_s,k_j)/d k_s,
//          Dkk[s,j] = dA_kk[s,j] (j < s) or dA_kk[j,s] (j > s)   (kappa is symmetric)
//   d kappa(x,y)/d x_g = 2 scale^2 sum_h (x_g.y_h) y_h
// The reference computes the same quantities with Triton kernels K14-K21
// (kata/spd/flash_delta.py:27-1116); its inter-chunk products round U and the kernel to bf16,
// these kernels keep fp32 throughout.
#include "attn_common.cuh"
#include "host_util.h"
#include "sm100.cuh"

namespace kata {
namespace {

constexpr int C = 64;      // chunk rows (the reference's C)
constexpr int NTH = 256;   // threads per CTA
constexpr int TB = 32;     // tile rows for the parallel passes
constexpr int MAXG2 = 16;  // max M*M group pairs

struct DeltaParams {
  const void* q;
  const void* k;
  const void* v;
  const float* beta;
  float* U;
  float* E;
  float* o;
  float* den;
  const float* dout;
  float* dq;
  float* dk;
  float* dv;
  float* dbeta;
  float* dnum;  // workspace (B,T,H,Dv)
  float* z;     // workspace (B,T,H)
  float* dU;    // workspace (B,T,H,Dv)
  float* Y;     // workspace (B,T,H,Dv)
  int B, T, H, D, Dv, M, normalize;
  float scale, eps;
  int strict;  // readout pass: 1 -> mask s < t (E = tril(kappa(k,k),-1) U with q := k)
};

// kappa(x, y) for rows x, y (length D, stride 1) and the M*M scaled group dots ip[g*M+h]
__device__ __forceinline__ float kappa_parts(const float* x, const float* y, int M, int E, float scale, float* ip) {
  float a = 0.f;
  for (int g = 0; g < M; ++g)
    for (int h = 0; h < M; ++h) {
      float d = 0.f;
      for (int e = 0; e < E; ++e) d = fmaf(x[g * E + e], y[h * E + e], d);
      d *= scale;
      ip[g * M + h] = d;
      a = fmaf(d, d, a);
    }
  return a;
}
__device__ __forceinline__ float kappa(const float* x, const float* y, int M, int E, float scale) {
  float ip[MAXG2];
  return kappa_parts(x, y, M, E, scale, ip);
}

template <typename T>
__device__ __forceinline__ void load_rows_f(float* dst, int ld, const T* src, size_t row_stride, int row0, int nrows,
                                            int ncols, int T_) {
  for (int i = threadIdx.x; i < nrows * ncols; i += NTH) {
    const int r = i / ncols, c = i - r * ncols;
    const int t = row0 + r;
    dst[r * ld + c] = (t < T_) ? to_f32<T>(src[static_cast<size_t>(t) * row_stride + c]) : 0.f;
  }
}

// ------------------------------------------------------------------------------------------------
// Forward 1: U and E, one CTA per (b,h), sequential over chunks.
// smem: Kc[C][D+1], Kp[C][D+1], A[C][C+1], Up[C][Dv+1] (previous chunk's U, then this chunk's rhs/U)
// ------------------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(NTH) delta_u_kernel(DeltaParams p) {
  extern __shared__ float sm[];
  const int D = p.D, Dv = p.Dv, M = p.M, E = D / M, T_ = p.T;
  const int ldk = D + 1, lda = C + 1, ldv = Dv + 1;
  float* sKc = sm;
  float* sKp = sKc + C * ldk;
  float* sA = sKp + C * ldk;
  float* sUp = sA + C * lda;
  float* sBeta = sUp + C * ldv;
  const int bh = blockIdx.x, b = bh / p.H, h = bh % p.H;
  const size_t rowstep = static_cast<size_t>(p.H);
  const T* k = static_cast<const T*>(p.k) + (static_cast<size_t>(b) * T_ * p.H + h) * D;
  const T* v = static_cast<const T*>(p.v) + (static_cast<size_t>(b) * T_ * p.H + h) * Dv;
  const float* beta = static_cast<const float*>(p.beta) + static_cast<size_t>(b) * T_ * p.H + h;
  float* U = p.U + (static_cast<size_t>(b) * T_ * p.H + h) * Dv;
  float* Eo = p.E ? p.E + (static_cast<size_t>(b) * T_ * p.H + h) * Dv : nullptr;
  const int tid = threadIdx.x;
  // thread -> (row r, columns cph + 8u) for C x Dv register tiles: r = tid/4 (0..63), 4 column phases
  const int er = tid >> 2, ec = tid & 3;
  const int nu = Dv / 4;  // columns per thread (<= 64 for Dv <= 256)
  const int nchunks = (T_ + C - 1) / C;
  for (int c = 0; c < nchunks; ++c) {
    const int c0 = c * C;
    __syncthreads();
    load_rows_f<T>(sKc, ldk, k, rowstep * D, c0, C, D, T_);
    for (int i = tid; i < C; i += NTH) sBeta[i] = (c0 + i < T_) ? (beta[static_cast<size_t>(c0 + i) * rowstep]) : 0.f;
    float ev[64];
#pragma unroll
    for (int u = 0; u < 64; ++u) ev[u] = 0.f;
    // inter-chunk erase: E_c += kappa(K_c, K_c') U_c'
    for (int cp = 0; cp < c; ++cp) {
      const int p0 = cp * C;
      __syncthreads();
      load_rows_f<T>(sKp, ldk, k, rowstep * D, p0, C, D, T_);
      for (int i = tid; i < C * Dv; i += NTH) {
        const int r = i / Dv, cc = i - r * Dv;
        sUp[r * ldv + cc] = U[static_cast<size_t>(p0 + r) * rowstep * Dv + cc];
      }
      __syncthreads();
      for (int i = tid; i < C * C; i += NTH) {
        const int r = i / C, s = i - r * C;
        sA[r * lda + s] = kappa(sKc + r * ldk, sKp + s * ldk, M, E, p.scale);
      }
      __syncthreads();
      for (int s = 0; s < C; ++s) {
        const float a = sA[er * lda + s];
#pragma unroll
        for (int u = 0; u < 64; ++u)
          if (u < nu) ev[u] = fmaf(a, sUp[s * ldv + ec + 4 * u], ev[u]);
      }
    }
    // diagonal block: A = kappa(K_c, K_c) (strictly lower used); rhs = beta (V - E_inter)
    __syncthreads();
    for (int i = tid; i < C * C; i += NTH) {
      const int r = i / C, s = i - r * C;
      sA[r * lda + s] = (s < r) ? kappa(sKc + r * ldk, sKc + s * ldk, M, E, p.scale) : 0.f;
    }
    {
      const int t = c0 + er;
      const float bt = sBeta[er];
#pragma unroll
      for (int u = 0; u < 64; ++u) {
        if (u < nu) {
          const int cc = ec + 4 * u;
          const float vv = (t < T_) ? to_f32<T>(v[static_cast<size_t>(t) * rowstep * Dv + cc]) : 0.f;
          sUp[er * ldv + cc] = bt * (vv - ev[u]);  // rhs
        }
      }
    }
    __syncthreads();
    // forward substitution: U[t] = rhs[t] - beta_t sum_{s<t} A[t,s] U[s]; columns in parallel
    for (int cc = tid; cc < Dv; cc += NTH) {
      for (int t = 1; t < C; ++t) {
        float acc = 0.f;
        for (int s = 0; s < t; ++s) acc = fmaf(sA[t * lda + s], sUp[s * ldv + cc], acc);
        sUp[t * ldv + cc] -= sBeta[t] * acc;
      }
    }
    __syncthreads();
    // E = E_inter + sum_{s<t} A[t,s] U[s];  store U, E
    {
      const int t = c0 + er;
#pragma unroll
      for (int u = 0; u < 64; ++u) {
        if (u < nu) {
          const int cc = ec + 4 * u;
          float e = ev[u];
          for (int s = 0; s < er; ++s) e = fmaf(sA[er * lda + s], sUp[s * ldv + cc], e);
          if (t < T_) {
            U[static_cast<size_t>(t) * rowstep * Dv + cc] = sUp[er * ldv + cc];
            if (p.E) Eo[static_cast<size_t>(t) * rowstep * Dv + cc] = e;
          }
        }
      }
    }
  }
}

// ------------------------------------------------------------------------------------------------
// Forward 2: num = P U, den = rowsum(P), o.  CTA per (32-query tile, b*h).  U == null -> den only;
// o / den null -> not written.  With strict = 1 and q := k the same pass yields E = L U.
// ------------------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(NTH) delta_readout_kernel(DeltaParams p) {
  extern __shared__ float sm[];
  const int D = p.D, Dv = p.Dv, M = p.M, E = D / M, T_ = p.T;
  const int ldk = D + 1, ldv = Dv + 1, lda = TB + 1;
  float* sQ = sm;
  float* sK = sQ + TB * ldk;
  float* sU = sK + TB * ldk;
  float* sA = sU + TB * ldv;
  const int nqt = (T_ + TB - 1) / TB;
  const int qt = nqt - 1 - blockIdx.x;
  const int bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const size_t base = static_cast<size_t>(b) * T_ * p.H + h;  // + t*H
  const T* q = static_cast<const T*>(p.q) + base * D;
  const T* k = static_cast<const T*>(p.k) + base * D;
  const float* U = p.U ? p.U + base * Dv : nullptr;
  const size_t sqk = static_cast<size_t>(p.H) * D, sv = static_cast<size_t>(p.H) * Dv;
  const int t0 = qt * TB;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  load_rows_f<T>(sQ, ldk, q, sqk, t0, TB, D, T_);
  const int orow = tid >> 3, ocol = tid & 7, nu = U ? Dv / 8 : 0;
  float acc[32];
#pragma unroll
  for (int u = 0; u < 32; ++u) acc[u] = 0.f;
  float den = 0.f;
  for (int s0 = 0; s0 < min(t0 + TB, T_); s0 += TB) {
    __syncthreads();
    load_rows_f<T>(sK, ldk, k, sqk, s0, TB, D, T_);
    if (U) load_rows_f<float>(sU, ldv, U, sv, s0, TB, Dv, T_);
    __syncthreads();
    for (int i = 0; i < TB / 8; ++i) {
      const int r = warp + 8 * i, s = lane;
      const int t = t0 + r, sg = s0 + s;
      sA[r * lda + s] = (sg <= t - p.strict && sg < T_ && t < T_) ? kappa(sQ + r * ldk, sK + s * ldk, M, E, p.scale) : 0.f;
    }
    __syncthreads();
    for (int s = 0; s < TB; ++s) {
      const float a = sA[orow * lda + s];
      den += a;
#pragma unroll
      for (int u = 0; u < 32; ++u)
        if (u < nu) acc[u] = fmaf(a, sU[s * ldv + ocol + 8 * u], acc[u]);
    }
  }
  const int t = t0 + orow;
  if (t < T_) {
    const float inv = p.normalize ? 1.f / (den + p.eps) : 1.f;
    if (p.o) {
      float* o = p.o + (base + static_cast<size_t>(t) * p.H) * Dv;
#pragma unroll
      for (int u = 0; u < 32; ++u)
        if (u < nu) o[ocol + 8 * u] = acc[u] * inv;
    }
    if (ocol == 0 && p.den) p.den[base + static_cast<size_t>(t) * p.H] = den;
  }
}

// ------------------------------------------------------------------------------------------------
// Backward 0: dnum, z.  One warp per row.
// ------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(NTH) delta_prep_kernel(DeltaParams p) {
  const int warp = (blockIdx.x * NTH + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const size_t rows = static_cast<size_t>(p.B) * p.T * p.H;
  if (static_cast<size_t>(warp) >= rows) return;
  const size_t r = warp;
  const float inv = p.normalize ? 1.f / (p.den[r] + p.eps) : 1.f;
  float zz = 0.f;
  for (int c = lane; c < p.Dv; c += 32) {
    const float g = p.dout[r * p.Dv + c];
    p.dnum[r * p.Dv + c] = g * inv;
    if (p.normalize) zz = fmaf(g, p.o[r * p.Dv + c], zz);
  }
  for (int off = 16; off; off >>= 1) zz += __shfl_xor_sync(0xffffffffu, zz, off);
  if (lane == 0) p.z[r] = zz * inv;
}

// ------------------------------------------------------------------------------------------------
// Backward 1: dU_s = sum_{t>=s} P[t,s] dnum_t.  CTA per (32-key tile, b*h).
// ------------------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(NTH) delta_du_kernel(DeltaParams p) {
  extern __shared__ float sm[];
  const int D = p.D, Dv = p.Dv, M = p.M, E = D / M, T_ = p.T;
  const int ldk = D + 1, ldv = Dv + 1, lda = TB + 1;
  float* sK = sm;
  float* sQ = sK + TB * ldk;
  float* sG = sQ + TB * ldk;
  float* sA = sG + TB * ldv;
  const int kt = blockIdx.x;
  const int bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const size_t base = static_cast<size_t>(b) * T_ * p.H + h;
  const T* q = static_cast<const T*>(p.q) + base * D;
  const T* k = static_cast<const T*>(p.k) + base * D;
  const float* dn = p.dnum + base * Dv;
  const size_t sqk = static_cast<size_t>(p.H) * D, sv = static_cast<size_t>(p.H) * Dv;
  const int s0 = kt * TB;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  load_rows_f<T>(sK, ldk, k, sqk, s0, TB, D, T_);
  const int orow = tid >> 3, ocol = tid & 7, nu = Dv / 8;
  float acc[32];
#pragma unroll
  for (int u = 0; u < 32; ++u) acc[u] = 0.f;
  for (int t0 = s0; t0 < T_; t0 += TB) {
    __syncthreads();
    load_rows_f<T>(sQ, ldk, q, sqk, t0, TB, D, T_);
    load_rows_f<float>(sG, ldv, dn, sv, t0, TB, Dv, T_);
    __syncthreads();
    for (int i = 0; i < TB / 8; ++i) {
      const int r = warp + 8 * i, s = lane;  // r: query row, s: key col
      const int t = t0 + r, sg = s0 + s;
      sA[s * lda + r] = (sg <= t && t < T_ && sg < T_) ? kappa(sQ + r * ldk, sK + s * ldk, M, E, p.scale) : 0.f;
    }
    __syncthreads();
    for (int r = 0; r < TB; ++r) {
      const float a = sA[orow * lda + r];
#pragma unroll
      for (int u = 0; u < 32; ++u)
        if (u < nu) acc[u] = fmaf(a, sG[r * ldv + ocol + 8 * u], acc[u]);
    }
  }
  const int sg = s0 + orow;
  if (sg < T_) {
    float* out = p.dU + (base + static_cast<size_t>(sg) * p.H) * Dv;
#pragma unroll
    for (int u = 0; u < 32; ++u)
      if (u < nu) out[ocol + 8 * u] = acc[u];
  }
}

// ------------------------------------------------------------------------------------------------
// Backward 2: Y = (I + diag(beta) L)^{-T} dU, one CTA per (b,h), chunks from last to first.
//   Y_c = (I + N_cc)^{-T} (dU_c - sum_{c'>c} L[c',c]^T (beta Y)_{c'})
// ------------------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(NTH) delta_y_kernel(DeltaParams p) {
  extern __shared__ float sm[];
  const int D = p.D, Dv = p.Dv, M = p.M, E = D / M, T_ = p.T;
  const int ldk = D + 1, lda = C + 1, ldv = Dv + 1;
  float* sKc = sm;
  float* sKp = sKc + C * ldk;
  float* sA = sKp + C * ldk;
  float* sY = sA + C * lda;
  float* sBeta = sY + C * ldv;
  float* sBp = sBeta + C;
  const int bh = blockIdx.x, b = bh / p.H, h = bh % p.H;
  const size_t rowstep = static_cast<size_t>(p.H);
  const T* k = static_cast<const T*>(p.k) + (static_cast<size_t>(b) * T_ * p.H + h) * D;
  const float* beta = static_cast<const float*>(p.beta) + static_cast<size_t>(b) * T_ * p.H + h;
  const float* dU = p.dU + (static_cast<size_t>(b) * T_ * p.H + h) * Dv;
  float* Y = p.Y + (static_cast<size_t>(b) * T_ * p.H + h) * Dv;
  const int tid = threadIdx.x;
  const int er = tid >> 2, ec = tid & 3, nu = Dv / 4;
  const int nchunks = (T_ + C - 1) / C;
  for (int c = nchunks - 1; c >= 0; --c) {
    const int c0 = c * C;
    __syncthreads();
    load_rows_f<T>(sKc, ldk, k, rowstep * D, c0, C, D, T_);
    for (int i = tid; i < C; i += NTH) sBeta[i] = (c0 + i < T_) ? (beta[static_cast<size_t>(c0 + i) * rowstep]) : 0.f;
    float fv[64];
#pragma unroll
    for (int u = 0; u < 64; ++u) fv[u] = 0.f;
    for (int cp = c + 1; cp < nchunks; ++cp) {
      const int p0 = cp * C;
      __syncthreads();
      load_rows_f<T>(sKp, ldk, k, rowstep * D, p0, C, D, T_);
      for (int i = tid; i < C; i += NTH) sBp[i] = (p0 + i < T_) ? (beta[static_cast<size_t>(p0 + i) * rowstep]) : 0.f;
      __syncthreads();
      for (int i = tid; i < C * Dv; i += NTH) {  // (beta Y)_{c'} into sY
        const int r = i / Dv, cc = i - r * Dv;
        sY[r * ldv + cc] = (p0 + r < T_) ? sBp[r] * Y[static_cast<size_t>(p0 + r) * rowstep * Dv + cc] : 0.f;
      }
      for (int i = tid; i < C * C; i += NTH) {  // sA[s][r] = L[c'(s), c(r)] = kappa(K_c'[s], K_c[r])
        const int s = i / C, r = i - s * C;
        sA[s * lda + r] = kappa(sKp + s * ldk, sKc + r * ldk, M, E, p.scale);
      }
      __syncthreads();
      for (int s = 0; s < C; ++s) {
        const float a = sA[s * lda + er];
#pragma unroll
        for (int u = 0; u < 64; ++u)
          if (u < nu) fv[u] = fmaf(a, sY[s * ldv + ec + 4 * u], fv[u]);
      }
    }
    __syncthreads();
    for (int i = tid; i < C * C; i += NTH) {  // strictly lower A of the diagonal block
      const int r = i / C, s = i - r * C;
      sA[r * lda + s] = (s < r) ? kappa(sKc + r * ldk, sKc + s * ldk, M, E, p.scale) : 0.f;
    }
    {
      const int t = c0 + er;
#pragma unroll
      for (int u = 0; u < 64; ++u) {
        if (u < nu) {
          const int cc = ec + 4 * u;
          const float g = (t < T_) ? dU[static_cast<size_t>(t) * rowstep * Dv + cc] : 0.f;
          sY[er * ldv + cc] = g - fv[u];
        }
      }
    }
    __syncthreads();
    // backward substitution: Y[t] = rhs[t] - sum_{s>t} beta_s A[s,t] Y[s]
    for (int cc = tid; cc < Dv; cc += NTH) {
      for (int t = C - 2; t >= 0; --t) {
        float acc = 0.f;
        for (int s = t + 1; s < C; ++s) acc = fmaf(sBeta[s] * sA[s * lda + t], sY[s * ldv + cc], acc);
        sY[t * ldv + cc] -= acc;
      }
    }
    __syncthreads();
    for (int i = tid; i < C * Dv; i += NTH) {
      const int r = i / Dv, cc = i - r * Dv;
      if (c0 + r < T_) Y[static_cast<size_t>(c0 + r) * rowstep * Dv + cc] = sY[r * ldv + cc];
    }
  }
}

// ------------------------------------------------------------------------------------------------
// Backward 3: dq.  CTA per (32-query tile, b*h); W_gh[t,s] = 2 scale dA_qk[t,s] ip_gh  so that
// dq_g[t] = sum_s sum_h W_gh[t,s] k_h[s]  (ip_gh already carries one factor of scale).
// ------------------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(NTH) delta_dq_kernel(DeltaParams p) {
  extern __shared__ float sm[];
  const int D = p.D, Dv = p.Dv, M = p.M, E = D / M, T_ = p.T;
  const int NP = M * M;
  const int ldk = D + 1, ldv = Dv + 1, lda = TB + 1;
  float* sQ = sm;
  float* sG = sQ + TB * ldk;  // dnum rows
  float* sK = sG + TB * ldv;
  float* sU = sK + TB * ldk;
  float* sW = sU + TB * ldv;  // NP x TB x lda
  float* sZ = sW + NP * TB * lda;
  const int nqt = (T_ + TB - 1) / TB;
  const int qt = nqt - 1 - blockIdx.x;
  const int bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const size_t base = static_cast<size_t>(b) * T_ * p.H + h;
  const T* q = static_cast<const T*>(p.q) + base * D;
  const T* k = static_cast<const T*>(p.k) + base * D;
  const size_t sqk = static_cast<size_t>(p.H) * D, sv = static_cast<size_t>(p.H) * Dv;
  const int t0 = qt * TB;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  load_rows_f<T>(sQ, ldk, q, sqk, t0, TB, D, T_);
  load_rows_f<float>(sG, ldv, p.dnum + base * Dv, sv, t0, TB, Dv, T_);
  for (int i = tid; i < TB; i += NTH) sZ[i] = (t0 + i < T_) ? p.z[base + static_cast<size_t>(t0 + i) * p.H] : 0.f;
  const int orow = tid >> 3, ocol = tid & 7, nu = D / 8;
  float dq[32];
#pragma unroll
  for (int u = 0; u < 32; ++u) dq[u] = 0.f;
  for (int s0 = 0; s0 < min(t0 + TB, T_); s0 += TB) {
    __syncthreads();
    load_rows_f<T>(sK, ldk, k, sqk, s0, TB, D, T_);
    load_rows_f<float>(sU, ldv, p.U + base * Dv, sv, s0, TB, Dv, T_);
    __syncthreads();
    for (int i = 0; i < TB / 8; ++i) {
      const int r = warp + 8 * i, s = lane;
      const int t = t0 + r, sg = s0 + s;
      const bool valid = (sg <= t) && (sg < T_) && (t < T_);
      float ip[MAXG2];
      kappa_parts(sQ + r * ldk, sK + s * ldk, M, E, p.scale, ip);
      float dA = 0.f;
      if (valid) {
        for (int j = 0; j < Dv; ++j) dA = fmaf(sG[r * ldv + j], sU[s * ldv + j], dA);
        dA -= sZ[r];
      }
      const float w = 2.f * p.scale * dA;
      for (int j = 0; j < NP; ++j) sW[(j * TB + r) * lda + s] = w * ip[j];
    }
    __syncthreads();
    for (int s = 0; s < TB; ++s) {
      for (int hh = 0; hh < M; ++hh) {
#pragma unroll
        for (int u = 0; u < 32; ++u) {
          if (u < nu) {
            const int d = ocol + 8 * u, g = d / E, e = d - g * E;
            dq[u] = fmaf(sW[((g * M + hh) * TB + orow) * lda + s], sK[s * ldk + hh * E + e], dq[u]);
          }
        }
      }
    }
  }
  const int t = t0 + orow;
  if (t < T_) {
    float* out = p.dq + (base + static_cast<size_t>(t) * p.H) * D;
#pragma unroll
    for (int u = 0; u < 32; ++u)
      if (u < nu) out[ocol + 8 * u] = dq[u];
  }
}

// ------------------------------------------------------------------------------------------------
// Backward 4: dk, dv, dbeta.  CTA per (32-key tile, b*h), looping over every other 32-row tile.
//   column role in A_qk:  W[t,s] = 2 scale dA_qk[t,s] ip(q_t,k_s);  dk_h[s] += sum_g W_gh q_g[t]
//   both roles in A_kk:   Dkk[s,j];  dk_g[s] += 2 scale Dkk[s,j] sum_h ip(k_s,k_j)_gh k_h[j]
// ------------------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(NTH) delta_dk_kernel(DeltaParams p) {
  extern __shared__ float sm[];
  const int D = p.D, Dv = p.Dv, M = p.M, E = D / M, T_ = p.T;
  const int NP = M * M;
  const int ldk = D + 1, ldv = Dv + 1, lda = TB + 1;
  float* sK = sm;              // own key tile rows s
  float* sU = sK + TB * ldk;   // own U rows
  float* sY = sU + TB * ldv;   // own Y rows
  float* sX = sY + TB * ldv;   // other tile rows (q or k)
  float* sG = sX + TB * ldk;   // other tile dnum or U
  float* sH = sG + TB * ldv;   // other tile Y (for A_kk)
  float* sW = sH + TB * ldv;   // NP x TB x lda   (entry [j][s][r])
  float* sZ = sW + NP * TB * lda;
  float* sB = sZ + TB;         // own beta
  float* sBo = sB + TB;        // other beta
  const int kt = blockIdx.x;
  const int bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const size_t base = static_cast<size_t>(b) * T_ * p.H + h;
  const T* q = static_cast<const T*>(p.q) + base * D;
  const T* k = static_cast<const T*>(p.k) + base * D;
  const float* beta = static_cast<const float*>(p.beta) + base;
  const size_t sqk = static_cast<size_t>(p.H) * D, sv = static_cast<size_t>(p.H) * Dv;
  const int s0 = kt * TB;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  load_rows_f<T>(sK, ldk, k, sqk, s0, TB, D, T_);
  load_rows_f<float>(sU, ldv, p.U + base * Dv, sv, s0, TB, Dv, T_);
  load_rows_f<float>(sY, ldv, p.Y + base * Dv, sv, s0, TB, Dv, T_);
  for (int i = tid; i < TB; i += NTH) sB[i] = (s0 + i < T_) ? (beta[static_cast<size_t>(s0 + i) * p.H]) : 0.f;
  const int orow = tid >> 3, ocol = tid & 7, nu = D / 8;
  float dk[32];
#pragma unroll
  for (int u = 0; u < 32; ++u) dk[u] = 0.f;
  const int ntiles = (T_ + TB - 1) / TB;
  // pass A: column role of A_qk, over query tiles t0 >= s0
  for (int t0 = s0; t0 < T_; t0 += TB) {
    __syncthreads();
    load_rows_f<T>(sX, ldk, q, sqk, t0, TB, D, T_);
    load_rows_f<float>(sG, ldv, p.dnum + base * Dv, sv, t0, TB, Dv, T_);
    for (int i = tid; i < TB; i += NTH) sZ[i] = (t0 + i < T_) ? p.z[base + static_cast<size_t>(t0 + i) * p.H] : 0.f;
    __syncthreads();
    for (int i = 0; i < TB / 8; ++i) {
      const int r = warp + 8 * i, s = lane;  // r: query row of the other tile, s: own key
      const int t = t0 + r, sg = s0 + s;
      const bool valid = (sg <= t) && (sg < T_) && (t < T_);
      float ip[MAXG2];
      kappa_parts(sX + r * ldk, sK + s * ldk, M, E, p.scale, ip);
      float dA = 0.f;
      if (valid) {
        for (int j = 0; j < Dv; ++j) dA = fmaf(sG[r * ldv + j], sU[s * ldv + j], dA);
        dA -= sZ[r];
      }
      const float w = 2.f * p.scale * dA;
      for (int j = 0; j < NP; ++j) sW[(j * TB + s) * lda + r] = w * ip[j];
    }
    __syncthreads();
    for (int r = 0; r < TB; ++r) {
      for (int g = 0; g < M; ++g) {
#pragma unroll
        for (int u = 0; u < 32; ++u) {
          if (u < nu) {
            const int d = ocol + 8 * u, hh = d / E, e = d - hh * E;
            dk[u] = fmaf(sW[((g * M + hh) * TB + orow) * lda + r], sX[r * ldk + g * E + e], dk[u]);
          }
        }
      }
    }
  }
  // pass B: A_kk, both roles, over all key tiles j
  for (int jt = 0; jt < ntiles; ++jt) {
    const int j0 = jt * TB;
    __syncthreads();
    load_rows_f<T>(sX, ldk, k, sqk, j0, TB, D, T_);
    load_rows_f<float>(sG, ldv, p.U + base * Dv, sv, j0, TB, Dv, T_);
    load_rows_f<float>(sH, ldv, p.Y + base * Dv, sv, j0, TB, Dv, T_);
    for (int i = tid; i < TB; i += NTH) sBo[i] = (j0 + i < T_) ? (beta[static_cast<size_t>(j0 + i) * p.H]) : 0.f;
    __syncthreads();
    for (int i = 0; i < TB / 8; ++i) {
      const int r = warp + 8 * i, s = lane;  // r: other key row j, s: own key
      const int jg = j0 + r, sg = s0 + s;
      float ip[MAXG2];
      kappa_parts(sK + s * ldk, sX + r * ldk, M, E, p.scale, ip);  // ip(k_s, k_j)
      float dkk = 0.f;
      if (jg < T_ && sg < T_ && jg != sg) {
        float yu = 0.f;
        if (jg < sg) {  // dA_kk[s, j] = -beta_s Y_s . U_j
          for (int c = 0; c < Dv; ++c) yu = fmaf(sY[s * ldv + c], sG[r * ldv + c], yu);
          dkk = -sB[s] * yu;
        } else {  // dA_kk[j, s] = -beta_j Y_j . U_s
          for (int c = 0; c < Dv; ++c) yu = fmaf(sH[r * ldv + c], sU[s * ldv + c], yu);
          dkk = -sBo[r] * yu;
        }
      }
      const float w = 2.f * p.scale * dkk;
      for (int j = 0; j < NP; ++j) sW[(j * TB + s) * lda + r] = w * ip[j];
    }
    __syncthreads();
    for (int r = 0; r < TB; ++r) {
      for (int hh = 0; hh < M; ++hh) {
#pragma unroll
        for (int u = 0; u < 32; ++u) {
          if (u < nu) {
            const int d = ocol + 8 * u, g = d / E, e = d - g * E;
            dk[u] = fmaf(sW[((g * M + hh) * TB + orow) * lda + r], sX[r * ldk + hh * E + e], dk[u]);
          }
        }
      }
    }
  }
  const int sg = s0 + orow;
  if (sg < T_) {
    float* out = p.dk + (base + static_cast<size_t>(sg) * p.H) * D;
#pragma unroll
    for (int u = 0; u < 32; ++u)
      if (u < nu) out[ocol + 8 * u] = dk[u];
  }
  // dv = beta * Y, dbeta = Y . (V - E): warp per row of the own tile
  const T* v = static_cast<const T*>(p.v) + base * Dv;
  for (int r = warp; r < TB; r += NTH / 32) {
    const int sgr = s0 + r;
    if (sgr >= T_) continue;
    const size_t ro = static_cast<size_t>(sgr) * p.H;
    float acc = 0.f;
    for (int c = lane; c < Dv; c += 32) {
      const float y = sY[r * ldv + c];
      p.dv[(base + ro) * Dv + c] = sB[r] * y;
      acc = fmaf(y, to_f32<T>(v[ro * Dv + c]) - p.E[(base + ro) * Dv + c], acc);
    }
    for (int off = 16; off; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) p.dbeta[base + ro] = acc;
  }
}

size_t smem_u(int D, int Dv) { return sizeof(float) * (2 * C * (D + 1) + C * (C + 1) + C * (Dv + 1) + C); }
size_t smem_y(int D, int Dv) { return sizeof(float) * (2 * C * (D + 1) + C * (C + 1) + C * (Dv + 1) + 2 * C); }
size_t smem_readout(int D, int Dv) { return sizeof(float) * (2 * TB * (D + 1) + TB * (Dv + 1) + TB * (TB + 1)); }
size_t smem_du(int D, int Dv) { return sizeof(float) * (2 * TB * (D + 1) + TB * (Dv + 1) + TB * (TB + 1)); }
size_t smem_dq(int D, int Dv, int M) {
  return sizeof(float) * (2 * TB * (D + 1) + 2 * TB * (Dv + 1) + M * M * TB * (TB + 1) + TB);
}
size_t smem_dk(int D, int Dv, int M) {
  return sizeof(float) * (2 * TB * (D + 1) + 4 * TB * (Dv + 1) + M * M * TB * (TB + 1) + 3 * TB);
}

template <typename K>
int launch(K kernel, dim3 grid, size_t smem, cudaStream_t st, const DeltaParams& p) {
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
    return KATA_ERR_CUDA;
  kernel<<<grid, NTH, smem, st>>>(p);
  return from_cuda(cudaGetLastError());
}


template <typename T>
int fwd_typed(const DeltaParams& p, int phases, cudaStream_t st) {
  if (phases != 2) {
    const int e = launch(delta_u_kernel<T>, dim3(p.B * p.H), smem_u(p.D, p.Dv), st, p);
    if (e || phases == 1) return e;
  }
  if (!p.o && !p.den) return KATA_OK;
  return launch(delta_readout_kernel<T>, dim3((p.T + TB - 1) / TB, p.B * p.H), smem_readout(p.D, p.Dv), st, p);
}

// Workspace: dnum | dU | Y | E (each B*T*H*Dv fp32) | z (B*T*H fp32).
template <typename T>
int bwd_typed(DeltaParams p, bool given_dnum, cudaStream_t st) {
  const size_t rows = static_cast<size_t>(p.B) * p.T * p.H;
  const dim3 tiles((p.T + TB - 1) / TB, p.B * p.H);
  int e = KATA_OK;
  if (!given_dnum) {
    delta_prep_kernel<<<static_cast<unsigned>((rows * 32 + NTH - 1) / NTH), NTH, 0, st>>>(p);
    e = from_cuda(cudaGetLastError());
  }
  if (!e && !p.E) {  // E = tril(kappa(k,k),-1) U, recomputed (the forward does not keep it)
    DeltaParams pe = p;
    pe.q = p.k;
    pe.o = pe.E = p.dU + 2 * rows * p.Dv;  // E slot of the workspace
    pe.den = nullptr;
    pe.normalize = 0;
    pe.strict = 1;
    e = launch(delta_readout_kernel<T>, tiles, smem_readout(p.D, p.Dv), st, pe);
    p.E = pe.E;
  }
  if (!e) e = launch(delta_du_kernel<T>, tiles, smem_du(p.D, p.Dv), st, p);
  if (!e) e = launch(delta_y_kernel<T>, dim3(p.B * p.H), smem_y(p.D, p.Dv), st, p);
  if (!e) e = launch(delta_dq_kernel<T>, tiles, smem_dq(p.D, p.Dv, p.M), st, p);
  if (!e) e = launch(delta_dk_kernel<T>, tiles, smem_dk(p.D, p.Dv, p.M), st, p);
  return e;
}

int check(int dtype, int B, int T, int H, int D, int Dv, int M) {
  if (dtype != KATA_DTYPE_F32 && dtype != KATA_DTYPE_BF16 && dtype != KATA_DTYPE_F16) return KATA_ERR_DTYPE;
  if (B < 1 || T < 1 || H < 1 || D < 1 || Dv < 1 || M < 1 || D % M) return KATA_ERR_SHAPE;
  if (M * M > MAXG2 || D > 256 || Dv > 256 || D % 8 || Dv % 8) return KATA_ERR_UNSUPPORTED;
  if (smem_dk(D, Dv, M) > 227 * 1024 || smem_u(D, Dv) > 227 * 1024) return KATA_ERR_UNSUPPORTED;
  return KATA_OK;
}

DeltaParams base_params(const void* q, const void* k, const void* v, const float* beta, int B, int T, int H, int D,
                        int Dv, int M, int normalize, float scale, float eps) {
  DeltaParams p{};
  p.q = q;
  p.k = k;
  p.v = v;
  p.beta = beta;
  p.B = B;
  p.T = T;
  p.H = H;
  p.D = D;
  p.Dv = Dv;
  p.M = M;
  p.normalize = normalize;
  p.scale = scale;
  p.eps = eps;
  p.strict = 0;
  return p;
}

}  // namespace
}  // namespace kata

using namespace kata;

extern "C" int kata_delta_fwd(const kata_delta_fwd_args* a, kata_stream_t stream) {
  if (!a) return KATA_ERR_INVALID;
  int e = check(a->dtype, a->B, a->T, a->H, a->D, a->Dv, a->M);
  if (e) return e;
  if (a->phases < 0 || a->phases > 2 || !a->q || !a->k) return KATA_ERR_INVALID;
  if (a->phases != 2 && (!a->v || !a->beta || !a->U)) return KATA_ERR_INVALID;
  if (a->phases == 0 && (!a->o || !a->den)) return KATA_ERR_INVALID;
  if (a->phases == 2 && a->o && !a->U) return KATA_ERR_INVALID;
  if (a->phases == 2 && a->normalize && a->o && !a->den) return KATA_ERR_INVALID;
  DeltaParams p = base_params(a->q, a->k, a->v, a->beta, a->B, a->T, a->H, a->D, a->Dv, a->M, a->normalize,
                              a->scale, a->eps);
  p.U = a->U;
  p.E = a->E;
  p.o = a->o;
  p.den = a->den;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (a->dtype) {
    case KATA_DTYPE_F32: return fwd_typed<float>(p, a->phases, st);
    case KATA_DTYPE_BF16: return fwd_typed<__nv_bfloat16>(p, a->phases, st);
    default: return fwd_typed<__half>(p, a->phases, st);
  }
}

extern "C" size_t kata_delta_bwd_workspace_bytes(const kata_delta_bwd_args* a) {
  if (!a || a->B < 1 || a->T < 1 || a->H < 1 || a->Dv < 1) return 0;
  const size_t rows = static_cast<size_t>(a->B) * a->T * a->H;
  return sizeof(float) * (4 * rows * a->Dv + rows);
}

extern "C" int kata_delta_bwd(const kata_delta_bwd_args* a, kata_stream_t stream) {
  if (!a) return KATA_ERR_INVALID;
  int e = check(a->dtype, a->B, a->T, a->H, a->D, a->Dv, a->M);
  if (e) return e;
  if (!a->q || !a->k || !a->v || !a->beta || !a->U || !a->dout || !a->dq || !a->dk || !a->dv || !a->dbeta)
    return KATA_ERR_INVALID;
  if (!a->z && (!a->o || !a->den)) return KATA_ERR_INVALID;
  const size_t need = kata_delta_bwd_workspace_bytes(a);
  if (!a->workspace || a->workspace_bytes < need) return KATA_ERR_WORKSPACE;
  const size_t rows = static_cast<size_t>(a->B) * a->T * a->H;
  float* ws = static_cast<float*>(a->workspace);
  DeltaParams p = base_params(a->q, a->k, a->v, a->beta, a->B, a->T, a->H, a->D, a->Dv, a->M,
                              a->z ? 0 : a->normalize, a->scale, a->eps);
  p.U = const_cast<float*>(a->U);
  p.E = const_cast<float*>(a->E);
  p.o = const_cast<float*>(a->o);
  p.den = const_cast<float*>(a->den);
  p.dout = a->dout;
  p.dq = a->dq;
  p.dk = a->dk;
  p.dv = a->dv;
  p.dbeta = a->dbeta;
  p.dnum = a->z ? const_cast<float*>(a->dout) : ws;
  p.dU = ws + rows * a->Dv;
  p.Y = ws + 2 * rows * a->Dv;
  p.z = a->z ? const_cast<float*>(a->z) : ws + 4 * rows * a->Dv;
  // dU at slot 1, Y at slot 2; the recomputed E takes slot 3 (bwd_typed addresses it from dU).
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (a->dtype) {
    case KATA_DTYPE_F32: return bwd_typed<float>(p, a->z != nullptr, st);
    case KATA_DTYPE_BF16: return bwd_typed<__nv_bfloat16>(p, a->z != nullptr, st);
    default: return bwd_typed<__half>(p, a->z != nullptr, st);
  }
}
