// delta_scan.cu -- SPD delta rule ("flash_delta", kata/spd/flash_delta.py) on B200.
//
// Kernel value (all M*M group pairs, E = D/M):  kappa(x,y) = sum_{g,h} (scale x_g . y_h)^2,
// which is exactly the "sum" score of the attention kernels, and which factors through the
// E^2-dimensional map psi(x)[a,b] = scale * sum_g x_{g,a} x_{g,b}:  kappa(x,y) = psi(x).psi(y)
// (its upper triangle, off-diagonal entries weighted by sqrt 2, is what the scans use).
//   L = tril(kappa(k,k), -1),  U = (I + diag(beta) L)^{-1} diag(beta) V,  num = tril(kappa(q,k)) U
// Forward
//   prep    (chunk-parallel): Tm_c = (I + diag(beta) L_cc)^{-1} for every 64-row chunk
//   u_scan  (sequential over chunks, O(T)): E_c = psi(K_c) H_c + L_cc U_c with the state
//           H_c = sum_{c'<c} psi(K_c')^T U_c'  (F x Dv, F = E^2), U_c = Tm_c beta (V_c - psi(K_c) H_c)
//   readout: the attention forward (sum score) with v := U gives num / den' and den
// Backward (dO' = dO/(den+eps), z = <dO,o>/(den+eps) when normalised)
//   attention backward (sum score, v := U, den := den+eps, delta := <dO,o>): dq, the key-role dk
//           and dU = tril(kappa(q,k))^T dO'
//   y_scan  (reverse, O(T)): Y_c = Tm_c^T (dU_c - psi(K_c) G_c),  G_c = sum_{c'>c} psi(K_c')^T (beta Y)_c'
//   attention backward with q := k, v := U, dO := -beta Y, den := 1, delta := 0: both roles of the
//           erase kernel A_kk (its diagonal term, which L excludes, is subtracted in finalize)
//   finalize: dk = sum of the three, dv = beta Y, dbeta = Y.(V - E)
// The reference computes the same quantities with Triton K14-K21 (kata/spd/flash_delta.py:27-1116);
// its O(T^2) chunk loops become the O(T) state scans here.
#include <algorithm>
#include <cuda_bf16.h>
#include <type_traits>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "attn_common.cuh"
#include "attn_internal.h"
#include "host_util.h"
#include "tc64.cuh"

namespace kata {
namespace {

constexpr int C = 64;     // chunk rows
constexpr int NT = 256;   // threads
constexpr int LDT = 65;   // padded fp32 row of a 64-wide tile

struct DP {
  const void* q;
  const void* k;
  const void* v;
  const float* beta;
  float* U;
  float* E;
  float* Tm;        // (B,T,H,64)
  float* Lm;        // (B,T,H,64): kappa(k_i, k_j) for j < i within the chunk, 0 elsewhere
  const void* dU;   // (B,T,H,Dv) dtype (attention dv output)
  float* Y;         // (B,T,H,Dv)
  float* S;         // (B,H,E*E,Dv) final state, or null
  int B, T, H, D, Dv, M;
  float scale;
};

// ------------------------------------------------------------------------------------------------
// 64 rows x `cols` values (row t0 + r at base + (t0 + r) * stride) into an fp32 tile with row stride
// lds; rows past T are zero.  16-byte vector loads, four in flight per thread.
// ------------------------------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ void load_tile_v(float* s, int lds, const T* base, size_t stride, int t0, int cols, int T_) {
  constexpr int VEC = 16 / sizeof(T);
  const int cpr = cols / VEC, total = C * cpr;
  for (int i0 = 0; i0 < total; i0 += NT * 4) {
    uint4 buf[4];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int idx = i0 + threadIdx.x + NT * m, r = idx / cpr, c = (idx - r * cpr) * VEC;
      buf[m] = (idx < total && t0 + r < T_)
                   ? *reinterpret_cast<const uint4*>(base + static_cast<size_t>(t0 + r) * stride + c)
                   : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int idx = i0 + threadIdx.x + NT * m, r = idx / cpr, c = (idx - r * cpr) * VEC;
      if (idx < total) {
        const T* e = reinterpret_cast<const T*>(&buf[m]);
#pragma unroll
        for (int x = 0; x < VEC; ++x) s[r * lds + c + x] = to_f32<T>(e[x]);
      }
    }
  }
}

// ------------------------------------------------------------------------------------------------
// prep: Tm = (I + diag(beta) L_cc)^{-1}, L_cc[i][j] = kappa(k_i, k_j) (j < i).  grid (chunks, B*H).
// ------------------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(NT) delta_prep_kernel(DP p) {
  extern __shared__ float sm[];
  const int D = p.D, M = p.M, E = D / M, ldk = D + 1;
  float* sK = sm;                 // 64 x (D+1)
  float* sL = sK + C * ldk;       // 64 x 65: L, then the identity -> Tm columns
  float* sX = sL + C * LDT;       // 64 x 65
  float* sB = sX + C * LDT;
  const int c0 = blockIdx.x * C, bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const size_t rowbase = static_cast<size_t>(b) * p.T * p.H + h;  // + t*H
  const T* k = static_cast<const T*>(p.k) + rowbase * D;
  load_tile_v<T>(sK, ldk, k, static_cast<size_t>(p.H) * D, c0, D, p.T);
  for (int i = threadIdx.x; i < C; i += NT) sB[i] = c0 + i < p.T ? p.beta[(rowbase + static_cast<size_t>(c0 + i) * p.H)] : 0.f;
  __syncthreads();
  const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
  float kap[4][4];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) kap[r][c] = 0.f;
  for (int g = 0; g < M; ++g)
    for (int hh = 0; hh < M; ++hh) {
      float s[4][4];
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) s[r][c] = 0.f;
      for (int e = 0; e < E; ++e) {
        float a[4], bb[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) a[r] = sK[(ty + 16 * r) * ldk + g * E + e];
#pragma unroll
        for (int c = 0; c < 4; ++c) bb[c] = sK[(tx + 16 * c) * ldk + hh * E + e];
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
          for (int c = 0; c < 4; ++c) s[r][c] = fmaf(a[r], bb[c], s[r][c]);
      }
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float x = p.scale * s[r][c];
          kap[r][c] = fmaf(x, x, kap[r][c]);
        }
    }
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int i = ty + 16 * r, j = tx + 16 * c;
      sL[i * LDT + j] = j < i ? sB[i] * kap[r][c] : 0.f;
      sX[i * LDT + j] = i == j ? 1.f : 0.f;
      if (c0 + i < p.T) p.Lm[(rowbase + static_cast<size_t>(c0 + i) * p.H) * C + j] = j < i ? kap[r][c] : 0.f;
    }
  __syncthreads();
  // forward substitution per column of the identity: x_i -= sum_{j<i} L_ij x_j
  if (threadIdx.x < C) {
    float* col = sX + threadIdx.x;
    for (int i = threadIdx.x + 1; i < C; ++i) {
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
      int j = threadIdx.x;  // Tm is lower triangular: column c is zero above row c
      for (; j + 3 < i; j += 4) {
        a0 = fmaf(sL[i * LDT + j], col[j * LDT], a0);
        a1 = fmaf(sL[i * LDT + j + 1], col[(j + 1) * LDT], a1);
        a2 = fmaf(sL[i * LDT + j + 2], col[(j + 2) * LDT], a2);
        a3 = fmaf(sL[i * LDT + j + 3], col[(j + 3) * LDT], a3);
      }
      for (; j < i; ++j) a0 = fmaf(sL[i * LDT + j], col[j * LDT], a0);
      col[i * LDT] = -((a0 + a1) + (a2 + a3));
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < C * C; i += NT) {
    const int r = i >> 6, c = i & 63, t = c0 + r;
    if (t < p.T) p.Tm[(rowbase + static_cast<size_t>(t) * p.H) * C + c] = sX[r * LDT + c];
  }
}

// ------------------------------------------------------------------------------------------------
// prep on the tensor cores (16-bit keys, E = D / M a multiple of 16, D in {64, 128}): the M^2 part
// products S_gh = K_g K_h^T of a chunk are M = 64 tcgen05 chains (one K step of 16 per 16 columns of
// a group) into tensor memory, four parts at a time, each issued twice (lane offsets 0 and 16) so
// that both lane halves of every warp hold all 64 rows; 8 warps square and sum them, thread (warp
// w, lane l) owning row 16 (w % 4) + l % 16 and 16 of the 64 columns.  bf16 / fp16 keys are exact
// in the fp32 accumulators, so kappa matches the CUDA-core form up to summation order.  The unit
// lower triangular inverse Tm = (I + diag(beta) L)^{-1} is then formed in fp32 by 16 x 16 blocks:
// the four diagonal blocks by forward substitution (64 threads, one column each), then the blocks
// at distance d = 1, 2, 3 below the diagonal as X_ij = -X_ii sum_{l=j}^{i-1} B_il X_lj.
// ------------------------------------------------------------------------------------------------
constexpr int kPrepThreads = 256;
constexpr int kPrepParts = 4;  // part accumulators in tensor memory at a time (64 columns each)

struct TcPrepSmem {
  uint8_t K[2][tc64::TB];  // the chunk's keys, 64 x 128 bytes per 64 columns, 128-byte swizzle
  float B[C][LDT];         // beta_i kappa(k_i, k_j), j < i
  float X[C][LDT];         // Tm
  float R[3][16][17];      // the sums of one distance level
  float beta[C];
  uint64_t bar;
  uint32_t tmem;
  int abort;
};

template <typename T, int D, int M>
__global__ void __launch_bounds__(kPrepThreads) delta_tc_prep_kernel(DP p) {
  using namespace tc64;
  constexpr int E = D / M, NP = M * M, NB = (NP + kPrepParts - 1) / kPrepParts;
  static_assert(E % 16 == 0 && (D == 64 || D == 128), "tensor-core prep geometry");
  extern __shared__ uint8_t smraw[];
  TcPrepSmem& sm = *reinterpret_cast<TcPrepSmem*>(align1k(smraw));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c0 = blockIdx.x * C, bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const size_t rowbase = static_cast<size_t>(b) * p.T * p.H + h;  // + t*H
  const T* kp = static_cast<const T*>(p.k) + rowbase * D;
  if (tid == 0) {
    sm.abort = 0;
    mbar_init(&sm.bar, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&sm.tmem, 256);
    tmem_relinquish();
  }
  // keys into the swizzled tiles (rows past T zero), beta
  for (int idx = tid; idx < C * (D / 8); idx += kPrepThreads) {
    const int r = idx / (D / 8), col = (idx - r * (D / 8)) * 8, t = c0 + r;
    const bool in = t < p.T;
    cp_async16(smem_u32(sm.K[col >> 6]) + toff(r, col & 63), kp + static_cast<size_t>(in ? t : c0) * p.H * D + col, in);
  }
  cp_async_commit();
  if (tid < C) sm.beta[tid] = c0 + tid < p.T ? p.beta[rowbase + static_cast<size_t>(c0 + tid) * p.H] : 0.f;
  cp_async_wait<0>();
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem;
  const int qd = warp & 3, chalf = warp >> 2, hl = lane >> 4;
  const int row = 16 * qd + (lane & 15);
  const int col0 = 32 * chalf + 16 * hl;  // this thread's 16 columns
  const uint32_t lane_base = static_cast<uint32_t>(32 * qd) << 16;
  constexpr uint32_t idesc = umma_idesc_f16(64, 64, is_bf16<T>(), false, false);
  // K-major descriptor of the 16 columns starting at column c of the key tiles
  auto kslice = [&](int c) -> uint64_t { return kdesc(sm.K[c >> 6]) + static_cast<uint64_t>(((c & 63) >> 4) * 2); };
  float kap[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) kap[j] = 0.f;
  uint32_t phase = 0;
  bool ok = true;
  for (int nb = 0; nb < NB && ok; ++nb) {
    if (tid == 0) {
      tc_fence_after();
      for (int q = 0; q < kPrepParts && nb * kPrepParts + q < NP; ++q) {
        const int pp = nb * kPrepParts + q, g = pp / M, hh = pp % M;
        const uint32_t d = tbase + static_cast<uint32_t>(q * 64);
#pragma unroll
        for (int kk = 0; kk < E / 16; ++kk) {
          const uint64_t ad = kslice(g * E + 16 * kk), bd = kslice(hh * E + 16 * kk);
          umma_ss(d, ad, bd, idesc, kk > 0 ? 1u : 0u);
          umma_ss(d + (16u << 16), ad, bd, idesc, kk > 0 ? 1u : 0u);
        }
      }
      umma_commit(&sm.bar);
    }
    ok = wait_mma(&sm.bar, phase, &sm.abort);
    if (!ok) break;
    for (int q = 0; q < kPrepParts && nb * kPrepParts + q < NP; ++q) {
      float x[16];
      ld_quarter(tbase + lane_base + static_cast<uint32_t>(q * 64 + 32 * chalf), hl, x);
#pragma unroll
      for (int j = 0; j < 16; ++j) kap[j] = fmaf(x[j], x[j], kap[j]);
    }
    tc_fence_before();
    __syncthreads();  // every part read before the next batch overwrites the accumulators
  }
  if (ok) {  // (a timed-out wait leaves Tm and L unwritten, as in the scans)
    const float sc2 = p.scale * p.scale, bt = sm.beta[row];
    const int t = c0 + row;
    float* lrow = p.Lm + (rowbase + static_cast<size_t>(t < p.T ? t : 0) * p.H) * C + col0;
#pragma unroll
    for (int j4 = 0; j4 < 4; ++j4) {
      float4 lv;
      float* l = &lv.x;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = col0 + 4 * j4 + j;
        l[j] = c < row ? sc2 * kap[4 * j4 + j] : 0.f;
        sm.B[row][c] = bt * l[j];
      }
      if (t < p.T) *reinterpret_cast<float4*>(lrow + 4 * j4) = lv;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, 256);
  if (!ok) return;
  // diagonal blocks: column cc of block blk by forward substitution; zeros above the diagonal blocks
  for (int i = tid; i < C * C; i += kPrepThreads) {
    const int r = i >> 6, c = i & 63;
    if ((r >> 4) < (c >> 4)) sm.X[r][c] = 0.f;
  }
  if (tid < C) {
    const int blk = tid >> 4, cc = tid & 15, o = 16 * blk;
    float x[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      float a = r == cc ? 1.f : 0.f;
#pragma unroll
      for (int j = 0; j < r; ++j) a = fmaf(-sm.B[o + r][o + j], x[j], a);
      x[r] = r < cc ? 0.f : a;
    }
#pragma unroll
    for (int r = 0; r < 16; ++r) sm.X[o + r][o + cc] = x[r];
  }
  __syncthreads();
  for (int d = 1; d < 4; ++d) {
    const int nblk = 4 - d;
    // R_(i, j) = sum_{l=j}^{i-1} B_il X_lj for the blocks (i, j = i - d)
    for (int idx = tid; idx < nblk * 256; idx += kPrepThreads) {
      const int q = idx >> 8, r = (idx >> 4) & 15, c = idx & 15;
      const int bi = d + q, bj = q;
      float a = 0.f;
      for (int l = 16 * bj; l < 16 * bi; ++l) a = fmaf(sm.B[16 * bi + r][l], sm.X[l][16 * bj + c], a);
      sm.R[q][r][c] = a;
    }
    __syncthreads();
    for (int idx = tid; idx < nblk * 256; idx += kPrepThreads) {
      const int q = idx >> 8, r = (idx >> 4) & 15, c = idx & 15;
      const int bi = d + q, bj = q;
      float a = 0.f;
#pragma unroll
      for (int m = 0; m < 16; ++m)
        if (m <= r) a = fmaf(sm.X[16 * bi + r][16 * bi + m], sm.R[q][m][c], a);
      sm.X[16 * bi + r][16 * bj + c] = -a;
    }
    __syncthreads();
  }
  for (int i = tid; i < C * (C / 4); i += kPrepThreads) {
    const int r = i >> 4, c = (i & 15) * 4, t = c0 + r;
    if (t < p.T)
      *reinterpret_cast<float4*>(p.Tm + (rowbase + static_cast<size_t>(t) * p.H) * C + c) =
          make_float4(sm.X[r][c], sm.X[r][c + 1], sm.X[r][c + 2], sm.X[r][c + 3]);
  }
}

// psi over the upper triangle a <= b (psi(x).psi(y) = kappa(x,y)):
//   psi_f(x) = w_ab * scale * sum_g x_{g,a} x_{g,b},  w = 1 (a == b) or sqrt(2) (a < b),
// features numbered row by row, f = start(a) + (b - a), start(a) = a E - a (a - 1) / 2, and padded
// with zeros to a multiple of 64.  The scans keep a table of (a, b) per feature (0xffff: padding)
// and build psi in blocks of 64 features.
constexpr int FB = 64;       // feature block
constexpr int LDP = FB + 4;  // psi tile row: 16-byte aligned for vector reads along the features

__device__ __forceinline__ int tri_start(int a, int E) { return a * E - (a * (a - 1)) / 2; }

__device__ __forceinline__ void build_feature_table(unsigned short* tab, int E, int F) {
  const int Fsym = E * (E + 1) / 2;
  for (int a = threadIdx.x; a < E; a += NT) {
    const int st = tri_start(a, E);
    for (int bcol = a; bcol < E; ++bcol) tab[st + bcol - a] = static_cast<unsigned short>((a << 8) | bcol);
  }
  for (int f = Fsym + threadIdx.x; f < F; f += NT) tab[f] = 0xffff;
}

// psi of the 64 chunk rows for features [f0, f0 + 64): thread = (feature tid & 63, rows tid >> 6 + 4 k)
__device__ __forceinline__ void build_psi(float* sPsi, const float* sK, int ldk, int E, int M, int f0,
                                          const unsigned short* tab, float scale) {
  const int fl = threadIdx.x & (FB - 1);
  const unsigned t = tab[f0 + fl];
  if (t == 0xffffu) {
#pragma unroll 4
    for (int i = threadIdx.x >> 6; i < C; i += NT / FB) sPsi[i * LDP + fl] = 0.f;
    return;
  }
  const int a = static_cast<int>(t >> 8), bcol = static_cast<int>(t & 0xffu);
  const float w = a == bcol ? scale : scale * 1.41421356237309515f;
#pragma unroll 4
  for (int i = threadIdx.x >> 6; i < C; i += NT / FB) {
    const float* kr = sK + i * ldk;
    float acc = 0.f;
    for (int g = 0; g < M; ++g) acc = fmaf(kr[g * E + a], kr[g * E + bcol], acc);
    sPsi[i * LDP + fl] = w * acc;
  }
}

// X (64 x VS) += sign * psi (64 x 64) . S[f0 : f0+64] (64 x VS); thread (ty, tx): rows ty + 16 r,
// columns tx + 16 cc; psi read four features at a time.
template <int VS>
__device__ __forceinline__ void psi_times_state(float* X, const float* sPsi, const float* S, int f0, float sign) {
  constexpr int CPT = VS / 16;
  const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
  float acc[4][CPT];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int cc = 0; cc < CPT; ++cc) acc[r][cc] = 0.f;
#pragma unroll 2
  for (int f = 0; f < FB; f += 4) {
    float4 a[4];
    float b[4][CPT];
#pragma unroll
    for (int r = 0; r < 4; ++r) a[r] = *reinterpret_cast<const float4*>(sPsi + (ty + 16 * r) * LDP + f);
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int cc = 0; cc < CPT; ++cc) b[j][cc] = S[(f0 + f + j) * VS + tx + 16 * cc];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int cc = 0; cc < CPT; ++cc) {
        float x = acc[r][cc];
        x = fmaf(a[r].x, b[0][cc], x);
        x = fmaf(a[r].y, b[1][cc], x);
        x = fmaf(a[r].z, b[2][cc], x);
        x = fmaf(a[r].w, b[3][cc], x);
        acc[r][cc] = x;
      }
  }
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int cc = 0; cc < CPT; ++cc) X[(ty + 16 * r) * VS + tx + 16 * cc] += sign * acc[r][cc];
}

// S[f0 : f0+64] (64 x VS) += psi^T (64 x 64) . W (64 x VS); thread (ty, tx): features 4 ty + j,
// columns tx + 16 cc.
template <int VS>
__device__ __forceinline__ void state_update(float* S, const float* sPsi, const float* W, int f0) {
  constexpr int CPT = VS / 16;
  const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
  float acc[4][CPT];
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int cc = 0; cc < CPT; ++cc) acc[j][cc] = 0.f;
#pragma unroll 4
  for (int i = 0; i < C; ++i) {
    const float4 a = *reinterpret_cast<const float4*>(sPsi + i * LDP + 4 * ty);
    float b[CPT];
#pragma unroll
    for (int cc = 0; cc < CPT; ++cc) b[cc] = W[i * VS + tx + 16 * cc];
#pragma unroll
    for (int cc = 0; cc < CPT; ++cc) {
      acc[0][cc] = fmaf(a.x, b[cc], acc[0][cc]);
      acc[1][cc] = fmaf(a.y, b[cc], acc[1][cc]);
      acc[2][cc] = fmaf(a.z, b[cc], acc[2][cc]);
      acc[3][cc] = fmaf(a.w, b[cc], acc[3][cc]);
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int cc = 0; cc < CPT; ++cc) S[(f0 + 4 * ty + j) * VS + tx + 16 * cc] += acc[j][cc];
}

// ------------------------------------------------------------------------------------------------
// u_scan (forward): U, E for every chunk, in order.  CTA = (VS-column slice of Dv, b*h); the
// F x VS state H lives in shared memory.
// ------------------------------------------------------------------------------------------------
template <typename T, int VS>
__global__ void __launch_bounds__(NT) delta_u_scan_kernel(DP p, int F) {
  extern __shared__ __align__(16) float sm[];
  const int D = p.D, M = p.M, E = D / M, ldk = D + 1;
  constexpr int CPT = VS / 16;
  float* sH = sm;                    // F x VS
  float* sPsi = sH + F * VS;         // 64 x LDP
  float* sK = sPsi + C * LDP;        // 64 x (D+1)
  float* sT = sK + C * ldk;          // 64 x 65 (Tm)
  float* sL = sT + C * LDT;          // 64 x 65 (kappa, strictly lower)
  float* sR = sL + C * LDT;          // 64 x VS: rhs, then U
  float* sE = sR + C * VS;           // 64 x VS
  float* sB = sE + C * VS;           // 64
  unsigned short* sTab = reinterpret_cast<unsigned short*>(sB + C);  // F
  const int v0 = blockIdx.x * VS, bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const size_t rowbase = static_cast<size_t>(b) * p.T * p.H + h;
  const T* k = static_cast<const T*>(p.k) + rowbase * D;
  const T* v = static_cast<const T*>(p.v) + rowbase * p.Dv + v0;
  for (int i = threadIdx.x; i < F * VS; i += NT) sH[i] = 0.f;
  build_feature_table(sTab, E, F);
  const int nch = (p.T + C - 1) / C;
  const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
  for (int ch = 0; ch < nch; ++ch) {
    const int c0 = ch * C;
    __syncthreads();
    load_tile_v<T>(sK, ldk, k, static_cast<size_t>(p.H) * D, c0, D, p.T);
    load_tile_v<float>(sT, LDT, p.Tm + rowbase * C, static_cast<size_t>(p.H) * C, c0, C, p.T);
    load_tile_v<float>(sL, LDT, p.Lm + rowbase * C, static_cast<size_t>(p.H) * C, c0, C, p.T);
    load_tile_v<T>(sR, VS, v, static_cast<size_t>(p.H) * p.Dv, c0, VS, p.T);  // V slice
    for (int i = threadIdx.x; i < C; i += NT)
      sB[i] = c0 + i < p.T ? p.beta[rowbase + static_cast<size_t>(c0 + i) * p.H] : 0.f;
    for (int i = threadIdx.x; i < C * VS; i += NT) sE[i] = 0.f;
    // E = psi(K) H, block by block over the features
    for (int f0 = 0; f0 < F; f0 += FB) {
      __syncthreads();
      build_psi(sPsi, sK, ldk, E, M, f0, sTab, p.scale);
      __syncthreads();
      psi_times_state<VS>(sE, sPsi, sH, f0, 1.f);
    }
    __syncthreads();
    // rhs = beta (V - E) in place of V
    for (int i = threadIdx.x; i < C * VS; i += NT) sR[i] = sB[i / VS] * (sR[i] - sE[i]);
    __syncthreads();
    // U = Tm rhs  (Tm lower triangular)
    float u[4][CPT];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int i = ty + 16 * r;
#pragma unroll
      for (int cc = 0; cc < CPT; ++cc) {
        float acc = 0.f;
        for (int j = 0; j <= i; ++j) acc = fmaf(sT[i * LDT + j], sR[j * VS + tx + 16 * cc], acc);
        u[r][cc] = acc;
      }
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int cc = 0; cc < CPT; ++cc) sR[(ty + 16 * r) * VS + tx + 16 * cc] = u[r][cc];
    __syncthreads();
    // E_i += sum_{j<i} kappa(k_i, k_j) U_j ; store U, E
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int i = ty + 16 * r, t = c0 + i;
#pragma unroll
      for (int cc = 0; cc < CPT; ++cc) {
        const int c = tx + 16 * cc;
        float acc = 0.f;
        for (int j = 0; j < i; ++j) acc = fmaf(sL[i * LDT + j], sR[j * VS + c], acc);
        if (t < p.T) {
          const size_t o = (rowbase + static_cast<size_t>(t) * p.H) * p.Dv + v0 + c;
          p.U[o] = u[r][cc];
          if (p.E) p.E[o] = sE[i * VS + c] + acc;
        }
      }
    }
    // H += psi(K)^T U  (psi of the last feature block is still in shared memory)
    for (int f0 = F - FB; f0 >= 0; f0 -= FB) {
      if (f0 != F - FB) {
        __syncthreads();
        build_psi(sPsi, sK, ldk, E, M, f0, sTab, p.scale);
      }
      __syncthreads();
      state_update<VS>(sH, sPsi, sR, f0);
    }
  }
  if (p.S) {  // final state, unpacked to the full E x E feature grid: S[a,b] = S[b,a] = H_f / w_ab
    __syncthreads();
    const int Fsym = E * (E + 1) / 2;
    float* out = p.S + static_cast<size_t>(bh) * E * E * p.Dv + v0;
    for (int idx = threadIdx.x; idx < Fsym * VS; idx += NT) {
      const int f = idx / VS, c = idx % VS;
      const int a = sTab[f] >> 8, bcol = sTab[f] & 0xff;
      const float val = sH[f * VS + c] * (a == bcol ? 1.f : 0.70710678118654752f);
      out[static_cast<size_t>(a * E + bcol) * p.Dv + c] = val;
      out[static_cast<size_t>(bcol * E + a) * p.Dv + c] = val;
    }
  }
}

// ------------------------------------------------------------------------------------------------
// y_scan (backward): Y_c = Tm_c^T (dU_c - psi(K_c) G),  G += psi(K_c)^T (beta Y_c), reverse order
// ------------------------------------------------------------------------------------------------
template <typename T, int VS>
__global__ void __launch_bounds__(NT) delta_y_scan_kernel(DP p, int F) {
  extern __shared__ __align__(16) float sm[];
  const int D = p.D, M = p.M, E = D / M, ldk = D + 1;
  constexpr int CPT = VS / 16;
  float* sG = sm;
  float* sPsi = sG + F * VS;
  float* sK = sPsi + C * LDP;
  float* sT = sK + C * ldk;
  float* sX = sT + C * LDT;   // 64 x VS: dU - psi G, then beta Y
  float* sB = sX + C * VS;
  unsigned short* sTab = reinterpret_cast<unsigned short*>(sB + C);
  const int v0 = blockIdx.x * VS, bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const size_t rowbase = static_cast<size_t>(b) * p.T * p.H + h;
  const T* k = static_cast<const T*>(p.k) + rowbase * D;
  const T* dU = static_cast<const T*>(p.dU) + rowbase * p.Dv + v0;
  for (int i = threadIdx.x; i < F * VS; i += NT) sG[i] = 0.f;
  build_feature_table(sTab, E, F);
  const int nch = (p.T + C - 1) / C;
  const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
  for (int ch = nch - 1; ch >= 0; --ch) {
    const int c0 = ch * C;
    __syncthreads();
    load_tile_v<T>(sK, ldk, k, static_cast<size_t>(p.H) * D, c0, D, p.T);
    load_tile_v<float>(sT, LDT, p.Tm + rowbase * C, static_cast<size_t>(p.H) * C, c0, C, p.T);
    load_tile_v<T>(sX, VS, dU, static_cast<size_t>(p.H) * p.Dv, c0, VS, p.T);
    for (int i = threadIdx.x; i < C; i += NT)
      sB[i] = c0 + i < p.T ? p.beta[rowbase + static_cast<size_t>(c0 + i) * p.H] : 0.f;
    for (int f0 = 0; f0 < F; f0 += FB) {
      __syncthreads();
      build_psi(sPsi, sK, ldk, E, M, f0, sTab, p.scale);
      __syncthreads();
      psi_times_state<VS>(sX, sPsi, sG, f0, -1.f);
    }
    __syncthreads();
    // Y = Tm^T X  (Y_i = sum_{j>=i} Tm[j][i] X_j)
    float y[4][CPT];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int i = ty + 16 * r;
#pragma unroll
      for (int cc = 0; cc < CPT; ++cc) {
        float acc = 0.f;
        for (int j = i; j < C; ++j) acc = fmaf(sT[j * LDT + i], sX[j * VS + tx + 16 * cc], acc);
        y[r][cc] = acc;
      }
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int i = ty + 16 * r, t = c0 + i;
#pragma unroll
      for (int cc = 0; cc < CPT; ++cc) {
        const int c = tx + 16 * cc;
        if (t < p.T) p.Y[(rowbase + static_cast<size_t>(t) * p.H) * p.Dv + v0 + c] = y[r][cc];
        sX[i * VS + c] = sB[i] * y[r][cc];
      }
    }
    for (int f0 = F - FB; f0 >= 0; f0 -= FB) {
      if (f0 != F - FB) {
        __syncthreads();
        build_psi(sPsi, sK, ldk, E, M, f0, sTab, p.scale);
      }
      __syncthreads();
      state_update<VS>(sG, sPsi, sX, f0);
    }
  }
}

// ================================================================================================
// Tensor-core scans (16-bit inputs, F <= 192 features, D <= 64, Dv = 64).  One CTA of 128 threads
// per (b, h) runs every chunk in order (REV: the y-scan, in reverse).  The F x 64 fp32 state lives
// in registers: thread (warp w, lane l) owns feature row 64 fb + 16 w + (l & 15) of every feature
// block fb and value columns [32 (l >> 4), +32).  Per chunk:
//   psi(K) as NFB 64 x 64 16-bit tiles (rows tokens, columns features) and the state as NFB tiles
//   (rows features, columns values); one M = 64 tcgen05 chain gives P = psi(K) . state in TMEM;
//   u-scan: rhs = beta (V - P), U = Tm rhs (fp32 on the CUDA cores), E = P + L U;
//   y-scan: X = dU - P, Y = Tm^T X, W = beta Y;
//   then the chains psi_fb^T . U (or W) (rows features) update the state, added in fp32.
// The products take 16-bit operands (psi, the state, U / beta Y rounded to the input type, as the
// reference's Triton kernels round their inter-chunk operands to bf16) with fp32 accumulation.
// ================================================================================================
template <int NFB>
struct TcScanSmem {
  uint8_t psi[NFB][tc64::TB];
  uint8_t st[NFB][tc64::TB];
  uint8_t w[tc64::TB];  // U (u-scan) or beta Y (y-scan): rows tokens, columns values, 16-bit
  // chunk inputs, double-buffered (the next chunk's copies land while this one computes)
  float Tm[2][C][68];
  float L[2][C][68];      // u-scan only: kappa(k_i, k_j), j < i
  uint16_t K[2][C * 64];  // chunk keys as loaded (16-bit), row r at r * 64
  float Kf[C][65];        // the chunk's keys in fp32, rows padded to 65 words: psi reads one column
                          // of 32 rows at a time, conflict-free (with the 128-byte rows of K it was
                          // a 32-way bank conflict on every load)
  float beta[2][C];
  float R[C][68];         // rhs, then U (u-scan) / X (y-scan): fp32, 16-byte aligned rows
  unsigned short tab[NFB * 64];
  uint64_t bar;
  uint32_t tmem;
  int abort;
};

// psi of token row pr, features [ph F / NPH, (ph + 1) F / NPH) (F = 64 NFB), into the 16-bit psi tiles,
// eight features per 16-byte store.  E and M are compile-time: the row sits in registers and every
// feature's (a, b) pair, weight and tile position are constants of the unrolled loops (a table
// lookup and two shared-memory loads per product otherwise).
template <typename T, int E, int M, int NFB, int NPH>
__device__ __forceinline__ void build_psi_row(const float* krow, int pr, int ph, float scale,
                                              uint8_t (*psi)[tc64::TB]) {
  constexpr int F = 64 * NFB, FH = F / NPH, FSYM = E * (E + 1) / 2;
  static_assert(FH % 8 == 0, "whole 16-byte stores per part");
  float k[M * E];
#pragma unroll
  for (int i = 0; i < M * E; ++i) k[i] = krow[i];
  const float w1 = scale, w2 = scale * 1.41421356237309515f;
  float buf[8];
#pragma unroll
  for (int f = 0; f < F; ++f) {
    // (a, b) of feature f: row a of the upper triangle starts at a E - a (a - 1) / 2
    int a = 0;
#pragma unroll
    for (int aa = 1; aa < E; ++aa)
      if (f >= aa * E - (aa * (aa - 1)) / 2) a = aa;
    const int bc = a + f - (a * E - (a * (a - 1)) / 2);
    float v = 0.f;
    if (f < FSYM && f / FH == ph) {
#pragma unroll
      for (int g = 0; g < M; ++g) v = fmaf(k[g * E + a], k[g * E + bc], v);
      v *= a == bc ? w1 : w2;
    }
    buf[f & 7] = v;
    if ((f & 7) == 7 && f / FH == ph) {
      const int fl = f - 7;
      tc64::st_shared_v4_at(psi[fl / 64], pr, fl % 64, pack2<T>(buf[0], buf[1]), pack2<T>(buf[2], buf[3]),
                            pack2<T>(buf[4], buf[5]), pack2<T>(buf[6], buf[7]));
    }
  }
}

constexpr int kScanThreads = 256;

// Thread mapping (8 warps): warp w reads TMEM lane quarter w % 4, where both lane halves hold rows
// 16 (w % 4) .. + 15 of every M = 64 accumulator (the MMAs are issued at lane offsets 0 and 16);
// thread (w, lane) owns row m = 16 (w % 4) + lane % 16 and the 16 value columns of group
// cg = 2 (w / 4) + lane / 16.  The state (F x 64) is held as 16 columns of NFB feature rows per thread.
template <typename T, int E, int M, bool REV>
__global__ void __launch_bounds__(kScanThreads) delta_tc_scan_kernel(DP p) {
  using namespace tc64;
  constexpr int NFB = (E * (E + 1) / 2 + 63) / 64;
  using Sm = TcScanSmem<NFB>;
  extern __shared__ uint8_t smraw[];
  Sm& sm = *reinterpret_cast<Sm*>(align1k(smraw));
  constexpr bool BF = is_bf16<T>();
  constexpr int F = NFB * 64;
  const int tid = threadIdx.x;
  const int bh = blockIdx.x, b = bh / p.H, h = bh % p.H;
  constexpr int D = E * M;
  const size_t rowbase = static_cast<size_t>(b) * p.T * p.H + h;
  const T* kp = static_cast<const T*>(p.k) + rowbase * D;
  if (tid == 0) {
    sm.abort = 0;
    mbar_init(&sm.bar, 1);
    fence_mbar_init();
  }
  if (tid < 32) {
    tmem_alloc(&sm.tmem, 256);
    tmem_relinquish();
  }
  build_feature_table(sm.tab, E, F);
  const int warp = tid >> 5, ln = tid & 31;
  const int m = 16 * (warp & 3) + (ln & 15), hl = ln >> 4;
  const int col0 = 16 * (2 * (warp >> 2) + hl);                    // this thread's 16 value columns
  const uint32_t lane_base = static_cast<uint32_t>(32 * (warp & 3)) << 16;
  const uint32_t tcol = 32u * static_cast<uint32_t>(warp >> 2);   // the 32 columns this warp loads
  float S[NFB][16];
#pragma unroll
  for (int fb = 0; fb < NFB; ++fb)
#pragma unroll
    for (int j = 0; j < 16; ++j) S[fb][j] = 0.f;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem;
  uint32_t phase = 0;
  bool ok = true;
  const int nch = (p.T + C - 1) / C;
  const int pr = tid & 63, ph = tid >> 6;  // psi building: token row, quarter of the features
  // chunk `chn`'s Tm (and L), keys and beta into buffer bf by cp.async (rows past T zero-filled)
  auto issue = [&](int chn, int bf) {
    const int cc0 = chn * C, kv = D / 8;
    for (int idx = tid; idx < C * 16; idx += kScanThreads) {
      const int r = idx >> 4, c = idx & 15, t = cc0 + r;
      const bool in = t < p.T;
      const size_t o = (rowbase + static_cast<size_t>(in ? t : 0) * p.H) * C + 4 * c;
      cp_async16(smem_u32(&sm.Tm[bf][r][4 * c]), p.Tm + o, in);
      if (!REV) cp_async16(smem_u32(&sm.L[bf][r][4 * c]), p.Lm + o, in);
    }
    for (int idx = tid; idx < C * kv; idx += kScanThreads) {
      const int r = idx / kv, c = idx - r * kv, t = cc0 + r;
      const bool in = t < p.T;
      cp_async16(smem_u32(&sm.K[bf][r * 64 + 8 * c]), kp + static_cast<size_t>(in ? t : 0) * p.H * D + 8 * c, in);
    }
    if (tid < C) {
      const int t = cc0 + tid;
      const bool in = t < p.T;
      cp_async4(smem_u32(&sm.beta[bf][tid]), p.beta + rowbase + static_cast<size_t>(in ? t : 0) * p.H, in);
    }
    cp_async_commit();
  };
  if (nch > 0) issue(REV ? nch - 1 : 0, 0);
  for (int it = 0; it < nch && ok; ++it) {
    const int ch = REV ? nch - 1 - it : it, c0 = ch * C, bf = it & 1;
    if (it + 1 < nch) {
      issue(REV ? ch - 1 : ch + 1, bf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    const float(*Tm)[68] = sm.Tm[bf];
    const float(*Lm)[68] = sm.L[bf];
    const float* beta = sm.beta[bf];
    {  // keys to fp32 (this thread's own copies have landed; the barrier below publishes them all)
      const T* kr = reinterpret_cast<const T*>(sm.K[bf]);
      __syncthreads();
      for (int i = tid; i < C * D; i += kScanThreads) {
        const int r = i / D, c = i - r * D;
        sm.Kf[r][c] = to_f32<T>(kr[r * 64 + c]);
      }
    }
    // the state as 16-bit tiles (rows features), the B operand of P = psi(K) state
#pragma unroll
    for (int fb = 0; fb < NFB; ++fb) st_row16<T>(sm.st[fb], m, col0, S[fb]);
    __syncthreads();
    // psi(K): thread (token pr, quarter ph) forms features [ph F / 4, (ph + 1) F / 4)
    build_psi_row<T, E, M, NFB, kScanThreads / 64>(sm.Kf[pr], pr, ph, p.scale, sm.psi);
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {  // P = psi(K) . state   (rows tokens)
      tc_fence_after();
#pragma unroll
      for (int fb = 0; fb < NFB; ++fb) mma64x2<BF, false, true>(tbase, sm.psi[fb], sm.st[fb], fb > 0);
      umma_commit(&sm.bar);
    }
    if (!(ok = wait_mma(&sm.bar, phase, &sm.abort))) break;
    float x[16];
    ld_quarter(tbase + lane_base + tcol, hl, x);
    const int t = c0 + m;
    const bool in = t < p.T;
    const size_t vrow = (rowbase + static_cast<size_t>(in ? t : 0) * p.H) * 64 + col0;
    {
      const T* src = static_cast<const T*>(REV ? p.dU : p.v) + vrow;
      float in16[16];
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const uint4 u4 = in ? reinterpret_cast<const uint4*>(src)[q] : make_uint4(0u, 0u, 0u, 0u);
        const T* e = reinterpret_cast<const T*>(&u4);
#pragma unroll
        for (int j = 0; j < 8; ++j) in16[8 * q + j] = to_f32<T>(e[j]);
      }
      const float bm = beta[m];
#pragma unroll
      for (int j = 0; j < 16; ++j) sm.R[m][col0 + j] = REV ? in16[j] - x[j] : bm * (in16[j] - x[j]);
    }
    __syncthreads();
    float y[16];  // u-scan: U = Tm rhs (row m);  y-scan: Y = Tm^T X (row m)
#pragma unroll
    for (int j = 0; j < 16; ++j) y[j] = 0.f;
    if (!REV) {
      for (int i = 0; i <= m; ++i) {
        const float tmi = Tm[m][i];
        const float4* rr = reinterpret_cast<const float4*>(&sm.R[i][col0]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 r4 = rr[q];
          y[4 * q] = fmaf(tmi, r4.x, y[4 * q]);
          y[4 * q + 1] = fmaf(tmi, r4.y, y[4 * q + 1]);
          y[4 * q + 2] = fmaf(tmi, r4.z, y[4 * q + 2]);
          y[4 * q + 3] = fmaf(tmi, r4.w, y[4 * q + 3]);
        }
      }
    } else {
      for (int i = m; i < C; ++i) {
        const float tim = Tm[i][m];
        const float4* rr = reinterpret_cast<const float4*>(&sm.R[i][col0]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 r4 = rr[q];
          y[4 * q] = fmaf(tim, r4.x, y[4 * q]);
          y[4 * q + 1] = fmaf(tim, r4.y, y[4 * q + 1]);
          y[4 * q + 2] = fmaf(tim, r4.z, y[4 * q + 2]);
          y[4 * q + 3] = fmaf(tim, r4.w, y[4 * q + 3]);
        }
      }
    }
    __syncthreads();  // every row of R has been read
    {
      float* dst = (REV ? p.Y : p.U) + vrow;
      if (in)
#pragma unroll
        for (int q = 0; q < 4; ++q)
          reinterpret_cast<float4*>(dst)[q] = make_float4(y[4 * q], y[4 * q + 1], y[4 * q + 2], y[4 * q + 3]);
      const float wsc = REV ? beta[m] : 1.f;  // the state update takes U, or beta Y
      float w0[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) w0[j] = wsc * y[j];
      st_row16<T>(sm.w, m, col0, w0);
      if (!REV)
#pragma unroll
        for (int j = 0; j < 16; ++j) sm.R[m][col0 + j] = y[j];
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {  // state update psi_fb^T . W   (rows features)
      tc_fence_after();
#pragma unroll
      for (int fb = 0; fb < NFB; ++fb) mma64x2<BF, true, true>(tbase + 64 + 64 * fb, sm.psi[fb], sm.w, false);
      umma_commit(&sm.bar);
    }
    if (!REV && p.E && in) {  // E = P + sum_{i<m} L[m][i] U_i  (overlaps the state-update MMAs)
      for (int i = 0; i < m; ++i) {
        const float lmi = Lm[m][i];
        const float4* rr = reinterpret_cast<const float4*>(&sm.R[i][col0]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 r4 = rr[q];
          x[4 * q] = fmaf(lmi, r4.x, x[4 * q]);
          x[4 * q + 1] = fmaf(lmi, r4.y, x[4 * q + 1]);
          x[4 * q + 2] = fmaf(lmi, r4.z, x[4 * q + 2]);
          x[4 * q + 3] = fmaf(lmi, r4.w, x[4 * q + 3]);
        }
      }
      float* dst = p.E + vrow;
#pragma unroll
      for (int q = 0; q < 4; ++q)
        reinterpret_cast<float4*>(dst)[q] = make_float4(x[4 * q], x[4 * q + 1], x[4 * q + 2], x[4 * q + 3]);
    }
    if (!(ok = wait_mma(&sm.bar, phase, &sm.abort))) break;
#pragma unroll
    for (int fb = 0; fb < NFB; ++fb) {
      float d[16];
      ld_quarter(tbase + lane_base + 64 + 64 * fb + tcol, hl, d);
#pragma unroll
      for (int j = 0; j < 16; ++j) S[fb][j] += d[j];
    }
    tc_fence_before();
    __syncthreads();  // tiles and R are rewritten by the next chunk
  }
  if (ok && !REV && p.S) {  // final state, unpacked to the full E x E feature grid (S[a,b] = S[b,a])
#pragma unroll
    for (int fb = 0; fb < NFB; ++fb) {
      const unsigned tb = sm.tab[64 * fb + m];
      if (tb == 0xffffu) continue;
      const int a = static_cast<int>(tb >> 8), bc = static_cast<int>(tb & 0xffu);
      const float wt = a == bc ? 1.f : 0.70710678118654752f;
      float* out = p.S + static_cast<size_t>(bh) * E * E * 64 + col0;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float val = S[fb][j] * wt;
        out[static_cast<size_t>(a * E + bc) * 64 + j] = val;
        out[static_cast<size_t>(bc * E + a) * 64 + j] = val;
      }
    }
  }
  cp_async_wait<0>();
  if (!ok && tid == 0) mbar_drain(&sm.bar, phase ^ 1u);
  tc_fence_before();
  __syncthreads();
  if (tid < 32) tmem_dealloc(tbase, 256);
}

// ------------------------------------------------------------------------------------------------
// elementwise helpers (one warp per token row)
// ------------------------------------------------------------------------------------------------
// out[r, :] = f(in[r, :]) * (rowscale ? -rowscale[r] : 1), converted to T
template <typename T, typename S>
__global__ void __launch_bounds__(NT) delta_cvt_kernel(const S* __restrict__ in, T* __restrict__ out,
                                                       const float* __restrict__ neg_rowscale, long rows, int cols) {
  const long warp = (static_cast<long>(blockIdx.x) * NT + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const float f = neg_rowscale ? -neg_rowscale[warp] : 1.f;
  for (int c = lane; c < cols; c += 32) out[warp * cols + c] = from_f32<T>(f * to_f32<S>(in[warp * cols + c]));
}

// den' and delta for the first attention backward; ones / zeros for the second
__global__ void __launch_bounds__(NT) delta_bwd_vecs_kernel(const float* __restrict__ dout, const float* __restrict__ o,
                                                            const float* __restrict__ den, const float* __restrict__ z,
                                                            float* __restrict__ den1, float* __restrict__ del1,
                                                            float* __restrict__ ones, float* __restrict__ zeros,
                                                            long rows, int Dv, int normalize, float eps) {
  const long warp = (static_cast<long>(blockIdx.x) * NT + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  float d = 0.f;
  if (!z && normalize)
    for (int c = lane; c < Dv; c += 32) d = fmaf(dout[warp * Dv + c], o[warp * Dv + c], d);
#pragma unroll
  for (int off = 16; off; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
  if (lane == 0) {
    den1[warp] = (!z && normalize) ? den[warp] + eps : 1.f;
    del1[warp] = z ? z[warp] : d;
    ones[warp] = 1.f;
    zeros[warp] = 0.f;
  }
}

// o = normalize ? num / (den + eps) : num,  num = o_attn * den'  (den' = den if den > 0 else 1)
template <typename T>
__global__ void __launch_bounds__(NT) delta_readout_finish_kernel(const T* __restrict__ oa, const float* __restrict__ den,
                                                                  float* __restrict__ o, long rows, int Dv, int normalize,
                                                                  float eps) {
  const long warp = (static_cast<long>(blockIdx.x) * NT + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const float dn = den[warp];
  const float f = (dn > 0.f ? dn : 1.f) * (normalize ? 1.f / (dn + eps) : 1.f);
  for (int c = lane; c < Dv; c += 32) o[warp * Dv + c] = f * to_f32<T>(oa[warp * Dv + c]);
}

// dq, dk, dv, dbeta.  dk = dk1 (key role of A_qk) + dq2 + dk2 (both roles of A_kk) minus the
// diagonal term of the second call, 2 dA_ss dkappa(x, k_s)/dx |_{x = k_s}, dA_ss = -beta_s Y_s.U_s.
template <typename T>
__global__ void __launch_bounds__(NT) delta_finish_kernel(const T* __restrict__ dq1, const T* __restrict__ dk1,
                                                          const T* __restrict__ dq2, const T* __restrict__ dk2,
                                                          const T* __restrict__ kk, const T* __restrict__ vv,
                                                          const float* __restrict__ beta, const float* __restrict__ U,
                                                          const float* __restrict__ Ew, const float* __restrict__ Y,
                                                          float* __restrict__ dq, float* __restrict__ dk,
                                                          float* __restrict__ dv, float* __restrict__ dbeta, long rows,
                                                          int D, int Dv, int M, float scale) {
  extern __shared__ float sk[];  // per warp: D values of k, then the M * M group inner products
  const long warp = (static_cast<long>(blockIdx.x) * NT + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31, wl = threadIdx.x >> 5;
  if (warp >= rows) return;
  float* kr = sk + wl * (D + 16);
  float* ip = kr + D;  // ip[g * M + h] = k_g . k_h
  for (int c = lane; c < D; c += 32) kr[c] = to_f32<T>(kk[warp * D + c]);
  __syncwarp();
  const int E = D / M;
  if (lane < M * M) {
    const int g = lane / M, hh = lane - g * M;
    float s = 0.f;
    for (int e = 0; e < E; ++e) s = fmaf(kr[g * E + e], kr[hh * E + e], s);
    ip[lane] = s;
  }
  __syncwarp();
  const float bt = beta[warp];
  float yu = 0.f, db = 0.f;
  for (int c = lane; c < Dv; c += 32) {
    const float y = Y[warp * Dv + c];
    yu = fmaf(y, U[warp * Dv + c], yu);
    db = fmaf(y, to_f32<T>(vv[warp * Dv + c]) - Ew[warp * Dv + c], db);
    dv[warp * Dv + c] = bt * y;
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) {
    yu += __shfl_xor_sync(0xffffffffu, yu, off);
    db += __shfl_xor_sync(0xffffffffu, db, off);
  }
  if (lane == 0) dbeta[warp] = db;
  const float dass = -bt * yu;
  for (int c = lane; c < D; c += 32) {
    const int g = c / E, e = c - g * E;
    // dkappa(x,y)/dx_g at x = y = k: 2 scale^2 sum_h (k_g . k_h) k_h
    float dg = 0.f;
    for (int hh = 0; hh < M; ++hh) dg = fmaf(ip[g * M + hh], kr[hh * E + e], dg);
    dg *= 2.f * scale * scale;
    dq[warp * D + c] = to_f32<T>(dq1[warp * D + c]);
    dk[warp * D + c] = to_f32<T>(dk1[warp * D + c]) + to_f32<T>(dq2[warp * D + c]) + to_f32<T>(dk2[warp * D + c]) -
                       2.f * dass * dg;
  }
}

unsigned warp_blocks(long rows) { return static_cast<unsigned>((rows * 32 + NT - 1) / NT); }

size_t al256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// Value columns per scan CTA: 32 when the F x 32 state fits beside the tiles (two CTAs per SM at
// E = 16), else 16.
int feat_dim(int E) { return (E * (E + 1) / 2 + 63) / 64 * 64; }
int pick_vs(int F, int Dv) { return (Dv % 32 == 0 && F <= 640) ? 32 : 16; }

size_t scan_smem(int F, int D, int vs, bool y) {
  const size_t f = static_cast<size_t>(F) * vs + C * LDP + C * (D + 1) + C * LDT * (y ? 1 : 2) + C +
                   C * vs * (y ? 1 : 2);
  return f * sizeof(float) + static_cast<size_t>(F) * sizeof(unsigned short);
}

template <typename K>
int launch_k(K kernel, dim3 grid, size_t smem, cudaStream_t st, const DP& p, int F) {
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
    return KATA_ERR_CUDA;
  kernel<<<grid, NT, smem, st>>>(p, F);
  return from_cuda(cudaGetLastError());
}

template <typename T, int D, int M>
int run_tc_prep(const DP& p, cudaStream_t st) {
  // at least 80 KB per CTA: at most two CTAs (2 x 256 tensor-memory columns) per SM
  const size_t smem = std::max<size_t>(sizeof(TcPrepSmem) + 1024, 80 * 1024);
  auto kern = delta_tc_prep_kernel<T, D, M>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
    return KATA_ERR_CUDA;
  kern<<<dim3((p.T + C - 1) / C, p.B * p.H), kPrepThreads, smem, st>>>(p);
  return from_cuda(cudaGetLastError());
}

template <typename T>
int run_prep(const DP& p, cudaStream_t st) {
  if constexpr (!std::is_same<T, float>::value) {
    if (p.D == 64 && p.M == 4) return run_tc_prep<T, 64, 4>(p, st);
    if (p.D == 64 && p.M == 2) return run_tc_prep<T, 64, 2>(p, st);
    if (p.D == 64 && p.M == 1) return run_tc_prep<T, 64, 1>(p, st);
    if (p.D == 128 && p.M == 4) return run_tc_prep<T, 128, 4>(p, st);
    if (p.D == 128 && p.M == 2) return run_tc_prep<T, 128, 2>(p, st);
    if (p.D == 128 && p.M == 1) return run_tc_prep<T, 128, 1>(p, st);
  }
  const size_t smem = sizeof(float) * (C * (p.D + 1) + 2 * C * LDT + C);
  auto kern = delta_prep_kernel<T>;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
    return KATA_ERR_CUDA;
  kern<<<dim3((p.T + C - 1) / C, p.B * p.H), NT, smem, st>>>(p);
  return from_cuda(cudaGetLastError());
}

// The tensor-core scans serve 16-bit inputs with Dv = 64 and E = D / M = 16, M in {1, 2, 4} (the
// mixer's geometry: D = 64, M = 4; F = 192 features); the fp32 CUDA-core scans serve everything
// else (and stay the fp32-exact mode).
template <typename T>
bool tc_scan_ok(const DP& p) {
  return !std::is_same<T, float>::value && p.Dv == 64 && p.D == 16 * p.M && (p.M == 1 || p.M == 2 || p.M == 4);
}

template <typename T, bool REV>
int run_tc_scan(const DP& p, cudaStream_t st) {
  auto go = [&](auto kern, size_t smem) -> int {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
      return KATA_ERR_CUDA;
    kern<<<p.B * p.H, kScanThreads, smem, st>>>(p);
    return from_cuda(cudaGetLastError());
  };
  constexpr size_t smem = sizeof(TcScanSmem<3>) + 1024;  // E = 16: 136 features in 3 blocks
  if (p.M == 1) return go(delta_tc_scan_kernel<T, 16, 1, REV>, smem);
  if (p.M == 2) return go(delta_tc_scan_kernel<T, 16, 2, REV>, smem);
  return go(delta_tc_scan_kernel<T, 16, 4, REV>, smem);
}

template <typename T>
int run_u_scan(const DP& p, cudaStream_t st) {
  if constexpr (!std::is_same<T, float>::value)
    if (tc_scan_ok<T>(p)) return run_tc_scan<T, false>(p, st);
  const int F = feat_dim(p.D / p.M), vs = pick_vs(F, p.Dv);
  const dim3 grid(p.Dv / vs, p.B * p.H);
  if (vs == 32) return launch_k(delta_u_scan_kernel<T, 32>, grid, scan_smem(F, p.D, 32, false), st, p, F);
  return launch_k(delta_u_scan_kernel<T, 16>, grid, scan_smem(F, p.D, 16, false), st, p, F);
}

template <typename T>
int run_y_scan(const DP& p, cudaStream_t st) {
  if constexpr (!std::is_same<T, float>::value)
    if (tc_scan_ok<T>(p)) return run_tc_scan<T, true>(p, st);
  const int F = feat_dim(p.D / p.M), vs = pick_vs(F, p.Dv);
  const dim3 grid(p.Dv / vs, p.B * p.H);
  if (vs == 32) return launch_k(delta_y_scan_kernel<T, 32>, grid, scan_smem(F, p.D, 32, true), st, p, F);
  return launch_k(delta_y_scan_kernel<T, 16>, grid, scan_smem(F, p.D, 16, true), st, p, F);
}

int check(int dtype, int B, int T, int H, int D, int Dv, int M) {
  if (dtype != KATA_DTYPE_F32 && dtype != KATA_DTYPE_BF16 && dtype != KATA_DTYPE_F16) return KATA_ERR_DTYPE;
  if (B < 1 || T < 1 || H < 1 || D < 1 || Dv < 1 || M < 1 || D % M) return KATA_ERR_SHAPE;
  const int E = D / M;
  if (M > 4 || D > 256 || Dv > 256 || Dv % 16 || E % 8 || E > 64) return KATA_ERR_UNSUPPORTED;
  if (scan_smem(feat_dim(E), D, pick_vs(feat_dim(E), Dv), false) > 227 * 1024) return KATA_ERR_UNSUPPORTED;
  return KATA_OK;
}

size_t esz(int dtype) { return dtype == KATA_DTYPE_F32 ? 4 : 2; }

// ---- workspace layouts (byte offsets, 256-aligned) ------------------------------------------------
// Workspace the readout / den attention forward (sum score) can use: the Gram features of q and k
// when that form applies (bf16, groups of 16), else 0.  dv = Dv for the readout, D for den alone.
size_t attn_fwd_ws_bytes(int dtype, int B, int T, int H, int D, int dv, int M) {
  kata_attn_fwd_args f{};
  f.dtype = dtype;
  f.B = B;
  f.T = T;
  f.H = H;
  f.HQ = H;
  f.D = D;
  f.Dv = dv;
  f.M = M;
  f.score = KATA_SCORE_SUM;
  f.algo = KATA_ALGO_AUTO;
  return kata_attn_fwd_workspace_bytes(&f);
}

struct FwdWs {
  size_t Tm, Lm, Ub, oa, E, zv, attn, attn_bytes, total;
};
FwdWs fwd_ws(int dtype, int B, int T, int H, int D, int Dv, int M) {
  const size_t rows = static_cast<size_t>(B) * T * H;
  FwdWs w{};
  size_t o = 0;
  w.Tm = o; o += al256(rows * C * 4);
  w.Lm = o; o += al256(rows * C * 4);
  w.Ub = o; o += al256(rows * (Dv > D ? Dv : D) * esz(dtype));
  w.oa = o; o += al256(rows * (Dv > D ? Dv : D) * esz(dtype));
  w.E = o; o += al256(rows * Dv * 4);
  w.zv = o; o += al256(rows * D * esz(dtype));
  const size_t a1 = attn_fwd_ws_bytes(dtype, B, T, H, D, Dv, M), a2 = attn_fwd_ws_bytes(dtype, B, T, H, D, D, M);
  w.attn_bytes = a1 > a2 ? a1 : a2;
  w.attn = o; o += al256(w.attn_bytes);
  w.total = o;
  return w;
}

struct BwdWs2 {
  size_t Tm, Lm, Ub, dOb, den1, del1, ones, zeros, attn, dq1, dk1, dU, Y, Yb, dq2, dk2, dv2, E, Us, total;
};
BwdWs2 bwd_ws(int dtype, int B, int T, int H, int D, int Dv, size_t attn_bytes) {
  const size_t rows = static_cast<size_t>(B) * T * H, es = esz(dtype);
  BwdWs2 w{};
  size_t o = 0;
  w.Tm = o; o += al256(rows * C * 4);
  w.Lm = o; o += al256(rows * C * 4);
  w.Ub = o; o += al256(rows * Dv * es);
  w.dOb = o; o += al256(rows * Dv * es);
  w.den1 = o; o += al256(rows * 4);
  w.del1 = o; o += al256(rows * 4);
  w.ones = o; o += al256(rows * 4);
  w.zeros = o; o += al256(rows * 4);
  w.attn = o; o += al256(attn_bytes);
  w.dq1 = o; o += al256(rows * D * es);
  w.dk1 = o; o += al256(rows * D * es);
  w.dU = o; o += al256(rows * Dv * es);
  w.Y = o; o += al256(rows * Dv * 4);
  w.Yb = o; o += al256(rows * Dv * es);
  w.dq2 = o; o += al256(rows * D * es);
  w.dk2 = o; o += al256(rows * D * es);
  w.dv2 = o; o += al256(rows * Dv * es);
  w.E = o; o += al256(rows * Dv * 4);
  w.Us = o; o += al256(rows * Dv * 4);
  w.total = o;
  return w;
}

// Workspace of the two attention backward calls (sum score; includes the Gram features and their
// gradients when that form applies)
size_t attn_ws_bytes(int dtype, int B, int T, int H, int D, int Dv, int M) {
  kata_attn_bwd_args a{};
  a.dtype = dtype;
  a.B = B;
  a.T = T;
  a.H = H;
  a.HQ = H;
  a.D = D;
  a.Dv = Dv;
  a.M = M;
  a.score = KATA_SCORE_SUM;
  a.algo = KATA_ALGO_AUTO;
  return kata_attn_bwd_workspace_bytes(&a);
}

template <typename T>
int cvt(const void* in, bool in_f32, void* out, const float* neg_rowscale, long rows, int cols, cudaStream_t st) {
  if (in_f32)
    delta_cvt_kernel<T, float><<<warp_blocks(rows), NT, 0, st>>>(static_cast<const float*>(in), static_cast<T*>(out),
                                                                 neg_rowscale, rows, cols);
  else
    delta_cvt_kernel<T, T><<<warp_blocks(rows), NT, 0, st>>>(static_cast<const T*>(in), static_cast<T*>(out),
                                                             neg_rowscale, rows, cols);
  return from_cuda(cudaGetLastError());
}

template <typename T>
int fwd_typed(const kata_delta_fwd_args* a, cudaStream_t st) {
  const FwdWs w = fwd_ws(a->dtype, a->B, a->T, a->H, a->D, a->Dv, a->M);
  uint8_t* ws = static_cast<uint8_t*>(a->workspace);
  const long rows = static_cast<long>(a->B) * a->T * a->H;
  DP p{};
  p.q = a->q;
  p.k = a->k;
  p.v = a->v;
  p.beta = a->beta;
  p.U = a->U;
  p.E = a->E;
  p.Tm = reinterpret_cast<float*>(ws + w.Tm);
  p.Lm = reinterpret_cast<float*>(ws + w.Lm);
  p.S = a->state;
  p.B = a->B;
  p.T = a->T;
  p.H = a->H;
  p.D = a->D;
  p.Dv = a->Dv;
  p.M = a->M;
  p.scale = a->scale;
  int e = KATA_OK;
  if (a->phases != 2) {
    e = run_prep<T>(p, st);
    if (!e) e = run_u_scan<T>(p, st);
    if (e || a->phases == 1) return e;
  }
  if (!a->o && !a->den) return KATA_OK;
  // readout through the attention forward (sum score): o_attn = num / den', den
  const bool den_only = a->U == nullptr;
  const int dv = den_only ? a->D : a->Dv;
  void* vb = ws + (den_only ? w.zv : w.Ub);
  if (den_only)
    e = from_cuda(cudaMemsetAsync(vb, 0, static_cast<size_t>(rows) * a->D * esz(a->dtype), st));
  else
    e = cvt<T>(a->U, true, vb, nullptr, rows, a->Dv, st);
  if (e) return e;
  float* den = a->den ? a->den : reinterpret_cast<float*>(ws + w.E);  // E slot is free here
  kata_attn_fwd_args f{};
  f.q = a->q;
  f.k = a->k;
  f.v = vb;
  f.o = ws + w.oa;
  f.den = den;
  f.dtype = a->dtype;
  f.B = a->B;
  f.T = a->T;
  f.H = a->H;
  f.HQ = a->H;
  f.D = a->D;
  f.Dv = dv;
  f.M = a->M;
  f.score = KATA_SCORE_SUM;
  f.algo = KATA_ALGO_AUTO;
  f.scale = a->scale;
  f.workspace = w.attn_bytes ? ws + w.attn : nullptr;
  f.workspace_bytes = w.attn_bytes;
  e = kata_attn_fwd(&f, reinterpret_cast<kata_stream_t>(st));
  if (e || den_only || !a->o) return e;
  delta_readout_finish_kernel<T><<<warp_blocks(rows), NT, 0, st>>>(static_cast<const T*>(f.o), den, a->o, rows, a->Dv,
                                                                  a->normalize, a->eps);
  return from_cuda(cudaGetLastError());
}

template <typename T>
int bwd_typed(const kata_delta_bwd_args* a, cudaStream_t st) {
  const size_t attn_bytes = attn_ws_bytes(a->dtype, a->B, a->T, a->H, a->D, a->Dv, a->M);
  const BwdWs2 w = bwd_ws(a->dtype, a->B, a->T, a->H, a->D, a->Dv, attn_bytes);
  uint8_t* ws = static_cast<uint8_t*>(a->workspace);
  auto F32 = [&](size_t off) { return reinterpret_cast<float*>(ws + off); };
  const long rows = static_cast<long>(a->B) * a->T * a->H;
  DP p{};
  p.q = a->q;
  p.k = a->k;
  p.v = a->v;
  p.beta = a->beta;
  p.Tm = F32(w.Tm);
  p.Lm = F32(w.Lm);
  p.B = a->B;
  p.T = a->T;
  p.H = a->H;
  p.D = a->D;
  p.Dv = a->Dv;
  p.M = a->M;
  p.scale = a->scale;
  int e = run_prep<T>(p, st);
  const float* Ew = a->E;
  if (!e && !Ew) {  // recompute the erase term with the forward scan
    p.U = F32(w.Us);
    p.E = F32(w.E);
    e = run_u_scan<T>(p, st);
    Ew = F32(w.E);
  }
  if (!e) e = cvt<T>(a->U, true, ws + w.Ub, nullptr, rows, a->Dv, st);
  if (!e) e = cvt<T>(a->dout, true, ws + w.dOb, nullptr, rows, a->Dv, st);
  if (e) return e;
  delta_bwd_vecs_kernel<<<warp_blocks(rows), NT, 0, st>>>(a->dout, a->o, a->den, a->z, F32(w.den1), F32(w.del1),
                                                          F32(w.ones), F32(w.zeros), rows, a->Dv,
                                                          a->z ? 0 : a->normalize, a->eps);
  if ((e = from_cuda(cudaGetLastError()))) return e;
  // attention backward 1: A_qk with v := U
  kata_attn_bwd_args g{};
  g.q = a->q;
  g.k = a->k;
  g.v = ws + w.Ub;
  g.o = nullptr;
  g.den = F32(w.den1);
  g.dout = ws + w.dOb;
  g.dq = ws + w.dq1;
  g.dk = ws + w.dk1;
  g.dv = ws + w.dU;
  g.workspace = ws + w.attn;
  g.workspace_bytes = attn_bytes;
  g.dtype = a->dtype;
  g.B = a->B;
  g.T = a->T;
  g.H = a->H;
  g.HQ = a->H;
  g.D = a->D;
  g.Dv = a->Dv;
  g.M = a->M;
  g.score = KATA_SCORE_SUM;
  g.algo = KATA_ALGO_AUTO;
  g.scale = a->scale;
  e = attn_bwd_impl(&g, F32(w.del1), reinterpret_cast<kata_stream_t>(st));
  if (e) return e;
  // reverse scan for Y
  p.dU = ws + w.dU;
  p.Y = F32(w.Y);
  if ((e = run_y_scan<T>(p, st))) return e;
  if ((e = cvt<T>(F32(w.Y), true, ws + w.Yb, a->beta, rows, a->Dv, st))) return e;  // -beta Y
  // attention backward 2: A_kk (q := k) with dO := -beta Y
  g.q = a->k;
  g.den = F32(w.ones);
  g.dout = ws + w.Yb;
  g.dq = ws + w.dq2;
  g.dk = ws + w.dk2;
  g.dv = ws + w.dv2;
  e = attn_bwd_impl(&g, F32(w.zeros), reinterpret_cast<kata_stream_t>(st));
  if (e) return e;
  const size_t smem = sizeof(float) * (NT / 32) * (a->D + 16);
  delta_finish_kernel<T><<<warp_blocks(rows), NT, smem, st>>>(
      static_cast<const T*>(static_cast<const void*>(ws + w.dq1)), static_cast<const T*>(static_cast<const void*>(ws + w.dk1)),
      static_cast<const T*>(static_cast<const void*>(ws + w.dq2)), static_cast<const T*>(static_cast<const void*>(ws + w.dk2)),
      static_cast<const T*>(a->k), static_cast<const T*>(a->v), a->beta, a->U, Ew, F32(w.Y), a->dq, a->dk, a->dv,
      a->dbeta, rows, a->D, a->Dv, a->M, a->scale);
  return from_cuda(cudaGetLastError());
}

}  // namespace
}  // namespace kata

using namespace kata;

extern "C" size_t kata_delta_fwd_workspace_bytes(const kata_delta_fwd_args* a) {
  if (!a || a->B < 1 || a->T < 1 || a->H < 1 || a->D < 1 || a->Dv < 1) return 0;
  return fwd_ws(a->dtype, a->B, a->T, a->H, a->D, a->Dv, a->M).total;
}

extern "C" int kata_delta_fwd(const kata_delta_fwd_args* a, kata_stream_t stream) {
  if (!a) return KATA_ERR_INVALID;
  int e = check(a->dtype, a->B, a->T, a->H, a->D, a->Dv, a->M);
  if (e) return e;
  if (a->phases < 0 || a->phases > 2 || !a->q || !a->k) return KATA_ERR_INVALID;
  if (a->phases != 2 && (!a->v || !a->beta || !a->U)) return KATA_ERR_INVALID;
  if (a->phases == 0 && (!a->o || !a->den)) return KATA_ERR_INVALID;
  if (a->phases == 2 && a->o && !a->U) return KATA_ERR_INVALID;
  if (a->phases == 2 && a->normalize && a->o && !a->den) return KATA_ERR_INVALID;
  if (!a->workspace || a->workspace_bytes < kata_delta_fwd_workspace_bytes(a)) return KATA_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (a->dtype) {
    case KATA_DTYPE_F32: return fwd_typed<float>(a, st);
    case KATA_DTYPE_BF16: return fwd_typed<__nv_bfloat16>(a, st);
    default: return fwd_typed<__half>(a, st);
  }
}

extern "C" size_t kata_delta_bwd_workspace_bytes(const kata_delta_bwd_args* a) {
  if (!a || a->B < 1 || a->T < 1 || a->H < 1 || a->D < 1 || a->Dv < 1) return 0;
  return bwd_ws(a->dtype, a->B, a->T, a->H, a->D, a->Dv,
                attn_ws_bytes(a->dtype, a->B, a->T, a->H, a->D, a->Dv, a->M)).total;
}

extern "C" int kata_delta_bwd(const kata_delta_bwd_args* a, kata_stream_t stream) {
  if (!a) return KATA_ERR_INVALID;
  int e = check(a->dtype, a->B, a->T, a->H, a->D, a->Dv, a->M);
  if (e) return e;
  if (!a->q || !a->k || !a->v || !a->beta || !a->U || !a->dout || !a->dq || !a->dk || !a->dv || !a->dbeta)
    return KATA_ERR_INVALID;
  if (!a->z && a->normalize && (!a->o || !a->den)) return KATA_ERR_INVALID;
  if (!a->workspace || a->workspace_bytes < kata_delta_bwd_workspace_bytes(a)) return KATA_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (a->dtype) {
    case KATA_DTYPE_F32: return bwd_typed<float>(a, st);
    case KATA_DTYPE_BF16: return bwd_typed<__nv_bfloat16>(a, st);
    default: return bwd_typed<__half>(a, st);
  }
}
