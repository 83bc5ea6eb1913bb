// gdn.cu -- gated delta rule (fla's chunk_gated_delta_rule), chunked WY form, fp32 arithmetic.
//
// Per (sequence, value head), token recurrence (fla/ops/gated_delta_rule/naive.py:13-60):
//   S <- exp(g_t) S;  u_t = beta_t (v_t - S^T k_t);  S <- S + k_t u_t^T;  o_t = scale S^T q_t.
// Chunks of C = 64 tokens, gamma = within-chunk cumulative sum of g, S0 = state entering the chunk:
//   L_ij = beta_i e^{gamma_i - gamma_j} k_i.k_j (j < i),  Tm = (I + L)^{-1}
//   W = Tm diag(beta e^gamma) K,  U0 = Tm diag(beta) V,  u = U0 - W S0
//   o_i = scale [e^{gamma_i} q_i^T S0 + sum_{j<=i} e^{gamma_i - gamma_j} (q_i.k_j) u_j]
//   S_end = e^{gamma_C} S0 + sum_j e^{gamma_C - gamma_j} k_j u_j^T
// Kernels: prep (gamma, Tm, W, U0; chunk-parallel), state (S0 per chunk and u; sequential over
// chunks, parallel over heads x 16-column slices of V), output (chunk-parallel).
// Backward: dvl (intra-chunk part of du; chunk-parallel), dstate (reverse scan of dS giving du and
// dS_end per chunk; sequential), grad (dq, dk, dv, dbeta, dg per chunk; chunk-parallel).
// The same quantities are produced by fla's Triton kernels chunk_gated_delta_rule_fwd/_bwd
// (fla/ops/gated_delta_rule/chunk.py:29-236); here every product is fp32.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "attn_common.cuh"
#include "gdn_tc.h"
#include "host_util.h"
#include "kata_b200.h"

namespace kata {
namespace {

constexpr int CH = 64;    // chunk length
constexpr int DK = 64;    // key dim (this build)
constexpr int DV = 64;    // value dim (this build)
constexpr int LD = 68;    // row of every 64-wide fp32 shared tile: 16-byte aligned, rows 4 banks apart
constexpr int TILE = CH * LD;
constexpr int NT = 256;   // threads of every kernel
constexpr int VS = 16;    // value columns per CTA of the sequential scans
constexpr int LDS_ = VS + 1;

struct GdnParams {
  const void* q;
  const void* k;
  const void* v;
  const float* g;
  const float* beta;
  const float* h0;
  void* o;
  float* ht;
  float* A;
  const int* cu;   // (N+1) token offsets or null (equal lengths T)
  const int* co;   // (N+1) chunk offsets or null
  float* gam;      // (BT, HV)
  float* W;        // (BT, HV, K)
  float* U0;       // (BT, HV, V)
  float* u;        // (BT, HV, V)
  float* hS;       // (NC, HV, K, V) state entering each chunk
  // backward
  const void* dout;
  const float* dht;
  float* dq;
  float* dk;
  float* dv;
  float* dg;
  float* dbeta;
  float* dh0;
  float* dvl;      // (BT, HV, V)
  float* du;       // (BT, HV, V)
  float* hD;       // (NC, HV, K, V) gradient of the state leaving each chunk
  int B, T, H, HV, N, NC, a_given, gva;
  float scale;
};

// chunk -> (sequence, first token (flattened over B*T), valid rows)
struct ChunkPos {
  int n, bos, len;
};

__device__ __forceinline__ ChunkPos chunk_pos(const GdnParams& p, int gc) {
  ChunkPos r;
  if (p.cu) {
    int lo = 0, hi = p.N;  // largest n with co[n] <= gc
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (p.co[mid] <= gc) lo = mid; else hi = mid;
    }
    r.n = lo;
    const int j = gc - p.co[lo];
    r.bos = p.cu[lo] + j * CH;
    r.len = min(CH, p.cu[lo + 1] - r.bos);
  } else {
    const int per = (p.T + CH - 1) / CH;
    r.n = gc / per;
    const int j = gc - r.n * per;
    r.bos = r.n * p.T + j * CH;
    r.len = min(CH, p.T - j * CH);
  }
  return r;
}

__device__ __forceinline__ void seq_range(const GdnParams& p, int n, int& bos, int& eos, int& c0, int& nc) {
  if (p.cu) {
    bos = p.cu[n];
    eos = p.cu[n + 1];
    c0 = p.co[n];
    nc = p.co[n + 1] - c0;
  } else {
    bos = n * p.T;
    eos = bos + p.T;
    nc = (p.T + CH - 1) / CH;
    c0 = n * nc;
  }
}

// ---- 64x64 fp32 tile products from shared memory (LD-strided rows): thread (ty, tx) owns rows
// ty+16r, columns tx+16c.  A(i,k) = TA ? A[k][i] : A[i][k];  B(k,j) = TB ? B[j][k] : B[k][j].
// Operands stored row-major along k (A with TA false, B with TB true) are read four k at a time
// with 16-byte loads.
template <bool TA, bool TB>
__device__ __forceinline__ void mm(float (&acc)[4][4], const float* A, const float* B) {
  const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
#pragma unroll 2
  for (int k = 0; k < 64; k += 4) {
    float a[4][4], b[4][4];  // a[r][j] = A(row ty+16r, k+j),  b[c][j] = B(k+j, col tx+16c)
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      if (!TA) {
        const float4 v = *reinterpret_cast<const float4*>(A + (ty + 16 * r) * LD + k);
        a[r][0] = v.x; a[r][1] = v.y; a[r][2] = v.z; a[r][3] = v.w;
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) a[r][j] = A[(k + j) * LD + ty + 16 * r];
      }
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      if (TB) {
        const float4 v = *reinterpret_cast<const float4*>(B + (tx + 16 * c) * LD + k);
        b[c][0] = v.x; b[c][1] = v.y; b[c][2] = v.z; b[c][3] = v.w;
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) b[c][j] = B[(k + j) * LD + tx + 16 * c];
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[r][c] = fmaf(a[r][j], b[c][j], acc[r][c]);
  }
}

__device__ __forceinline__ void zero(float (&a)[4][4]) {
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) a[r][c] = 0.f;
}

__device__ __forceinline__ void store_acc(float* C, const float (&a)[4][4]) {
  const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) C[(ty + 16 * r) * LD + tx + 16 * c] = a[r][c];
}

// Sum over the 16 threads that share a row (tx varies inside one half-warp).
__device__ __forceinline__ float row_reduce(float x) {
#pragma unroll
  for (int o = 8; o; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Load 64 rows of 64 values into a 64 x LD fp32 tile: row r starts at base + r * stride (elements);
// rows >= len are zero.  Vector loads (16 bytes), all issued before any shared store.
template <typename T>
__device__ __forceinline__ void load_rows(float* s, const T* base, size_t stride, int len) {
  constexpr int VEC = 16 / sizeof(T);       // elements per 16-byte load
  constexpr int PERROW = 64 / VEC;
  constexpr int PER = CH * PERROW / NT;     // loads per thread
  uint4 buf[PER];
#pragma unroll
  for (int m = 0; m < PER; ++m) {
    const int idx = threadIdx.x + NT * m, r = idx / PERROW, c = (idx % PERROW) * VEC;
    buf[m] = r < len ? *reinterpret_cast<const uint4*>(base + r * stride + c) : make_uint4(0u, 0u, 0u, 0u);
  }
#pragma unroll
  for (int m = 0; m < PER; ++m) {
    const int idx = threadIdx.x + NT * m, r = idx / PERROW, c = (idx % PERROW) * VEC;
    const T* e = reinterpret_cast<const T*>(&buf[m]);
#pragma unroll
    for (int x = 0; x < VEC; ++x) s[r * LD + c + x] = to_f32<T>(e[x]);
  }
}

// Rows [bos, bos+len) of a (tokens, heads, 64) tensor, head h.
template <typename T>
__device__ __forceinline__ void load_tile(float* s, const T* base, int heads, int h, int bos, int len) {
  load_rows<T>(s, base + (static_cast<size_t>(bos) * heads + h) * 64, static_cast<size_t>(heads) * 64, len);
}

__device__ __forceinline__ void load_vec(float* s, const float* base, int heads, int h, int bos, int len) {
  for (int i = threadIdx.x; i < CH; i += NT) s[i] = i < len ? base[static_cast<size_t>(bos + i) * heads + h] : 0.f;
}

template <typename T>
__device__ __forceinline__ void store_out(T* dst, float x) {
  *dst = from_f32<T>(x);
}

// Within-chunk inclusive cumulative sum of g (rows >= len hold g = 0, so gamma there = gamma_last).
__device__ __forceinline__ void chunk_cumsum(float* sGam, const float* sg) {
  if (threadIdx.x < 32) {
    const int l = threadIdx.x;
    float a = sg[2 * l], b = a + sg[2 * l + 1];
    float x = b;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, x, o);
      if (l >= o) x += y;
    }
    const float excl = x - b;
    sGam[2 * l] = excl + a;
    sGam[2 * l + 1] = excl + b;
  }
}

// ------------------------------------------------------------------------------------------------
// prep: gamma, Tm = (I+L)^{-1} (or the saved one), W, U0.  grid (NC, HV).
// ------------------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(NT) gdn_prep_kernel(GdnParams p) {
  extern __shared__ __align__(16) float sm[];
  float* sK = sm;            // k rows
  float* sL = sK + TILE;     // L, then Tm
  float* sX0 = sL + TILE;    // identity -> Tm
  float* sX1 = sX0 + TILE;   // beta e^gamma k -> W
  float* sX2 = sX1 + TILE;   // beta v -> U0
  float* sGam = sX2 + TILE;
  float* sB = sGam + CH;
  float* sg = sB + CH;
  const int gc = blockIdx.x, hv = blockIdx.y, hq = hv / (p.HV / p.H);
  const ChunkPos cp = chunk_pos(p, gc);
  load_tile<T>(sK, static_cast<const T*>(p.k), p.H, hq, cp.bos, cp.len);
  load_tile<T>(sX2, static_cast<const T*>(p.v), p.HV, hv, cp.bos, cp.len);
  load_vec(sB, p.beta, p.HV, hv, cp.bos, cp.len);
  load_vec(sg, p.g, p.HV, hv, cp.bos, cp.len);
  __syncthreads();
  chunk_cumsum(sGam, sg);
  __syncthreads();
  const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
  for (int i = threadIdx.x; i < CH * 64; i += NT) {
    const int r = i >> 6, c = i & 63;
    const float bk = sB[r] * __expf(sGam[r]);
    sX1[r * LD + c] = bk * sK[r * LD + c];
    sX2[r * LD + c] *= sB[r];
  }
  if (!p.a_given) {
    float e[4][4];
    zero(e);
    mm<false, true>(e, sK, sK);
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int i = ty + 16 * r, j = tx + 16 * c;
        sL[i * LD + j] = j < i ? sB[i] * __expf(sGam[i] - sGam[j]) * e[r][c] : 0.f;
        sX0[i * LD + j] = i == j ? 1.f : 0.f;
      }
    __syncthreads();
    // forward substitution, one column per thread: x_i -= sum_{j<i} L_ij x_j
    if (threadIdx.x < 192) {
      float* col = threadIdx.x < 64 ? sX0 + threadIdx.x : (threadIdx.x < 128 ? sX1 + threadIdx.x - 64 : sX2 + threadIdx.x - 128);
      for (int i = 1; i < CH; ++i) {
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
        int j = 0;
        for (; j + 3 < i; j += 4) {
          a0 = fmaf(sL[i * LD + j], col[j * LD], a0);
          a1 = fmaf(sL[i * LD + j + 1], col[(j + 1) * LD], a1);
          a2 = fmaf(sL[i * LD + j + 2], col[(j + 2) * LD], a2);
          a3 = fmaf(sL[i * LD + j + 3], col[(j + 3) * LD], a3);
        }
        for (; j < i; ++j) a0 = fmaf(sL[i * LD + j], col[j * LD], a0);
        col[i * LD] -= (a0 + a1) + (a2 + a3);
      }
    }
    __syncthreads();
  } else {
    // Tm given (the forward's A): W = Tm X1, U0 = Tm X2
    load_tile<float>(sX0, p.A, p.HV, hv, cp.bos, cp.len);
    __syncthreads();
    for (int i = cp.len + threadIdx.x; i < CH; i += NT) sX0[i * LD + i] = 1.f;
    __syncthreads();
    float w[4][4], uu[4][4];
    zero(w);
    zero(uu);
    mm<false, false>(w, sX0, sX1);
    mm<false, false>(uu, sX0, sX2);
    __syncthreads();
    store_acc(sX1, w);
    store_acc(sX2, uu);
    __syncthreads();
  }
  for (int i = threadIdx.x; i < cp.len * 64; i += NT) {
    const int r = i >> 6, c = i & 63;
    const size_t row = static_cast<size_t>(cp.bos + r) * p.HV + hv;
    if (!p.a_given) p.A[row * CH + c] = sX0[r * LD + c];
    p.W[row * DK + c] = sX1[r * LD + c];
    p.U0[row * DV + c] = sX2[r * LD + c];
  }
  for (int i = threadIdx.x; i < cp.len; i += NT) p.gam[static_cast<size_t>(cp.bos + i) * p.HV + hv] = sGam[i];
}

// ------------------------------------------------------------------------------------------------
// Asynchronous global -> shared copies (16 bytes; src_bytes 0 zero-fills) for the chunk pipelines.
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool pred) {
  const unsigned d = static_cast<unsigned>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(src), "r"(pred ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src, bool pred) {
  const unsigned d = static_cast<unsigned>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(d), "l"(src), "r"(pred ? 4 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

constexpr int LDW = 68;  // fp32 row of W tiles in the scans (16-byte aligned, rows 4 banks apart)

// 64 rows x 64 values of a (tokens, heads, 64) tensor, row stride `rs` elements in shared memory.
template <typename T>
__device__ __forceinline__ void cp_rows64(T* dst, int rs, const T* base, int heads, int h, int t0, int len) {
  constexpr int VEC = 16 / sizeof(T), PERROW = 64 / VEC, PER = CH * PERROW / NT;
#pragma unroll
  for (int m = 0; m < PER; ++m) {
    const int idx = threadIdx.x + NT * m, r = idx / PERROW, c = (idx % PERROW) * VEC;
    const int rr = r < len ? r : 0;
    cp_async16(dst + r * rs + c, base + (static_cast<size_t>(t0 + rr) * heads + h) * 64 + c, r < len);
  }
}
// 64 rows x VS values (columns v0..v0+VS) of a (tokens, heads, 64) tensor, dense VS-wide rows.
template <typename T>
__device__ __forceinline__ void cp_rows_slice(T* dst, const T* base, int heads, int h, int v0, int t0, int len) {
  constexpr int VEC = 16 / sizeof(T), PERROW = VS / VEC;
  for (int idx = threadIdx.x; idx < CH * PERROW; idx += NT) {
    const int r = idx / PERROW, c = (idx % PERROW) * VEC;
    const int rr = r < len ? r : 0;
    cp_async16(dst + r * VS + c, base + (static_cast<size_t>(t0 + rr) * heads + h) * 64 + v0 + c, r < len);
  }
}
__device__ __forceinline__ void cp_vec64(float* dst, const float* base, int heads, int h, int t0, int len) {
  if (threadIdx.x < CH) {
    const int r = threadIdx.x, rr = r < len ? r : 0;
    cp_async4(dst + r, base + static_cast<size_t>(t0 + rr) * heads + h, r < len);
  }
}

// ------------------------------------------------------------------------------------------------
// state: sequential over the chunks of one sequence; CTA = (16-column slice of V, n*HV + hv).
// Stores S0 of every chunk (hS) and u = U0 - W S0; final state to ht.  The next chunk's W, k, U0
// and gamma stream into the other half of a double buffer while this chunk computes.
// ------------------------------------------------------------------------------------------------
template <typename T>
struct StateSmem {
  float W[2][CH * LDW];
  T k[2][CH * (64 + 16 / sizeof(T))];
  float U0[2][CH * VS];
  float gam[2][CH];
  float S[DK * LDS_];
  float Ut[CH * LDS_];
};

template <typename T>
__global__ void __launch_bounds__(NT) gdn_state_kernel(GdnParams p) {
  extern __shared__ __align__(16) unsigned char smraw[];
  StateSmem<T>& sm = *reinterpret_cast<StateSmem<T>*>(smraw);
  constexpr int KR = 64 + 16 / sizeof(T);
  const int v0 = blockIdx.x * VS;
  const int n = blockIdx.y / p.HV, hv = blockIdx.y % p.HV, hq = hv / (p.HV / p.H);
  int bos, eos, c0, nc;
  seq_range(p, n, bos, eos, c0, nc);
  const int tr = threadIdx.x >> 4, tc = threadIdx.x & 15;
  const T* kb = static_cast<const T*>(p.k);
  auto issue = [&](int j, int b) {
    const int t0 = bos + j * CH, len = min(CH, eos - t0);
    cp_rows64<float>(sm.W[b], LDW, p.W, p.HV, hv, t0, len);
    cp_rows64<T>(sm.k[b], KR, kb, p.H, hq, t0, len);
    cp_rows_slice<float>(sm.U0[b], p.U0, p.HV, hv, v0, t0, len);
    cp_vec64(sm.gam[b], p.gam, p.HV, hv, t0, len);
    cp_async_commit();
  };
  if (nc > 0) issue(0, 0);
  for (int i = threadIdx.x; i < DK * VS; i += NT) {
    const int kk = i / VS, c = i % VS;
    sm.S[kk * LDS_ + c] = p.h0 ? p.h0[((static_cast<size_t>(n) * p.HV + hv) * DK + kk) * DV + v0 + c] : 0.f;
  }
  for (int j = 0; j < nc; ++j) {
    const int b = j & 1, gc = c0 + j, t0 = bos + j * CH, len = min(CH, eos - t0);
    if (j + 1 < nc) {
      issue(j + 1, b ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const float gC = sm.gam[b][len - 1];
    float* hs = p.hS + (static_cast<size_t>(gc) * p.HV + hv) * DK * DV;
#pragma unroll
    for (int r = 0; r < 4; ++r) hs[(tr + 16 * r) * DV + v0 + tc] = sm.S[(tr + 16 * r) * LDS_ + tc];
    // u = U0 - W S0 ; Ut = e^{gamma_C - gamma} u
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
    for (int kk = 0; kk < DK; ++kk) {
      const float sv = sm.S[kk * LDS_ + tc];
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[r] = fmaf(sm.W[b][(tr + 16 * r) * LDW + kk], sv, acc[r]);
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int i = tr + 16 * r;
      const float uu = i < len ? sm.U0[b][i * VS + tc] - acc[r] : 0.f;
      if (i < len) p.u[(static_cast<size_t>(t0 + i) * p.HV + hv) * DV + v0 + tc] = uu;
      sm.Ut[i * LDS_ + tc] = uu * __expf(gC - sm.gam[b][i]);
    }
    __syncthreads();
    // S = e^{gamma_C} S + k^T Ut
    const float eC = __expf(gC);
    float sacc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
    for (int i = 0; i < CH; ++i) {
      const float uv = sm.Ut[i * LDS_ + tc];
#pragma unroll
      for (int r = 0; r < 4; ++r) sacc[r] = fmaf(to_f32<T>(sm.k[b][i * KR + tr + 16 * r]), uv, sacc[r]);
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int kk = tr + 16 * r;
      sm.S[kk * LDS_ + tc] = eC * sm.S[kk * LDS_ + tc] + sacc[r];
    }
    __syncthreads();
  }
  if (p.ht)
    for (int i = threadIdx.x; i < DK * VS; i += NT) {
      const int kk = i / VS, c = i % VS;
      p.ht[((static_cast<size_t>(n) * p.HV + hv) * DK + kk) * DV + v0 + c] = sm.S[kk * LDS_ + c];
    }
}

// ------------------------------------------------------------------------------------------------
// output: o = scale [e^gamma (Q S0) + (tril(Q K^T) o Gamma) u].  grid (NC, HV).
// ------------------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(NT) gdn_out_kernel(GdnParams p) {
  extern __shared__ __align__(16) float sm[];
  float* sQ = sm;
  float* sK = sQ + TILE;
  float* sS = sK + TILE;
  float* sU = sS + TILE;
  float* sP = sU + TILE;
  float* sGam = sP + TILE;
  const int gc = blockIdx.x, hv = blockIdx.y, hq = hv / (p.HV / p.H);
  const ChunkPos cp = chunk_pos(p, gc);
  load_tile<T>(sQ, static_cast<const T*>(p.q), p.H, hq, cp.bos, cp.len);
  load_tile<T>(sK, static_cast<const T*>(p.k), p.H, hq, cp.bos, cp.len);
  load_tile<float>(sU, p.u, p.HV, hv, cp.bos, cp.len);
  load_vec(sGam, p.gam, p.HV, hv, cp.bos, cp.len);
  load_rows<float>(sS, p.hS + (static_cast<size_t>(gc) * p.HV + hv) * DK * DV, DV, DK);
  __syncthreads();
  const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
  float acc[4][4], e[4][4];
  zero(acc);
  zero(e);
  mm<false, false>(acc, sQ, sS);
  mm<false, true>(e, sQ, sK);
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = ty + 16 * r;
    const float eg = __expf(sGam[i]);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int j = tx + 16 * c;
      acc[r][c] *= eg;
      sP[i * LD + j] = j <= i ? __expf(sGam[i] - sGam[j]) * e[r][c] : 0.f;
    }
  }
  __syncthreads();
  mm<false, false>(acc, sP, sU);
  T* o = static_cast<T*>(p.o);
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = ty + 16 * r;
    if (i < cp.len)
#pragma unroll
      for (int c = 0; c < 4; ++c)
        store_out<T>(o + (static_cast<size_t>(cp.bos + i) * p.HV + hv) * DV + tx + 16 * c, p.scale * acc[r][c]);
  }
}

// ------------------------------------------------------------------------------------------------
// backward 0: dvl_j = scale sum_{i>=j} e^{gamma_i - gamma_j} (q_i.k_j) dO_i.  grid (NC, HV).
// ------------------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(NT) gdn_dvl_kernel(GdnParams p) {
  extern __shared__ __align__(16) float sm[];
  float* sQ = sm;
  float* sK = sQ + TILE;
  float* sDO = sK + TILE;
  float* sP = sDO + TILE;
  float* sGam = sP + TILE;
  const int gc = blockIdx.x, hv = blockIdx.y, hq = hv / (p.HV / p.H);
  const ChunkPos cp = chunk_pos(p, gc);
  load_tile<T>(sQ, static_cast<const T*>(p.q), p.H, hq, cp.bos, cp.len);
  load_tile<T>(sK, static_cast<const T*>(p.k), p.H, hq, cp.bos, cp.len);
  load_tile<T>(sDO, static_cast<const T*>(p.dout), p.HV, hv, cp.bos, cp.len);
  load_vec(sGam, p.gam, p.HV, hv, cp.bos, cp.len);
  __syncthreads();
  const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
  float e[4][4];
  zero(e);
  mm<false, true>(e, sK, sQ);  // [j][i] = k_j . q_i
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int j = ty + 16 * r, i = tx + 16 * c;
      sP[j * LD + i] = i >= j ? p.scale * __expf(sGam[i] - sGam[j]) * e[r][c] : 0.f;
    }
  __syncthreads();
  float acc[4][4];
  zero(acc);
  mm<false, false>(acc, sP, sDO);
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int j = ty + 16 * r;
    if (j < cp.len)
#pragma unroll
      for (int c = 0; c < 4; ++c) p.dvl[(static_cast<size_t>(cp.bos + j) * p.HV + hv) * DV + tx + 16 * c] = acc[r][c];
  }
}

// ------------------------------------------------------------------------------------------------
// backward 1: reverse scan of dS; CTA = (16-column slice of V, n*HV + hv).
//   dS_end(c) stored to hD;  du = dvl + e^{gamma_C - gamma} (k dS);
//   dS <- e^{gamma_C} dS + (scale e^gamma q)^T dO - W^T du;  dh0 = dS after the first chunk.
// The previous chunk's W, k, q, dvl, dO and gamma are prefetched into a double buffer.
// ------------------------------------------------------------------------------------------------
template <typename T>
struct DstateSmem {
  float W[2][CH * LDW];
  T k[2][CH * (64 + 16 / sizeof(T))];
  T q[2][CH * (64 + 16 / sizeof(T))];
  float dvl[2][CH * VS];
  T dO[2][CH * VS];
  float gam[2][CH];
  float S[DK * LDS_];
  float DU[CH * LDS_];
  float f[CH];
};

template <typename T>
__global__ void __launch_bounds__(NT) gdn_dstate_kernel(GdnParams p) {
  extern __shared__ __align__(16) unsigned char smraw[];
  DstateSmem<T>& sm = *reinterpret_cast<DstateSmem<T>*>(smraw);
  constexpr int KR = 64 + 16 / sizeof(T);
  const int v0 = blockIdx.x * VS;
  const int n = blockIdx.y / p.HV, hv = blockIdx.y % p.HV, hq = hv / (p.HV / p.H);
  int bos, eos, c0, nc;
  seq_range(p, n, bos, eos, c0, nc);
  const int tr = threadIdx.x >> 4, tc = threadIdx.x & 15;
  const T* kb = static_cast<const T*>(p.k);
  const T* qb = static_cast<const T*>(p.q);
  const T* dob = static_cast<const T*>(p.dout);
  auto issue = [&](int j, int b) {
    const int t0 = bos + j * CH, len = min(CH, eos - t0);
    cp_rows64<float>(sm.W[b], LDW, p.W, p.HV, hv, t0, len);
    cp_rows64<T>(sm.k[b], KR, kb, p.H, hq, t0, len);
    cp_rows64<T>(sm.q[b], KR, qb, p.H, hq, t0, len);
    cp_rows_slice<float>(sm.dvl[b], p.dvl, p.HV, hv, v0, t0, len);
    cp_rows_slice<T>(sm.dO[b], dob, p.HV, hv, v0, t0, len);
    cp_vec64(sm.gam[b], p.gam, p.HV, hv, t0, len);
    cp_async_commit();
  };
  if (nc > 0) issue(nc - 1, 0);
  for (int i = threadIdx.x; i < DK * VS; i += NT) {
    const int kk = i / VS, c = i % VS;
    sm.S[kk * LDS_ + c] = p.dht ? p.dht[((static_cast<size_t>(n) * p.HV + hv) * DK + kk) * DV + v0 + c] : 0.f;
  }
  for (int it = 0; it < nc; ++it) {
    const int j = nc - 1 - it, b = it & 1, gc = c0 + j, t0 = bos + j * CH, len = min(CH, eos - t0);
    if (j > 0) {
      issue(j - 1, b ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const float gC = sm.gam[b][len - 1];
    if (threadIdx.x < CH) sm.f[threadIdx.x] = threadIdx.x < len ? p.scale * __expf(sm.gam[b][threadIdx.x]) : 0.f;
    float* hd = p.hD + (static_cast<size_t>(gc) * p.HV + hv) * DK * DV;
#pragma unroll
    for (int r = 0; r < 4; ++r) hd[(tr + 16 * r) * DV + v0 + tc] = sm.S[(tr + 16 * r) * LDS_ + tc];
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
    for (int kk = 0; kk < DK; ++kk) {
      const float sv = sm.S[kk * LDS_ + tc];
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[r] = fmaf(to_f32<T>(sm.k[b][(tr + 16 * r) * KR + kk]), sv, acc[r]);
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int i = tr + 16 * r;
      const float d = i < len ? sm.dvl[b][i * VS + tc] + __expf(gC - sm.gam[b][i]) * acc[r] : 0.f;
      sm.DU[i * LDS_ + tc] = d;
      if (i < len) p.du[(static_cast<size_t>(t0 + i) * p.HV + hv) * DV + v0 + tc] = d;
    }
    __syncthreads();
    const float eC = __expf(gC);
    float sacc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
    for (int i = 0; i < CH; ++i) {
      const float dov = sm.f[i] * to_f32<T>(sm.dO[b][i * VS + tc]);
      const float duv = sm.DU[i * LDS_ + tc];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int kk = tr + 16 * r;
        sacc[r] = fmaf(to_f32<T>(sm.q[b][i * KR + kk]), dov, fmaf(-sm.W[b][i * LDW + kk], duv, sacc[r]));
      }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int kk = tr + 16 * r;
      sm.S[kk * LDS_ + tc] = eC * sm.S[kk * LDS_ + tc] + sacc[r];
    }
    __syncthreads();
  }
  if (p.dh0)
    for (int i = threadIdx.x; i < DK * VS; i += NT) {
      const int kk = i / VS, c = i % VS;
      p.dh0[((static_cast<size_t>(n) * p.HV + hv) * DK + kk) * DV + v0 + c] = sm.S[kk * LDS_ + c];
    }
}

// ------------------------------------------------------------------------------------------------
// backward 2: per-chunk gradients dq, dk, dv, dbeta, dg.  grid (NC, HV).
// ------------------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(NT) gdn_grad_kernel(GdnParams p) {
  extern __shared__ __align__(16) float sm[];
  float* sQ = sm;
  float* sK = sQ + TILE;
  float* sU = sK + TILE;
  float* sDU = sU + TILE;
  float* sDO = sDU + TILE;
  float* sS = sDO + TILE;
  float* sD = sS + TILE;
  float* sT = sD + TILE;
  float* X1 = sT + TILE;
  float* X2 = X1 + TILE;
  float* X3 = X2 + TILE;
  float* sGam = X3 + TILE;
  float* sB = sGam + CH;
  float* sDg = sB + CH;
  float* sDb = sDg + CH;
  float* sRed = sDb + CH;
  const int gc = blockIdx.x, hv = blockIdx.y, hq = hv / (p.HV / p.H);
  const ChunkPos cp = chunk_pos(p, gc);
  const int len = cp.len;
  load_tile<T>(sQ, static_cast<const T*>(p.q), p.H, hq, cp.bos, len);
  load_tile<T>(sK, static_cast<const T*>(p.k), p.H, hq, cp.bos, len);
  load_tile<float>(sU, p.u, p.HV, hv, cp.bos, len);
  load_tile<float>(sDU, p.du, p.HV, hv, cp.bos, len);
  load_tile<T>(sDO, static_cast<const T*>(p.dout), p.HV, hv, cp.bos, len);
  const size_t st = (static_cast<size_t>(gc) * p.HV + hv) * DK * DV;
  load_rows<float>(sS, p.hS + st, DV, DK);
  load_rows<float>(sD, p.hD + st, DV, DK);
  load_tile<float>(sT, p.A, p.HV, hv, cp.bos, len);
  load_vec(sGam, p.gam, p.HV, hv, cp.bos, len);
  load_vec(sB, p.beta, p.HV, hv, cp.bos, len);
  for (int i = threadIdx.x; i < CH; i += NT) {
    sDg[i] = 0.f;
    sDb[i] = 0.f;
  }
  if (threadIdx.x == 0) sRed[0] = 0.f;
  __syncthreads();
  if (len < CH)  // rows past the end: gamma_last (their g is 0) and identity rows of Tm
    for (int i = threadIdx.x; i < CH; i += NT)
      if (i >= len) {
        sGam[i] = sGam[len - 1];
        sT[i * LD + i] = 1.f;
      }
  __syncthreads();
  const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
  const float gC = sGam[CH - 1];
  float dq[4][4], dk[4][4], t[4][4], e[4][4];
  zero(dq);
  zero(dk);
  // (1) dW = -du S0^T
  zero(t);
  mm<false, true>(t, sDU, sS);
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) t[r][c] = -t[r][c];
  store_acc(X1, t);
  __syncthreads();
  // (2) Y_V = Tm^T du -> X2;  (3) Y_K = Tm^T dW -> X3
  zero(t);
  mm<true, false>(t, sT, sDU);
  store_acc(X2, t);
  zero(e);
  mm<true, false>(e, sT, X1);
  store_acc(X3, e);
  // (4) dv = beta Y_V; dbeta += v.Y_V + e^gamma k.Y_K; dk += beta e^gamma Y_K; dgamma += beta e^gamma k.Y_K
  const T* vb = static_cast<const T*>(p.v);
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = ty + 16 * r;
    const float eg = __expf(sGam[i]), bi = sB[i];
    float db = 0.f, dgm = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int col = tx + 16 * c;
      const size_t row = static_cast<size_t>(cp.bos + i) * p.HV + hv;
      const float vv = i < len ? to_f32<T>(vb[row * DV + col]) : 0.f;
      const float kk = sK[i * LD + col];
      if (i < len) p.dv[row * DV + col] = bi * t[r][c];
      dk[r][c] += bi * eg * e[r][c];
      db = fmaf(vv, t[r][c], fmaf(eg * kk, e[r][c], db));
      dgm = fmaf(bi * eg * kk, e[r][c], dgm);
    }
    db = row_reduce(db);
    dgm = row_reduce(dgm);
    if (tx == 0) {
      sDb[i] += db;
      sDg[i] += dgm;
    }
  }
  __syncthreads();
  // (5) dL = -(Y_V U0^T + Y_K W^T) (j < i); load U0 -> sT, W -> X1
  load_tile<float>(sT, p.U0, p.HV, hv, cp.bos, len);
  load_tile<float>(X1, p.W, p.HV, hv, cp.bos, len);
  __syncthreads();
  zero(t);
  mm<false, true>(t, X2, sT);
  mm<false, true>(t, X3, X1);
  zero(e);
  mm<false, true>(e, sK, sK);
  __syncthreads();  // X3 is rewritten below
  // (6) with E_ij = e^{gamma_i - gamma_j} k_i.k_j:  dbeta_i += sum_j dL E;  G = beta_i dL E;
  //     dgamma_i += sum_j G, dgamma_j -= sum_i G;  P = beta_i dL e^{gamma_i - gamma_j} -> X3
  {
    float colsum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int i = ty + 16 * r;
      float db = 0.f, dgm = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int j = tx + 16 * c;
        float P = 0.f;
        if (j < i) {
          const float dl = -t[r][c];
          const float dec = __expf(sGam[i] - sGam[j]);
          const float E = dec * e[r][c];
          db = fmaf(dl, E, db);
          const float G = sB[i] * dl * E;
          dgm += G;
          colsum[c] += G;
          P = sB[i] * dl * dec;
        }
        X3[i * LD + j] = P;
      }
      db = row_reduce(db);
      dgm = row_reduce(dgm);
      if (tx == 0) {
        sDb[i] += db;
        sDg[i] += dgm;
      }
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) atomicAdd(&sDg[tx + 16 * c], -colsum[c]);
  }
  __syncthreads();
  // (7) dk += P K + P^T K
  mm<false, false>(dk, X3, sK);
  mm<true, false>(dk, X3, sK);
  // (8) M'_ij = scale e^{gamma_i - gamma_j} dO_i.u_j (j <= i); Mg = M' q_i.k_j
  zero(t);
  mm<false, true>(t, sDO, sU);
  zero(e);
  mm<false, true>(e, sQ, sK);
  __syncthreads();
  {
    float colsum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int i = ty + 16 * r;
      float dgm = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int j = tx + 16 * c;
        float Mp = 0.f;
        if (j <= i) {
          Mp = p.scale * __expf(sGam[i] - sGam[j]) * t[r][c];
          const float Mg = Mp * e[r][c];
          dgm += Mg;
          colsum[c] += Mg;
        }
        X3[i * LD + j] = Mp;
      }
      dgm = row_reduce(dgm);
      if (tx == 0) sDg[i] += dgm;
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) atomicAdd(&sDg[tx + 16 * c], -colsum[c]);
  }
  __syncthreads();
  // (9) dq += M' K;  dk += M'^T Q
  mm<false, false>(dq, X3, sK);
  mm<true, false>(dk, X3, sQ);
  // (10) inter-chunk query term: dq += scale e^gamma (dO S0^T); dgamma_i += q_i . that
  zero(t);
  mm<false, true>(t, sDO, sS);
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = ty + 16 * r;
    const float f = p.scale * __expf(sGam[i]);
    float dgm = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float x = f * t[r][c];
      dq[r][c] += x;
      dgm = fmaf(sQ[i * LD + tx + 16 * c], x, dgm);
    }
    dgm = row_reduce(dgm);
    if (tx == 0) sDg[i] += dgm;
  }
  // (11) state-leaving term: Z = u dS_end^T; dk += e^{gamma_C - gamma_j} Z;
  //      r_j = e^{gamma_C - gamma_j} k_j.Z_j: dgamma_j -= r_j, dgamma_C += sum_j r_j + e^{gamma_C} <S0, dS_end>
  zero(t);
  mm<false, true>(t, sU, sD);
  float tot = 0.f;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int j = ty + 16 * r;
    const float f = __expf(gC - sGam[j]);
    float rr = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float x = f * t[r][c];
      dk[r][c] += x;
      rr = fmaf(sK[j * LD + tx + 16 * c], x, rr);
    }
    rr = row_reduce(rr);
    if (tx == 0) {
      sDg[j] -= rr;
      tot += rr;
    }
  }
  {
    float sd = 0.f;
    for (int i = threadIdx.x; i < DK * DV; i += NT) sd = fmaf(sS[(i >> 6) * LD + (i & 63)], sD[(i >> 6) * LD + (i & 63)], sd);
    sd = sd * __expf(gC) + tot;
#pragma unroll
    for (int o = 16; o; o >>= 1) sd += __shfl_xor_sync(0xffffffffu, sd, o);
    if ((threadIdx.x & 31) == 0) atomicAdd(sRed, sd);
  }
  __syncthreads();
  if (threadIdx.x == 0) sDg[CH - 1] += sRed[0];
  __syncthreads();
  // (12) dg = reverse cumulative sum of dgamma within the chunk
  if (threadIdx.x < 32) {
    const int l = threadIdx.x;
    // reverse order: element m = 63 - idx
    const float a = sDg[CH - 1 - 2 * l], b2 = a + sDg[CH - 2 - 2 * l];
    float x = b2;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, x, o);
      if (l >= o) x += y;
    }
    const float excl = x - b2;
    const int i0 = CH - 1 - 2 * l, i1 = CH - 2 - 2 * l;
    if (i0 < len) p.dg[static_cast<size_t>(cp.bos + i0) * p.HV + hv] = excl + a;
    if (i1 < len) p.dg[static_cast<size_t>(cp.bos + i1) * p.HV + hv] = excl + b2;
  }
  for (int i = threadIdx.x; i < len; i += NT) p.dbeta[static_cast<size_t>(cp.bos + i) * p.HV + hv] = sDb[i];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = ty + 16 * r;
    if (i < len)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const size_t off = (static_cast<size_t>(cp.bos + i) * p.H + hq) * DK + tx + 16 * c;
        if (p.gva) {
          atomicAdd(p.dq + off, dq[r][c]);
          atomicAdd(p.dk + off, dk[r][c]);
        } else {
          p.dq[off] = dq[r][c];
          p.dk[off] = dk[r][c];
        }
      }
  }
}

constexpr size_t kSmemPrep = sizeof(float) * (5 * TILE + 3 * CH);

constexpr size_t kSmemOut = sizeof(float) * (5 * TILE + CH);
constexpr size_t kSmemDvl = sizeof(float) * (4 * TILE + CH);

constexpr size_t kSmemGrad = sizeof(float) * (11 * TILE + 4 * CH + 4);

template <typename K>
int launch(K kernel, dim3 grid, size_t smem, cudaStream_t st, const GdnParams& p) {
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
    return KATA_ERR_CUDA;
  kernel<<<grid, NT, smem, st>>>(p);
  return from_cuda(cudaGetLastError());
}

struct WsLayout {
  size_t gam, W, U0, u, hS, dvl, du, hD, fwd_total, total;
};

// Forward part (gam, W, U0, u, hS) then, for the backward, its own part (dvl, du, hD).  With
// `reuse` the forward part lives in the forward call's workspace and is not counted here.
WsLayout ws_layout(int B, int T, int HV, int NC, bool bwd, bool reuse = false) {
  const size_t rows = static_cast<size_t>(B) * T * HV;
  const size_t st = static_cast<size_t>(NC) * HV * DK * DV;
  auto al = [](size_t x) { return (x + 63) & ~static_cast<size_t>(63); };  // 256-byte aligned (floats)
  WsLayout w{};
  size_t o = 0;
  w.gam = o; o += al(rows);
  w.W = o; o += al(rows * DK);
  w.U0 = o; o += al(rows * DV);
  w.u = o; o += al(rows * DV);
  w.hS = o; o += al(st);
  w.fwd_total = o * sizeof(float);
  if (bwd) {
    if (reuse) o = 0;
    w.dvl = o; o += al(rows * DV);
    w.du = o; o += al(rows * DV);
    w.hD = o; o += al(st);
  }
  w.total = o * sizeof(float);
  return w;
}

int check_dims(int dtype, int B, int T, int H, int HV, int K, int V, int N, int NC, const int* cu, const int* co) {
  if (dtype != KATA_DTYPE_F32 && dtype != KATA_DTYPE_BF16 && dtype != KATA_DTYPE_F16) return KATA_ERR_DTYPE;
  if (B < 1 || T < 1 || H < 1 || HV < H || HV % H || N < 1 || NC < 1) return KATA_ERR_SHAPE;
  if (K != DK || V != DV) return KATA_ERR_UNSUPPORTED;
  if ((cu == nullptr) != (co == nullptr)) return KATA_ERR_INVALID;
  if (!cu && (N != B || NC != B * ((T + CH - 1) / CH))) return KATA_ERR_SHAPE;
  if (cu && B != 1) return KATA_ERR_SHAPE;
  return KATA_OK;
}

template <typename T>
int fwd_typed(GdnParams p, cudaStream_t st) {
  int e = launch(gdn_prep_kernel<T>, dim3(p.NC, p.HV), kSmemPrep, st, p);
  if (!e) e = launch(gdn_state_kernel<T>, dim3(DV / VS, p.N * p.HV), sizeof(StateSmem<T>), st, p);
  if (!e) e = launch(gdn_out_kernel<T>, dim3(p.NC, p.HV), kSmemOut, st, p);
  return e;
}

template <typename T>
int bwd_typed(GdnParams p, bool reuse, cudaStream_t st) {
  const size_t rows = static_cast<size_t>(p.B) * p.T;
  if (p.gva) {
    int e = from_cuda(cudaMemsetAsync(p.dq, 0, rows * p.H * DK * sizeof(float), st));
    if (!e) e = from_cuda(cudaMemsetAsync(p.dk, 0, rows * p.H * DK * sizeof(float), st));
    if (e) return e;
  }
  int e = KATA_OK;
  if (!reuse) {  // recompute gamma, W, U0 (from the saved Tm), then u and the chunk states
    e = launch(gdn_prep_kernel<T>, dim3(p.NC, p.HV), kSmemPrep, st, p);
    if (!e) e = launch(gdn_state_kernel<T>, dim3(DV / VS, p.N * p.HV), sizeof(StateSmem<T>), st, p);
  }
  if (!e) e = launch(gdn_dvl_kernel<T>, dim3(p.NC, p.HV), kSmemDvl, st, p);
  if (!e) e = launch(gdn_dstate_kernel<T>, dim3(DV / VS, p.N * p.HV), sizeof(DstateSmem<T>), st, p);
  if (!e) e = launch(gdn_grad_kernel<T>, dim3(p.NC, p.HV), kSmemGrad, st, p);
  return e;
}

int dispatch_fwd(int dtype, const GdnParams& p, cudaStream_t st) {
  switch (dtype) {
    case KATA_DTYPE_F32: return fwd_typed<float>(p, st);
    case KATA_DTYPE_BF16: return fwd_typed<__nv_bfloat16>(p, st);
    default: return fwd_typed<__half>(p, st);
  }
}
int dispatch_bwd(int dtype, const GdnParams& p, bool reuse, cudaStream_t st) {
  switch (dtype) {
    case KATA_DTYPE_F32: return bwd_typed<float>(p, reuse, st);
    case KATA_DTYPE_BF16: return bwd_typed<__nv_bfloat16>(p, reuse, st);
    default: return bwd_typed<__half>(p, reuse, st);
  }
}

void bind_ws(GdnParams& p, void* ws, const WsLayout& w, bool bwd, void* fwd_ws = nullptr) {
  float* f = static_cast<float*>(fwd_ws ? fwd_ws : ws);
  p.gam = f + w.gam;
  p.W = f + w.W;
  p.U0 = f + w.U0;
  p.u = f + w.u;
  p.hS = f + w.hS;
  if (bwd) {
    float* b = static_cast<float*>(ws);
    p.dvl = b + w.dvl;
    p.du = b + w.du;
    p.hD = b + w.hD;
  }
}

// Kernel family: 1 = tensor cores (16-bit inputs), 2 = fp32-exact CUDA cores, or a negative error.
int gdn_family(int algo, int dtype) {
  if (algo == KATA_ALGO_TC) return dtype == KATA_DTYPE_F32 ? KATA_ERR_UNSUPPORTED : 1;
  if (algo == KATA_ALGO_SIMT) return 2;
  if (algo != KATA_ALGO_AUTO) return KATA_ERR_INVALID;
  return dtype == KATA_DTYPE_F32 ? 2 : 1;
}

}  // namespace
}  // namespace kata

using namespace kata;

extern "C" size_t kata_gdn_fwd_workspace_bytes(const kata_gdn_fwd_args* a) {
  if (!a || a->B < 1 || a->T < 1 || a->HV < 1 || a->num_chunks < 1) return 0;
  if (gdn_family(a->algo, a->dtype) == 1) return gdn_tc_fwd_workspace_bytes(a->B, a->T, a->HV, a->num_chunks);
  return ws_layout(a->B, a->T, a->HV, a->num_chunks, false).total;
}

extern "C" int kata_gdn_fwd(const kata_gdn_fwd_args* a, kata_stream_t stream) {
  if (!a) return KATA_ERR_INVALID;
  int e = check_dims(a->dtype, a->B, a->T, a->H, a->HV, a->K, a->V, a->N, a->num_chunks, a->cu_seqlens,
                     a->chunk_offsets);
  if (e) return e;
  if (!a->q || !a->k || !a->v || !a->g || !a->beta || !a->o || !a->A) return KATA_ERR_INVALID;
  const int fam = gdn_family(a->algo, a->dtype);
  if (fam < 0) return fam;
  if (fam == 1) return gdn_tc_fwd(a, reinterpret_cast<cudaStream_t>(stream));
  const WsLayout w = ws_layout(a->B, a->T, a->HV, a->num_chunks, false);
  if (!a->workspace || a->workspace_bytes < w.total) return KATA_ERR_WORKSPACE;
  GdnParams p{};
  p.q = a->q;
  p.k = a->k;
  p.v = a->v;
  p.g = a->g;
  p.beta = a->beta;
  p.h0 = a->h0;
  p.o = a->o;
  p.ht = a->ht;
  p.A = a->A;
  p.cu = a->cu_seqlens;
  p.co = a->chunk_offsets;
  p.B = a->B;
  p.T = a->T;
  p.H = a->H;
  p.HV = a->HV;
  p.N = a->N;
  p.NC = a->num_chunks;
  p.scale = a->scale;
  p.a_given = 0;
  bind_ws(p, a->workspace, w, false);
  return dispatch_fwd(a->dtype, p, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" size_t kata_gdn_bwd_workspace_bytes(const kata_gdn_bwd_args* a) {
  if (!a || a->B < 1 || a->T < 1 || a->HV < 1 || a->num_chunks < 1) return 0;
  if (gdn_family(a->algo, a->dtype) == 1)
    return gdn_tc_bwd_workspace_bytes(a->B, a->T, a->HV, a->num_chunks, a->fwd_workspace != nullptr);
  return ws_layout(a->B, a->T, a->HV, a->num_chunks, true, a->fwd_workspace != nullptr).total;
}

extern "C" int kata_gdn_bwd(const kata_gdn_bwd_args* a, kata_stream_t stream) {
  if (!a) return KATA_ERR_INVALID;
  int e = check_dims(a->dtype, a->B, a->T, a->H, a->HV, a->K, a->V, a->N, a->num_chunks, a->cu_seqlens,
                     a->chunk_offsets);
  if (e) return e;
  if (!a->q || !a->k || !a->v || !a->g || !a->beta || !a->A || !a->dout || !a->dq || !a->dk || !a->dv || !a->dg ||
      !a->dbeta)
    return KATA_ERR_INVALID;
  const int fam = gdn_family(a->algo, a->dtype);
  if (fam < 0) return fam;
  if (a->grad_dtype != KATA_DTYPE_F32 && (a->grad_dtype != a->dtype || fam != 1 || a->HV != a->H))
    return a->grad_dtype == a->dtype ? KATA_ERR_UNSUPPORTED : KATA_ERR_DTYPE;
  if (fam == 1) return gdn_tc_bwd(a, reinterpret_cast<cudaStream_t>(stream));
  const bool reuse = a->fwd_workspace != nullptr;
  const WsLayout w = ws_layout(a->B, a->T, a->HV, a->num_chunks, true, reuse);
  if (!a->workspace || a->workspace_bytes < w.total) return KATA_ERR_WORKSPACE;
  GdnParams p{};
  p.q = a->q;
  p.k = a->k;
  p.v = a->v;
  p.g = a->g;
  p.beta = a->beta;
  p.h0 = a->h0;
  p.A = const_cast<float*>(a->A);
  p.cu = a->cu_seqlens;
  p.co = a->chunk_offsets;
  p.dout = a->dout;
  p.dht = a->dht;
  p.dq = static_cast<float*>(a->dq);
  p.dk = static_cast<float*>(a->dk);
  p.dv = static_cast<float*>(a->dv);
  p.dg = a->dg;
  p.dbeta = a->dbeta;
  p.dh0 = a->dh0;
  p.B = a->B;
  p.T = a->T;
  p.H = a->H;
  p.HV = a->HV;
  p.N = a->N;
  p.NC = a->num_chunks;
  p.scale = a->scale;
  p.a_given = 1;
  p.gva = a->HV != a->H;
  bind_ws(p, a->workspace, w, true, const_cast<void*>(a->fwd_workspace));
  return dispatch_bwd(a->dtype, p, reuse, reinterpret_cast<cudaStream_t>(stream));
}
