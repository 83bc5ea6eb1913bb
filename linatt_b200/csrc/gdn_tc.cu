// gdn_tc.cu -- gated delta rule (fla's chunk_gated_delta_rule) on the tensor cores, bf16 / fp16 inputs.
//
// Same chunked WY algebra as gdn.cu (the fp32-exact CUDA-core path); every 64 x 64 x 64 chunk
// product here is a tcgen05.mma with M = 64 (a 64-token chunk is one tile), operands in 128-byte
// swizzled shared memory written by the threads themselves, accumulators in tensor memory.  With
// M = 64 an accumulator row m lives in TMEM lane (m % 16) + 32 * (m / 16) (+ 16 for a second tile
// interleaved in the same columns), so warp w of a 128-thread CTA reads rows 16w..16w+15 of two
// chunks at once with one 32-lane load: lanes 0-15 hold chunk slot 0, lanes 16-31 slot 1.
//
// Per (sequence, value head), chunks of C = 64 tokens, gamma = within-chunk cumulative log gate:
//   L_ij = beta_i e^{gamma_i - gamma_j} k_i.k_j (j < i),  Tm = (I + L)^{-1}  (fla's A)
//   W = Tm diag(beta e^gamma) K,  U0 = Tm diag(beta) V,  u = U0 - W S0
//   o = scale [e^gamma (Q S0) + (tril(Q K^T) o Gamma) u],  S_end = e^{gamma_C} S0 + K^T diag(e^{gamma_C-gamma}) u
// Kernels: prep (Gram on the tensor cores, Tm by forward substitution in registers, W / U0 on the
// tensor cores; two chunks per CTA), state (sequential chunk scan per head: W S0 and K^T u~ on the
// tensor cores, the fp32 state in registers), out (two chunks per CTA).  Backward: dvl (two chunks
// per CTA), dstate (reverse scan: K dS, q^T dO~ and W^T du on the tensor cores), grad (one chunk per
// CTA: seven independent products, then Y_K, dq and dk, dL, and the P K terms, all accumulated in
// tensor memory).  Products take 16-bit operands (the state, u, W, Tm, and the masked score tiles
// are rounded to the input type, as fla's kernels do) and accumulate in fp32; the recurrent state
// itself is carried in fp32 registers.  Reference arithmetic: fla/ops/gated_delta_rule/chunk.py:29-236
// (third-party, fla 0.5.x), restated in oracle/gdn_oracle.py.
#include <type_traits>

#include "attn_common.cuh"
#include "gdn_tc.h"
#include "host_util.h"
#include "sm100.cuh"
#include "tc64.cuh"

namespace kata {
namespace gdntc {
namespace {
using namespace tc64;

constexpr int CH = 64;

struct Params {
  const void* q;
  const void* k;
  const void* v;
  const float* g;
  const float* beta;
  const float* h0;
  void* o;
  float* ht;
  float* A;
  const int* cu;
  const int* co;
  float* gam;  // (rows) fp32
  void* W;     // (rows, 64) 16-bit
  float* U0;   // (rows, 64) fp32
  void* u;     // (rows, 64) 16-bit
  void* hS;    // (NC, HV, 64, 64) 16-bit: state entering each chunk
  const void* dout;
  const float* dht;
  void* dq;    // fp32, or 16-bit when grad16
  void* dk;
  void* dv;
  float* dg;
  float* dbeta;
  float* dh0;
  float* dvl;  // (rows, 64) fp32
  void* du;    // (rows, 64) 16-bit
  void* hD;    // (NC, HV, 64, 64) 16-bit: gradient of the state leaving each chunk
  int B, T, H, HV, N, NC, a_given, gva, grad16;
  float scale;
};

struct ChunkPos {
  int n, bos, len;
};

__device__ __forceinline__ ChunkPos chunk_pos(const Params& p, int gc) {
  ChunkPos r;
  if (p.cu) {
    int lo = 0, hi = p.N;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (p.co[mid] <= gc) lo = mid; else hi = mid;
    }
    r.n = lo;
    r.bos = p.cu[lo] + (gc - p.co[lo]) * CH;
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

__device__ __forceinline__ void seq_range(const Params& p, int n, int& bos, int& eos, int& c0, int& nc) {
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

// Chunk item (= chunk index * HV + value head) of slot s of a two-chunk CTA: scalars, so that no
// per-slot array is indexed with a runtime slot (which would put it in local memory).
struct Item {
  int gc, bos, len, hv, hq;
};
__device__ __forceinline__ Item item_of(const Params& p, int s, int items) {
  const int item = 2 * blockIdx.x + s;
  const bool valid = item < items;
  Item it;
  it.gc = valid ? item / p.HV : 0;
  it.hv = valid ? item % p.HV : 0;
  it.hq = it.hv / (p.HV / p.H);
  const ChunkPos cp = chunk_pos(p, it.gc);
  it.bos = cp.bos;
  it.len = valid ? cp.len : 0;
  return it;
}

// ------------------------------------------------------------------------------------------------
// tiles and MMAs
// ------------------------------------------------------------------------------------------------
// 64 fp32 columns of this thread's TMEM lane (warp-collective).
__device__ __forceinline__ void ld64(uint32_t taddr, float (&x)[64]) {
  uint32_t a[32], b[32];
  tmem_ld32(taddr, a);
  tmem_ld32(taddr + 32, b);
  tmem_wait_ld();
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    x[j] = __uint_as_float(a[j]);
    x[32 + j] = __uint_as_float(b[j]);
  }
}
__device__ __forceinline__ void st64(uint32_t taddr, const float (&x)[64]) {
  uint32_t a[32], b[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    a[j] = __float_as_uint(x[j]);
    b[j] = __float_as_uint(x[32 + j]);
  }
  tmem_st32(taddr, a);
  tmem_st32(taddr + 32, b);
}

// Row r of a tile from / to 64 floats.
template <typename T>
__device__ __forceinline__ void st_row(uint8_t* tile, int r, const float (&x)[64]) {
  const uint32_t base = smem_u32(tile);
#pragma unroll
  for (int c = 0; c < 8; ++c)
    st_shared_v4(base + toff(r, 8 * c), pack2<T>(x[8 * c], x[8 * c + 1]), pack2<T>(x[8 * c + 2], x[8 * c + 3]),
                 pack2<T>(x[8 * c + 4], x[8 * c + 5]), pack2<T>(x[8 * c + 6], x[8 * c + 7]));
}
template <typename T>
__device__ __forceinline__ void ld_row(const uint8_t* tile, int r, float (&x)[64]) {
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const uint4 u4 = *reinterpret_cast<const uint4*>(tile + toff(r, 8 * c));
    const T* e = reinterpret_cast<const T*>(&u4);
#pragma unroll
    for (int j = 0; j < 8; ++j) x[8 * c + j] = to_f32<T>(e[j]);
  }
}
// 64 16-bit values from global memory (16-byte aligned) into row r of a tile; zeros when !ok.
__device__ __forceinline__ void cp_row(uint8_t* tile, int r, const void* src, bool ok) {
  const uint4* s = reinterpret_cast<const uint4*>(src);
  uint4 v[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) v[c] = ok ? s[c] : make_uint4(0u, 0u, 0u, 0u);
  const uint32_t base = smem_u32(tile);
#pragma unroll
  for (int c = 0; c < 8; ++c) st_shared_v4(base + toff(r, 8 * c), v[c].x, v[c].y, v[c].z, v[c].w);
}
// 64 fp32 values from global memory into row r of a 16-bit tile (rounded); `diag` >= 0 writes the
// identity row instead (used for the rows of Tm past a ragged chunk's end).
template <typename T>
__device__ __forceinline__ void cvt_row(uint8_t* tile, int r, const float* src, bool ok, int diag) {
  float x[64];
  const float4* s = reinterpret_cast<const float4*>(src);
#pragma unroll
  for (int c = 0; c < 16; ++c) {
    const float4 f = ok ? s[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    x[4 * c] = f.x;
    x[4 * c + 1] = f.y;
    x[4 * c + 2] = f.z;
    x[4 * c + 3] = f.w;
  }
  if (diag >= 0)
#pragma unroll
    for (int c = 0; c < 64; ++c) x[c] = c == diag ? 1.f : 0.f;
  st_row<T>(tile, r, x);
}
// 64 floats to global memory as 16-bit values (16-byte stores).
template <typename T>
__device__ __forceinline__ void st_g16(void* dst, const float (&x)[64]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int c = 0; c < 8; ++c)
    d[c] = make_uint4(pack2<T>(x[8 * c], x[8 * c + 1]), pack2<T>(x[8 * c + 2], x[8 * c + 3]),
                      pack2<T>(x[8 * c + 4], x[8 * c + 5]), pack2<T>(x[8 * c + 6], x[8 * c + 7]));
}
__device__ __forceinline__ void st_g32(float* dst, const float (&x)[64]) {
  float4* d = reinterpret_cast<float4*>(dst);
#pragma unroll
  for (int c = 0; c < 16; ++c) d[c] = make_float4(x[4 * c], x[4 * c + 1], x[4 * c + 2], x[4 * c + 3]);
}
template <typename T>
__device__ __forceinline__ void ld_g16(const void* src, float (&x)[64], bool ok) {
  const uint4* s = reinterpret_cast<const uint4*>(src);
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const uint4 u4 = ok ? s[c] : make_uint4(0u, 0u, 0u, 0u);
    const T* e = reinterpret_cast<const T*>(&u4);
#pragma unroll
    for (int j = 0; j < 8; ++j) x[8 * c + j] = to_f32<T>(e[j]);
  }
}

// 64 rows (first `len` valid) of a (tokens, heads, 64) 16-bit tensor into a swizzled tile.
__device__ __forceinline__ void cpa_tile(uint8_t* tile, const void* base, int heads, int h, int t0, int len) {
  const uint8_t* b = static_cast<const uint8_t*>(base);
  const uint32_t dst = smem_u32(tile);
  for (int idx = threadIdx.x; idx < 512; idx += blockDim.x) {
    const int r = idx >> 3, c = idx & 7;
    const int rr = r < len ? r : 0;
    cp_async16(dst + toff(r, 8 * c), b + ((static_cast<size_t>(t0 + rr) * heads + h) * 64 + 8 * c) * 2, r < len);
  }
}
// 64 rows of a (tokens, heads, 64) fp32 tensor into a dense [64][64] fp32 array.
__device__ __forceinline__ void cpa_f32(float* dst, const float* base, int heads, int h, int t0, int len) {
  const uint32_t d = smem_u32(dst);
  for (int idx = threadIdx.x; idx < 1024; idx += blockDim.x) {
    const int r = idx >> 4, c = idx & 15;
    const int rr = r < len ? r : 0;
    cp_async16(d + (r * 64 + 4 * c) * 4, base + (static_cast<size_t>(t0 + rr) * heads + h) * 64 + 4 * c, r < len);
  }
}
__device__ __forceinline__ void cpa_vec(float* dst, const float* base, int heads, int h, int t0, int len) {
  if (threadIdx.x < CH) {
    const int r = threadIdx.x, rr = r < len ? r : 0;
    cp_async4(smem_u32(dst + r), base + static_cast<size_t>(t0 + rr) * heads + h, r < len);
  }
}

// Unit lower-triangular solve (I + L) x = e_c for one column, in registers (L[i][j] = 0 for j >= i).
__device__ __forceinline__ void solve_column(const float (*L)[68], int c, float (&x)[64]) {
#pragma unroll
  for (int i = 0; i < 64; ++i) x[i] = i == c ? 1.f : 0.f;
#pragma unroll
  for (int i = 1; i < 64; ++i) {
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int j = 0; j < i; j += 4) {
      const float4 l = *reinterpret_cast<const float4*>(&L[i][j]);
      a0 = fmaf(l.x, x[j], a0);
      a1 = fmaf(l.y, x[j + 1], a1);
      a0 = fmaf(l.z, x[j + 2], a0);
      a1 = fmaf(l.w, x[j + 3], a1);
    }
    x[i] -= a0 + a1;
  }
}

// ------------------------------------------------------------------------------------------------
// prep: gamma, Tm (or the given A), W, U0.  Two chunks per CTA, 128 threads.
// ------------------------------------------------------------------------------------------------

struct PrepSmem {
  uint8_t tK[2][TB];  // k, then X1 = beta e^gamma k
  uint8_t tV[2][TB];  // v, then X2 = beta v
  uint8_t tT[2][TB];  // Tm
  float L[2][CH][68];
  float gam[2][CH];
  float beta[2][CH];
  uint64_t bar;
  uint32_t tmem;
  int abort;
};

template <typename T>
__global__ void __launch_bounds__(128) gdn_tc_prep_kernel(Params p, int items) {
  extern __shared__ uint8_t smraw[];
  PrepSmem& sm = *reinterpret_cast<PrepSmem*>(align1k(smraw));
  constexpr bool BF = is_bf16<T>();
  const int tid = threadIdx.x;
  // two views of the chunk pair: by column / load row (slot tid >> 6) and by accumulator row (slot =
  // lane half)
  const Item ia = item_of(p, tid >> 6, items);
  const Item ib = item_of(p, (tid & 31) >> 4, items);
  if (tid == 0) {
    sm.abort = 0;
    mbar_init(&sm.bar, 1);
    fence_mbar_init();
  }
  if (tid < 32) {
    tmem_alloc(&sm.tmem, 128);
    tmem_relinquish();
  }
  float gsum;
  {
    const int s = tid >> 6, r = tid & 63;
    const bool ok = r < ia.len;
    const size_t tok = static_cast<size_t>(ia.bos + (ok ? r : 0));
    cp_row(sm.tK[s], r, static_cast<const T*>(p.k) + (tok * p.H + ia.hq) * 64, ok);
    cp_row(sm.tV[s], r, static_cast<const T*>(p.v) + (tok * p.HV + ia.hv) * 64, ok);
    sm.beta[s][r] = ok ? p.beta[tok * p.HV + ia.hv] : 0.f;
    sm.gam[s][r] = ok ? p.g[tok * p.HV + ia.hv] : 0.f;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem;
  {  // gamma: inclusive cumulative sum within the chunk (rows past the end add g = 0)
    const int s = tid >> 6, r = tid & 63;
    gsum = 0.f;
    for (int j = 0; j <= r; ++j) gsum += sm.gam[s][j];
  }
  __syncthreads();
  sm.gam[tid >> 6][tid & 63] = gsum;
  fence_proxy_async_smem();
  __syncthreads();
  uint32_t phase = 0;
  bool ok = true;
  do {
    const RowMap rm = rowmap();
    if (!p.a_given) {
      if (tid == 0) {
        tc_fence_after();
#pragma unroll
        for (int s = 0; s < 2; ++s) mma64<BF, false, false>(tbase + (16u * s << 16), sm.tK[s], sm.tK[s], false);
        umma_commit(&sm.bar);
      }
      if (!(ok = wait_mma(&sm.bar, phase, &sm.abort))) break;
      float x[64];
      ld64(tbase + rm.lane, x);
      const int s = rm.slot, r = rm.row;
      const float br = sm.beta[s][r], gr = sm.gam[s][r];
#pragma unroll
      for (int j = 0; j < 64; ++j) sm.L[s][r][j] = j < r ? br * __expf(gr - sm.gam[s][j]) * x[j] : 0.f;
    }
    {  // X1 = beta e^gamma k, X2 = beta v (rows past the end have beta = 0)
      const int s = rm.slot, r = rm.row;
      const float br = sm.beta[s][r], f = br * __expf(sm.gam[s][r]);
      float x[64];
      ld_row<T>(sm.tK[s], r, x);
#pragma unroll
      for (int j = 0; j < 64; ++j) x[j] *= f;
      st_row<T>(sm.tK[s], r, x);
      ld_row<T>(sm.tV[s], r, x);
#pragma unroll
      for (int j = 0; j < 64; ++j) x[j] *= br;
      st_row<T>(sm.tV[s], r, x);
    }
    tc_fence_before();
    __syncthreads();
    if (!p.a_given) {  // Tm by forward substitution: thread = one column of one chunk
      const int s = tid >> 6, c = tid & 63;
      float x[64];
      solve_column(sm.L[s], c, x);
      uint8_t* tt = sm.tT[s];
      float* arow = p.A + (static_cast<size_t>(ia.bos) * p.HV + ia.hv) * 64 + c;
      const size_t astride = static_cast<size_t>(p.HV) * 64;
#pragma unroll
      for (int r = 0; r < 64; ++r) {
        *reinterpret_cast<T*>(tt + toff(r, c)) = from_f32<T>(x[r]);
        if (r < ia.len) arow[r * astride] = x[r];
      }
    } else {  // the forward's Tm; rows past a ragged chunk's end are identity rows
      const int s = tid >> 6, r = tid & 63;
      const bool in = r < ia.len;
      cvt_row<T>(sm.tT[s], r, p.A + (static_cast<size_t>(ia.bos + (in ? r : 0)) * p.HV + ia.hv) * 64, in,
                 in ? -1 : r);
    }
    fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        mma64<BF, false, true>(tbase + (16u * s << 16), sm.tT[s], sm.tK[s], false);
        mma64<BF, false, true>(tbase + (16u * s << 16) + 64, sm.tT[s], sm.tV[s], false);
      }
      umma_commit(&sm.bar);
    }
    if (!(ok = wait_mma(&sm.bar, phase, &sm.abort))) break;
    {
      const int s = rm.slot, r = rm.row;
      const bool in = r < ib.len;
      const size_t row = static_cast<size_t>(ib.bos + (in ? r : 0)) * p.HV + ib.hv;
      float x[64];
      ld64(tbase + rm.lane, x);
      if (in) st_g16<T>(static_cast<T*>(p.W) + row * 64, x);
      ld64(tbase + rm.lane + 64, x);
      if (in) {
        st_g32(p.U0 + row * 64, x);
        p.gam[row] = sm.gam[s][r];
      }
    }
  } while (0);
  if (!ok && tid == 0) mbar_drain(&sm.bar, phase ^ 1u);
  tc_fence_before();
  __syncthreads();
  if (tid < 32) tmem_dealloc(tbase, 128);
}

// ------------------------------------------------------------------------------------------------
// Column-split scans.  A sequential chunk scan is latency-bound: every chunk is two dependent MMA
// round trips plus a row-wise update.  So a CTA takes one half of the 64 value columns (the two
// halves of a head are independent), each MMA is issued twice, into TMEM lane offsets 0 and 16 of
// the same columns, and thread (warp w, lane l) handles row 16w + (l & 15) and the 16 value columns
// vh * 32 + 16 * (l >> 4) .. +16: every lane works, on a quarter of a row.  The B-operand tiles that
// the threads write (state, u~, ...) carry only the CTA's 32 columns; the other columns stay zero and
// their MMA outputs are never read.
// ------------------------------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ void ld_row16(const uint8_t* tile, int r, int c0, float (&x)[16]) {
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const uint4 u4 = *reinterpret_cast<const uint4*>(tile + toff(r, c0 + 8 * c));
    const T* e = reinterpret_cast<const T*>(&u4);
#pragma unroll
    for (int j = 0; j < 8; ++j) x[8 * c + j] = to_f32<T>(e[j]);
  }
}
template <typename T>
__device__ __forceinline__ void st_g16x16(void* dst, const float (&x)[16]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int c = 0; c < 2; ++c)
    d[c] = make_uint4(pack2<T>(x[8 * c], x[8 * c + 1]), pack2<T>(x[8 * c + 2], x[8 * c + 3]),
                      pack2<T>(x[8 * c + 4], x[8 * c + 5]), pack2<T>(x[8 * c + 6], x[8 * c + 7]));
}
// 64 rows x 32 fp32 columns [c0, c0 + 32) of a (tokens, heads, 64) tensor into a dense [64][32] array.
__device__ __forceinline__ void cpa_f32_half(float* dst, const float* base, int heads, int h, int c0, int t0, int len) {
  const uint32_t d = smem_u32(dst);
  for (int idx = threadIdx.x; idx < 512; idx += blockDim.x) {
    const int r = idx >> 3, c = idx & 7;
    const int rr = r < len ? r : 0;
    cp_async16(d + (r * 32 + 4 * c) * 4, base + (static_cast<size_t>(t0 + rr) * heads + h) * 64 + c0 + 4 * c, r < len);
  }
}
// ------------------------------------------------------------------------------------------------
// state: sequential over the chunks of one sequence; CTA = (sequence, value head, value half).
//   hS[c] = S (16-bit);  u = U0 - W S;  S <- e^{gamma_C} S + K^T diag(e^{gamma_C - gamma}) u
// The fp32 state lives in registers (16 values per thread).  The next chunk's W, k, U0 and gamma
// stream into the other half of a double buffer (cp.async).
// ------------------------------------------------------------------------------------------------
struct StateSmem {
  uint8_t tW[2][TB];
  uint8_t tK[2][TB];
  uint8_t tS[TB];  // state, [key][value] (this CTA's 32 columns)
  uint8_t tU[TB];  // e^{gamma_C - gamma} u, [token][value]
  float U0[2][CH * 32];
  float gam[2][CH];
  uint64_t bar;
  uint32_t tmem;
  int abort;
};

template <typename T>
__global__ void __launch_bounds__(128) gdn_tc_state_kernel(Params p) {
  extern __shared__ uint8_t smraw[];
  StateSmem& sm = *reinterpret_cast<StateSmem*>(align1k(smraw));
  constexpr bool BF = is_bf16<T>();
  const int tid = threadIdx.x, ln = tid & 31;
  const int vh = blockIdx.x & 1, nh = blockIdx.x >> 1;
  const int n = nh / p.HV, hv = nh % p.HV, hq = hv / (p.HV / p.H);
  int bos, eos, c0, nc;
  seq_range(p, n, bos, eos, c0, nc);
  auto issue = [&](int j, int b) {
    const int t0 = bos + j * CH, len = min(CH, eos - t0);
    cpa_tile(sm.tW[b], p.W, p.HV, hv, t0, len);
    cpa_tile(sm.tK[b], p.k, p.H, hq, t0, len);
    cpa_f32_half(sm.U0[b], p.U0, p.HV, hv, 32 * vh, t0, len);
    cpa_vec(sm.gam[b], p.gam, p.HV, hv, t0, len);
    cp_async_commit();
  };
  if (tid == 0) {
    sm.abort = 0;
    mbar_init(&sm.bar, 1);
    fence_mbar_init();
  }
  if (tid < 32) {
    tmem_alloc(&sm.tmem, 128);
    tmem_relinquish();
  }
  if (nc > 0) issue(0, 0);
  zero_tile(sm.tS);
  zero_tile(sm.tU);
  __syncthreads();
  const RowMap rm = rowmap();
  const int m = rm.row;
  const int vc = 32 * vh + 16 * (ln >> 4);  // this thread's first value column
  float S[16];
  {
    const float* h0 = p.h0 ? p.h0 + ((static_cast<size_t>(n) * p.HV + hv) * 64 + m) * 64 + vc : nullptr;
#pragma unroll
    for (int c = 0; c < 16; ++c) S[c] = h0 ? h0[c] : 0.f;
    st_row16<T>(sm.tS, m, vc, S);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem;
  uint32_t phase = 0;
  bool ok = true;
  for (int j = 0; j < nc; ++j) {
    const int b = j & 1, gc = c0 + j, t0 = bos + j * CH, len = min(CH, eos - t0);
    if (j + 1 < nc) {
      issue(j + 1, b ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    st_g16x16<T>(static_cast<T*>(p.hS) + ((static_cast<size_t>(gc) * p.HV + hv) * 64 + m) * 64 + vc, S);
    fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      mma64x2<BF, false, true>(tbase, sm.tW[b], sm.tS, false);  // W S
      umma_commit(&sm.bar);
    }
    if (!(ok = wait_mma(&sm.bar, phase, &sm.abort))) break;
    const float gC = sm.gam[b][len - 1];
    {
      float x[16];
      ld_quarter(tbase + rm.lane + 32 * vh, ln >> 4, x);
      const int r = m;
      const bool in = r < len;
      const float f = in ? __expf(gC - sm.gam[b][r]) : 0.f;
      const float* u0 = sm.U0[b] + r * 32 + (vc - 32 * vh);
#pragma unroll
      for (int c = 0; c < 16; ++c) x[c] = u0[c] - x[c];
      if (in) st_g16x16<T>(static_cast<T*>(p.u) + (static_cast<size_t>(t0 + r) * p.HV + hv) * 64 + vc, x);
#pragma unroll
      for (int c = 0; c < 16; ++c) x[c] *= f;
      st_row16<T>(sm.tU, r, vc, x);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      mma64x2<BF, true, true>(tbase + 64, sm.tK[b], sm.tU, false);  // K^T u~
      umma_commit(&sm.bar);
    }
    if (!(ok = wait_mma(&sm.bar, phase, &sm.abort))) break;
    {
      float x[16];
      ld_quarter(tbase + rm.lane + 64 + 32 * vh, ln >> 4, x);
      const float eC = __expf(gC);
#pragma unroll
      for (int c = 0; c < 16; ++c) S[c] = fmaf(eC, S[c], x[c]);
      st_row16<T>(sm.tS, m, vc, S);
    }
    tc_fence_before();
    __syncthreads();
  }
  if (ok && p.ht) {
    float* d = p.ht + ((static_cast<size_t>(n) * p.HV + hv) * 64 + m) * 64 + vc;
#pragma unroll
    for (int c = 0; c < 16; ++c) d[c] = S[c];
  }
  cp_async_wait<0>();
  if (!ok && tid == 0) mbar_drain(&sm.bar, phase ^ 1u);
  tc_fence_before();
  __syncthreads();
  if (tid < 32) tmem_dealloc(tbase, 128);
}

// ------------------------------------------------------------------------------------------------
// output: o = scale [e^gamma (Q S0) + (tril(Q K^T) o Gamma) u].  Two chunks per CTA.
// ------------------------------------------------------------------------------------------------
struct OutSmem {
  uint8_t tQ[2][TB];
  uint8_t tK[2][TB];
  uint8_t tU[2][TB];
  uint8_t tS[2][TB];
  uint8_t tP[2][TB];
  float gam[2][CH];
  uint64_t bar;
  uint32_t tmem;
  int abort;
};

template <typename T>
__global__ void __launch_bounds__(128) gdn_tc_out_kernel(Params p, int items) {
  extern __shared__ uint8_t smraw[];
  OutSmem& sm = *reinterpret_cast<OutSmem*>(align1k(smraw));
  constexpr bool BF = is_bf16<T>();
  const int tid = threadIdx.x;
  const Item ia = item_of(p, tid >> 6, items);         // load rows
  const Item ib = item_of(p, (tid & 31) >> 4, items);  // accumulator rows
  if (tid == 0) {
    sm.abort = 0;
    mbar_init(&sm.bar, 1);
    fence_mbar_init();
  }
  if (tid < 32) {
    tmem_alloc(&sm.tmem, 128);
    tmem_relinquish();
  }
  {
    const int s = tid >> 6, r = tid & 63;
    const bool in = r < ia.len;
    const size_t tok = static_cast<size_t>(ia.bos + (in ? r : 0));
    cp_row(sm.tQ[s], r, static_cast<const T*>(p.q) + (tok * p.H + ia.hq) * 64, in);
    cp_row(sm.tK[s], r, static_cast<const T*>(p.k) + (tok * p.H + ia.hq) * 64, in);
    cp_row(sm.tU[s], r, static_cast<const T*>(p.u) + (tok * p.HV + ia.hv) * 64, in);
    cp_row(sm.tS[s], r, static_cast<const T*>(p.hS) + ((static_cast<size_t>(ia.gc) * p.HV + ia.hv) * 64 + r) * 64,
           ia.len > 0);
    sm.gam[s][r] = in ? p.gam[tok * p.HV + ia.hv] : 0.f;
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem;
  uint32_t phase = 0;
  bool ok = true;
  do {
    if (tid == 0) {
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        mma64<BF, false, true>(tbase + (16u * s << 16), sm.tQ[s], sm.tS[s], false);        // Q S0
        mma64<BF, false, false>(tbase + (16u * s << 16) + 64, sm.tQ[s], sm.tK[s], false);  // Q K^T
      }
      umma_commit(&sm.bar);
    }
    if (!(ok = wait_mma(&sm.bar, phase, &sm.abort))) break;
    const RowMap rm = rowmap();
    const int s = rm.slot, r = rm.row;
    const float gr = sm.gam[s][r];
    {
      float x[64];
      ld64(tbase + rm.lane + 64, x);
#pragma unroll
      for (int j = 0; j < 64; ++j) x[j] = j <= r ? __expf(gr - sm.gam[s][j]) * x[j] : 0.f;
      st_row<T>(sm.tP[s], r, x);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int t = 0; t < 2; ++t) mma64<BF, false, true>(tbase + (16u * t << 16) + 64, sm.tP[t], sm.tU[t], false);
      umma_commit(&sm.bar);
    }
    if (!(ok = wait_mma(&sm.bar, phase, &sm.abort))) break;
    float a[64], x[64];
    ld64(tbase + rm.lane, a);
    ld64(tbase + rm.lane + 64, x);
    const float eg = __expf(gr);
#pragma unroll
    for (int c = 0; c < 64; ++c) x[c] = p.scale * fmaf(eg, a[c], x[c]);
    if (r < ib.len) st_g16<T>(static_cast<T*>(p.o) + (static_cast<size_t>(ib.bos + r) * p.HV + ib.hv) * 64, x);
  } while (0);
  if (!ok && tid == 0) mbar_drain(&sm.bar, phase ^ 1u);
  tc_fence_before();
  __syncthreads();
  if (tid < 32) tmem_dealloc(tbase, 128);
}

// ------------------------------------------------------------------------------------------------
// backward 0: dvl_j = scale sum_{i>=j} e^{gamma_i - gamma_j} (q_i.k_j) dO_i.  Two chunks per CTA.
// ------------------------------------------------------------------------------------------------
struct DvlSmem {
  uint8_t tQ[2][TB];
  uint8_t tK[2][TB];
  uint8_t tO[2][TB];
  uint8_t tP[2][TB];
  float gam[2][CH];
  uint64_t bar;
  uint32_t tmem;
  int abort;
};

template <typename T>
__global__ void __launch_bounds__(128) gdn_tc_dvl_kernel(Params p, int items) {
  extern __shared__ uint8_t smraw[];
  DvlSmem& sm = *reinterpret_cast<DvlSmem*>(align1k(smraw));
  constexpr bool BF = is_bf16<T>();
  const int tid = threadIdx.x;
  const Item ia = item_of(p, tid >> 6, items);         // load rows
  const Item ib = item_of(p, (tid & 31) >> 4, items);  // accumulator rows
  if (tid == 0) {
    sm.abort = 0;
    mbar_init(&sm.bar, 1);
    fence_mbar_init();
  }
  if (tid < 32) {
    tmem_alloc(&sm.tmem, 128);
    tmem_relinquish();
  }
  {
    const int s = tid >> 6, r = tid & 63;
    const bool in = r < ia.len;
    const size_t tok = static_cast<size_t>(ia.bos + (in ? r : 0));
    cp_row(sm.tQ[s], r, static_cast<const T*>(p.q) + (tok * p.H + ia.hq) * 64, in);
    cp_row(sm.tK[s], r, static_cast<const T*>(p.k) + (tok * p.H + ia.hq) * 64, in);
    cp_row(sm.tO[s], r, static_cast<const T*>(p.dout) + (tok * p.HV + ia.hv) * 64, in);
    sm.gam[s][r] = in ? p.gam[tok * p.HV + ia.hv] : 0.f;
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem;
  uint32_t phase = 0;
  bool ok = true;
  do {
    if (tid == 0) {
#pragma unroll
      for (int s = 0; s < 2; ++s) mma64<BF, false, false>(tbase + (16u * s << 16), sm.tK[s], sm.tQ[s], false);
      umma_commit(&sm.bar);
    }
    if (!(ok = wait_mma(&sm.bar, phase, &sm.abort))) break;
    const RowMap rm = rowmap();
    const int s = rm.slot, j = rm.row;
    {
      float x[64];
      ld64(tbase + rm.lane, x);  // row j: k_j . q_i
      const float gj = sm.gam[s][j];
#pragma unroll
      for (int i = 0; i < 64; ++i) x[i] = i >= j ? p.scale * __expf(sm.gam[s][i] - gj) * x[i] : 0.f;
      st_row<T>(sm.tP[s], j, x);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int t = 0; t < 2; ++t) mma64<BF, false, true>(tbase + (16u * t << 16) + 64, sm.tP[t], sm.tO[t], false);
      umma_commit(&sm.bar);
    }
    if (!(ok = wait_mma(&sm.bar, phase, &sm.abort))) break;
    float x[64];
    ld64(tbase + rm.lane + 64, x);
    if (j < ib.len) st_g32(p.dvl + (static_cast<size_t>(ib.bos + j) * p.HV + ib.hv) * 64, x);
  } while (0);
  if (!ok && tid == 0) mbar_drain(&sm.bar, phase ^ 1u);
  tc_fence_before();
  __syncthreads();
  if (tid < 32) tmem_dealloc(tbase, 128);
}

// ------------------------------------------------------------------------------------------------
// backward 1: reverse scan of dS; CTA = (sequence, value head, value half), column split as above.
//   hD[c] = dS (16-bit);  du = dvl + e^{gamma_C - gamma} (K dS);
//   dS <- e^{gamma_C} dS + q^T diag(scale e^gamma) dO - W^T du;  dh0 = dS after the first chunk.
// ------------------------------------------------------------------------------------------------
struct DstateSmem {
  uint8_t tW[2][TB];
  uint8_t tK[2][TB];
  uint8_t tQ[2][TB];
  uint8_t tO[2][TB];
  uint8_t tDS[TB];   // dS, [key][value] (this CTA's 32 columns)
  uint8_t tOs[TB];   // scale e^gamma dO, [token][value]
  uint8_t tDU[TB];   // -du, [token][value]
  float dvl[2][CH * 32];
  float gam[2][CH];
  uint64_t bar;
  uint32_t tmem;
  int abort;
};

template <typename T>
__global__ void __launch_bounds__(128) gdn_tc_dstate_kernel(Params p) {
  extern __shared__ uint8_t smraw[];
  DstateSmem& sm = *reinterpret_cast<DstateSmem*>(align1k(smraw));
  constexpr bool BF = is_bf16<T>();
  const int tid = threadIdx.x, ln = tid & 31;
  const int vh = blockIdx.x & 1, nh = blockIdx.x >> 1;
  const int n = nh / p.HV, hv = nh % p.HV, hq = hv / (p.HV / p.H);
  int bos, eos, c0, nc;
  seq_range(p, n, bos, eos, c0, nc);
  auto issue = [&](int j, int b) {
    const int t0 = bos + j * CH, len = min(CH, eos - t0);
    cpa_tile(sm.tW[b], p.W, p.HV, hv, t0, len);
    cpa_tile(sm.tK[b], p.k, p.H, hq, t0, len);
    cpa_tile(sm.tQ[b], p.q, p.H, hq, t0, len);
    cpa_tile(sm.tO[b], p.dout, p.HV, hv, t0, len);
    cpa_f32_half(sm.dvl[b], p.dvl, p.HV, hv, 32 * vh, t0, len);
    cpa_vec(sm.gam[b], p.gam, p.HV, hv, t0, len);
    cp_async_commit();
  };
  if (tid == 0) {
    sm.abort = 0;
    mbar_init(&sm.bar, 1);
    fence_mbar_init();
  }
  if (tid < 32) {
    tmem_alloc(&sm.tmem, 128);
    tmem_relinquish();
  }
  if (nc > 0) issue(nc - 1, 0);
  zero_tile(sm.tDS);
  zero_tile(sm.tOs);
  zero_tile(sm.tDU);
  __syncthreads();
  const RowMap rm = rowmap();
  const int m = rm.row;
  const int vc = 32 * vh + 16 * (ln >> 4);
  float dS[16];
  {
    const float* d0 = p.dht ? p.dht + ((static_cast<size_t>(n) * p.HV + hv) * 64 + m) * 64 + vc : nullptr;
#pragma unroll
    for (int c = 0; c < 16; ++c) dS[c] = d0 ? d0[c] : 0.f;
    st_row16<T>(sm.tDS, m, vc, dS);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem;
  uint32_t phase = 0;
  bool ok = true;
  for (int it = 0; it < nc; ++it) {
    const int j = nc - 1 - it, b = it & 1, gc = c0 + j, t0 = bos + j * CH, len = min(CH, eos - t0);
    if (j > 0) {
      issue(j - 1, b ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    st_g16x16<T>(static_cast<T*>(p.hD) + ((static_cast<size_t>(gc) * p.HV + hv) * 64 + m) * 64 + vc, dS);
    __syncthreads();  // the chunk's tiles (cp.async) are complete in every thread's view
    {  // dO rows scaled by scale e^gamma (this thread's 16 columns)
      const int r = m;
      float x[16];
      ld_row16<T>(sm.tO[b], r, vc, x);
      const float f = r < len ? p.scale * __expf(sm.gam[b][r]) : 0.f;
#pragma unroll
      for (int c = 0; c < 16; ++c) x[c] *= f;
      st_row16<T>(sm.tOs, r, vc, x);
    }
    fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      mma64x2<BF, false, true>(tbase, sm.tK[b], sm.tDS, false);      // K dS
      mma64x2<BF, true, true>(tbase + 64, sm.tQ[b], sm.tOs, false);  // q^T dO~
      umma_commit(&sm.bar);
    }
    if (!(ok = wait_mma(&sm.bar, phase, &sm.abort))) break;
    const float gC = sm.gam[b][len - 1];
    {
      float x[16];
      ld_quarter(tbase + rm.lane + 32 * vh, ln >> 4, x);
      const int r = m;
      const bool in = r < len;
      const float f = in ? __expf(gC - sm.gam[b][r]) : 0.f;
      const float* dv = sm.dvl[b] + r * 32 + (vc - 32 * vh);
#pragma unroll
      for (int c = 0; c < 16; ++c) x[c] = in ? fmaf(f, x[c], dv[c]) : 0.f;
      if (in) st_g16x16<T>(static_cast<T*>(p.du) + (static_cast<size_t>(t0 + r) * p.HV + hv) * 64 + vc, x);
#pragma unroll
      for (int c = 0; c < 16; ++c) x[c] = -x[c];
      st_row16<T>(sm.tDU, r, vc, x);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      mma64x2<BF, true, true>(tbase + 64, sm.tW[b], sm.tDU, true);  // - W^T du
      umma_commit(&sm.bar);
    }
    if (!(ok = wait_mma(&sm.bar, phase, &sm.abort))) break;
    {
      float x[16];
      ld_quarter(tbase + rm.lane + 64 + 32 * vh, ln >> 4, x);
      const float eC = __expf(gC);
#pragma unroll
      for (int c = 0; c < 16; ++c) dS[c] = fmaf(eC, dS[c], x[c]);
      st_row16<T>(sm.tDS, m, vc, dS);
    }
    tc_fence_before();
    __syncthreads();
  }
  if (ok && p.dh0) {
    float* d = p.dh0 + ((static_cast<size_t>(n) * p.HV + hv) * 64 + m) * 64 + vc;
#pragma unroll
    for (int c = 0; c < 16; ++c) d[c] = dS[c];
  }
  cp_async_wait<0>();
  if (!ok && tid == 0) mbar_drain(&sm.bar, phase ^ 1u);
  tc_fence_before();
  __syncthreads();
  if (tid < 32) tmem_dealloc(tbase, 128);
}

// ------------------------------------------------------------------------------------------------
// backward 2: per-chunk dq, dk, dv, dbeta, dg.  One chunk per CTA of 256 threads, two CTAs per SM (so
// one CTA's loads and MMAs overlap the other's epilogues): at most four accumulators live in 256
// TMEM columns (R0..R3), and twelve 16-bit tiles (U0 and W arrive late, into the tiles of dO and u).
// Every MMA is issued into both TMEM lane halves (mma64x2).  Warp w reads the lanes of subpartition
// w % 4 and columns 32 (w / 4) .. +32, of which its lane half h keeps 16: thread (w, l) handles row
// 16 (w % 4) + (l & 15) and columns 32 (w / 4) + 16 h .. +16.  Row sums combine the four threads of a
// row (shuffle + shared memory); column sums reduce the 16 rows of a half-warp by shuffles.
//   batch 1a: R0 du S0^T (-dW), R1 Tm^T du (Y_V), R2 dO u^T, R3 Q K^T
//   batch 1b: R0 dO S0^T (dq), R2 u dS_end^T (dk), R3 Tm^T dW (Y_K)
//   batch 2:  R0 += M' K, R2 += M'^T Q, R1 = Y_V U0^T + Y_K W^T (-dL), R3 K K^T
//   batch 3:  R2 += P K + P^T K
// ------------------------------------------------------------------------------------------------
struct GradSmem {
  uint8_t tQ[TB], tK[TB], tO[TB], tU[TB], tDU[TB], tS0[TB], tHD[TB], tTm[TB];
  uint8_t tDW[TB];  // dW, later P
  uint8_t tYV[TB], tYK[TB], tM[TB];
  float colpart[4][CH];  // column sums of the dgamma_j terms, per subpartition (16 rows each)
  float part[3][2][CH];  // per-row partial sums (dgamma, dbeta, tot) of the two column groups
  float gam[CH], beta[CH], dgam[CH], red[4];
  uint64_t bar;
  uint32_t tmem;
  int abort;
};

// 16 columns of this thread's TMEM lane (its lane half h of the warp's 32 columns at taddr) and the
// matching store, written into both 16-column halves (the half a lane does not own is never read).
__device__ __forceinline__ void st_quarter(uint32_t taddr, const float (&x)[16]) {
  uint32_t a[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) a[j] = __float_as_uint(x[j]);
  tmem_st16(taddr, a);
  tmem_st16(taddr + 16, a);
}

// 16 gradient values at element offset `off` of an fp32 or (grad16) 16-bit output.
template <typename T>
__device__ __forceinline__ void st_grad16(void* base, size_t off, const float (&x)[16], int grad16) {
  if (grad16) {
    st_g16x16<T>(static_cast<T*>(base) + off, x);
  } else {
    float4* d = reinterpret_cast<float4*>(static_cast<float*>(base) + off);
#pragma unroll
    for (int c = 0; c < 4; ++c) d[c] = make_float4(x[4 * c], x[4 * c + 1], x[4 * c + 2], x[4 * c + 3]);
  }
}

// Sum over the 16 rows of a half-warp of each of the thread's 16 column values; lane (l & 15) == j of
// the half ends with column j's sum in the return value.
__device__ __forceinline__ float colsum16(const float (&c)[16]) {
  const int me = threadIdx.x & 15;
  float mine = 0.f;
#pragma unroll
  for (int jj = 0; jj < 16; ++jj) {
    float v = c[jj];
    v += __shfl_xor_sync(0xffffffffu, v, 8);
    v += __shfl_xor_sync(0xffffffffu, v, 4);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    if (jj == me) mine = v;
  }
  return mine;
}

template <typename T>
__global__ void __launch_bounds__(256, 2) gdn_tc_grad_kernel(Params p) {
  extern __shared__ uint8_t smraw[];
  GradSmem& sm = *reinterpret_cast<GradSmem*>(align1k(smraw));
  constexpr bool BF = is_bf16<T>();
  const int tid = threadIdx.x, ln = tid & 31, w = tid >> 5;
  const int gc = blockIdx.x / p.HV, hv = blockIdx.x % p.HV, hq = hv / (p.HV / p.H);
  const ChunkPos cp = chunk_pos(p, gc);
  const int len = cp.len;
  if (tid == 0) {
    sm.abort = 0;
    mbar_init(&sm.bar, 1);
    fence_mbar_init();
  }
  if (w == 0) {
    tmem_alloc(&sm.tmem, 256);
    tmem_relinquish();
  }
  {  // loads: thread = (group, row)
    const int r = tid & 63, grp = tid >> 6;
    const bool in = r < len;
    const size_t tok = static_cast<size_t>(cp.bos + (in ? r : 0));
    const size_t rowv = tok * p.HV + hv;
    const size_t st = (static_cast<size_t>(gc) * p.HV + hv) * 64 * 64;
    if (grp == 0) {
      cp_row(sm.tQ, r, static_cast<const T*>(p.q) + (tok * p.H + hq) * 64, in);
      cp_row(sm.tK, r, static_cast<const T*>(p.k) + (tok * p.H + hq) * 64, in);
      sm.gam[r] = in ? p.gam[rowv] : 0.f;
      sm.beta[r] = in ? p.beta[rowv] : 0.f;
    } else if (grp == 1) {
      cp_row(sm.tO, r, static_cast<const T*>(p.dout) + rowv * 64, in);
      cp_row(sm.tU, r, static_cast<const T*>(p.u) + rowv * 64, in);
    } else if (grp == 2) {
      cp_row(sm.tDU, r, static_cast<const T*>(p.du) + rowv * 64, in);
      cp_row(sm.tS0, r, static_cast<const T*>(p.hS) + st + r * 64, true);
      cp_row(sm.tHD, r, static_cast<const T*>(p.hD) + st + r * 64, true);
    } else {
      cvt_row<T>(sm.tTm, r, p.A + rowv * 64, in, in ? -1 : r);
    }
    if (tid < 4) sm.red[tid] = 0.f;
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (tid < CH && tid >= len) sm.gam[tid] = sm.gam[len - 1];  // rows past the end: gamma_last (g = 0)
  __syncthreads();
  const uint32_t tbase = sm.tmem;
  const int spq = w & 3, cg = w >> 2, hh = ln >> 4;
  const int r = 16 * spq + (ln & 15), ch = 32 * cg + 16 * hh;  // this thread's row and first column
  const uint32_t T0 = tbase + (static_cast<uint32_t>(32 * spq) << 16) + 32 * cg;  // warp-uniform TMEM address
  const uint32_t R0 = T0, R1 = T0 + 64, R2 = T0 + 128, R3 = T0 + 192;
  uint32_t phase = 0;
  bool ok = true;
  const float gC = sm.gam[CH - 1], gr = sm.gam[r], br = sm.beta[r], egr = __expf(gr);
  float dgr = 0.f, dbr = 0.f, tot = 0.f;  // this thread's parts of the row sums
  const bool in = r < len;
  const size_t rowv = static_cast<size_t>(cp.bos + (in ? r : 0)) * p.HV + hv;
  do {
    if (tid == 0) {
      mma64x2<BF, false, false>(tbase, sm.tDU, sm.tS0, false);     // du S0^T  (= -dW)
      mma64x2<BF, true, true>(tbase + 64, sm.tTm, sm.tDU, false);  // Tm^T du  (= Y_V)
      mma64x2<BF, false, false>(tbase + 128, sm.tO, sm.tU, false);  // dO u^T
      mma64x2<BF, false, false>(tbase + 192, sm.tQ, sm.tK, false);  // Q K^T
      umma_commit(&sm.bar);
    }
    if (!(ok = wait_mma(&sm.bar, phase, &sm.abort))) break;
    {  // epilogue 1a
      float x[16];
      ld_quarter(R0, hh, x);  // dW = -(du S0^T)
#pragma unroll
      for (int c = 0; c < 16; ++c) x[c] = -x[c];
      st_row16<T>(sm.tDW, r, ch, x);
      ld_quarter(R1, hh, x);  // Y_V
      st_row16<T>(sm.tYV, r, ch, x);
      float vv[16];
      {
        const uint4* s4 = reinterpret_cast<const uint4*>(static_cast<const T*>(p.v) + rowv * 64 + ch);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const uint4 u4 = in ? s4[c] : make_uint4(0u, 0u, 0u, 0u);
          const T* e = reinterpret_cast<const T*>(&u4);
#pragma unroll
          for (int j = 0; j < 8; ++j) vv[8 * c + j] = to_f32<T>(e[j]);
        }
      }
      float s1 = 0.f;
#pragma unroll
      for (int c = 0; c < 16; ++c) s1 = fmaf(vv[c], x[c], s1);
      dbr += s1;
#pragma unroll
      for (int c = 0; c < 16; ++c) x[c] *= br;
      if (in) st_grad16<T>(p.dv, rowv * 64 + ch, x, p.grad16);
      float t[16], e[16];
      ld_quarter(R2, hh, t);  // dO_r . u_j
      ld_quarter(R3, hh, e);  // q_r . k_j
      float rs = 0.f;
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) {
        const int j = ch + jj;
        const float mp = j <= r ? p.scale * __expf(gr - sm.gam[j]) * t[jj] : 0.f;
        t[jj] = mp;
        e[jj] *= mp;  // Mg_rj = M'_rj (q_r . k_j): into dgamma_r, out of dgamma_j
        rs += e[jj];
      }
      dgr += rs;
      st_row16<T>(sm.tM, r, ch, t);
      const float cs = colsum16(e);
      sm.colpart[spq][ch + (ln & 15)] = cs;
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      mma64x2<BF, false, false>(tbase, sm.tO, sm.tS0, false);         // dO S0^T
      mma64x2<BF, false, false>(tbase + 128, sm.tU, sm.tHD, false);   // u dS_end^T
      mma64x2<BF, true, true>(tbase + 192, sm.tTm, sm.tDW, false);    // Y_K = Tm^T dW
      umma_commit(&sm.bar);
    }
    if (!(ok = wait_mma(&sm.bar, phase, &sm.abort))) break;
    {  // U0 and W into the tiles of dO and u (their last reader, batch 1b, has completed)
      const int rr = tid & 63, grp = tid >> 6;
      const bool rin = rr < len;
      const size_t rv = static_cast<size_t>(cp.bos + (rin ? rr : 0)) * p.HV + hv;
      if (grp == 0) cvt_row<T>(sm.tO, rr, p.U0 + rv * 64, rin, -1);
      else if (grp == 1) cp_row(sm.tU, rr, static_cast<const T*>(p.W) + rv * 64, rin);
    }
    {  // epilogue 1b
      float x[16], y[16], qq[16], kk[16];
      ld_quarter(R0, hh, x);  // dq term scale e^gamma (dO S0^T)
      ld_row16<T>(sm.tQ, r, ch, qq);
      float s1 = 0.f;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        x[c] *= p.scale * egr;
        s1 = fmaf(qq[c], x[c], s1);
      }
      dgr += s1;
      st_quarter(R0, x);
      ld_quarter(R2, hh, x);  // dk term e^{gamma_C - gamma} (u dS_end^T)
      ld_quarter(R3, hh, y);  // Y_K
      ld_row16<T>(sm.tK, r, ch, kk);
      st_row16<T>(sm.tYK, r, ch, y);
      const float f = __expf(gC - gr);
      float s2 = 0.f, s3 = 0.f;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        x[c] *= f;
        s2 = fmaf(kk[c], x[c], s2);
        s3 = fmaf(kk[c], y[c], s3);
        x[c] = fmaf(br * egr, y[c], x[c]);  // + beta e^gamma Y_K
      }
      dgr += br * egr * s3 - s2;
      dbr += egr * s3;
      tot += s2;
      st_quarter(R2, x);
    }
    tmem_wait_st();
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      mma64x2<BF, false, true>(tbase, sm.tM, sm.tK, true);           // dq += M' K
      mma64x2<BF, true, true>(tbase + 128, sm.tM, sm.tQ, true);      // dk += M'^T Q
      mma64x2<BF, false, false>(tbase + 64, sm.tYV, sm.tO, false);   // Y_V U0^T
      mma64x2<BF, false, false>(tbase + 64, sm.tYK, sm.tU, true);    // + Y_K W^T  (= -dL)
      mma64x2<BF, false, false>(tbase + 192, sm.tK, sm.tK, false);   // K K^T
      umma_commit(&sm.bar);
    }
    if (!(ok = wait_mma(&sm.bar, phase, &sm.abort))) break;
    {  // epilogue 2
      float t[16], e[16];
      ld_quarter(R1, hh, t);
      ld_quarter(R3, hh, e);
      float db = 0.f, dg = 0.f;
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) {
        const int j = ch + jj;
        float P = 0.f, G = 0.f;
        if (j < r) {
          const float dl = -t[jj];
          const float dec = __expf(gr - sm.gam[j]);
          const float E = dec * e[jj];
          db = fmaf(dl, E, db);
          G = br * dl * E;
          dg += G;
          P = br * dl * dec;
        }
        t[jj] = P;
        e[jj] = G;
      }
      dbr += db;
      dgr += dg;
      st_row16<T>(sm.tDW, r, ch, t);
      const float cs = colsum16(e);
      sm.colpart[spq][ch + (ln & 15)] += cs;
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      mma64x2<BF, false, true>(tbase + 128, sm.tDW, sm.tK, true);  // dk += P K
      mma64x2<BF, true, true>(tbase + 128, sm.tDW, sm.tK, true);   // dk += P^T K
      umma_commit(&sm.bar);
    }
    if (!(ok = wait_mma(&sm.bar, phase, &sm.abort))) break;
    {
      float x[16];
      const size_t off = (static_cast<size_t>(cp.bos + (in ? r : 0)) * p.H + hq) * 64 + ch;
      ld_quarter(R0, hh, x);
      if (in) {
        if (p.gva) {
#pragma unroll
          for (int c = 0; c < 16; ++c) atomicAdd(static_cast<float*>(p.dq) + off + c, x[c]);
        } else {
          st_grad16<T>(p.dq, off, x, p.grad16);
        }
      }
      ld_quarter(R2, hh, x);
      if (in) {
        if (p.gva) {
#pragma unroll
          for (int c = 0; c < 16; ++c) atomicAdd(static_cast<float*>(p.dk) + off + c, x[c]);
        } else {
          st_grad16<T>(p.dk, off, x, p.grad16);
        }
      }
    }
    // row sums: the two lane halves of a warp (shuffle), then the two column groups (shared memory)
    dgr += __shfl_xor_sync(0xffffffffu, dgr, 16);
    dbr += __shfl_xor_sync(0xffffffffu, dbr, 16);
    tot += __shfl_xor_sync(0xffffffffu, tot, 16);
    if (hh == 0) {
      sm.part[0][cg][r] = dgr;
      sm.part[1][cg][r] = dbr;
      sm.part[2][cg][r] = tot;
    }
    {
      float sd = 0.f;  // <S0, dS_end>
      for (int i = tid; i < CH * CH; i += blockDim.x) {
        const int rr = i >> 6, cc = i & 63;
        const T a = *reinterpret_cast<const T*>(sm.tS0 + toff(rr, cc));
        const T d = *reinterpret_cast<const T*>(sm.tHD + toff(rr, cc));
        sd = fmaf(to_f32<T>(a), to_f32<T>(d), sd);
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) sd += __shfl_xor_sync(0xffffffffu, sd, o);
      if (ln == 0) atomicAdd(&sm.red[1], sd);
    }
    __syncthreads();
    if (tid < CH) {
      const float col = sm.colpart[0][tid] + sm.colpart[1][tid] + sm.colpart[2][tid] + sm.colpart[3][tid];
      sm.dgam[tid] = sm.part[0][0][tid] + sm.part[0][1][tid] - col;
      atomicAdd(&sm.red[0], sm.part[2][0][tid] + sm.part[2][1][tid]);
      if (tid < len) p.dbeta[static_cast<size_t>(cp.bos + tid) * p.HV + hv] = sm.part[1][0][tid] + sm.part[1][1][tid];
    }
    __syncthreads();
    if (tid == 0) sm.dgam[CH - 1] += sm.red[0] + __expf(gC) * sm.red[1];
    __syncthreads();
    if (tid < 32) {  // dg = reverse cumulative sum of dgamma within the chunk
      const int l = tid;
      const float a = sm.dgam[CH - 1 - 2 * l], b2 = a + sm.dgam[CH - 2 - 2 * l];
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
  } while (0);
  if (!ok && tid == 0) mbar_drain(&sm.bar, phase ^ 1u);
  tc_fence_before();
  __syncthreads();
  if (w == 0) tmem_dealloc(tbase, 256);
}

// ------------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------------
template <typename K>
int launch(K kernel, int grid, size_t smem, cudaStream_t st, const Params& p, int threads = 128) {
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
    return KATA_ERR_CUDA;
  kernel<<<grid, threads, smem, st>>>(p);
  return from_cuda(cudaGetLastError());
}
template <typename K>
int launch2(K kernel, int grid, size_t smem, cudaStream_t st, const Params& p, int items) {
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
    return KATA_ERR_CUDA;
  kernel<<<grid, 128, smem, st>>>(p, items);
  return from_cuda(cudaGetLastError());
}

struct Ws {
  size_t gam, W, U0, u, hS, fwd_total, dvl, du, hD, total;
};

// Byte offsets (256-byte aligned) of the workspace parts.  With `reuse` the forward part lives in the
// forward call's workspace and is not counted in the backward's.
Ws ws_layout(int B, int T, int HV, int NC, bool bwd, bool reuse) {
  const size_t rows = static_cast<size_t>(B) * T * HV;
  const size_t st = static_cast<size_t>(NC) * HV * 64 * 64;
  auto al = [](size_t x) { return (x + 255) & ~static_cast<size_t>(255); };
  Ws w{};
  size_t o = 0;
  w.gam = o; o += al(rows * 4);
  w.W = o; o += al(rows * 64 * 2);
  w.U0 = o; o += al(rows * 64 * 4);
  w.u = o; o += al(rows * 64 * 2);
  w.hS = o; o += al(st * 2);
  w.fwd_total = o;
  if (bwd) {
    if (reuse) o = 0;
    w.dvl = o; o += al(rows * 64 * 4);
    w.du = o; o += al(rows * 64 * 2);
    w.hD = o; o += al(st * 2);
  }
  w.total = o;
  return w;
}

void bind(Params& p, void* ws, const Ws& w, bool bwd, const void* fwd_ws) {
  uint8_t* f = static_cast<uint8_t*>(const_cast<void*>(fwd_ws ? fwd_ws : ws));
  p.gam = reinterpret_cast<float*>(f + w.gam);
  p.W = f + w.W;
  p.U0 = reinterpret_cast<float*>(f + w.U0);
  p.u = f + w.u;
  p.hS = f + w.hS;
  if (bwd) {
    uint8_t* b = static_cast<uint8_t*>(ws);
    p.dvl = reinterpret_cast<float*>(b + w.dvl);
    p.du = b + w.du;
    p.hD = b + w.hD;
  }
}

constexpr size_t smem_of(size_t bytes) { return bytes + 1024; }

template <typename T>
int fwd_typed(const Params& p, cudaStream_t st) {
  const int items = p.NC * p.HV, pairs = (items + 1) / 2;
  int e = launch2(gdn_tc_prep_kernel<T>, pairs, smem_of(sizeof(PrepSmem)), st, p, items);
  if (!e) e = launch(gdn_tc_state_kernel<T>, 2 * p.N * p.HV, smem_of(sizeof(StateSmem)), st, p);
  if (!e) e = launch2(gdn_tc_out_kernel<T>, pairs, smem_of(sizeof(OutSmem)), st, p, items);
  return e;
}

template <typename T>
int bwd_typed(const Params& p, bool reuse, cudaStream_t st) {
  const int items = p.NC * p.HV, pairs = (items + 1) / 2;
  const size_t rows = static_cast<size_t>(p.B) * p.T;
  if (p.gva) {
    int e = from_cuda(cudaMemsetAsync(p.dq, 0, rows * p.H * 64 * sizeof(float), st));
    if (!e) e = from_cuda(cudaMemsetAsync(p.dk, 0, rows * p.H * 64 * sizeof(float), st));
    if (e) return e;
  }
  int e = KATA_OK;
  if (!reuse) {  // rebuild gamma, W, U0 from the saved Tm, then u and the chunk states
    e = launch2(gdn_tc_prep_kernel<T>, pairs, smem_of(sizeof(PrepSmem)), st, p, items);
    if (!e) e = launch(gdn_tc_state_kernel<T>, 2 * p.N * p.HV, smem_of(sizeof(StateSmem)), st, p);
  }
  if (!e) e = launch2(gdn_tc_dvl_kernel<T>, pairs, smem_of(sizeof(DvlSmem)), st, p, items);
  if (!e) e = launch(gdn_tc_dstate_kernel<T>, 2 * p.N * p.HV, smem_of(sizeof(DstateSmem)), st, p);
  if (!e) e = launch(gdn_tc_grad_kernel<T>, p.NC * p.HV, smem_of(sizeof(GradSmem)), st, p, 256);
  return e;
}

}  // namespace
}  // namespace gdntc

size_t gdn_tc_fwd_workspace_bytes(int B, int T, int HV, int NC) {
  return gdntc::ws_layout(B, T, HV, NC, false, false).total;
}
size_t gdn_tc_bwd_workspace_bytes(int B, int T, int HV, int NC, bool reuse) {
  return gdntc::ws_layout(B, T, HV, NC, true, reuse).total;
}

int gdn_tc_fwd(const kata_gdn_fwd_args* a, cudaStream_t st) {
  using namespace gdntc;
  const Ws w = ws_layout(a->B, a->T, a->HV, a->num_chunks, false, false);
  if (!a->workspace || a->workspace_bytes < w.total) return KATA_ERR_WORKSPACE;
  const auto al16 = [](const void* x) { return (reinterpret_cast<uintptr_t>(x) & 15u) == 0; };
  if (!al16(a->q) || !al16(a->k) || !al16(a->v) || !al16(a->o) || !al16(a->A) || !al16(a->workspace) ||
      (a->h0 && !al16(a->h0)) || (a->ht && !al16(a->ht)))
    return KATA_ERR_ALIGN;
  Params p{};
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
  bind(p, a->workspace, w, false, nullptr);
  return a->dtype == KATA_DTYPE_BF16 ? fwd_typed<__nv_bfloat16>(p, st) : fwd_typed<__half>(p, st);
}

int gdn_tc_bwd(const kata_gdn_bwd_args* a, cudaStream_t st) {
  using namespace gdntc;
  const bool reuse = a->fwd_workspace != nullptr;
  const Ws w = ws_layout(a->B, a->T, a->HV, a->num_chunks, true, reuse);
  if (!a->workspace || a->workspace_bytes < w.total) return KATA_ERR_WORKSPACE;
  const auto al16 = [](const void* x) { return (reinterpret_cast<uintptr_t>(x) & 15u) == 0; };
  if (!al16(a->q) || !al16(a->k) || !al16(a->v) || !al16(a->A) || !al16(a->dout) || !al16(a->dq) ||
      !al16(a->dk) || !al16(a->dv) || !al16(a->workspace) || (a->fwd_workspace && !al16(a->fwd_workspace)) ||
      (a->h0 && !al16(a->h0)) || (a->dht && !al16(a->dht)) || (a->dh0 && !al16(a->dh0)))
    return KATA_ERR_ALIGN;
  Params p{};
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
  p.dq = a->dq;
  p.dk = a->dk;
  p.dv = a->dv;
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
  p.grad16 = a->grad_dtype != KATA_DTYPE_F32;
  bind(p, a->workspace, w, true, a->fwd_workspace);
  return a->dtype == KATA_DTYPE_BF16 ? bwd_typed<__nv_bfloat16>(p, reuse, st) : bwd_typed<__half>(p, reuse, st);
}

}  // namespace kata
