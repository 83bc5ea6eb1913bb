// sp_tc.cu -- the quadratic-feature contractions of the sequence-parallel and decode paths on tcgen05.
//
// With psi(x)[g,a,b] = scale * x_{g,a} x_{g,b} (concat score, F = M E^2 features; E = D / M) or
// psi(x)[a,b] = scale * sum_g x_{g,a} x_{g,b} (sum score, F = E^2), KATA-SPD attention of a query on
// an earlier block of keys is psi(q)^T P with the additive state P = sum_s psi(k_s) [v_s | 1].  The
// products here never materialise psi in global memory: every kernel forms its psi tiles in shared
// memory from the 16-bit token rows and feeds them to tcgen05.mma with fp32 accumulation in TMEM.
// The tiles hold the unscaled products x_a x_b rounded to bf16 (for bf16 rows one packed
// mul.rn.bf16x2 per two features: the product of two bf16 values is exact in fp32, so this is the
// same single rounding), or for the sum score the fp32 sum over groups rounded to bf16; the scale
// multiplies the fp32 result in the epilogue.
//
//   state  S[f, n]  = sum_t psi(x_t)[f] W[t, n]      one CTA per (256 features, head): two M = 128
//                                                    MMAs per K step, N = NW (the [v | 1 | 0] row
//                                                    rounded up to 16), K = tokens in blocks of 64
//   apply  Y[t, n]  = sum_f psi(x_t)[f] P[f, n]      one CTA per (256 tokens, head): two M = 128 MMAs,
//                                                    N = NW, K = features in blocks of 64; psi goes
//                                                    to TMEM (the A operand read from tensor memory)
//   grad   dx[t, (g,a)] += c * sum_b (W P^T)[t, (g,a,b)] x[t, (g,b)]
//                                                    one CTA per (256 features, head, token range):
//                                                    the P^T slice stays in shared memory, W streams
//                                                    by 128-token tiles; M = 128, N = 256, K = NW
// The operand that streams is the one whose reuse the CTA cannot hold: W (tokens) in `state` and
// `grad`, P^T (features) in `apply`; each CTA makes 256 rows of output per streamed byte, twice the
// reuse of a single 128-row MMA.
//
// Shared memory bandwidth (128 B per clock per SM) is what these kernels share out: every M = 128 MMA
// reads its A and B tiles from it, TMA writes the streamed tiles into it and the psi producers
// store into it.  `apply`, whose psi rows are token rows (TMEM lanes), keeps psi out of it.
//
// Every kernel runs 320 threads: warps 0-7 form psi (or run the epilogue of `grad`), warp 8 issues
// the TMA loads of a ring of stages, warp 9 issues the MMAs.  Stages are handed over by mbarriers
// only -- no CTA-wide barrier inside the main loops -- so psi for block i+1 is formed while the MMAs
// of block i run and the copies of blocks i+2.. are in flight.  Every wait is bounded (2 s); a wait
// that runs out sets the shared abort flag and the optional device status word, every role leaves
// its loop, and the CTA waits (bounded) for its own copies and MMAs in flight before it frees TMEM.
//
// The state is stored transposed, S^T (B*H, ldw, F) (rows n), so that P^T is the K-major B operand of
// `apply` and the MN-major B operand of `grad`; the decode path asks `state` for the untransposed
// (B*H, F, lds) layout instead.  W (B*H, T, ldw) and P^T (B*H, ldw, F) are bf16, and the token rows
// of `state` and `grad` arrive by TMA as well (no multicast); `apply` reads each token's row with
// plain 16-byte loads.  ldw <= 144, a multiple of 8.
#include <type_traits>

#include "attn_common.cuh"
#include "attn_tc_common.cuh"
#include "host_util.h"
#include "sm100.cuh"

namespace kata {
namespace sptc {
namespace {

constexpr uint32_t kRowB = 128;  // bytes of a 64-element 16-bit row (128-byte swizzle)
constexpr int kCompute = 256;    // psi / epilogue threads: warps 0-7
constexpr int kProducerWarp = 8;
constexpr int kIssuerWarp = 9;
constexpr int kThreads = kCompute + 64;
constexpr uint32_t kTmemCols = 512;  // two fp32 accumulators of up to 256 columns

__device__ __forceinline__ uint8_t* align1k(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~static_cast<uintptr_t>(1023));
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cta.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
          "r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ uint32_t par(int phase_index) { return static_cast<uint32_t>(phase_index & 1); }

// Abort path: wait (bounded) for the last phase armed on each barrier of a ring whose uses
// 0..count-1 went to bars[j % ring], phase j / ring, so that no copy or MMA still writes this CTA's
// shared memory or TMEM when it exits.
__device__ void drain_ring(uint64_t* bars, int ring, int count) {
  for (int k = 1; k <= ring && k <= count; ++k) {
    const int j = count - k;
    mbar_drain(&bars[j % ring], par(j / ring));
  }
}

struct Params {
  const void* x;  // (B, T, H, D) 16-bit token rows (q or k); `apply` reads them directly
  float* out;     // state: S^T (B*H, ldw, F) or S (B*H, F, lds);  apply: Y (B*H, T, ldw) or dv (B,T,H,Dv)
  float* dx;      // grad: (B, T, H, D) fp32, accumulated
  int* status;    // optional device status word
  int B, T, H, D, M, F, ldw, lds, Dv;
  int G;              // state: W has H*G heads, head hw reads x head hw / G;  apply: P head = x head / G
  int trans;          // state: 1 = S^T layout, 0 = (F, lds) layout
  int mode;           // apply: 0 = store Y, 1 = dv += Y[:, :Dv]
  int tiles_per_cta;  // grad: 128-token tiles of one CTA
  float scale;        // psi scale
  float factor;       // grad: c
};

// N 16-bit values (N a multiple of 8, src 16-byte aligned) to fp32.
template <typename T, int N>
__device__ __forceinline__ void load_vals(const T* src, float (&out)[N]) {
#pragma unroll
  for (int c = 0; c < N / 8; ++c) {
    const uint4 v = *reinterpret_cast<const uint4*>(src + 8 * c);
    const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
    for (int j = 0; j < 8; ++j) out[8 * c + j] = to_f32<T>(e[j]);
  }
}
// The E values of row `row` of a [rows][E] 16-bit tile that TMA wrote with the 2E-byte swizzle (the
// 16-byte chunks of each row permuted by row, so that a warp reading 32 consecutive rows spreads over
// all banks), and one element of it.
template <typename T, int E>
__device__ __forceinline__ void load_row_swz(const T* tile, int row, float (&out)[E]) {
  const uint8_t* base = reinterpret_cast<const uint8_t*>(tile);
#pragma unroll
  for (int c = 0; c < E / 8; ++c) {
    const uint4 v = *reinterpret_cast<const uint4*>(base + swz_offset(row, 16 * c, 2 * E));
    const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
    for (int j = 0; j < 8; ++j) out[8 * c + j] = to_f32<T>(e[j]);
  }
}
template <typename T, int E>
__device__ __forceinline__ float elem_swz(const T* tile, int row, int e) {
  return to_f32<T>(*reinterpret_cast<const T*>(reinterpret_cast<const uint8_t*>(tile) + swz_offset(row, 2 * e, 2 * E)));
}
__device__ __forceinline__ uint32_t bf16x2(float2 v) { return pack2<__nv_bfloat16>(v.x, v.y); }
// Two bf16 products a * b, each rounded once to nearest even.
__device__ __forceinline__ uint32_t bmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// The 16-bit half `hi` of a word in both halves.
__device__ __forceinline__ uint32_t bcast16(uint32_t w, int hi) { return __byte_perm(w, 0, hi ? 0x3232 : 0x1010); }
// The E / 2 words (16-bit pairs) of row `row` of a [rows][E] tile written with the 2E-byte swizzle.
template <int E>
__device__ __forceinline__ void load_words_swz(const void* tile, int row, uint32_t (&w)[E / 2]) {
  const uint8_t* base = static_cast<const uint8_t*>(tile);
#pragma unroll
  for (int c = 0; c < E / 8; ++c) {
    const uint4 v = *reinterpret_cast<const uint4*>(base + swz_offset(row, 16 * c, 2 * E));
    w[4 * c] = v.x, w[4 * c + 1] = v.y, w[4 * c + 2] = v.z, w[4 * c + 3] = v.w;
  }
}
template <typename T>
constexpr bool kIsBf16 = std::is_same<T, __nv_bfloat16>::value;
// One arrival per compute warp (barriers of the compute warps count kComputeWarps): the warp's
// shared-memory writes or reads, ordered by __syncwarp, are released by lane 0's arrive.
constexpr int kComputeWarps = kCompute / 32;
__device__ __forceinline__ void warp_arrive(uint64_t* bar) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

// ------------------------------------------------------------------------------------------------
// state: one CTA per (256-feature slice, W head); K-loop over the head's tokens in blocks of 64.
// A = psi^T, MN-major: four 64-feature boxes [64 tokens][128 B]; features 0-127 feed accumulator 0
// (TMEM columns 0..NW-1), 128-255 accumulator 1 (columns 256..).  B = the W tile, MN-major.
// Compute thread (t, q) forms token row t of feature box q.
// ------------------------------------------------------------------------------------------------
template <typename T, int E, bool SUM, int NW>
struct StateSmem {
  static constexpr int NWB = (NW + 63) / 64;
  static constexpr int SW = SUM ? 3 : 4;     // W / token-row ring
  static constexpr int XW = SUM ? 4 * E : E;  // 16-bit values per token row held (sum: all M <= 4 groups)
  uint8_t W[SW][NWB][64 * kRowB];
  static constexpr int SP = 3;                 // psi ring
  uint8_t psi[SP][4][64 * kRowB];
  T xs[SW][64 * XW];  // token rows: concat [64][E] with the 2E-byte swizzle, sum [64][D] dense
  uint64_t tfull[SW], mdone[SW], pfull[SP];
  uint32_t tmem;
  int abort;
};

template <typename T, int E, bool SUM, int NW>
__global__ void __launch_bounds__(kThreads, 1)
    sp_state_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, Params p) {
  using L = StateSmem<T, E, SUM, NW>;
  constexpr int SW = L::SW, SP = L::SP, NWB = L::NWB, EE = E * E, CPB = 64 / E;
  extern __shared__ uint8_t smraw[];
  L& sm = *reinterpret_cast<L*>(align1k(smraw));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int HW = p.H * p.G;  // heads of W and of the state
  const int bh = blockIdx.y, b = bh / HW, h = (bh % HW) / p.G;
  const int f0 = blockIdx.x * 256;
  const int g = SUM ? 0 : f0 / EE;
  const int a0 = (f0 % EE) / E;  // first a-value of the slice
  const int xw = SUM ? p.D : E;  // 16-bit values per token row in the tile
  const int nblk = (p.T + 63) / 64;
  if (tid == 0) {
    sm.abort = 0;
    for (int s = 0; s < SW; ++s) {
      mbar_init(&sm.tfull[s], 1);
      mbar_init(&sm.mdone[s], 1);
    }
    for (int s = 0; s < SP; ++s) mbar_init(&sm.pfull[s], kComputeWarps);
    fence_mbar_init();
  }
  if (warp == kProducerWarp) {
    tmem_alloc(&sm.tmem, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem;
  const WaitCtx wc{p.status, &sm.abort};
  int issued = 0, committed = 0;
  if (warp == kProducerWarp) {
    if (lane == 0) {
      tma_prefetch_desc(&tmW);
      tma_prefetch_desc(&tmX);
      const uint32_t bytes = NWB * 64 * kRowB + 64u * static_cast<uint32_t>(xw) * 2u;
      for (int j = 0; j < nblk; ++j) {
        const int s = j % SW;
        if (j >= SW && !mbar_wait(&sm.mdone[s], par((j - SW) / SW), wc)) break;
        mbar_arrive_expect_tx(&sm.tfull[s], bytes);
        for (int q = 0; q < NWB; ++q) tma_load_3d(sm.W[s][q], &tmW, &sm.tfull[s], 64 * q, 64 * j, bh);
        tma_load_4d(sm.xs[s], &tmX, &sm.tfull[s], g * E, h, 64 * j, b);
        issued = j + 1;
      }
    }
    __syncwarp();
  } else if (warp == kIssuerWarp) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(128, NW, true, true, true);
      for (int i = 0; i < nblk; ++i) {
        const int s = i % SW, ps = i % SP;
        if (!mbar_wait(&sm.tfull[s], par(i / SW), wc) || !mbar_wait(&sm.pfull[ps], par(i / SP), wc)) break;
        tc_fence_after();
        const uint64_t ad0 = umma_smem_desc(smem_u32(sm.psi[ps][0]), 64 * kRowB, 1024, 128);
        const uint64_t ad1 = umma_smem_desc(smem_u32(sm.psi[ps][2]), 64 * kRowB, 1024, 128);
        const uint64_t bd = umma_smem_desc(smem_u32(sm.W[s][0]), 64 * kRowB, 1024, 128);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {  // 16 tokens = 16 rows of 128 B per K step
          const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
          umma_ss(tbase, ad0 + 128u * kk, bd + 128u * kk, idesc, acc);
          umma_ss(tbase + 256u, ad1 + 128u * kk, bd + 128u * kk, idesc, acc);
        }
        umma_commit(&sm.mdone[s]);
        committed = i + 1;
      }
    }
    __syncwarp();
  } else {
    const int t = tid & 63, q = tid >> 6;  // token row of the block, 64-feature box
    const int aq = a0 + (64 * q) / E;      // first a-value of the box
    for (int i = 0; i < nblk; ++i) {
      const int s = i % SW, ps = i % SP;
      if (!mbar_wait_w(&sm.tfull[s], par(i / SW), wc)) break;
      if (i >= SP && !mbar_wait_w(&sm.mdone[(i - SP) % SW], par((i - SP) / SW), wc)) break;  // psi[ps] is free
      uint32_t v[32];  // the box row as bf16 pairs: features 2c, 2c+1 = (a = aq + 2c / E, b = 2c % E and + 1)
      if constexpr (SUM) {  // rows of xw = D values, unswizzled; fp32 sums over the groups
        const T* xr = sm.xs[s] + t * xw;
        float2 acc[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) acc[c] = make_float2(0.f, 0.f);
#pragma unroll
        for (int gg = 0; gg < 4; ++gg) {
          if (gg < p.M) {
            float xb[E], xa[CPB];
            load_vals<T, E>(xr + gg * E, xb);
#pragma unroll
            for (int k = 0; k < CPB; ++k) xa[k] = to_f32<T>(xr[gg * E + aq + k]);
#pragma unroll
            for (int c = 0; c < 32; ++c) {
              const int k = (2 * c) / E, bb = (2 * c) % E;
              acc[c] = ffma2(make_float2(xa[k], xa[k]), make_float2(xb[bb], xb[bb + 1]), acc[c]);
            }
          }
        }
#pragma unroll
        for (int c = 0; c < 32; ++c) v[c] = bf16x2(acc[c]);
      } else if constexpr (kIsBf16<T>) {  // rows of E values, 2E-byte swizzle: packed bf16 products
        uint32_t xw2[E / 2], xa[CPB];
        load_words_swz<E>(sm.xs[s], t, xw2);
        const uint8_t* xt = reinterpret_cast<const uint8_t*>(sm.xs[s]);
#pragma unroll
        for (int k = 0; k < CPB; ++k)
          xa[k] = bcast16(*reinterpret_cast<const uint16_t*>(xt + swz_offset(t, 2 * (aq + k), 2 * E)), 0);
#pragma unroll
        for (int c = 0; c < 32; ++c) v[c] = bmul2(xa[(2 * c) / E], xw2[((2 * c) % E) / 2]);
      } else {  // fp16 rows: fp32 products, one rounding to bf16
        float xb[E], xa[CPB];
        load_row_swz<T, E>(sm.xs[s], t, xb);
#pragma unroll
        for (int k = 0; k < CPB; ++k) xa[k] = elem_swz<T, E>(sm.xs[s], t, aq + k);
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const int k = (2 * c) / E, bb = (2 * c) % E;
          v[c] = bf16x2(fmul2(make_float2(xa[k], xa[k]), make_float2(xb[bb], xb[bb + 1])));
        }
      }
      const uint32_t base = smem_u32(sm.psi[ps][q]);
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8)
        st_shared_v4(base + swz_offset(t, 16 * c8, 128), v[4 * c8], v[4 * c8 + 1], v[4 * c8 + 2], v[4 * c8 + 3]);
      fence_proxy_async_smem();
      warp_arrive(&sm.pfull[ps]);
    }
  }
  __syncthreads();
  if (warp < kProducerWarp && __all_sync(0xffffffffu, sm.abort == 0) &&
      mbar_wait_w(&sm.mdone[(nblk - 1) % SW], par((nblk - 1) / SW), wc)) {
    tc_fence_after();
    const int lq = warp & 3, hh = warp >> 2;
    const int fl = f0 + 128 * hh + 32 * lq + lane;
    const uint32_t taddr = tbase + (static_cast<uint32_t>(32 * lq) << 16) + 256u * hh;
    float* out = p.out + static_cast<size_t>(bh) * p.F * (p.trans ? p.ldw : p.lds);
#pragma unroll
    for (int c0 = 0; c0 < NW; c0 += 16) {
      uint32_t r[16];
      tmem_ld16(taddr + c0, r);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int n = c0 + j;
        if (n < p.ldw) {
          const float y = p.scale * __uint_as_float(r[j]);
          if (p.trans) out[static_cast<size_t>(n) * p.F + fl] = y;
          else out[static_cast<size_t>(fl) * p.lds + n] = y;
        }
      }
    }
    if (!p.trans)
      for (int n = p.ldw; n < p.lds; ++n) out[static_cast<size_t>(fl) * p.lds + n] = 0.f;
  }
  tc_fence_before();
  __syncthreads();
  if (sm.abort != 0 && lane == 0) {
    if (warp == kIssuerWarp) drain_ring(sm.mdone, SW, committed);
    if (warp == kProducerWarp) drain_ring(sm.tfull, SW, issued);
  }
  __syncthreads();
  if (warp == kProducerWarp) tmem_dealloc(tbase, kTmemCols);
}

// ------------------------------------------------------------------------------------------------
// apply: one CTA per (256-token tile, head); K-loop over the F features in blocks of 64.  A = psi
// in TMEM, [128 lanes = tokens][32 columns = 64 features as bf16 pairs] per MMA: tokens 0-127 feed
// accumulator 0, tokens 128-255 accumulator 1.  B = the P^T block [NW rows][64 features], K-major,
// in shared memory.  Compute thread r owns token t0 + r (TMEM lane r % 128 of its half's A tile): it
// keeps its current group's E values in registers (the next group's loaded one group ahead) and
// writes its 32 psi columns with one tcgen05.st per block.
// TMEM columns: accumulator 0 at 0, accumulator 1 at 256; the three psi stages take the 32-column
// halves {144, 176}, {400, 432} and {208, 464} (free for both N = 80 and N = 144).
// ------------------------------------------------------------------------------------------------
template <int NW>
struct ApplySmem {
  static constexpr int SW = 4;  // P^T ring
  static constexpr int SP = 3;  // psi ring (TMEM)
  uint8_t P[SW][NW * kRowB];
  uint64_t pfull[SW], mdone[SW], sfull[SP];
  uint32_t tmem;
  int abort;
};
__device__ __forceinline__ uint32_t apply_psi_col(int stage, int half) {
  if (stage == 2) return half ? 464u : 208u;
  return (stage ? 400u : 144u) + 32u * static_cast<uint32_t>(half);
}

template <typename T, int E, int D, int NW>
__global__ void __launch_bounds__(kThreads, 1) sp_apply_kernel(const __grid_constant__ CUtensorMap tmP, Params p) {
  using L = ApplySmem<NW>;
  constexpr int SW = L::SW, SP = L::SP, EE = E * E, BPG = EE / 64;  // 64-feature blocks per group
  extern __shared__ uint8_t smraw[];
  L& sm = *reinterpret_cast<L*>(align1k(smraw));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const int bhp = b * (p.H / p.G) + h / p.G;  // the state's head
  const int t0 = blockIdx.x * 256;
  const int nblk = p.F / 64;
  if (tid == 0) {
    sm.abort = 0;
    for (int s = 0; s < SW; ++s) {
      mbar_init(&sm.pfull[s], 1);
      mbar_init(&sm.mdone[s], 1);
    }
    for (int s = 0; s < SP; ++s) mbar_init(&sm.sfull[s], kComputeWarps);
    fence_mbar_init();
  }
  if (warp == kProducerWarp) {
    tmem_alloc(&sm.tmem, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem;
  const WaitCtx wc{p.status, &sm.abort};
  int issued = 0, committed = 0;
  if (warp == kProducerWarp) {
    if (lane == 0) {
      tma_prefetch_desc(&tmP);
      for (int j = 0; j < nblk; ++j) {
        const int s = j % SW;
        if (j >= SW && !mbar_wait(&sm.mdone[s], par((j - SW) / SW), wc)) break;
        mbar_arrive_expect_tx(&sm.pfull[s], NW * kRowB);
        tma_load_3d(sm.P[s], &tmP, &sm.pfull[s], 64 * j, 0, bhp);
        issued = j + 1;
      }
    }
    __syncwarp();
  } else if (warp == kIssuerWarp) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(128, NW, true, false, false);
      for (int i = 0; i < nblk; ++i) {
        const int s = i % SW, ps = i % SP;
        if (!mbar_wait(&sm.pfull[s], par(i / SW), wc) || !mbar_wait(&sm.sfull[ps], par(i / SP), wc)) break;
        tc_fence_after();
        const uint32_t a0 = tbase + apply_psi_col(ps, 0), a1 = tbase + apply_psi_col(ps, 1);
        const uint64_t bd = umma_smem_desc(smem_u32(sm.P[s]), 16, 1024, 128);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {  // 16 features = 8 TMEM columns of A, 32 bytes of each B row
          const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
          umma_ts(tbase, a0 + 8u * kk, bd + 2u * kk, idesc, acc);
          umma_ts(tbase + 256u, a1 + 8u * kk, bd + 2u * kk, idesc, acc);
        }
        umma_commit(&sm.mdone[s]);
        committed = i + 1;
      }
    }
    __syncwarp();
  } else {
    const int r = tid, t = t0 + r;
    const bool tin = t < p.T;
    const T* xrow = static_cast<const T*>(p.x) + ((static_cast<size_t>(b) * p.T + (tin ? t : 0)) * p.H + h) * D;
    uint4 nxt[E / 8];  // the next group's values, loaded one group ahead
#pragma unroll
    for (int c = 0; c < E / 8; ++c)
      nxt[c] = tin ? reinterpret_cast<const uint4*>(xrow)[c] : make_uint4(0u, 0u, 0u, 0u);
    const uint32_t lane_base = tbase + (static_cast<uint32_t>(32 * (warp & 3)) << 16);
    bool ok = true;
    for (int g = 0; g < p.M && ok; ++g) {
      uint32_t xw2[E / 2];  // the group's values as 16-bit pairs
      float xg[kIsBf16<T> ? 1 : E];
#pragma unroll
      for (int c = 0; c < E / 8; ++c) {
        xw2[4 * c] = nxt[c].x, xw2[4 * c + 1] = nxt[c].y, xw2[4 * c + 2] = nxt[c].z, xw2[4 * c + 3] = nxt[c].w;
        if constexpr (!kIsBf16<T>) {
          const T* e = reinterpret_cast<const T*>(&nxt[c]);
#pragma unroll
          for (int j = 0; j < 8; ++j) xg[8 * c + j] = to_f32<T>(e[j]);
        }
      }
      if (g + 1 < p.M) {
#pragma unroll
        for (int c = 0; c < E / 8; ++c)
          nxt[c] = tin ? reinterpret_cast<const uint4*>(xrow + (g + 1) * E)[c] : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int ii = 0; ii < BPG; ++ii) {
        const int i = g * BPG + ii, ps = i % SP;
        if (i >= SP && !(ok = mbar_wait_w(&sm.mdone[(i - SP) % SW], par((i - SP) / SW), wc))) break;
        uint32_t wv[32];  // column c: features 2c, 2c+1 of the block
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const int j0 = 64 * ii + 2 * c;  // feature within the group (even)
          const int a = j0 / E, bb = j0 % E;
          if constexpr (kIsBf16<T>) wv[c] = bmul2(bcast16(xw2[a / 2], a & 1), xw2[bb / 2]);
          else wv[c] = bf16x2(fmul2(make_float2(xg[a], xg[a]), make_float2(xg[bb], xg[bb + 1])));
        }
        tmem_st32(lane_base + apply_psi_col(ps, warp >> 2), wv);
        tmem_wait_st();
        tc_fence_before();
        warp_arrive(&sm.sfull[ps]);
      }
    }
  }
  __syncthreads();
  if (warp < kProducerWarp && __all_sync(0xffffffffu, sm.abort == 0) &&
      mbar_wait_w(&sm.mdone[(nblk - 1) % SW], par((nblk - 1) / SW), wc)) {
    tc_fence_after();
    const int lq = warp & 3, hh = warp >> 2;
    const int t = t0 + 128 * hh + 32 * lq + lane;
    const uint32_t taddr = tbase + (static_cast<uint32_t>(32 * lq) << 16) + 256u * hh;
    const bool tin = t < p.T;
    const bool vec = p.mode == 0 || (p.Dv % 4) == 0;
    float* row = p.mode == 0 ? p.out + (static_cast<size_t>(bh) * p.T + (tin ? t : 0)) * p.ldw
                             : p.out + ((static_cast<size_t>(b) * p.T + (tin ? t : 0)) * p.H + h) * p.Dv;
    const int ncols = p.mode == 0 ? p.ldw : p.Dv;
#pragma unroll
    for (int c0 = 0; c0 < NW; c0 += 16) {
      uint32_t rv[16];
      tmem_ld16(taddr + c0, rv);
      tmem_wait_ld();
      if (!tin) continue;
      if (vec) {
#pragma unroll
        for (int j = 0; j < 16; j += 4) {
          if (c0 + j < ncols) {
            float4* d4 = reinterpret_cast<float4*>(row + c0 + j);
            float4 y = make_float4(p.scale * __uint_as_float(rv[j]), p.scale * __uint_as_float(rv[j + 1]),
                                   p.scale * __uint_as_float(rv[j + 2]), p.scale * __uint_as_float(rv[j + 3]));
            if (p.mode) {
              const float4 o = *d4;
              y.x += o.x, y.y += o.y, y.z += o.z, y.w += o.w;
            }
            *d4 = y;
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (c0 + j < ncols) row[c0 + j] += p.scale * __uint_as_float(rv[j]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (sm.abort != 0 && lane == 0) {
    if (warp == kIssuerWarp) drain_ring(sm.mdone, SW, committed);
    if (warp == kProducerWarp) drain_ring(sm.pfull, SW, issued);
  }
  __syncthreads();
  if (warp == kProducerWarp) tmem_dealloc(tbase, kTmemCols);
}

// ------------------------------------------------------------------------------------------------
// grad: one CTA per (256-feature slice, head, range of 128-token tiles).  B = the P^T slice
// [NW rows][256 features], MN-major, loaded once.  Per tile: A = W [128 tokens][NW], K-major, and
// the tile's token rows of the slice's group; D = W P^T (128 x 256) in one of two TMEM buffers, so
// the MMAs of tile j+1 run during the epilogue of tile j.  Epilogue warp w reads token rows
// 32 (w & 3).. and columns 128 (w >> 2).. (128 / E whole a-values): dx[t, g E + a] gets
// c * sum_b D[t, (a, b)] x[t, g E + b].
// ------------------------------------------------------------------------------------------------
template <typename T, int E, int NW>
struct GradSmem {
  static constexpr int NWB = (NW + 63) / 64;
  static constexpr int SW = NWB == 3 ? 2 : 3;  // W / token-row ring
  uint8_t B[4][NW * kRowB];
  uint8_t A[SW][NWB][128 * kRowB];
  T xs[SW][128 * E];  // token rows [128][E] of the slice's group, 2E-byte swizzle
  uint64_t bfull, afull[SW], afree[SW], xfree[SW], mdone[2], accfree[2];
  uint32_t tmem;
  int abort;
};

template <typename T, int E, int D, int NW>
__global__ void __launch_bounds__(kThreads, 1)
    sp_grad_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmP,
                   const __grid_constant__ CUtensorMap tmX, Params p) {
  using L = GradSmem<T, E, NW>;
  constexpr int SW = L::SW, NWB = L::NWB, EE = E * E, KSTEPS = NW / 16, NA = 128 / E;
  extern __shared__ uint8_t smraw[];
  L& sm = *reinterpret_cast<L*>(align1k(smraw));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const int f0 = blockIdx.x * 256, g = f0 / EE, a0 = (f0 % EE) / E;
  const int tile0 = blockIdx.z * p.tiles_per_cta;
  const int ntile = min(p.tiles_per_cta, (p.T + 127) / 128 - tile0);  // >= 1 by the grid's construction
  if (tid == 0) {
    sm.abort = 0;
    mbar_init(&sm.bfull, 1);
    for (int s = 0; s < SW; ++s) {
      mbar_init(&sm.afull[s], 1);
      mbar_init(&sm.afree[s], 1);
      mbar_init(&sm.xfree[s], kComputeWarps);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.mdone[s], 1);
      mbar_init(&sm.accfree[s], kComputeWarps);
    }
    fence_mbar_init();
  }
  if (warp == kProducerWarp) {
    tmem_alloc(&sm.tmem, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem;
  const WaitCtx wc{p.status, &sm.abort};
  int issued = 0, committed = 0;
  bool bissued = false;
  if (warp == kProducerWarp) {
    if (lane == 0) {
      tma_prefetch_desc(&tmW);
      tma_prefetch_desc(&tmP);
      tma_prefetch_desc(&tmX);
      mbar_arrive_expect_tx(&sm.bfull, 4 * NW * kRowB);
      for (int q = 0; q < 4; ++q) tma_load_3d(sm.B[q], &tmP, &sm.bfull, f0 + 64 * q, 0, bh);
      bissued = true;
      const uint32_t bytes = NWB * 128 * kRowB + 128u * E * 2u;
      for (int j = 0; j < ntile; ++j) {
        const int s = j % SW, tok = 128 * (tile0 + j);
        if (j >= SW && (!mbar_wait(&sm.afree[s], par((j - SW) / SW), wc) ||
                        !mbar_wait(&sm.xfree[s], par((j - SW) / SW), wc)))
          break;
        mbar_arrive_expect_tx(&sm.afull[s], bytes);
        for (int q = 0; q < NWB; ++q) tma_load_3d(sm.A[s][q], &tmW, &sm.afull[s], 64 * q, tok, bh);
        tma_load_4d(sm.xs[s], &tmX, &sm.afull[s], g * E, h, tok, b);
        issued = j + 1;
      }
    }
    __syncwarp();
  } else if (warp == kIssuerWarp) {
    if (lane == 0 && mbar_wait(&sm.bfull, 0, wc)) {
      constexpr uint32_t idesc = umma_idesc_f16(128, 256, true, false, true);
      const uint64_t bd = umma_smem_desc(smem_u32(sm.B[0]), NW * kRowB, 1024, 128);
      for (int j = 0; j < ntile; ++j) {
        const int s = j % SW, ab = j & 1;
        if (!mbar_wait(&sm.afull[s], par(j / SW), wc)) break;
        if (j >= 2 && !mbar_wait(&sm.accfree[ab], par((j - 2) >> 1), wc)) break;
        tc_fence_after();
        const uint64_t ad = umma_smem_desc(smem_u32(sm.A[s][0]), 16, 1024, 128);
        const uint32_t d = tbase + 256u * ab;
#pragma unroll
        for (int kk = 0; kk < KSTEPS; ++kk)
          umma_ss(d, ad + static_cast<uint64_t>(((kk >> 2) * 128 * kRowB + (kk & 3) * 32) >> 4),
                  bd + static_cast<uint64_t>(128 * kk), idesc, kk > 0 ? 1u : 0u);
        umma_commit(&sm.afree[s]);
        umma_commit(&sm.mdone[ab]);
        committed = j + 1;
      }
    }
    __syncwarp();
  } else {
    const int lq = warp & 3, hh = warp >> 2, r = 32 * lq + lane;
    const uint32_t lanebase = tbase + (static_cast<uint32_t>(32 * lq) << 16) + 128u * hh;
    for (int j = 0; j < ntile; ++j) {
      const int s = j % SW, ab = j & 1;
      if (!mbar_wait_w(&sm.afull[s], par(j / SW), wc)) break;
      float xg[E];
      load_row_swz<T, E>(sm.xs[s], r, xg);
      warp_arrive(&sm.xfree[s]);
      // this tile's dx values, loaded while the MMAs run
      const int t = 128 * (tile0 + j) + r;
      const bool tin = t < p.T;
      float4* d4 = reinterpret_cast<float4*>(p.dx + ((static_cast<size_t>(b) * p.T + (tin ? t : 0)) * p.H + h) * D +
                                             g * E + a0 + NA * hh);
      float4 dv[NA / 4];
#pragma unroll
      for (int c = 0; c < NA / 4; ++c) dv[c] = tin ? d4[c] : make_float4(0.f, 0.f, 0.f, 0.f);
      if (!mbar_wait_w(&sm.mdone[ab], par(j >> 1), wc)) break;
      tc_fence_after();
      float sums[NA];
#pragma unroll
      for (int c0 = 0; c0 < 128; c0 += 64) {  // two 32-column loads per wait
        uint32_t rv[64];
        tmem_ld32(lanebase + 256u * ab + c0, *reinterpret_cast<uint32_t(*)[32]>(rv));
        tmem_ld32(lanebase + 256u * ab + c0 + 32, *reinterpret_cast<uint32_t(*)[32]>(rv + 32));
        tmem_wait_ld();
        if (c0 == 64) {  // the accumulator buffer is read: tile j+2's MMAs may overwrite it
          tc_fence_before();
          warp_arrive(&sm.accfree[ab]);
        }
#pragma unroll
        for (int part = 0; part < 64 / E; ++part) {
          float sacc = 0.f;
#pragma unroll
          for (int jj = 0; jj < E; ++jj) sacc = fmaf(__uint_as_float(rv[part * E + jj]), xg[jj], sacc);
          sums[(c0 + part * E) / E] = sacc;
        }
      }
      if (tin) {
#pragma unroll
        for (int c = 0; c < NA / 4; ++c) {
          dv[c].x = fmaf(p.factor, sums[4 * c], dv[c].x);
          dv[c].y = fmaf(p.factor, sums[4 * c + 1], dv[c].y);
          dv[c].z = fmaf(p.factor, sums[4 * c + 2], dv[c].z);
          dv[c].w = fmaf(p.factor, sums[4 * c + 3], dv[c].w);
          d4[c] = dv[c];
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (sm.abort != 0 && lane == 0) {
    if (warp == kIssuerWarp) {
      drain_ring(sm.afree, SW, committed);
      drain_ring(sm.mdone, 2, committed);
    }
    if (warp == kProducerWarp) {
      if (bissued) mbar_drain(&sm.bfull, 0);
      drain_ring(sm.afull, SW, issued);
    }
  }
  __syncthreads();
  if (warp == kProducerWarp) tmem_dealloc(tbase, kTmemCols);
}

// ------------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------------
int nw_of(int ldw) { return ldw <= 80 ? 80 : 144; }

// W (B*H, T, ldw) bf16 with boxes of [64 cols][rows][1]
int map_w(CUtensorMap* m, const void* W, int BH, int T, int ldw, int rows) {
  const uint64_t dims[3] = {static_cast<uint64_t>(ldw), static_cast<uint64_t>(T), static_cast<uint64_t>(BH)};
  const uint64_t str[2] = {static_cast<uint64_t>(ldw) * 2, static_cast<uint64_t>(ldw) * 2 * T};
  const uint32_t box[3] = {64, static_cast<uint32_t>(rows), 1};
  return encode_tmap_16bit(m, W, 3, dims, str, box, 128);
}
// P^T (B*H, ldw, F) bf16 with boxes of [64 features][NW rows][1]
int map_p(CUtensorMap* m, const void* P, int BH, int ldw, int F, int nw) {
  const uint64_t dims[3] = {static_cast<uint64_t>(F), static_cast<uint64_t>(ldw), static_cast<uint64_t>(BH)};
  const uint64_t str[2] = {static_cast<uint64_t>(F) * 2, static_cast<uint64_t>(F) * 2 * ldw};
  const uint32_t box[3] = {64, static_cast<uint32_t>(nw), 1};
  return encode_tmap_16bit(m, P, 3, dims, str, box, 128);
}
// x (B, T, H, D) 16-bit with boxes of [cols values][1 head][rows tokens][1]; swizzle 0 (dense rows)
// or 2 cols bytes (cols in {16, 32})
int map_x(CUtensorMap* m, const void* x, int B, int T, int H, int D, int cols, int rows, int swizzle) {
  const uint64_t dims[4] = {static_cast<uint64_t>(D), static_cast<uint64_t>(H), static_cast<uint64_t>(T),
                            static_cast<uint64_t>(B)};
  const uint64_t str[3] = {static_cast<uint64_t>(D) * 2, static_cast<uint64_t>(H) * D * 2,
                           static_cast<uint64_t>(T) * H * D * 2};
  const uint32_t box[4] = {static_cast<uint32_t>(cols), 1, static_cast<uint32_t>(rows), 1};
  return encode_tmap_16bit(m, x, 4, dims, str, box, swizzle);
}

template <typename K>
int launch_cfg(K kernel, size_t smem) {
  return from_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
}

template <typename T, int E, bool SUM, int NW>
int state_launch(const Params& p, const CUtensorMap& tmW, const CUtensorMap& tmX, cudaStream_t st) {
  auto k = sp_state_kernel<T, E, SUM, NW>;
  const size_t smem = sizeof(StateSmem<T, E, SUM, NW>) + 1024;
  int e = launch_cfg(k, smem);
  if (e) return e;
  k<<<dim3(p.F / 256, p.B * p.H * p.G), kThreads, smem, st>>>(tmW, tmX, p);
  return from_cuda(cudaGetLastError());
}
template <typename T, int E, int D, int NW>
int apply_launch(const Params& p, const CUtensorMap& tmP, cudaStream_t st) {
  auto k = sp_apply_kernel<T, E, D, NW>;
  const size_t smem = sizeof(ApplySmem<NW>) + 1024;
  int e = launch_cfg(k, smem);
  if (e) return e;
  k<<<dim3((p.T + 255) / 256, p.B * p.H), kThreads, smem, st>>>(tmP, p);
  return from_cuda(cudaGetLastError());
}
template <typename T, int E, int D, int NW>
int grad_launch(const Params& p, const CUtensorMap& tmW, const CUtensorMap& tmP, const CUtensorMap& tmX,
                cudaStream_t st) {
  auto k = sp_grad_kernel<T, E, D, NW>;
  const size_t smem = sizeof(GradSmem<T, E, NW>) + 1024;
  int e = launch_cfg(k, smem);
  if (e) return e;
  const int ntt = (p.T + 127) / 128;
  const dim3 grid(p.F / 256, p.B * p.H, (ntt + p.tiles_per_cta - 1) / p.tiles_per_cta);
  k<<<grid, kThreads, smem, st>>>(tmW, tmP, tmX, p);
  return from_cuda(cudaGetLastError());
}

// Shapes covered: concat score with E in {16, 32} and D = M E in {64, 128}; the sum score (state only)
// with E in {16, 32} and M <= 4.  ldw <= 144, a multiple of 8.
bool shape_ok(int D, int M, int ldw, bool sum) {
  if (M < 1 || D % M || ldw < 8 || ldw > 144 || ldw % 8) return false;
  const int E = D / M;
  if (E != 16 && E != 32) return false;
  if (sum) return M <= 4;
  return D == 64 || D == 128;
}

template <typename T, int E, bool SUM>
int state_nw(const Params& p, const CUtensorMap& tmW, const CUtensorMap& tmX, cudaStream_t st) {
  return nw_of(p.ldw) == 80 ? state_launch<T, E, SUM, 80>(p, tmW, tmX, st) : state_launch<T, E, SUM, 144>(p, tmW, tmX, st);
}
template <typename T>
int state_dispatch(const Params& p, const CUtensorMap& tmW, const CUtensorMap& tmX, bool sum, cudaStream_t st) {
  const int E = p.D / p.M;
  if (sum) return E == 16 ? state_nw<T, 16, true>(p, tmW, tmX, st) : state_nw<T, 32, true>(p, tmW, tmX, st);
  return E == 16 ? state_nw<T, 16, false>(p, tmW, tmX, st) : state_nw<T, 32, false>(p, tmW, tmX, st);
}
template <typename T, int E, int D>
int apply_nw(const Params& p, const CUtensorMap& tmP, cudaStream_t st) {
  return nw_of(p.ldw) == 80 ? apply_launch<T, E, D, 80>(p, tmP, st) : apply_launch<T, E, D, 144>(p, tmP, st);
}
template <typename T>
int apply_dispatch(const Params& p, const CUtensorMap& tmP, cudaStream_t st) {
  const int E = p.D / p.M;
  if (p.D == 64) return E == 16 ? apply_nw<T, 16, 64>(p, tmP, st) : apply_nw<T, 32, 64>(p, tmP, st);
  return E == 16 ? apply_nw<T, 16, 128>(p, tmP, st) : apply_nw<T, 32, 128>(p, tmP, st);
}
template <typename T, int E, int D>
int grad_nw(const Params& p, const CUtensorMap& tmW, const CUtensorMap& tmP, const CUtensorMap& tmX, cudaStream_t st) {
  return nw_of(p.ldw) == 80 ? grad_launch<T, E, D, 80>(p, tmW, tmP, tmX, st)
                            : grad_launch<T, E, D, 144>(p, tmW, tmP, tmX, st);
}
template <typename T>
int grad_dispatch(const Params& p, const CUtensorMap& tmW, const CUtensorMap& tmP, const CUtensorMap& tmX,
                  cudaStream_t st) {
  const int E = p.D / p.M;
  if (p.D == 64)
    return E == 16 ? grad_nw<T, 16, 64>(p, tmW, tmP, tmX, st) : grad_nw<T, 32, 64>(p, tmW, tmP, tmX, st);
  return E == 16 ? grad_nw<T, 16, 128>(p, tmW, tmP, tmX, st) : grad_nw<T, 32, 128>(p, tmW, tmP, tmX, st);
}

// 128-token tiles per gradient CTA: 32 (one P^T slice load per 4096 tokens), fewer when the grid
// would otherwise not fill two waves of the 148 SMs.
int grad_tiles_per_cta(int F, int BH, int T) {
  const int ntt = (T + 127) / 128;
  const long long slices = static_cast<long long>(F / 256) * BH;
  int tpc = 32;
  while (tpc > 4 && slices * ((ntt + tpc - 1) / tpc) < 2 * 148) tpc /= 2;
  return tpc;
}

bool al16(const void* x) { return (reinterpret_cast<uintptr_t>(x) & 15u) == 0; }

}  // namespace
}  // namespace sptc
}  // namespace kata

using namespace kata;

extern "C" int kata_sp_state(const void* x, const void* W, float* S, int dtype, int B, int T, int H, int G, int D,
                             int M, int score, int ldw, float scale, int trans, int lds, int* status,
                             kata_stream_t stream) {
  using namespace sptc;
  if (!x || !W || !S) return KATA_ERR_INVALID;
  if (dtype != KATA_DTYPE_BF16 && dtype != KATA_DTYPE_F16) return KATA_ERR_DTYPE;
  const bool sum = score == KATA_SCORE_SUM;
  if (B < 1 || T < 1 || H < 1 || G < 1 || !shape_ok(D, M, ldw, sum)) return KATA_ERR_SHAPE;
  if (!trans && (lds < ldw || lds % 4)) return KATA_ERR_SHAPE;
  if (!al16(x) || !al16(W) || !al16(S)) return KATA_ERR_ALIGN;
  const int E = D / M;
  Params p{};
  p.x = x;
  p.out = S;
  p.status = status;
  p.B = B;
  p.T = T;
  p.H = H;
  p.D = D;
  p.M = M;
  p.F = sum ? E * E : M * E * E;
  p.ldw = ldw;
  p.lds = lds;
  p.G = G;
  p.trans = trans;
  p.scale = scale;
  CUtensorMap tmW, tmX;
  int e = map_w(&tmW, W, B * H * G, T, ldw, 64);
  if (!e) e = map_x(&tmX, x, B, T, H, D, sum ? D : E, 64, sum ? 0 : 2 * E);
  if (e) return e;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return dtype == KATA_DTYPE_BF16 ? state_dispatch<__nv_bfloat16>(p, tmW, tmX, sum, st)
                                  : state_dispatch<__half>(p, tmW, tmX, sum, st);
}

extern "C" int kata_sp_apply(const void* x, const void* P, float* Y, int dtype, int B, int T, int H, int G, int D,
                             int M, int ldw, float scale, int dv_mode, int Dv, int* status, kata_stream_t stream) {
  using namespace sptc;
  if (!x || !P || !Y) return KATA_ERR_INVALID;
  if (dtype != KATA_DTYPE_BF16 && dtype != KATA_DTYPE_F16) return KATA_ERR_DTYPE;
  if (B < 1 || T < 1 || H < 1 || G < 1 || H % G || !shape_ok(D, M, ldw, false)) return KATA_ERR_SHAPE;
  if (dv_mode && (Dv < 1 || Dv > ldw)) return KATA_ERR_SHAPE;
  if (!al16(x) || !al16(P) || !al16(Y)) return KATA_ERR_ALIGN;
  const int E = D / M;
  Params p{};
  p.x = x;
  p.out = Y;
  p.status = status;
  p.B = B;
  p.T = T;
  p.H = H;
  p.D = D;
  p.M = M;
  p.F = M * E * E;
  p.ldw = ldw;
  p.Dv = Dv;
  p.G = G;
  p.mode = dv_mode;
  p.scale = scale;
  CUtensorMap tmP;
  int e = map_p(&tmP, P, B * (H / G), ldw, p.F, nw_of(ldw));
  if (e) return e;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return dtype == KATA_DTYPE_BF16 ? apply_dispatch<__nv_bfloat16>(p, tmP, st) : apply_dispatch<__half>(p, tmP, st);
}

extern "C" int kata_sp_grad(const void* W, const void* P, const void* x, float* dx, int dtype, int B, int T, int H,
                            int D, int M, int ldw, float factor, int* status, kata_stream_t stream) {
  using namespace sptc;
  if (!x || !P || !W || !dx) return KATA_ERR_INVALID;
  if (dtype != KATA_DTYPE_BF16 && dtype != KATA_DTYPE_F16) return KATA_ERR_DTYPE;
  if (B < 1 || T < 1 || H < 1 || !shape_ok(D, M, ldw, false)) return KATA_ERR_SHAPE;
  if (!al16(x) || !al16(P) || !al16(W) || !al16(dx)) return KATA_ERR_ALIGN;
  const int E = D / M;
  Params p{};
  p.x = x;
  p.dx = dx;
  p.status = status;
  p.B = B;
  p.T = T;
  p.H = H;
  p.D = D;
  p.M = M;
  p.F = M * E * E;
  p.ldw = ldw;
  p.G = 1;
  p.factor = factor;
  p.tiles_per_cta = grad_tiles_per_cta(p.F, B * H, T);
  CUtensorMap tmW, tmP, tmX;
  int e = map_w(&tmW, W, B * H, T, ldw, 128);
  if (!e) e = map_p(&tmP, P, B * H, ldw, p.F, nw_of(ldw));
  if (!e) e = map_x(&tmX, x, B, T, H, D, E, 128, 2 * E);
  if (e) return e;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return dtype == KATA_DTYPE_BF16 ? grad_dispatch<__nv_bfloat16>(p, tmW, tmP, tmX, st)
                                  : grad_dispatch<__half>(p, tmW, tmP, tmX, st);
}
