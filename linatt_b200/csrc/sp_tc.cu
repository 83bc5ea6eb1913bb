// sp_tc.cu -- the quadratic-feature contractions of the sequence-parallel and decode paths on tcgen05.
//
// With psi(x)[g,a,b] = scale * x_{g,a} x_{g,b} (concat score, F = M E^2 features; E = D / M) or
// psi(x)[a,b] = scale * sum_g x_{g,a} x_{g,b} (sum score, F = E^2), KATA-SPD attention of a query on
// an earlier block of keys is psi(q)^T P with the additive state P = sum_s psi(k_s) [v_s | 1].  The
// products here never materialise psi in global memory: every kernel forms its psi tiles in shared
// memory from the 16-bit token rows, rounded to bf16 exactly as a materialised feature tensor would
// be (product first, then the scale), and feeds them to tcgen05.mma with fp32 accumulation in TMEM.
//
//   state  S[f, n]  = sum_t psi(x_t)[f] W[t, n]      M = 128 features, N = NW (the [v | 1 | 0] row
//                                                    rounded up to 16), K = tokens in blocks of 64
//   apply  Y[t, n]  = sum_f psi(x_t)[f] P[f, n]      M = 128 tokens, N = NW, K = features (blocks of 64)
//   grad   dx[t, (g,a)] += c * sum_b (W P^T)[t, (g,a,b)] x[t, (g,b)]
//                                                    M = 128 tokens, N = 256 features, K = NW
// The state is stored transposed, S^T (B*H, ldw, F) (rows n), so that P^T is the K-major B operand of
// `apply` and the MN-major B operand of `grad`; the decode path asks `state` for the untransposed
// (B*H, F, lds) layout instead.  W (B*H, T, ldw) and P^T (B*H, ldw, F) are bf16 and arrive by TMA
// (no multicast); token rows are read with plain 16-byte loads.  ldw <= 144, a multiple of 8.
#include "attn_common.cuh"
#include "attn_tc_common.cuh"
#include "host_util.h"
#include "sm100.cuh"

namespace kata {
namespace sptc {
namespace {

constexpr uint32_t kRowB = 128;          // bytes of a 64-element 16-bit row (128-byte swizzle)
constexpr int kStages = 4;  // ring depth of the state / apply pipelines (prefetch distance 2)

__device__ __forceinline__ uint8_t* align1k(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~static_cast<uintptr_t>(1023));
}
__device__ __forceinline__ uint32_t toff(int r, int c) { return swz_offset(r, c * 2, 128); }
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(pred ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cta.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
          "r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
// Uniform bounded wait of all threads of the CTA on one barrier phase; false when any timed out.
__device__ __forceinline__ bool wait_all(uint64_t* bar, uint32_t parity, volatile int* abort, int* status) {
  WaitCtx wc{status, abort};
  const bool ok = mbar_wait(bar, parity, wc);
  return !__syncthreads_or(!ok);
}

struct Params {
  const void* x;     // (B, T, H, D) 16-bit token rows (q or k)
  const void* W;     // unused on the device (TMA)
  float* out;        // state: S^T (B*H, ldw, F) or S (B*H, F, lds);  apply: Y (B*H, T, ldw) or dv (B,T,H,Dv)
  float* dx;         // grad: (B, T, H, D) fp32, accumulated
  int* status;
  int B, T, H, D, M, F, ldw, lds, Dv;
  int G;             // state: W has H*G heads, head hw reads x head hw / G;  apply: P head = x head / G
  int trans;         // state: 1 = S^T layout, 0 = (F, lds) layout
  int mode;          // apply: 0 = store Y, 1 = dv += Y[:, :Dv]
  float scale;       // psi scale
  float factor;      // grad: c
};

template <typename T>
__device__ __forceinline__ float bf(T v) { return to_f32<T>(v); }

// Element i (a compile-time index after unrolling) of a token row held as packed 16-bit pairs.
template <typename T>
__device__ __forceinline__ float xunpack(uint32_t w, int odd) {
  const uint16_t hb = odd ? static_cast<uint16_t>(w >> 16) : static_cast<uint16_t>(w & 0xffffu);
  return to_f32<T>(*reinterpret_cast<const T*>(&hb));
}
// The E values of group g (a runtime value) of the token row: an unrolled compare over the groups,
// so every register index stays a compile-time constant (no local-memory copy of the row).
template <typename T, int E, int D>
__device__ __forceinline__ void group_vals(const uint32_t (&xr)[D / 2], int g, float (&xg)[E]) {
#pragma unroll
  for (int gg = 0; gg < D / E; ++gg)
    if (gg == g) {
#pragma unroll
      for (int e = 0; e < E; ++e) xg[e] = xunpack<T>(xr[(gg * E + e) >> 1], (gg * E + e) & 1);
    }
}

// ------------------------------------------------------------------------------------------------
// state: one CTA per (128-feature tile, head); K-loop over the head's tokens in blocks of 64.
// Thread f of 128 owns feature f0 + f: it forms row f of the K-major psi tile [f][t] for each block.
// ------------------------------------------------------------------------------------------------
template <typename T, int E, bool SUM, int NW>
struct StateSmem {
  static constexpr int NWB = (NW + 63) / 64;
  static constexpr int XW = SUM ? 4 * E : E;  // 16-bit values of a token row held per block (SUM: all M <= 4 groups)
  uint8_t W[kStages][NWB][64 * kRowB];
  uint8_t psi[kStages][128 * kRowB];
  T xs[kStages][64][XW];
  uint64_t wfull[kStages], mdone[kStages];
  uint32_t tmem;
  int abort;
};

template <typename T, int E, bool SUM, int NW>
__global__ void __launch_bounds__(128, 1) sp_state_kernel(const __grid_constant__ CUtensorMap tmW, Params p) {
  using L = StateSmem<T, E, SUM, NW>;
  extern __shared__ uint8_t smraw[];
  L& sm = *reinterpret_cast<L*>(align1k(smraw));
  constexpr int EE = E * E;
  constexpr int NWB = L::NWB;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int HW = p.H * p.G;  // heads of W and of the state
  const int bh = blockIdx.y, b = bh / HW, h = (bh % HW) / p.G;
  const int f0 = blockIdx.x * 128;
  const int g = SUM ? 0 : f0 / EE;
  const int rem = (f0 + tid) % EE, fa = rem / E, fb = rem % E;
  const int M = SUM ? p.M : 1;
  const int nblk = (p.T + 63) / 64;
  if (tid == 0) {
    sm.abort = 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.wfull[s], 1);
      mbar_init(&sm.mdone[s], 1);
    }
    fence_mbar_init();
    tma_prefetch_desc(&tmW);
  }
  if (warp == 0) {
    tmem_alloc(&sm.tmem, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem;
  const T* xb = static_cast<const T*>(p.x);
  // block j's W tile (TMA, thread 0) and its token rows (cp.async, every thread)
  auto issue = [&](int j) {
    const int s = j % kStages;
    if (tid == 0) {
      mbar_arrive_expect_tx(&sm.wfull[s], NWB * 64 * kRowB);
      for (int q = 0; q < NWB; ++q) tma_load_3d(sm.W[s][q], &tmW, &sm.wfull[s], 64 * q, 64 * j, bh);
    }
    const int CPR = (SUM ? p.D : E) * 2 / 16;  // 16-byte chunks of the token row this tile needs
    for (int i = tid; i < 64 * CPR; i += 128) {
      const int r = i / CPR, c = i % CPR, t = 64 * j + r;
      const bool ok = t < p.T;
      const T* src = xb + ((static_cast<size_t>(b) * p.T + (ok ? t : 0)) * p.H + h) * p.D + g * E + 8 * c;
      cp_async16(smem_u32(&sm.xs[s][r][8 * c]), src, ok);
    }
    cp_async_commit();
  };
  issue(0);
  if (nblk > 1) issue(1);
  constexpr uint32_t idesc = umma_idesc_f16(128, NW, true, false, true);
  bool ok = true;
  for (int i = 0; i < nblk && ok; ++i) {
    const int s = i % kStages;
    if (i + 2 < nblk) {
      // stage (i+2) % 4 held block i-2: its W tile is free once that block's MMAs completed
      if (tid == 0 && i >= 2) {
        WaitCtx wc{p.status, &sm.abort};
        mbar_wait(&sm.mdone[(i - 2) % kStages], static_cast<uint32_t>(((i - 2) / kStages) & 1), wc);
      }
      issue(i + 2);
      cp_async_wait<2>();
    } else if (i + 1 < nblk) {
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    // psi[s] was last read by block i-4's MMAs
    if (i >= kStages &&
        !(ok = wait_all(&sm.mdone[s], static_cast<uint32_t>(((i - kStages) / kStages) & 1), &sm.abort, p.status)))
      break;
    __syncthreads();
    {  // row tid of psi[s]: 64 tokens
      const uint32_t base = smem_u32(sm.psi[s]);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t wv[4];
#pragma unroll
        for (int e2 = 0; e2 < 4; ++e2) {
          float v2[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int t = 8 * c + 2 * e2 + u;
            if constexpr (SUM) {
              float acc = 0.f;
              for (int gg = 0; gg < M; ++gg) acc = fmaf(bf(sm.xs[s][t][gg * E + fa]), bf(sm.xs[s][t][gg * E + fb]), acc);
              v2[u] = p.scale * acc;
            } else {
              v2[u] = p.scale * (bf(sm.xs[s][t][fa]) * bf(sm.xs[s][t][fb]));
            }
          }
          wv[e2] = pack2<__nv_bfloat16>(v2[0], v2[1]);
        }
        st_shared_v4(base + toff(tid, 8 * c), wv[0], wv[1], wv[2], wv[3]);
      }
    }
    fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0) {
      WaitCtx wc{p.status, &sm.abort};
      if (mbar_wait(&sm.wfull[s], static_cast<uint32_t>((i / kStages) & 1), wc)) {
        tc_fence_after();
        const uint64_t ad = umma_smem_desc(smem_u32(sm.psi[s]), 16, 1024, 128);
        const uint64_t bd = umma_smem_desc(smem_u32(sm.W[s][0]), 64 * kRowB, 1024, 128);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_ss(tbase, ad + static_cast<uint64_t>(2 * kk), bd + static_cast<uint64_t>(128 * kk), idesc,
                  (i > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&sm.mdone[s]);
      }
    }
    ok = !__syncthreads_or(sm.abort != 0);
  }
  if (ok && nblk > 0)
    ok = wait_all(&sm.mdone[(nblk - 1) % kStages], static_cast<uint32_t>(((nblk - 1) / kStages) & 1), &sm.abort,
                  p.status);
  if (ok && nblk > 0) {
    tc_fence_after();
    const int fl = f0 + tid;
    const uint32_t lane = static_cast<uint32_t>(32 * warp) << 16;
    float* out = p.out + static_cast<size_t>(bh) * p.F * (p.trans ? p.ldw : p.lds);
#pragma unroll
    for (int c0 = 0; c0 < NW; c0 += 16) {
      uint32_t r[16];
      tmem_ld16(tbase + lane + c0, r);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int n = c0 + j;
        if (n < p.ldw) {
          if (p.trans) out[static_cast<size_t>(n) * p.F + fl] = __uint_as_float(r[j]);
          else out[static_cast<size_t>(fl) * p.lds + n] = __uint_as_float(r[j]);
        }
      }
    }
    if (!p.trans)
      for (int n = p.ldw; n < p.lds; ++n) out[static_cast<size_t>(fl) * p.lds + n] = 0.f;
  }
  cp_async_wait<0>();
  if (!ok && tid == 0)
    for (int s = 0; s < kStages; ++s) mbar_drain(&sm.mdone[s], 0), mbar_drain(&sm.mdone[s], 1);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, 256);
}

// ------------------------------------------------------------------------------------------------
// apply: one CTA per (128-token tile, head); K-loop over the F features in blocks of 64.  Thread t
// of 128 owns token t0 + t (its 16-bit row in registers) and forms row t of the K-major psi tile.
// ------------------------------------------------------------------------------------------------
template <int NW>
struct ApplySmem {
  uint8_t P[kStages][NW * kRowB];
  uint8_t psi[kStages][128 * kRowB];
  uint64_t pfull[kStages], mdone[kStages];
  uint32_t tmem;
  int abort;
};

template <typename T, int E, int D, int NW>
__global__ void __launch_bounds__(128, 1) sp_apply_kernel(const __grid_constant__ CUtensorMap tmP, Params p) {
  using L = ApplySmem<NW>;
  extern __shared__ uint8_t smraw[];
  L& sm = *reinterpret_cast<L*>(align1k(smraw));
  constexpr int EE = E * E;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const int bhp = b * (p.H / p.G) + h / p.G;  // the state's head
  const int t = blockIdx.x * 128 + tid;
  const bool tin = t < p.T;
  const int nblk = p.F / 64;
  if (tid == 0) {
    sm.abort = 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.pfull[s], 1);
      mbar_init(&sm.mdone[s], 1);
    }
    fence_mbar_init();
    tma_prefetch_desc(&tmP);
  }
  if (warp == 0) {
    tmem_alloc(&sm.tmem, 256);
    tmem_relinquish();
  }
  // this thread's token row, packed 16-bit pairs
  uint32_t xr[D / 2];
  {
    const uint4* src = reinterpret_cast<const uint4*>(static_cast<const T*>(p.x) +
                                                      ((static_cast<size_t>(b) * p.T + (tin ? t : 0)) * p.H + h) * D);
#pragma unroll
    for (int c = 0; c < D / 8; ++c) {
      const uint4 v = tin ? src[c] : make_uint4(0u, 0u, 0u, 0u);
      xr[4 * c] = v.x;
      xr[4 * c + 1] = v.y;
      xr[4 * c + 2] = v.z;
      xr[4 * c + 3] = v.w;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem;
  auto issue = [&](int j) {
    if (tid == 0) {
      const int s = j % kStages;
      mbar_arrive_expect_tx(&sm.pfull[s], NW * kRowB);
      tma_load_3d(sm.P[s], &tmP, &sm.pfull[s], 64 * j, 0, bhp);
    }
  };
  issue(0);
  if (nblk > 1) issue(1);
  constexpr uint32_t idesc = umma_idesc_f16(128, NW, true, false, false);
  constexpr int BPG = EE / 64;  // 64-feature blocks per group
  bool ok = true;
  for (int g = 0; g < p.F / EE && ok; ++g) {
    float xg[E];
    group_vals<T, E, D>(xr, g, xg);
#pragma unroll
    for (int ii = 0; ii < BPG; ++ii) {
      const int i = g * BPG + ii;
      const int s = i % kStages;
      if (i + 2 < nblk) {
        if (tid == 0 && i >= 2) {  // stage (i+2) % 4 held block i-2
          WaitCtx wc{p.status, &sm.abort};
          mbar_wait(&sm.mdone[(i - 2) % kStages], static_cast<uint32_t>(((i - 2) / kStages) & 1), wc);
        }
        issue(i + 2);
      }
      if (i >= kStages &&
          !(ok = wait_all(&sm.mdone[s], static_cast<uint32_t>(((i - kStages) / kStages) & 1), &sm.abort, p.status)))
        break;
      {  // row tid of psi[s]: features 64 i .. 64 i + 63 = (g, a0 + j / E, j % E)
        const uint32_t base = smem_u32(sm.psi[s]);
        constexpr int a0 = 0;  // (64 ii) / E is added below as a compile-time offset
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t wv[4];
#pragma unroll
          for (int e2 = 0; e2 < 4; ++e2) {
            const int j0 = 8 * c + 2 * e2;  // feature offset within the block (even)
            const int a = a0 + (64 * ii + j0) / E, bb = (64 * ii + j0) % E;
            const float xa = xg[a];
            wv[e2] = pack2<__nv_bfloat16>(p.scale * (xa * xg[bb]), p.scale * (xa * xg[bb + 1]));
          }
          st_shared_v4(base + toff(tid, 8 * c), wv[0], wv[1], wv[2], wv[3]);
        }
      }
      fence_proxy_async_smem();
      __syncthreads();
      if (tid == 0) {
        WaitCtx wc{p.status, &sm.abort};
        if (mbar_wait(&sm.pfull[s], static_cast<uint32_t>((i / kStages) & 1), wc)) {
          tc_fence_after();
          const uint64_t ad = umma_smem_desc(smem_u32(sm.psi[s]), 16, 1024, 128);
          const uint64_t bd = umma_smem_desc(smem_u32(sm.P[s]), 16, 1024, 128);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_ss(tbase, ad + static_cast<uint64_t>(2 * kk), bd + static_cast<uint64_t>(2 * kk), idesc,
                    (i > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&sm.mdone[s]);
        }
      }
      ok = !__syncthreads_or(sm.abort != 0);
      if (!ok) break;
    }
  }
  if (ok && nblk > 0)
    ok = wait_all(&sm.mdone[(nblk - 1) % kStages], static_cast<uint32_t>(((nblk - 1) / kStages) & 1), &sm.abort,
                  p.status);
  if (ok && nblk > 0) {
    tc_fence_after();
    const uint32_t lane = static_cast<uint32_t>(32 * warp) << 16;
#pragma unroll
    for (int c0 = 0; c0 < NW; c0 += 16) {
      uint32_t r[16];
      tmem_ld16(tbase + lane + c0, r);
      tmem_wait_ld();
      if (tin) {
        if (p.mode == 0) {
          float* y = p.out + (static_cast<size_t>(bh) * p.T + t) * p.ldw;
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (c0 + j < p.ldw) y[c0 + j] = __uint_as_float(r[j]);
        } else {
          float* dv = p.out + ((static_cast<size_t>(b) * p.T + t) * p.H + h) * p.Dv;
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (c0 + j < p.Dv) dv[c0 + j] += __uint_as_float(r[j]);
        }
      }
    }
  }
  if (!ok && tid == 0)
    for (int s = 0; s < kStages; ++s) mbar_drain(&sm.mdone[s], 0), mbar_drain(&sm.mdone[s], 1);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, 256);
}

// ------------------------------------------------------------------------------------------------
// grad: one CTA per (128-token tile, head).  A = W tile (128 tokens x NW, K-major, loaded once);
// per 256-feature tile, B = P^T (NW rows x 256 features, MN-major, four TMA boxes) and
// D = W P^T (128 x 256) in one of two TMEM buffers, so the MMAs of tile i+1 run during the epilogue
// of tile i.  Epilogue: thread t contracts its row of D with its token's group values.
// ------------------------------------------------------------------------------------------------
template <int NW>
struct GradSmem {
  static constexpr int NWB = (NW + 63) / 64;
  uint8_t A[NWB][128 * kRowB];
  uint8_t B[2][4][NW * kRowB];
  float dxs[32][128];  // a group's per-(a, token) results, [a][thread]
  uint64_t afull, bfull[2], mdone[2];
  uint32_t tmem;
  int abort;
};

template <typename T, int E, int D, int NW>
__global__ void __launch_bounds__(128, 1) sp_grad_kernel(const __grid_constant__ CUtensorMap tmW,
                                                         const __grid_constant__ CUtensorMap tmP, Params p) {
  using L = GradSmem<NW>;
  extern __shared__ uint8_t smraw[];
  L& sm = *reinterpret_cast<L*>(align1k(smraw));
  constexpr int EE = E * E;
  constexpr int NWB = L::NWB;
  constexpr int KSTEPS = NW / 16;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const int t0 = blockIdx.x * 128, t = t0 + tid;
  const bool tin = t < p.T;
  const int ntile = p.F / 256;
  if (tid == 0) {
    sm.abort = 0;
    mbar_init(&sm.afull, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.bfull[s], 1);
      mbar_init(&sm.mdone[s], 1);
    }
    fence_mbar_init();
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmP);
  }
  if (warp == 0) {
    tmem_alloc(&sm.tmem, 512);
    tmem_relinquish();
  }
  // this thread's token row (each group's E values are read when the group starts)
  const T* xrow = static_cast<const T*>(p.x) + ((static_cast<size_t>(b) * p.T + (tin ? t : 0)) * p.H + h) * D;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem;
  auto issue_b = [&](int j) {
    const int s = j & 1;
    mbar_arrive_expect_tx(&sm.bfull[s], 4 * NW * kRowB);
    for (int q = 0; q < 4; ++q) tma_load_3d(sm.B[s][q], &tmP, &sm.bfull[s], 256 * j + 64 * q, 0, bh);
  };
  constexpr uint32_t idesc = umma_idesc_f16(128, 256, true, false, true);
  auto issue_mma = [&](int j) {  // thread 0
    WaitCtx wc{p.status, &sm.abort};
    if (!mbar_wait(&sm.bfull[j & 1], static_cast<uint32_t>((j >> 1) & 1), wc)) return;
    tc_fence_after();
    const uint64_t ad = umma_smem_desc(smem_u32(sm.A[0]), 16, 1024, 128);
    const uint64_t bd = umma_smem_desc(smem_u32(sm.B[j & 1][0]), NW * kRowB, 1024, 128);
    const uint32_t d = tbase + 256u * static_cast<uint32_t>(j & 1);
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk)
      umma_ss(d, ad + static_cast<uint64_t>(((kk >> 2) * 128 * kRowB + (kk & 3) * 32) >> 4),
              bd + static_cast<uint64_t>(128 * kk), idesc, kk > 0 ? 1u : 0u);
    umma_commit(&sm.mdone[j & 1]);
  };
  if (tid == 0) {
    mbar_arrive_expect_tx(&sm.afull, NWB * 128 * kRowB);
    for (int q = 0; q < NWB; ++q) tma_load_3d(sm.A[q], &tmW, &sm.afull, 64 * q, t0, bh);
    issue_b(0);
    if (ntile > 1) issue_b(1);
    WaitCtx wc{p.status, &sm.abort};
    if (mbar_wait(&sm.afull, 0, wc)) issue_mma(0);
  }
  bool ok = true;
  float* dxrow = p.dx + ((static_cast<size_t>(b) * p.T + (tin ? t : 0)) * p.H + h) * D;
  const uint32_t lane = static_cast<uint32_t>(32 * warp) << 16;
  constexpr int TPG = EE / 256;  // 256-feature tiles per group
  for (int g = 0; g < p.F / EE && ok; ++g) {
    float xg[E];
    {
      const uint4* src = reinterpret_cast<const uint4*>(xrow + g * E);
#pragma unroll
      for (int c = 0; c < E / 8; ++c) {
        const uint4 v = tin ? src[c] : make_uint4(0u, 0u, 0u, 0u);
        const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
        for (int j = 0; j < 8; ++j) xg[8 * c + j] = to_f32<T>(e[j]);
      }
    }
#pragma unroll
    for (int ii = 0; ii < TPG; ++ii) {
      const int i = g * TPG + ii;
      // the MMAs of tile i+1 (its accumulator buffer was last read by tile i-1's epilogue, finished)
      if (tid == 0 && i + 1 < ntile) issue_mma(i + 1);
      if (!(ok = wait_all(&sm.mdone[i & 1], static_cast<uint32_t>((i >> 1) & 1), &sm.abort, p.status))) break;
      tc_fence_after();
      // B stage i & 1 is free again: prefetch tile i+2 into it
      if (tid == 0 && i + 2 < ntile) issue_b(i + 2);
      const uint32_t acc = tbase + lane + 256u * static_cast<uint32_t>(i & 1);
      // 256 features = 256 / E values of a (from a0 = 256 ii / E), E values of b each
#pragma unroll
      for (int c0 = 0; c0 < 256; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(acc + c0, r);
        tmem_wait_ld();
#pragma unroll
        for (int part = 0; part < 32 / E; ++part) {
          const int col = c0 + part * E;
          const int a = (256 * ii + col) / E;
          float sacc = 0.f;
#pragma unroll
          for (int j = 0; j < E; ++j) sacc = fmaf(__uint_as_float(r[part * E + j]), xg[j], sacc);
          sm.dxs[a][tid] = sacc;  // each a of the group is one tile's: written exactly once
        }
      }
      tc_fence_before();
      __syncthreads();  // the accumulator buffer i & 1 is read: tile i+2's MMAs may overwrite it
    }
    if (ok && tin) {  // the group's E values: one read-modify-write of E contiguous floats
      float4* d4 = reinterpret_cast<float4*>(dxrow + g * E);
      float4 v[E / 4];
#pragma unroll
      for (int c = 0; c < E / 4; ++c) v[c] = d4[c];
#pragma unroll
      for (int c = 0; c < E / 4; ++c) {
        v[c].x = fmaf(p.factor, sm.dxs[4 * c][tid], v[c].x);
        v[c].y = fmaf(p.factor, sm.dxs[4 * c + 1][tid], v[c].y);
        v[c].z = fmaf(p.factor, sm.dxs[4 * c + 2][tid], v[c].z);
        v[c].w = fmaf(p.factor, sm.dxs[4 * c + 3][tid], v[c].w);
        d4[c] = v[c];
      }
    }
  }
  if (!ok && tid == 0) {
    mbar_drain(&sm.mdone[0], 0), mbar_drain(&sm.mdone[0], 1);
    mbar_drain(&sm.mdone[1], 0), mbar_drain(&sm.mdone[1], 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, 512);
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

template <typename K>
int launch_cfg(K kernel, size_t smem) {
  return from_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
}

template <typename T, int E, bool SUM, int NW>
int state_launch(const Params& p, const CUtensorMap& tmW, cudaStream_t st) {
  using L = StateSmem<T, E, SUM, NW>;
  auto k = sp_state_kernel<T, E, SUM, NW>;
  const size_t smem = sizeof(L) + 1024;
  int e = launch_cfg(k, smem);
  if (e) return e;
  k<<<dim3(p.F / 128, p.B * p.H * p.G), 128, smem, st>>>(tmW, p);
  return from_cuda(cudaGetLastError());
}
template <typename T, int E, int D, int NW>
int apply_launch(const Params& p, const CUtensorMap& tmP, cudaStream_t st) {
  auto k = sp_apply_kernel<T, E, D, NW>;
  const size_t smem = sizeof(ApplySmem<NW>) + 1024;
  int e = launch_cfg(k, smem);
  if (e) return e;
  k<<<dim3((p.T + 127) / 128, p.B * p.H), 128, smem, st>>>(tmP, p);
  return from_cuda(cudaGetLastError());
}
template <typename T, int E, int D, int NW>
int grad_launch(const Params& p, const CUtensorMap& tmW, const CUtensorMap& tmP, cudaStream_t st) {
  auto k = sp_grad_kernel<T, E, D, NW>;
  const size_t smem = sizeof(GradSmem<NW>) + 1024;
  int e = launch_cfg(k, smem);
  if (e) return e;
  k<<<dim3((p.T + 127) / 128, p.B * p.H), 128, smem, st>>>(tmW, tmP, p);
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

template <typename T>
int state_dispatch(const Params& p, const CUtensorMap& tmW, bool sum, cudaStream_t st) {
  const int E = p.D / p.M, nw = nw_of(p.ldw);
  if (sum) {
    if (E == 16) return nw == 80 ? state_launch<T, 16, true, 80>(p, tmW, st) : state_launch<T, 16, true, 144>(p, tmW, st);
    return nw == 80 ? state_launch<T, 32, true, 80>(p, tmW, st) : state_launch<T, 32, true, 144>(p, tmW, st);
  }
  if (E == 16) return nw == 80 ? state_launch<T, 16, false, 80>(p, tmW, st) : state_launch<T, 16, false, 144>(p, tmW, st);
  return nw == 80 ? state_launch<T, 32, false, 80>(p, tmW, st) : state_launch<T, 32, false, 144>(p, tmW, st);
}
template <typename T>
int apply_dispatch(const Params& p, const CUtensorMap& tmP, cudaStream_t st) {
  const int E = p.D / p.M, nw = nw_of(p.ldw);
  if (p.D == 64) {
    if (E == 16) return nw == 80 ? apply_launch<T, 16, 64, 80>(p, tmP, st) : apply_launch<T, 16, 64, 144>(p, tmP, st);
    return nw == 80 ? apply_launch<T, 32, 64, 80>(p, tmP, st) : apply_launch<T, 32, 64, 144>(p, tmP, st);
  }
  if (E == 16) return nw == 80 ? apply_launch<T, 16, 128, 80>(p, tmP, st) : apply_launch<T, 16, 128, 144>(p, tmP, st);
  return nw == 80 ? apply_launch<T, 32, 128, 80>(p, tmP, st) : apply_launch<T, 32, 128, 144>(p, tmP, st);
}
template <typename T>
int grad_dispatch(const Params& p, const CUtensorMap& tmW, const CUtensorMap& tmP, cudaStream_t st) {
  const int E = p.D / p.M, nw = nw_of(p.ldw);
  if (p.D == 64) {
    if (E == 16) return nw == 80 ? grad_launch<T, 16, 64, 80>(p, tmW, tmP, st) : grad_launch<T, 16, 64, 144>(p, tmW, tmP, st);
    return nw == 80 ? grad_launch<T, 32, 64, 80>(p, tmW, tmP, st) : grad_launch<T, 32, 64, 144>(p, tmW, tmP, st);
  }
  if (E == 16) return nw == 80 ? grad_launch<T, 16, 128, 80>(p, tmW, tmP, st) : grad_launch<T, 16, 128, 144>(p, tmW, tmP, st);
  return nw == 80 ? grad_launch<T, 32, 128, 80>(p, tmW, tmP, st) : grad_launch<T, 32, 128, 144>(p, tmW, tmP, st);
}

bool al16(const void* x) { return (reinterpret_cast<uintptr_t>(x) & 15u) == 0; }

}  // namespace
}  // namespace sptc
}  // namespace kata

using namespace kata;

extern "C" int kata_sp_state(const void* x, const void* W, float* S, int dtype, int B, int T, int H, int G, int D,
                             int M, int score, int ldw, float scale, int trans, int lds, kata_stream_t stream) {
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
  CUtensorMap tmW;
  int e = map_w(&tmW, W, B * H * G, T, ldw, 64);
  if (e) return e;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return dtype == KATA_DTYPE_BF16 ? state_dispatch<__nv_bfloat16>(p, tmW, sum, st) : state_dispatch<__half>(p, tmW, sum, st);
}

extern "C" int kata_sp_apply(const void* x, const void* P, float* Y, int dtype, int B, int T, int H, int G, int D,
                             int M, int ldw, float scale, int dv_mode, int Dv, kata_stream_t stream) {
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
                            int D, int M, int ldw, float factor, kata_stream_t stream) {
  using namespace sptc;
  if (!x || !P || !W || !dx) return KATA_ERR_INVALID;
  if (dtype != KATA_DTYPE_BF16 && dtype != KATA_DTYPE_F16) return KATA_ERR_DTYPE;
  if (B < 1 || T < 1 || H < 1 || !shape_ok(D, M, ldw, false)) return KATA_ERR_SHAPE;
  if ((M * (D / M) * (D / M)) % 256) return KATA_ERR_SHAPE;
  if (!al16(x) || !al16(P) || !al16(W) || !al16(dx)) return KATA_ERR_ALIGN;
  const int E = D / M;
  Params p{};
  p.x = x;
  p.dx = dx;
  p.B = B;
  p.T = T;
  p.H = H;
  p.D = D;
  p.M = M;
  p.F = M * E * E;
  p.ldw = ldw;
  p.G = 1;
  p.factor = factor;
  CUtensorMap tmW, tmP;
  int e = map_w(&tmW, W, B * H, T, ldw, 128);
  if (!e) e = map_p(&tmP, P, B * H, ldw, p.F, nw_of(ldw));
  if (e) return e;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return dtype == KATA_DTYPE_BF16 ? grad_dispatch<__nv_bfloat16>(p, tmW, tmP, st)
                                  : grad_dispatch<__half>(p, tmW, tmP, st);
}
