// attn_tc_bwd.cu -- tcgen05 tensor-core backward of causal KATA-SPD attention (bf16 / fp16).
//
// Math (kata/parallel_kata_attn.py:49-146 concat, :579-653 sum; decay as autograd of :291-310):
//   S_p = <q_a, k_b>,  A = scale^2 sum_p S_p^2 * dec,  P = A / den,  delta_t = <o_t, dO_t>
//   dA[t,s]  = (dO_t . v_s - delta_t) / den_t                       (causal)
//   W_p[t,s] = 2 scale^2 S_p[t,s] dec[t,s] dA[t,s]   (= d(loss)/d(q_a.k_b))
//   dq_a = sum_b W_(a,b) k_b,  dk_b = sum_a W_(a,b)^T q_a,  dv = P^T dO
//   dc_t = sum_s G[t,s] - sum_t' G[t',t],  G = dA * A on pairs with c_t - c_s <= 0
//
// Two kernels, each warp-specialised like the forward (warp 0 TMA, warp 1 TMEM owner and MMA
// issuer, warps 2..9 two compute warpgroups splitting the 128 columns of every score tile):
//   dq kernel   one CTA per (query tile, batch*query head).  dN = dO V^T and the score parts pass
//               through a 3-slot TMEM ring, dQ accumulates at columns 384..; W_p goes back into
//               its slot as the TMEM operand of the dQ chains, which a second issuer warp (warp 10)
//               issues.  Prologue computes delta and writes delta and the per-query vectors for the
//               second kernel; with decay it also writes dc_t = sum_s G[t,s].
//   dkdv kernel one CTA per (key tile, batch*kv head) looping over the query tiles of every query
//               head of its GQA group.  dN^T and the transposed score parts pass through a 2-slot
//               TMEM ring, dK and dV accumulate at columns 256.. and 384..; W^T_p and, for the last
//               part, P^T go back into the slot as the TMEM operands of dK += W^T Q and
//               dV += P^T dO (Q, dO read MN-major); with decay it atomically subtracts
//               sum_t G[t,s] from dc.
// Every mbarrier wait is bounded; named barriers are only used outside the main loops so that an
// aborting warp never strands the others.
#include "attn_tc_common.cuh"

namespace kata {
namespace {

constexpr int kThreads = 320;
constexpr int kComputeWarp0 = 2;
// The dq ring kernel adds an eleventh warp that issues the dQ chains; warp 10 runs on the third
// scheduler (warp % 4 == 2), apart from the score issuer (warp 1).  (The dk/dv ring kernel keeps
// one issuer: with only two TMEM slots, a second issuer's chain would have to complete before the
// slot could be refilled, where a single issuer may queue the refill behind it in order.)
constexpr int kThreadsRing = 352;
constexpr int kChainWarp = 10;

struct BwdWs {
  // workspace views (fp32), each 16-byte aligned:
  //   delta (B,T,HQ) | rden (B,HQ,Tp) | delta*rden (B,HQ,Tp) [| c (B,HQ,Tp), decay only]
  // with Tp = T rounded up to 128, so that the 128 values of every tile are one contiguous,
  // in-bounds, 512-byte run that a bulk copy can move into shared memory (rows past T hold
  // rden = 1, delta*rden = 0, c = 0).  The head-major copy of the decay cumsum c lets both kernels
  // stage a tile's 128 values with one bulk copy instead of 128 strided loads per thread.
  float* delta;
  float* rden;
  float* dr;
  float* cT;
  int Tp;
};
// With packed documents (nseq > 0) the head-major vectors are indexed by tile number * 128 + row
// (Tp covers the tile bound), so every tile's 128 values stay one aligned run.
__host__ __device__ inline BwdWs ws_views(float* base, int B, int T, int HQ, int nseq = 0) {
  const int Tp = nseq > 0 ? varlen_tile_bound(T, nseq) * 128 : (T + 127) & ~127;
  const size_t n0 = (static_cast<size_t>(B) * T * HQ + 3) & ~static_cast<size_t>(3);
  const size_t n1 = static_cast<size_t>(B) * HQ * Tp;
  return BwdWs{base, base + n0, base + n0 + n1, base + n0 + 2 * n1, Tp};
}

template <int D, int DV>
struct BwdSmem {
  static constexpr int Q_BYTES = kTile * D * 2;
  static constexpr int O_BYTES = kTile * DV * 2;
  static constexpr int ITEM = Q_BYTES > O_BYTES ? Q_BYTES : O_BYTES;
  // dq kernel: Q, dO resident; a ring of four K/V tiles (two key tiles)
  static constexpr int DQ_OFF_Q = 0;
  static constexpr int DQ_OFF_O = DQ_OFF_Q + Q_BYTES;
  static constexpr int DQ_OFF_RING = DQ_OFF_O + O_BYTES;
  static constexpr int DQ_OFF_C = DQ_OFF_RING + 4 * ITEM;  // decay only: c of the key tile in ring slot r
  static constexpr int DQ_OFF_F = DQ_OFF_C + 4 * kTile * 4;  // decay only: per-compute-warp column factors
  static constexpr int dqr_total(bool decay) { return DQ_OFF_C + (decay ? 4 * kTile * 4 + 8 * 64 * 4 : 0); }
  // dkdv kernel: K, V resident; a ring of four dO/Q tiles (two query tiles); the W / P operands
  // stay in tensor memory
  static constexpr int KV_OFF_K = 0;
  static constexpr int KV_OFF_V = KV_OFF_K + Q_BYTES;
  static constexpr int KV_OFF_RING = KV_OFF_V + O_BYTES;
  static constexpr int KR_RING = 4;
  static constexpr int KR_OFF_RING = KV_OFF_RING;
  static constexpr int KR_OFF_VEC = KR_OFF_RING + KR_RING * ITEM;
  // [stage][v0, v1 (, c with decay)][128]; the barrier block follows the vectors
  static constexpr int kr_nvec(bool decay) { return decay ? 3 : 2; }
  static constexpr int kr_off_bars(bool decay) { return KR_OFF_VEC + 2 * kr_nvec(decay) * kTile * 4; }
  static constexpr int kr_total(bool decay) { return kr_off_bars(decay) + 256; }
};

struct DkvRingBars {
  uint64_t kv_full;
  uint64_t vec_full[2], vec_empty[2];
  uint64_t ring_full[4], ring_empty[4];
  uint64_t i_full[3], i_free[3];
  uint64_t acc_done, drain;
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ float2 u2f2(uint32_t a, uint32_t b) { return make_float2(__uint_as_float(a), __uint_as_float(b)); }

// bf16 pair <-> float2 for values kept in registers between the items of one tile
__device__ __forceinline__ uint32_t bf2_pack(float2 v) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(v.x, v.y);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ float2 bf2_unpack(uint32_t u) {
  return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
}
// Packed bf16 product (round to nearest even), one instruction for two elements.
__device__ __forceinline__ uint32_t bf2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Head-major copy of the decay cumsum: cT[(b*HQ + hq)*Tp + t] = c[(b*T + t)*HQ + hq], 0 past T.
__global__ void decay_c_transpose(const float* __restrict__ c, float* __restrict__ cT, int B, int T, int HQ, int Tp) {
  const size_t n = static_cast<size_t>(B) * Tp * HQ;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int hq = static_cast<int>(i % HQ);
    const size_t bt = i / HQ;
    const int t = static_cast<int>(bt % Tp), b = static_cast<int>(bt / Tp);
    cT[(static_cast<size_t>(b) * HQ + hq) * Tp + t] = t < T ? c[(static_cast<size_t>(b) * T + t) * HQ + hq] : 0.f;
  }
}

// The same copy for packed documents (B == 1): indexed by tile number (documents cut into their own
// 128-row tiles, numbered in document order), rows past a document's end 0.  One CTA of 128
// threads per tile, one row per thread.
__global__ void __launch_bounds__(128) decay_c_transpose_var(const float* __restrict__ c, float* __restrict__ cT,
                                                             int T, int HQ, int Tp, const int* __restrict__ cu,
                                                             int nseq) {
  __shared__ SeqTile seq;
  if (threadIdx.x < 32) {
    SeqTile st{};
    const bool have = varlen_tile(cu, nseq, T, static_cast<int>(blockIdx.x), st);
    if (threadIdx.x == 0) seq = have ? st : SeqTile{0, 0, -1, 0, 0};
  }
  __syncthreads();
  if (seq.j < 0) return;
  const int t = seq.start + seq.j * kTile + static_cast<int>(threadIdx.x);
  const size_t col = static_cast<size_t>(blockIdx.x) * kTile + threadIdx.x;
  for (int hq = 0; hq < HQ; ++hq) cT[static_cast<size_t>(hq) * Tp + col] = t < seq.end ? c[static_cast<size_t>(t) * HQ + hq] : 0.f;
}

// ================================================================================================
// dq kernel (tensor-memory ring)
// ================================================================================================
// TMEM: a ring of three 128-column slots that the items of every key tile pass through in order
// -- dN = dO V^T, then the score parts S_0..S_{NP-1} -- and dQ at columns 384..511.  The compute
// warps read dN once per tile and keep dA' = 2 scale^2 (dN - delta)/den (masked) in registers, so
// the dN slot is handed back at once; each S_p slot is overwritten in place by W_p = S_p dA' (bf16
// pairs), which the dQ chain reads as its A operand.  Two issuers on different schedulers: the
// score issuer (warp 1) issues dN and the score parts; the chain issuer (warp 10) waits for the
// compute warps to release each slot, issues the dQ chain of the W it holds, and signals w_done,
// after which the score issuer may refill the slot.  One thread's MMAs run in issue order, so the
// dQ accumulation order is that of the single-issuer form.  Score MMAs run up to two items ahead.
constexpr int kRingDQ = 4;  // K/V ring depth of the dq ring kernel (two key tiles in flight)

struct DqRingBars {
  uint64_t qo_full;
  uint64_t ring_full[kRingDQ], ring_empty[kRingDQ];
  uint64_t i_full[3], i_free[3], w_done[3];
  uint64_t acc_done, drain, drain2;
  uint32_t tmem_base;
  int abort_flag;
  float xch_delta[2][kTile];  // halves of delta_t; with decay, at the end, halves of the dc row sums
};

template <typename T, int D, int DV, int M, bool SUM, bool DECAY, bool GRAM, bool VAR>
__global__ void __launch_bounds__(kThreadsRing, 1)
    attn_bwd_dq_ring_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                        AttnBwdParams p) {
  constexpr int E = D / M;
  constexpr int CW = ScoreBoxW<E, GRAM>::value;
  constexpr int NBOX = D / CW;
  constexpr int VCW = BoxW<DV>::value;
  constexpr int NVBOX = DV / VCW;
  constexpr int NP = SUM ? M * M : M;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  static_assert(!GRAM || (M == 1 && !SUM && !DECAY), "Gram features: one linear score part");
  // Gram features: dQ (= d phi(q), kGramFP columns) does not fit beside three slots, and the linear
  // score needs no S here (d phi(q) = dA phi(K)), so the ring has two slots of dN items only, each
  // overwritten in place by dA' as the TMEM operand of its dQ chain.
  constexpr int NS = GRAM ? 2 : 3;  // TMEM ring slots
  constexpr uint32_t kColDQ = GRAM ? 256 : 384;
  constexpr int kItems = GRAM ? 1 : 1 + NP;  // items per key tile: dN, then S_0..S_{NP-1}
  constexpr int NPL = GRAM ? 0 : NP;         // score parts the compute warps read
  using L = BwdSmem<D, DV>;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ DqRingBars bars;
  __shared__ SeqTile seq;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int T_ = p.T;
  const int bh = blockIdx.y, hq = bh % p.HQ, h = hq / p.G;
  // query tile qi of a sequence with rows [kbase, t_end) of batch b (packed documents: the tile's
  // document, B == 1; past the last tile the CTA exits before it allocates anything); vt0 = the
  // tile's first row in the head-major per-query vectors
  int qi, b, kbase, t_end, vt0;
  if constexpr (VAR) {
    if (warp == 0) {
      SeqTile st{};
      const bool have = varlen_tile(p.cu, p.nseq, T_, static_cast<int>(blockIdx.x), st);
      if (lane == 0) seq = have ? st : SeqTile{0, 0, -1, 0, 0};
    }
    __syncthreads();
    if (seq.j < 0) return;
    qi = seq.j;
    b = 0;
    kbase = seq.start;
    t_end = seq.end;
    vt0 = (seq.base + seq.j) * kTile;
  } else {
    qi = (T_ + kTile - 1) / kTile - 1 - static_cast<int>(blockIdx.x);
    b = bh / p.HQ;
    kbase = 0;
    t_end = T_;
    vt0 = qi * kTile;
  }
  const int t0 = kbase + qi * kTile;
  const int nk = qi + 1;
  WaitCtx wc{p.status, &bars.abort_flag};

  if (threadIdx.x == 0) {
    bars.abort_flag = 0;
    mbar_init(&bars.qo_full, 1);
    for (int i = 0; i < kRingDQ; ++i) {
      mbar_init(&bars.ring_full[i], 1);
      mbar_init(&bars.ring_empty[i], 1);
    }
    for (int i = 0; i < 3; ++i) {
      mbar_init(&bars.i_full[i], 1);
      mbar_init(&bars.i_free[i], 8);
    }
    for (int i = 0; i < 3; ++i) mbar_init(&bars.w_done[i], 1);
    mbar_init(&bars.acc_done, 1);
    mbar_init(&bars.drain, 1);
    mbar_init(&bars.drain2, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars.tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmO);
      mbar_arrive_expect_tx(&bars.qo_full, L::Q_BYTES + L::O_BYTES);
      for (int bx = 0; bx < NBOX; ++bx)
        tma_load_4d(smem + L::DQ_OFF_Q + bx * (kTile * CW * 2), &tmQ, &bars.qo_full, bx * CW, hq, t0, b);
      for (int bx = 0; bx < NVBOX; ++bx)
        tma_load_4d(smem + L::DQ_OFF_O + bx * (kTile * VCW * 2), &tmO, &bars.qo_full, bx * VCW, hq, t0, b);
      int r = 0;
      bool ok = true;
      for (int j = 0; j < nk && ok; ++j) {
        for (int item = 0; item < 2; ++item, ++r) {  // V_j then K_j
          const int slot = r % kRingDQ;
          if (!mbar_wait(&bars.ring_empty[slot], ((r / kRingDQ) & 1) ^ 1, wc)) {
            ok = false;
            break;
          }
          uint8_t* dst = smem + L::DQ_OFF_RING + slot * L::ITEM;
          if (item == 0) {
            mbar_arrive_expect_tx(&bars.ring_full[slot], L::O_BYTES);
            for (int bx = 0; bx < NVBOX; ++bx)
              tma_load_4d(dst + bx * (kTile * VCW * 2), &tmV, &bars.ring_full[slot], bx * VCW, h, kbase + j * kTile, b);
          } else {
            // with decay, the key tile's c (head-major copy) rides with K_j, whose slot is held
            // until the tile's last dQ chain, i.e. after the compute warps have read it
            mbar_arrive_expect_tx(&bars.ring_full[slot], L::Q_BYTES + (DECAY ? kTile * 4 : 0));
            for (int bx = 0; bx < NBOX; ++bx)
              tma_load_4d(dst + bx * (kTile * CW * 2), &tmK, &bars.ring_full[slot], bx * CW, h, kbase + j * kTile, b);
            if (DECAY && !VAR)
              bulk_load(smem + L::DQ_OFF_C + slot * (kTile * 4),
                        ws_views(p.delta, p.B, T_, p.HQ).cT + (static_cast<size_t>(b) * p.HQ + hq) *
                            static_cast<size_t>((T_ + 127) & ~127) + static_cast<size_t>(j) * kTile,
                        kTile * 4, &bars.ring_full[slot]);
            if constexpr (DECAY && VAR) {  // packed documents: the copy of c is indexed by tile number
              const BwdWs wv = ws_views(p.delta, p.B, T_, p.HQ, p.nseq);
              bulk_load(smem + L::DQ_OFF_C + slot * (kTile * 4),
                        wv.cT + static_cast<size_t>(hq) * wv.Tp + static_cast<size_t>(seq.base + j) * kTile,
                        kTile * 4, &bars.ring_full[slot]);
            }
          }
        }
      }
      if (!ok) {
        for (int rr = (r > kRingDQ ? r - kRingDQ : 0); rr < r; ++rr)
          mbar_drain(&bars.ring_full[rr % kRingDQ], (rr / kRingDQ) & 1);
      }
    }
  } else if (warp == 1) {
    {  // warp-wide issue (every lane runs the loop; one elected lane issues)
      // Score issuer: dN and the score parts.  Item `it` = j * kItems + q lives in slot it % NS; the
      // slot is reused once the chain warp has released the item NS back (w_done: its dQ chain,
      // if any, has completed).  The ring holds V_j at position 2j and K_j at 2j + 1 (kRingDQ = 4:
      // slot (2j + c) & 3, use parity (j >> 1) & 1).
      const uint32_t id_nn = umma_idesc_f16(128, 128, kBF16, false, false);
      const uint32_t sRing = smem_u32(smem + L::DQ_OFF_RING);
      // Descriptor bases; every operand below is a compile-time or ring-slot-multiple offset from
      // one of these (no descriptor is rebuilt inside the loops).
      const uint64_t od0 = kmajor_desc<VCW>(smem_u32(smem + L::DQ_OFF_O), 0, DV, 0);  // dO, K-major
      const uint64_t qd0 = kmajor_desc<CW>(smem_u32(smem + L::DQ_OFF_Q), 0, E, 0);    // Q, K-major
      const uint64_t rv0 = kmajor_desc<VCW>(sRing, 0, DV, 0);  // V in ring slot 0, K-major
      const uint64_t rk0 = kmajor_desc<CW>(sRing, 0, E, 0);    // K in ring slot 0, K-major
      static_assert(kRingDQ == 4, "ring positions below assume four slots");
      bool ok = mbar_wait_w_inl(&bars.qo_full, 0, wc);
      int it = 0, x = 0;       // x = it % NS
      uint32_t use_par = 0;    // parity of (it / NS), i.e. of the current use of slot x
      for (int j = 0; ok && j < nk; ++j) {
        const uint32_t ring_par = static_cast<uint32_t>(j >> 1) & 1u;
#pragma unroll
        for (int q = 0; q < kItems; ++q) {
          if (it >= NS && !mbar_wait_w_inl(&bars.w_done[x], use_par ^ 1, wc)) {
            ok = false;
            break;
          }
          const uint32_t sd = tbase + static_cast<uint32_t>(x) * 128u;
          if (q == 0) {  // dN = dO V_j^T
            const int slotV = (2 * j) & 3;
            if (!mbar_wait_w_inl(&bars.ring_full[slotV], ring_par, wc)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t vd = rv0 + desc_units(static_cast<uint32_t>(slotV) * L::ITEM);
#pragma unroll
            for (int kk = 0; kk < DV / 16; ++kk)
              umma_ss_w(sd, od0 + kstep<VCW>(kk), vd + kstep<VCW>(kk), id_nn, kk > 0 ? 1u : 0u);
            umma_commit_w(&bars.i_full[x]);
            umma_commit_w(&bars.ring_empty[slotV]);
            if (!GRAM && !mbar_wait_w_inl(&bars.ring_full[(2 * j + 1) & 3], ring_par, wc)) {  // K_j
              ok = false;
              break;
            }
          } else {  // S_p = Q_a K_b^T
            const int pp = q - 1;
            const int ga = SUM ? pp / M : pp, gb = SUM ? pp % M : pp;
            const int slotK = (2 * j + 1) & 3;
            tc_fence_after();
            const uint64_t qd = qd0 + kmajor_goff<CW>(ga, E);
            const uint64_t kd = rk0 + desc_units(static_cast<uint32_t>(slotK) * L::ITEM) + kmajor_goff<CW>(gb, E);
#pragma unroll
            for (int kk = 0; kk < E / 16; ++kk)
              umma_ss_w(sd, qd + kstep<CW>(kk), kd + kstep<CW>(kk), id_nn, kk > 0 ? 1u : 0u);
            umma_commit_w(&bars.i_full[x]);
          }
          ++it;
          if (++x == NS) {
            x = 0;
            use_par ^= 1;
          }
        }
      }
      umma_commit_w(&bars.drain);
      mbar_drain(&bars.drain, 0);
    }
  } else if (warp == kChainWarp) {
    {  // warp-wide issue (every lane runs the loop; one elected lane issues)
      // Chain issuer (a scheduler of its own, so its issue stream does not queue behind the score
      // issuer's): for every item in order, once the compute warps release the slot, the dQ chain
      // of the W it holds (score parts), then w_done for the score issuer.  All dQ MMAs come from
      // this thread, so they execute in order; the K tile of key tile j is released after its
      // last chain.
      const uint32_t id_dq = umma_idesc_f16(128, E, kBF16, false, true);
      const uint64_t rkm0 = mnmajor_desc<CW>(smem_u32(smem + L::DQ_OFF_RING), 0, 0);  // K in ring slot 0, MN-major
      bool ok = true;
      int x = 0;
      uint32_t use_par = 0;
      for (int j = 0; ok && j < nk; ++j) {
#pragma unroll
        for (int q = 0; q < kItems; ++q) {
          if (!mbar_wait_w_inl(&bars.i_free[x], use_par, wc)) {
            ok = false;
            break;
          }
          if (GRAM) {  // dQ += dA' phi(K_j): the K tile's first and only use
            const int kslot = (2 * j + 1) & 3;
            if (!mbar_wait_w_inl(&bars.ring_full[kslot], static_cast<uint32_t>(j >> 1) & 1u, wc)) {
              ok = false;
              break;
            }
            const uint64_t kd = rkm0 + desc_units(static_cast<uint32_t>(kslot) * L::ITEM);
            const uint32_t wa = tbase + static_cast<uint32_t>(x) * 128u;
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < kTile / 16; ++kk)
              umma_ts_w(tbase + kColDQ, wa + packed_col(kk), kd + mnstep<CW>(kk), id_dq, (j > 0 || kk > 0) ? 1u : 0u);
            umma_commit_w(&bars.ring_empty[kslot]);
          } else if (q > 0) {
            const int pp = q - 1;
            const int ga = SUM ? pp / M : pp, gb = SUM ? pp % M : pp;
            const bool first = (j == 0) && (!SUM || gb == 0);
            const int kslot = (2 * j + 1) & 3;
            const uint64_t kd = rkm0 + desc_units(static_cast<uint32_t>(kslot) * L::ITEM) + mnmajor_boff<CW>(gb * E / CW);
            const uint32_t wa = tbase + static_cast<uint32_t>(x) * 128u;
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < kTile / 16; ++kk)
              umma_ts_w(tbase + kColDQ + ga * E, wa + packed_col(kk), kd + mnstep<CW>(kk), id_dq,
                      (!first || kk > 0) ? 1u : 0u);
            if (pp == NP - 1) umma_commit_w(&bars.ring_empty[kslot]);  // K tile no longer needed
          }
          umma_commit_w(&bars.w_done[x]);
          if (++x == NS) {
            x = 0;
            use_par ^= 1;
          }
        }
      }
      if (ok) umma_commit_w(&bars.acc_done);
      umma_commit_w(&bars.drain2);
      mbar_drain(&bars.drain2, 0);
    }
  } else {
    const int cw = warp - kComputeWarp0;
    const int hc = cw >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int tg = t0 + row;
    const bool live = tg < t_end;
    const uint32_t lane_addr = tbase + (static_cast<uint32_t>(quarter * 32) << 16);
    const size_t rowidx = (static_cast<size_t>(b) * T_ + tg) * p.HQ + hq;  // (b, tg, hq)
    const BwdWs ws = ws_views(p.delta, p.B, T_, p.HQ, VAR ? p.nseq : 0);
    // ---- delta_t = <o_t, dO_t> over this thread's half of Dv, then exchanged
    float dpart = 0.f;
    if (live && p.delta_in) {
      dpart = hc == 0 ? p.delta_in[rowidx] : 0.f;
    } else if (live) {
      constexpr int HV = DV / 2;
      const T* orow = static_cast<const T*>(p.o) + rowidx * DV + hc * HV;
      const T* grow = static_cast<const T*>(p.dout) + rowidx * DV + hc * HV;
#pragma unroll
      for (int c8 = 0; c8 < HV; c8 += 8) {
        const uint4 a = *reinterpret_cast<const uint4*>(orow + c8);
        const uint4 g = *reinterpret_cast<const uint4*>(grow + c8);
        const T* ah = reinterpret_cast<const T*>(&a);
        const T* gh = reinterpret_cast<const T*>(&g);
#pragma unroll
        for (int e = 0; e < 8; ++e) dpart = fmaf(to_f32<T>(ah[e]), to_f32<T>(gh[e]), dpart);
      }
    }
    bars.xch_delta[hc][row] = dpart;
    named_bar_sync(1, 256);
    const float delta = bars.xch_delta[0][row] + bars.xch_delta[1][row];
    float rden = 1.f;
    if (live) {
      const float dn = p.den[rowidx];
      rden = 1.f / (dn > 0.f ? dn : 1.f);
      if (hc == 0) ws.delta[rowidx] = delta;
    }
    if (hc == 0) {  // every row of the tile, including rows past T (rden 1, delta 0)
      // For the ring dk/dv kernel, pre-scaled: scale^2 / den and -scale^2 delta / den, so that
      // there P^T = sum S^2 * v0 and dA''^T = dN * v0 + v1 are one packed op each (dK is doubled
      // in its epilogue: W = 2 S dA'').  Rows past a packed document's end hold the next
      // document's tokens (not zeros as past T), so their v0 is 0 as well: no P, no dA.
      const size_t hm = (static_cast<size_t>(b) * p.HQ + hq) * ws.Tp + vt0 + row;  // head-major (b, hq, t)
      const float scale2 = p.scale * p.scale;
      ws.rden[hm] = live || !VAR ? rden * scale2 : 0.f;
      ws.dr[hm] = live ? -delta * rden * scale2 : 0.f;
    }
    const float w_scale = GRAM ? 1.f : 2.f * p.scale * p.scale;  // Gram: W = dA (linear score)
    const float2 rden_w = make_float2(rden * w_scale, rden * w_scale);
    const float2 ndr_w = make_float2(-delta * rden * w_scale, -delta * rden * w_scale);
    // decay: e(t,s) = exp(min(c_t - c_s, 0)) is folded into dA' once per key tile; the dc row sum
    // R_t = sum_s (dN - delta) rden A_ts over pairs with c_t - c_s <= 0 is 0.5 sum_s dA'_dec S^2
    float c_t = 0.f;
    const float* cb = nullptr;
    if (DECAY) {
      cb = p.c + static_cast<size_t>(b) * T_ * p.HQ + hq;
      c_t = live ? cb[static_cast<size_t>(tg) * p.HQ] : 0.f;
    }
    float2 r2 = make_float2(0.f, 0.f);
    bool ok = true;
    int it = 0;
    for (int j = 0; j < nk && ok; ++j) {
      const bool diag = (j == qi);
      float2 da[32];  // dA' of this thread's 64 key columns
      uint32_t cm[2] = {0u, 0u};  // decay: columns with c_t - c_s > 0 (no dc contribution)
      {
        const int x = static_cast<int>(static_cast<unsigned>(it) % NS);  // it >= 0
        if (!mbar_wait(&bars.i_full[x], (static_cast<unsigned>(it) / NS) & 1u, wc)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t nbase = lane_addr + x * 128u + hc * 64u;
        uint32_t rn[2][16];
        tmem_ld16(nbase, rn[0]);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int cur = c & 1;
          if (c < 3) tmem_ld16(nbase + (c + 1) * 16u, rn[cur ^ 1]);
#pragma unroll
          for (int x2 = 0; x2 < 8; ++x2) da[8 * c + x2] = ffma2(u2f2(rn[cur][2 * x2], rn[cur][2 * x2 + 1]), rden_w, ndr_w);
          if (c < 3) tmem_wait_ld();
        }
        if constexpr (!GRAM) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars.i_free[x]);
        }
        ++it;
        if (diag) {
#pragma unroll
          for (int x2 = 0; x2 < 32; ++x2) {
            const int s0 = hc * 64 + 2 * x2;
            if (s0 > row) da[x2].x = 0.f;
            if (s0 + 1 > row) da[x2].y = 0.f;
          }
        }
        if constexpr (GRAM) {  // dA' back into the slot (packed) as the A operand of the dQ chain
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t wv[8];
#pragma unroll
            for (int x2 = 0; x2 < 8; ++x2) wv[x2] = pack2<T>(da[8 * c + x2].x, da[8 * c + x2].y);
            tmem_st8(nbase + c * 8u, wv);
          }
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars.i_free[x]);
        }
        if (DECAY) {
          // the key tile's c, staged with K_j: wait for that load (the slot is not refilled before
          // the tile's last dQ chain, which follows this warp's release of the tile's parts)
          if (!mbar_wait_w(&bars.ring_full[(2 * j + 1) & 3], static_cast<uint32_t>(j >> 1) & 1u, wc)) {
            ok = false;
            break;
          }
          const float* cs = reinterpret_cast<const float*>(smem + L::DQ_OFF_C + ((2 * j + 1) & 3) * (kTile * 4)) + hc * 64;
          // Factored decay: with lo = min of c over this warp's 64 columns, a row with c_t <= lo has
          // every c_t - c_s <= 0 and e = exp(c_t - lo) * exp(lo - c_s), both factors <= 1 (no
          // overflow; an underflow only flushes values below 1e-38).  The column factors are made
          // once per warp (two per lane) instead of one exponential per element and thread.
          float* fb = reinterpret_cast<float*>(smem + L::DQ_OFF_F) + (warp - kComputeWarp0) * 64;
          const float2 cl = *reinterpret_cast<const float2*>(cs + 2 * lane);
          float lo = fminf(cl.x, cl.y);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
          *reinterpret_cast<float2*>(fb + 2 * lane) = make_float2(__expf(lo - cl.x), __expf(lo - cl.y));
          __syncwarp();
          if (!__any_sync(0xffffffffu, c_t > lo)) {
            const float rt = __expf(c_t - lo);
#pragma unroll
            for (int x4 = 0; x4 < 16; ++x4) {
              const float4 f = *reinterpret_cast<const float4*>(fb + 4 * x4);
              da[2 * x4] = fmul2(da[2 * x4], make_float2(rt * f.x, rt * f.y));
              da[2 * x4 + 1] = fmul2(da[2 * x4 + 1], make_float2(rt * f.z, rt * f.w));
            }
          } else {  // some row of this warp has c_t > c_s somewhere: exponentials per element
#pragma unroll
            for (int x2 = 0; x2 < 32; ++x2) {
              const float2 csv = *reinterpret_cast<const float2*>(cs + 2 * x2);
              const float x0 = c_t - csv.x, x1 = c_t - csv.y;
              da[x2].x *= __expf(fminf(x0, 0.f));
              da[x2].y *= __expf(fminf(x1, 0.f));
              if (x0 > 0.f) cm[x2 >> 4] |= 1u << ((2 * x2) & 31);
              if (x1 > 0.f) cm[x2 >> 4] |= 1u << ((2 * x2 + 1) & 31);
            }
          }
          __syncwarp();  // every lane has read the factors before the next tile rewrites them
        }
      }
      const bool any_clamp = DECAY && (cm[0] | cm[1]) != 0u;
      for (int pp = 0; pp < NPL; ++pp, ++it) {
        const int x = static_cast<int>(static_cast<unsigned>(it) % NS);  // it >= 0
        if (!mbar_wait(&bars.i_full[x], (static_cast<unsigned>(it) / NS) & 1u, wc)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sbase = lane_addr + x * 128u + hc * 64u;
        uint32_t rs[2][16];
        tmem_ld16(sbase, rs[0]);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int cur = c & 1;
          if (c < 3) tmem_ld16(sbase + (c + 1) * 16u, rs[cur ^ 1]);
          uint32_t wv[8];
#pragma unroll
          for (int x2 = 0; x2 < 8; ++x2) {
            const float2 sv = u2f2(rs[cur][2 * x2], rs[cur][2 * x2 + 1]);
            const float2 w = fmul2(sv, da[8 * c + x2]);
            wv[x2] = pack2<T>(w.x, w.y);
            if (DECAY) {
              float2 dm = da[8 * c + x2];
              if (any_clamp) {
                const int bit = 16 * c + 2 * x2;
                if (cm[bit >> 5] & (1u << (bit & 31))) dm.x = 0.f;
                if (cm[bit >> 5] & (1u << ((bit + 1) & 31))) dm.y = 0.f;
              }
              r2 = ffma2(fmul2(sv, sv), dm, r2);
            }
          }
          tmem_st8(sbase + c * 8u, wv);  // columns of S already in registers
          if (c < 3) tmem_wait_ld();
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars.i_free[x]);
      }
    }
    // ---- epilogue: dQ -> global; decay: dc_t = R_t (the dk/dv pass adds the column part).  The
    // delta exchange slots are free again: every compute warp read them right after the first named
    // barrier, before it released its first item, and no warp gets past the first three items
    // before all warps have released the first one.
    if (DECAY) bars.xch_delta[hc][row] = 0.5f * (r2.x + r2.y);
    named_bar_sync(1, 256);
    if (DECAY && ok && live && hc == 0) p.dc[rowidx] = bars.xch_delta[0][row] + bars.xch_delta[1][row];
    if (ok && mbar_wait(&bars.acc_done, 0, wc)) {
      tc_fence_after();
      // column halves of dQ: D / 2 each, or 80 + 64 for the kGramFP = 144 Gram columns
      constexpr int HD0 = GRAM ? 80 : D / 2;
      T* dqrow = static_cast<T*>(p.dq) + rowidx * D;
      constexpr int kSteps = (HD0 > D - HD0 ? HD0 : D - HD0) / 16;  // compile-time trip count
      const int cbeg = hc ? HD0 : 0, cend = hc ? D : HD0;
#pragma unroll
      for (int i = 0; i < kSteps; ++i) {
        const int c0 = cbeg + 16 * i;
        if (c0 >= cend) break;  // warp-uniform
        uint32_t r[16];
        tmem_ld16(lane_addr + kColDQ + c0, r);
        tmem_wait_ld();
        if (live) {
#pragma unroll
          for (int v2 = 0; v2 < 2; ++v2) {
            uint4 w;
            w.x = pack2<T>(__uint_as_float(r[8 * v2 + 0]), __uint_as_float(r[8 * v2 + 1]));
            w.y = pack2<T>(__uint_as_float(r[8 * v2 + 2]), __uint_as_float(r[8 * v2 + 3]));
            w.z = pack2<T>(__uint_as_float(r[8 * v2 + 4]), __uint_as_float(r[8 * v2 + 5]));
            w.w = pack2<T>(__uint_as_float(r[8 * v2 + 6]), __uint_as_float(r[8 * v2 + 7]));
            *reinterpret_cast<uint4*>(dqrow + c0 + 8 * v2) = w;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tbase, 512);
}

// ================================================================================================
// dk / dv kernel (tensor-memory ring)
// ================================================================================================
// TMEM: a ring of two 128-column slots that the items of every (key tile, query tile) pair pass
// through in order -- dN^T = V dO^T, then the transposed score parts S^T_0..S^T_{NP-1} (rows: keys)
// -- with dK at columns 256..383 and dV at 384..511.  The compute warps read dN^T once per pair and
// keep dA'^T = 2 scale^2 (dN - delta)/den (masked) in registers as bf16 pairs next to the fp32 sum
// of squared parts; each S^T_p slot is overwritten in place by W^T_p = S^T_p dA'^T (packed bf16,
// columns [0,32) and [64,96) of the slot), and the last part's slot also receives P^T = A/den in the
// other half (columns [32,64) and [96,128)).  The issuer reuses a slot only after the compute warps
// release it, issuing first the dK chain of the W it holds (and, for the last part, the dV chain of
// P) as tensor-memory-operand MMAs; MMAs of one CTA execute in issue order.
template <typename T, int D, int DV, int M, bool SUM, bool DECAY, bool GRAM, bool VAR>
__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_dkdv_ring_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                          AttnBwdParams p) {
  constexpr int E = D / M;
  constexpr int CW = ScoreBoxW<E, GRAM>::value;
  constexpr int NBOX = D / CW;
  constexpr int VCW = BoxW<DV>::value;
  constexpr int NVBOX = DV / VCW;
  constexpr int NP = SUM ? M * M : M;
  constexpr int kItems = 1 + NP;
  constexpr int kR = 4;  // dO / Q ring depth (two query tiles in flight)
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  static_assert(!GRAM || (M == 1 && !SUM && !DECAY && DV <= 64), "Gram features: one linear score part");
  // TMEM: NS 128-column slots for the items, then dK and dV.  At D = Dv = 64 the accumulators take
  // 64 columns each, which leaves room for a third slot (three items in flight); Gram features: dK
  // (= d phi(k)) takes kGramFP = 144 columns from 256, dV the last 64
  constexpr int NS = (!GRAM && D <= 64 && DV <= 64) ? 3 : 2;
  constexpr uint32_t kColDK = NS * 128, kColDV = GRAM ? 448 : (NS == 3 ? 448 : 384);
  static_assert(kColDV + DV <= 512 && kColDK + (GRAM ? kGramFP : D) <= (GRAM ? 448u : kColDV), "TMEM budget");
  using L = BwdSmem<D, DV>;
  static_assert(sizeof(DkvRingBars) <= 256, "barrier block");
  static_assert(L::KR_RING == kR, "ring depth");

  extern __shared__ __align__(1024) uint8_t smem[];
  constexpr int kNV = L::kr_nvec(DECAY);  // per-query vectors per stage
  DkvRingBars& bars = *reinterpret_cast<DkvRingBars*>(smem + L::kr_off_bars(DECAY));
  if ((smem_u32(smem) & 1023u) != 0) {
    if (threadIdx.x == 0 && p.status) atomicCAS(p.status, 0, kStatusWaitTimeout + 1);
    return;
  }

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Packed documents (VAR): the key tile's document (B == 1), in the last bytes of the 256-byte
  // barrier block; the regular kernel never touches it.  Past the last tile the CTA exits before it
  // allocates anything.
  SeqTile& seq = *reinterpret_cast<SeqTile*>(smem + L::kr_off_bars(DECAY) + 256 - sizeof(SeqTile));
  static_assert(sizeof(DkvRingBars) + sizeof(SeqTile) <= 256, "barrier block");
  if constexpr (VAR) {
    if (warp == 0) {
      SeqTile st{};
      const bool have = varlen_tile(p.cu, p.nseq, p.T, static_cast<int>(blockIdx.x), st);
      if (lane == 0) seq = have ? st : SeqTile{0, 0, -1, 0, 0};
    }
    __syncthreads();
    if (seq.j < 0) return;
  }
  const int T_ = p.T;
  const int nqt = (T_ + kTile - 1) / kTile;
  const int kj = VAR ? seq.j : static_cast<int>(blockIdx.x);
  const int bh = blockIdx.y, b = VAR ? 0 : bh / p.H, h = bh % p.H;
  const int s0 = (VAR ? seq.start : 0) + kj * kTile;
  const int nq = (VAR ? seq.ntiles : nqt) - kj;
  const int nwork = p.G * nq;
  const BwdWs ws = ws_views(p.delta, p.B, T_, p.HQ, VAR ? p.nseq : 0);
  WaitCtx wc{p.status, &bars.abort_flag};

  if (threadIdx.x == 0) {
    bars.abort_flag = 0;
    mbar_init(&bars.kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars.vec_full[i], 1);
      mbar_init(&bars.vec_empty[i], 8);
    }
    for (int i = 0; i < NS; ++i) {
      mbar_init(&bars.i_full[i], 1);
      mbar_init(&bars.i_free[i], 8);
    }
    for (int i = 0; i < kR; ++i) {
      mbar_init(&bars.ring_full[i], 1);
      mbar_init(&bars.ring_empty[i], 1);
    }
    mbar_init(&bars.acc_done, 1);
    mbar_init(&bars.drain, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars.tmem_base;
  float* vec = reinterpret_cast<float*>(smem + L::KR_OFF_VEC);  // [stage][0: v0, 1: v1, 2: c (decay)][128]

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmO);
      mbar_arrive_expect_tx(&bars.kv_full, L::Q_BYTES + L::O_BYTES);
      for (int bx = 0; bx < NBOX; ++bx)
        tma_load_4d(smem + L::KV_OFF_K + bx * (kTile * CW * 2), &tmK, &bars.kv_full, bx * CW, h, s0, b);
      for (int bx = 0; bx < NVBOX; ++bx)
        tma_load_4d(smem + L::KV_OFF_V + bx * (kTile * VCW * 2), &tmV, &bars.kv_full, bx * VCW, h, s0, b);
      int r = 0, nv = 0;
      bool ok = true;
      for (int n = 0; n < nwork && ok; ++n) {
        const int hq = h * p.G + n / nq;
        const int ti = (kj + n % nq) * kTile;  // within the sequence (packed: from its first row)
        const int vs = n & 1;
        if (!mbar_wait(&bars.vec_empty[vs], ((n >> 1) & 1) ^ 1, wc)) {
          ok = false;
          break;
        }
        const size_t hm = (static_cast<size_t>(b) * p.HQ + hq) * ws.Tp + ti + (VAR ? seq.base * kTile : 0);
        mbar_arrive_expect_tx(&bars.vec_full[vs], (DECAY ? 3 : 2) * kTile * 4);
        bulk_load(vec + (vs * kNV + 0) * kTile, ws.rden + hm, kTile * 4, &bars.vec_full[vs]);
        bulk_load(vec + (vs * kNV + 1) * kTile, ws.dr + hm, kTile * 4, &bars.vec_full[vs]);
        if (DECAY) bulk_load(vec + (vs * kNV + 2) * kTile, ws.cT + hm, kTile * 4, &bars.vec_full[vs]);
        nv = n + 1;
        for (int item = 0; item < 2; ++item, ++r) {  // dO_n then Q_n (dN is the first MMA of a pair)
          const int slot = r % kR;
          if (!mbar_wait(&bars.ring_empty[slot], ((r / kR) & 1) ^ 1, wc)) {
            ok = false;
            break;
          }
          uint8_t* dst = smem + L::KR_OFF_RING + slot * L::ITEM;
          if (item == 0) {
            mbar_arrive_expect_tx(&bars.ring_full[slot], L::O_BYTES);
            for (int bx = 0; bx < NVBOX; ++bx)
              tma_load_4d(dst + bx * (kTile * VCW * 2), &tmO, &bars.ring_full[slot], bx * VCW, hq,
                          ti + (VAR ? seq.start : 0), b);
          } else {
            mbar_arrive_expect_tx(&bars.ring_full[slot], L::Q_BYTES);
            for (int bx = 0; bx < NBOX; ++bx)
              tma_load_4d(dst + bx * (kTile * CW * 2), &tmQ, &bars.ring_full[slot], bx * CW, hq,
                          ti + (VAR ? seq.start : 0), b);
          }
        }
      }
      if (!ok) {
        for (int rr = (r > kR ? r - kR : 0); rr < r; ++rr) mbar_drain(&bars.ring_full[rr % kR], (rr / kR) & 1);
        for (int n = (nv > 2 ? nv - 2 : 0); n < nv; ++n) mbar_drain(&bars.vec_full[n & 1], (n >> 1) & 1);
      }
    }
  } else if (warp == 1) {
    {  // warp-wide issue (every lane runs the loop; one elected lane issues)
      const uint32_t id_nn = umma_idesc_f16(128, 128, kBF16, false, false);
      const uint32_t id_dk = umma_idesc_f16(128, E, kBF16, false, true);
      const uint32_t id_dv = umma_idesc_f16(128, DV, kBF16, false, true);
      const uint32_t sRing = smem_u32(smem + L::KR_OFF_RING);
      // Descriptor bases; every operand below is a compile-time or ring-slot-multiple offset from
      // one of these (no descriptor is rebuilt inside the loops).
      const uint64_t kd0 = kmajor_desc<CW>(smem_u32(smem + L::KV_OFF_K), 0, E, 0);     // K, K-major
      const uint64_t vd0 = kmajor_desc<VCW>(smem_u32(smem + L::KV_OFF_V), 0, DV, 0);  // V, K-major
      const uint64_t ro0 = kmajor_desc<VCW>(sRing, 0, DV, 0);  // dO in ring slot 0, K-major
      const uint64_t rom0 = mnmajor_desc<VCW>(sRing, 0, 0);    // dO in ring slot 0, MN-major
      const uint64_t rq0 = kmajor_desc<CW>(sRing, 0, E, 0);    // Q in ring slot 0, K-major
      const uint64_t rqm0 = mnmajor_desc<CW>(sRing, 0, 0);     // Q in ring slot 0, MN-major
      bool ok = mbar_wait_w(&bars.kv_full, 0, wc);
      // Item `it` = n * kItems + q lives in slot it % NS; before reuse, the pending chains of item
      // it - NS are issued.  After the last pair, NS claims drain the pending chains.  The ring
      // holds dO_n at position 2n and Q_n at 2n + 1 (kR = 4: slot (2n + c) & 3, use parity
      // (n >> 1) & 1).
      static_assert(kR == 4, "ring positions below assume four slots");
      int it = 0, x = 0;
      uint32_t use_par = 0;
      const int n_claims = nwork * kItems + NS;
      for (int n = 0; ok && it < n_claims; ++n) {
        const int slotO = (2 * n) & 3, slotQ = (2 * n + 1) & 3;
        const uint32_t ring_par = static_cast<uint32_t>(n >> 1) & 1u;
#pragma unroll
        for (int q = 0; q < kItems; ++q) {
          if (it >= n_claims) break;
          if (it >= NS) {
            if (!mbar_wait_w(&bars.i_free[x], use_par ^ 1, wc)) {
              ok = false;
              break;
            }
            // item it - NS: type pq and pair n + pdn, both compile-time offsets of (n, q)
            const int pq = ((q - NS) % kItems + kItems) % kItems;
            const int pdn = (q - NS - pq) / kItems;
            if (pq > 0) {
              const int pn = n + pdn, pp = pq - 1;
              const int ga = SUM ? pp / M : pp, gb = SUM ? pp % M : pp;
              const bool first = (pn == 0) && (!SUM || ga == 0);
              const int psQ = (2 * pn + 1) & 3;
              const uint64_t qd = rqm0 + desc_units(static_cast<uint32_t>(psQ) * L::ITEM) + mnmajor_boff<CW>(ga * E / CW);
              const uint32_t wa = tbase + static_cast<uint32_t>(x) * 128u;
              tc_fence_after();
#pragma unroll
              for (int kk = 0; kk < kTile / 16; ++kk)
                umma_ts_w(tbase + kColDK + gb * E, wa + packed_col(kk), qd + mnstep<CW>(kk), id_dk,
                        (!first || kk > 0) ? 1u : 0u);
              if (pp == NP - 1) {  // dV += P^T dO, then this pair's dO and Q tiles are free
                const int psO = (2 * pn) & 3;
                const uint64_t od = rom0 + desc_units(static_cast<uint32_t>(psO) * L::ITEM);
#pragma unroll
                for (int kk = 0; kk < kTile / 16; ++kk)
                  umma_ts_w(tbase + kColDV, wa + packed_col(kk) + 32u, od + mnstep<VCW>(kk), id_dv,
                          (pn > 0 || kk > 0) ? 1u : 0u);
                umma_commit_w(&bars.ring_empty[psO]);
                umma_commit_w(&bars.ring_empty[psQ]);
              }
            }
          }
          if (n >= nwork) {
            ++it;
            if (++x == NS) { x = 0; use_par ^= 1; }
            continue;
          }
          const uint32_t sd = tbase + static_cast<uint32_t>(x) * 128u;
          if (q == 0) {  // dN^T = V dO_n^T
            if (!mbar_wait_w(&bars.ring_full[slotO], ring_par, wc)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t od = ro0 + desc_units(static_cast<uint32_t>(slotO) * L::ITEM);
#pragma unroll
            for (int kk = 0; kk < DV / 16; ++kk)
              umma_ss_w(sd, vd0 + kstep<VCW>(kk), od + kstep<VCW>(kk), id_nn, kk > 0 ? 1u : 0u);
            umma_commit_w(&bars.i_full[x]);
            if (!mbar_wait_w(&bars.ring_full[slotQ], ring_par, wc)) {  // Q_n for the parts
              ok = false;
              break;
            }
          } else {  // S^T_p = K_b Q_a^T
            const int pp = q - 1;
            const int ga = SUM ? pp / M : pp, gb = SUM ? pp % M : pp;
            tc_fence_after();
            const uint64_t kd = kd0 + kmajor_goff<CW>(gb, E);
            const uint64_t qd = rq0 + desc_units(static_cast<uint32_t>(slotQ) * L::ITEM) + kmajor_goff<CW>(ga, E);
#pragma unroll
            for (int kk = 0; kk < E / 16; ++kk)
              umma_ss_w(sd, kd + kstep<CW>(kk), qd + kstep<CW>(kk), id_nn, kk > 0 ? 1u : 0u);
            umma_commit_w(&bars.i_full[x]);
          }
          ++it;
          if (++x == NS) {
            x = 0;
            use_par ^= 1;
          }
        }
      }
      if (ok) umma_commit_w(&bars.acc_done);
      umma_commit_w(&bars.drain);
      mbar_drain(&bars.drain, 0);
    }
  } else {
    const int cw = warp - kComputeWarp0;
    const int hc = cw >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;  // key row within the tile
    const int sg = s0 + row;
    const bool live = sg < (VAR ? seq.end : T_);
    const uint32_t lane_addr = tbase + (static_cast<uint32_t>(quarter * 32) << 16);
    // The vectors hold v0 = scale^2 / den and v1 = -scale^2 delta / den per query (written by the
    // dq pass), so dA''^T = dN^T v0 + v1 and P^T = v0 sum_p (S^T_p)^2; W''^T_p = S^T_p dA''^T is
    // half of the true W^T_p, and the dK epilogue doubles the accumulator.
    // decay: e(t,s) = exp(min(c_t - c_s, 0)) is folded into dA''^T when it is formed and again
    // into P^T; the column part of dc, sum_t (dN - delta) rden A_ts over pairs with c_t - c_s <= 0,
    // is sum_t dA''_dec S^2 (S^2 summed over the parts), added to dc once per query head.
    float csum = 0.f;
    float c_s = 0.f;  // decay: c of this thread's key row for the current query head
    bool ok = true;
    int it = 0;
    for (int n = 0; n < nwork && ok; ++n) {
      const int qi = kj + n % nq;
      const bool diag = (qi == kj);
      const int vs = n & 1;
      const float* v_rd = vec + (vs * kNV + 0) * kTile;
      const float* v_dr = vec + (vs * kNV + 1) * kTile;
      const float* v_c = vec + (vs * kNV + 2) * kTile;  // decay: c of the query tile
      if (DECAY && live && n % nq == 0)  // this row's c for the query head of pairs n .. n + nq - 1
        c_s = p.c[(static_cast<size_t>(b) * T_ + sg) * p.HQ + h * p.G + n / nq];
      if (!mbar_wait(&bars.vec_full[vs], (n >> 1) & 1, wc)) {
        ok = false;
        break;
      }
      uint32_t dap[32];  // dA'^T of this thread's 64 query columns, bf16 pairs
      {
        const int x = static_cast<int>(static_cast<unsigned>(it) % NS);  // it >= 0: a mask for NS = 2
        if (!mbar_wait(&bars.i_full[x], (static_cast<unsigned>(it) / NS) & 1u, wc)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t nbase = lane_addr + x * 128u + hc * 64u;
        // one copy of the item for the diagonal tile (causal mask: query t >= key s), one without
        const auto dn_item = [&](auto diag_c) {
          uint32_t rn[2][16];
          tmem_ld16(nbase, rn[0]);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int cur = c & 1;
            if (c < 3) tmem_ld16(nbase + (c + 1) * 16u, rn[cur ^ 1]);
            const int cbase = hc * 64 + c * 16;
#pragma unroll
            for (int x4 = 0; x4 < 4; ++x4) {
              const float4 rd = *reinterpret_cast<const float4*>(v_rd + cbase + 4 * x4);
              const float4 dr = *reinterpret_cast<const float4*>(v_dr + cbase + 4 * x4);
              float2 d0 = ffma2(u2f2(rn[cur][4 * x4], rn[cur][4 * x4 + 1]), make_float2(rd.x, rd.y),
                                make_float2(dr.x, dr.y));
              float2 d1 = ffma2(u2f2(rn[cur][4 * x4 + 2], rn[cur][4 * x4 + 3]), make_float2(rd.z, rd.w),
                                make_float2(dr.z, dr.w));
              if (decltype(diag_c)::value && diag) {
                const int tl = cbase + 4 * x4;
                if (tl < row) d0.x = 0.f;
                if (tl + 1 < row) d0.y = 0.f;
                if (tl + 2 < row) d1.x = 0.f;
                if (tl + 3 < row) d1.y = 0.f;
              }
              if (DECAY) {
                const float4 ct = *reinterpret_cast<const float4*>(v_c + cbase + 4 * x4);
                d0.x *= __expf(fminf(ct.x - c_s, 0.f));
                d0.y *= __expf(fminf(ct.y - c_s, 0.f));
                d1.x *= __expf(fminf(ct.z - c_s, 0.f));
                d1.y *= __expf(fminf(ct.w - c_s, 0.f));
              }
              dap[8 * c + 2 * x4] = bf2_pack(d0);
              dap[8 * c + 2 * x4 + 1] = bf2_pack(d1);
            }
            if (c < 3) tmem_wait_ld();
          }
        };
        // (with decay, one copy that tests the tile: the second copy made the decayed variant spill)
        if (DECAY || diag)
          dn_item(std::true_type{});
        else
          dn_item(std::false_type{});
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars.i_free[x]);
        ++it;
      }
      float2 acc[32];
      for (int pp = 0; pp < NP; ++pp, ++it) {
        const int x = static_cast<int>(static_cast<unsigned>(it) % NS);  // it >= 0: a mask for NS = 2
        if (!mbar_wait(&bars.i_full[x], (static_cast<unsigned>(it) / NS) & 1u, wc)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sbase = lane_addr + x * 128u + hc * 64u;
        uint32_t rs[2][16];
        tmem_ld16(sbase, rs[0]);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int cur = c & 1;
          if (c < 3) tmem_ld16(sbase + (c + 1) * 16u, rs[cur ^ 1]);
          uint32_t wv[8];
#pragma unroll
          for (int x2 = 0; x2 < 8; ++x2) {
            const float2 sv = u2f2(rs[cur][2 * x2], rs[cur][2 * x2 + 1]);
            if constexpr (GRAM) {  // linear score: P^T from S itself, W^T = dA''^T
              acc[8 * c + x2] = sv;
              wv[x2] = dap[8 * c + x2];
            } else {
              acc[8 * c + x2] = pp == 0 ? fmul2(sv, sv) : ffma2(sv, sv, acc[8 * c + x2]);
              if constexpr (kBF16) {  // S rounded to bf16, packed product (same operand precision as the MMA)
                wv[x2] = bf2_mul(pack2<T>(sv.x, sv.y), dap[8 * c + x2]);
              } else {
                const float2 w = fmul2(sv, bf2_unpack(dap[8 * c + x2]));
                wv[x2] = pack2<T>(w.x, w.y);
              }
            }
          }
          tmem_st8(sbase + c * 8u, wv);  // columns of S already in registers
          if (c < 3) tmem_wait_ld();
        }
        if (pp == NP - 1) {  // P^T = scale^2 A / den into the other half of the slot (all S is read)
          // one copy of the stage for the diagonal tile (causal mask) and one without any mask
          const auto p_stage = [&](auto diag_c) {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const int cbase = hc * 64 + c * 16;
              uint32_t pv[8];
#pragma unroll
              for (int x2 = 0; x2 < 8; ++x2) {
                const int tl = cbase + 2 * x2;
                const float2 a = fmul2(acc[8 * c + x2], *reinterpret_cast<const float2*>(v_rd + tl));
                float a0 = a.x, a1 = a.y;
                if (DECAY) {
                  const float2 ct = *reinterpret_cast<const float2*>(v_c + tl);
                  const float x0 = ct.x - c_s, x1 = ct.y - c_s;
                  a0 *= __expf(fminf(x0, 0.f));
                  a1 *= __expf(fminf(x1, 0.f));
                  const float2 dd = bf2_unpack(dap[8 * c + x2]);  // dA''_dec, causally masked
                  if (x0 <= 0.f) csum = fmaf(dd.x, acc[8 * c + x2].x, csum);
                  if (x1 <= 0.f) csum = fmaf(dd.y, acc[8 * c + x2].y, csum);
                }
                if (decltype(diag_c)::value && diag) {
                  if (tl < row) a0 = 0.f;
                  if (tl + 1 < row) a1 = 0.f;
                }
                pv[x2] = pack2<T>(a0, a1);
              }
              tmem_st8(sbase + 32u + c * 8u, pv);
            }
          };
          if (DECAY || diag)
            p_stage(std::true_type{});
          else
            p_stage(std::false_type{});
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&bars.i_free[x]);
          if (pp == NP - 1) mbar_arrive(&bars.vec_empty[vs]);
        }
      }
      if (DECAY && n % nq == nq - 1) {  // last query tile of this query head: dc_s -= column sum
        if (ok && live) atomicAdd(p.dc + (static_cast<size_t>(b) * T_ + sg) * p.HQ + h * p.G + n / nq, -csum);
        csum = 0.f;
      }
    }
    // ---- epilogue: dK, dV -> global
    named_bar_sync(1, 256);
    if (ok && mbar_wait(&bars.acc_done, 0, wc)) {
      tc_fence_after();
      constexpr int HV = DV / 2;
      const size_t rowkv = (static_cast<size_t>(b) * T_ + sg) * p.H + h;
      T* dvrow = static_cast<T*>(p.dv) + rowkv * DV + hc * HV;
      if constexpr (!GRAM) {
        constexpr int HD = D / 2;
        T* dkrow = static_cast<T*>(p.dk) + rowkv * D + hc * HD;
#pragma unroll
        for (int c0 = 0; c0 < HD; c0 += 16) {
          uint32_t r[16];
          tmem_ld16(lane_addr + kColDK + hc * HD + c0, r);
          tmem_wait_ld();
          if (live) {  // dK = 2 * (sum of W''^T Q)
            const auto f = [&](int i) { return 2.f * __uint_as_float(r[i]); };
#pragma unroll
            for (int v2 = 0; v2 < 2; ++v2) {
              uint4 w;
              w.x = pack2<T>(f(8 * v2 + 0), f(8 * v2 + 1));
              w.y = pack2<T>(f(8 * v2 + 2), f(8 * v2 + 3));
              w.z = pack2<T>(f(8 * v2 + 4), f(8 * v2 + 5));
              w.w = pack2<T>(f(8 * v2 + 6), f(8 * v2 + 7));
              *reinterpret_cast<uint4*>(dkrow + c0 + 8 * v2) = w;
            }
          }
        }
      } else {  // Gram: d phi(k) over kGramFP = 144 columns, halves of 80 and 64, no doubling
        T* dkrow = static_cast<T*>(p.dk) + rowkv * D;
        const int cbeg = hc ? 80 : 0, cend = hc ? D : 80;
        for (int c0 = cbeg; c0 < cend; c0 += 16) {
          uint32_t r[16];
          tmem_ld16(lane_addr + kColDK + c0, r);
          tmem_wait_ld();
          if (live) {
#pragma unroll
            for (int v2 = 0; v2 < 2; ++v2) {
              uint4 w;
              w.x = pack2<T>(__uint_as_float(r[8 * v2 + 0]), __uint_as_float(r[8 * v2 + 1]));
              w.y = pack2<T>(__uint_as_float(r[8 * v2 + 2]), __uint_as_float(r[8 * v2 + 3]));
              w.z = pack2<T>(__uint_as_float(r[8 * v2 + 4]), __uint_as_float(r[8 * v2 + 5]));
              w.w = pack2<T>(__uint_as_float(r[8 * v2 + 6]), __uint_as_float(r[8 * v2 + 7]));
              *reinterpret_cast<uint4*>(dkrow + c0 + 8 * v2) = w;
            }
          }
        }
      }
#pragma unroll
      for (int c0 = 0; c0 < HV; c0 += 16) {
        uint32_t r[16];
        tmem_ld16(lane_addr + kColDV + hc * HV + c0, r);
        tmem_wait_ld();
        if (live) {
#pragma unroll
          for (int v2 = 0; v2 < 2; ++v2) {
            uint4 w;
            w.x = pack2<T>(__uint_as_float(r[8 * v2 + 0]), __uint_as_float(r[8 * v2 + 1]));
            w.y = pack2<T>(__uint_as_float(r[8 * v2 + 2]), __uint_as_float(r[8 * v2 + 3]));
            w.z = pack2<T>(__uint_as_float(r[8 * v2 + 4]), __uint_as_float(r[8 * v2 + 5]));
            w.w = pack2<T>(__uint_as_float(r[8 * v2 + 6]), __uint_as_float(r[8 * v2 + 7]));
            *reinterpret_cast<uint4*>(dvrow + c0 + 8 * v2) = w;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tbase, 512);
}

// ================================================================================================
// host side
// ================================================================================================
template <typename T, int D, int DV, int M, bool SUM, bool DECAY, bool GRAM = false, bool VAR = false>
int launch_bwd(const AttnBwdParams& p, cudaStream_t st) {
  constexpr int E = D / M;
  constexpr int CW = ScoreBoxW<E, GRAM>::value;
  constexpr int VCW = BoxW<DV>::value;
  using L = BwdSmem<D, DV>;
  CUtensorMap tq, tk, tv, to;
  int e = make_tm_tokens(&tq, p.q, p.B, p.T, p.HQ, D, CW);
  if (!e) e = make_tm_tokens(&tk, p.k, p.B, p.T, p.H, D, CW);
  if (!e) e = make_tm_tokens(&tv, p.v, p.B, p.T, p.H, DV, VCW);
  if (!e) e = make_tm_tokens(&to, p.dout, p.B, p.T, p.HQ, DV, VCW);
  if (e) return e;
  const int nt = (p.T + kTile - 1) / kTile;
  if (DECAY && !VAR) {  // head-major copy of c for both passes' bulk copies
    const BwdWs ws = ws_views(p.delta, p.B, p.T, p.HQ);
    decay_c_transpose<<<296, 256, 0, st>>>(p.c, ws.cT, p.B, p.T, p.HQ, ws.Tp);
    if (cudaGetLastError() != cudaSuccess) return KATA_ERR_CUDA;
  }
  if (DECAY && VAR) {
    const BwdWs ws = ws_views(p.delta, p.B, p.T, p.HQ, p.nseq);
    decay_c_transpose_var<<<varlen_tile_bound(p.T, p.nseq), kTile, 0, st>>>(p.c, ws.cT, p.T, p.HQ, ws.Tp, p.cu, p.nseq);
    if (cudaGetLastError() != cudaSuccess) return KATA_ERR_CUDA;
  }
  if (p.phases != 2) {
    // dq pass: tensor-memory ring with two issuers (decay: dc row sums written here)
    auto kern = attn_bwd_dq_ring_tc<T, D, DV, M, SUM, DECAY, GRAM, VAR>;
    const size_t smem = L::dqr_total(DECAY) + 1024;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
        cudaSuccess)
      return KATA_ERR_CUDA;
    kern<<<dim3(VAR ? varlen_tile_bound(p.T, p.nseq) : nt, p.B * p.HQ), kThreadsRing, smem, st>>>(tq, tk, tv, to, p);
    if (cudaGetLastError() != cudaSuccess) return KATA_ERR_CUDA;
  }
  if (p.phases != 1) {
    // dk/dv pass: tensor-memory ring (decay: dc column sums added here)
    auto kern = attn_bwd_dkdv_ring_tc<T, D, DV, M, SUM, DECAY, GRAM, VAR>;
    const size_t smem = L::kr_total(DECAY);  // no static shared memory: no alignment slack
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
        cudaSuccess)
      return KATA_ERR_CUDA;
    kern<<<dim3(VAR ? varlen_tile_bound(p.T, p.nseq) : nt, p.B * p.H), kThreads, smem, st>>>(tq, tk, tv, to, p);
    if (cudaGetLastError() != cudaSuccess) return KATA_ERR_CUDA;
  }
  return KATA_OK;
}

template <typename T, int D, int DV, int M>
int bwd_variant(const AttnBwdParams& p, bool sum, cudaStream_t st) {
  const bool dec = p.c != nullptr;
  // packed documents (p.cu): the VAR instantiations
  if (sum) {
    if constexpr (M * M <= 16) {
      if (!dec)
        return p.cu ? launch_bwd<T, D, DV, M, true, false, false, true>(p, st) : launch_bwd<T, D, DV, M, true, false>(p, st);
    }
    return KATA_ERR_UNSUPPORTED;
  }
  if (p.cu)
    return dec ? launch_bwd<T, D, DV, M, false, true, false, true>(p, st) : launch_bwd<T, D, DV, M, false, false, false, true>(p, st);
  return dec ? launch_bwd<T, D, DV, M, false, true>(p, st) : launch_bwd<T, D, DV, M, false, false>(p, st);
}

template <typename T, int D, int DV>
int bwd_m(const AttnBwdParams& p, bool sum, cudaStream_t st) {
  switch (p.M) {
    case 1: return bwd_variant<T, D, DV, 1>(p, sum, st);
    case 2: return bwd_variant<T, D, DV, 2>(p, sum, st);
    case 4: return bwd_variant<T, D, DV, 4>(p, sum, st);
    default: break;
  }
  if constexpr (D / 8 >= 16) {
    if (p.M == 8) return bwd_variant<T, D, DV, 8>(p, sum, st);
  }
  return KATA_ERR_UNSUPPORTED;
}

template <typename T>
int bwd_dims(const AttnBwdParams& p, bool sum, cudaStream_t st) {
  if (p.D == 128 && p.Dv == 128) return bwd_m<T, 128, 128>(p, sum, st);
  if (p.D == 64 && p.Dv == 64) return bwd_m<T, 64, 64>(p, sum, st);
  if (p.D == 128 && p.Dv == 64) return bwd_m<T, 128, 64>(p, sum, st);
  return KATA_ERR_UNSUPPORTED;
}

}  // namespace

size_t tc_bwd_workspace_bytes(int B, int T, int HQ, bool decay, int nseq) {
  const size_t Tp = nseq > 0 ? static_cast<size_t>(varlen_tile_bound(T, nseq)) * 128
                             : (static_cast<size_t>(T) + 127) & ~static_cast<size_t>(127);
  const size_t n0 = (static_cast<size_t>(B) * T * HQ + 3) & ~static_cast<size_t>(3);
  return sizeof(float) * (n0 + (decay ? 3 : 2) * static_cast<size_t>(B) * HQ * Tp);
}

bool tc_bwd_supported(int dtype, int D, int Dv, int M, bool sum) {
  if (dtype != KATA_DTYPE_BF16 && dtype != KATA_DTYPE_F16) return false;
  if (!((D == 64 && Dv == 64) || (D == 128 && Dv == 128) || (D == 128 && Dv == 64))) return false;
  if (!(M == 1 || M == 2 || M == 4 || M == 8) || D % M) return false;
  if ((D / M) % 16) return false;
  if (sum && M * M > 16) return false;
  return true;
}

int tc_attn_bwd(const AttnBwdParams& p, int dtype, bool sum, cudaStream_t st) {
  if (!tc_bwd_supported(dtype, p.D, p.Dv, p.M, sum)) return KATA_ERR_UNSUPPORTED;
  return dtype == KATA_DTYPE_BF16 ? bwd_dims<__nv_bfloat16>(p, sum, st) : bwd_dims<__half>(p, sum, st);
}

// Linear-score backward over bf16 Gram features: p.q, p.k hold phi (kGramFP columns), p.dq, p.dk
// receive d phi (bf16, kGramFP columns), p.D = kGramFP, p.M = 1, p.scale = 1.
int tc_attn_bwd_gram(const AttnBwdParams& p, cudaStream_t st) {
  if (p.D != kGramFP || p.M != 1 || p.Dv != 64 || p.c) return KATA_ERR_UNSUPPORTED;
  return launch_bwd<__nv_bfloat16, kGramFP, 64, 1, false, false, true>(p, st);
}

}  // namespace kata
