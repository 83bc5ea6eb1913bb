// attn_tc_fwd.cu -- tcgen05 tensor-core forward of causal KATA-SPD attention (bf16 / fp16).
//
// Math (kata/kernels/parallel_kata.py:10-197 concat, :202-345 sum):
//   S_p[t,s] = <q_a[t], k_b[s]>      for score parts p = (a,b): concat (g,g), sum all (a,b)
//   A[t,s]   = scale^2 * sum_p S_p^2 (* exp(min(c_t - c_s, 0)))   causal
//   O[t]     = sum_s half(A[t,s]) v_s,  den_t = sum_s A[t,s],  o_t = O[t] / (den_t > 0 ? den_t : 1)
//
// One CTA per (128-query tile, batch*head).  Warp roles (320 threads):
//   warp 0      TMA producer: Q once, K and V tiles through 3-stage rings (4-D tensor maps over
//               the time-major (B,T,H,D) tensors, so rows past T are zero-filled per batch).
//   warp 1      TMEM owner + MMA issuer (the whole warp runs the issue loop, one elected lane
//               issues every MMA and commit): for each key tile, one tcgen05.mma chain
//               per score part into a 3-slot TMEM ring (128 fp32 columns per slot), then the
//               P*V chain into the O accumulator (columns 384..384+Dv).  P is read straight from
//               tensor memory (A operand in TMEM), so P never touches shared memory.
//   warps 2..9  two compute warpgroups.  Thread (warp%4, lane) owns TMEM lane = query row;
//               warpgroup 0 owns key columns 0..63, warpgroup 1 owns 64..127.  They square and
//               accumulate the parts (packed fp32x2 FMAs), apply mask/decay, accumulate the row
//               sum, and store P = half(A) as packed pairs into the first 32 columns of their half
//               of the tile's last score slot (already read), where the P*V MMA reads it.
//               Finally they read O from TMEM, divide by den and store o and den.
// Slot reuse: the issuer never issues a score MMA into the slot that holds a P before it has
// issued the P*V chain reading it (tcgen05 MMAs of one CTA execute in issue order).
// Every mbarrier wait is bounded (see sm100.cuh); a timeout records a status code and drains.
#include "attn_tc_common.cuh"

namespace kata {
namespace {

constexpr int kBT = 128;  // query rows per tile (= UMMA M)
constexpr int kBK = 128;  // keys per tile (= UMMA N of the score MMAs, K of the P*V MMA)
constexpr int kSlots = 3;
constexpr int kStages = 3;
constexpr int kThreads = 320;
constexpr int kComputeWarp0 = 2;
constexpr uint32_t kOCol = 384;

template <int D, int DV>
struct FwdSmem {
  static constexpr int Q_BYTES = kBT * D * 2;
  static constexpr int K_BYTES = kBK * D * 2;
  static constexpr int V_BYTES = kBK * DV * 2;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + Q_BYTES;
  static constexpr int OFF_V = OFF_K + kStages * K_BYTES;
  static constexpr int TOTAL = OFF_V + kStages * V_BYTES;
};

struct FwdBarriers {
  uint64_t q_full;
  uint64_t k_full[kStages], k_empty[kStages];
  uint64_t v_full[kStages], v_empty[kStages];
  uint64_t s_full[kSlots], s_free[kSlots];
  uint64_t p_full[2];
  uint64_t o_full;
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  alignas(16) float den_x[2][kBT];  // partial row sums of the two column halves (decay: c staging)
};

template <typename T, int D, int DV, int M, bool SUM, bool DECAY, bool GRAM, bool VAR>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, AttnFwdParams p) {
  constexpr int E = D / M;
  constexpr int CW = ScoreBoxW<E, GRAM>::value;  // group box width (elements); swizzle = 2*CW bytes
  constexpr int NBOX = D / CW;
  constexpr int VCW = DV < 64 ? DV : 64;
  constexpr int NVBOX = DV / VCW;
  constexpr int NP = SUM ? M * M : M;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  static_assert(!GRAM || (M == 1 && !SUM && !DECAY), "Gram features: one linear score part");
  using L = FwdSmem<D, DV>;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ FwdBarriers bars;
  __shared__ SeqTile seq;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int T_ = p.T;
  const int bh = blockIdx.y, hq = bh % p.HQ, h = hq / p.G;
  // Rows of this CTA: query tile qt of a sequence whose rows are [kbase, t_end) of batch b; its key
  // tiles 0..qt start at kbase.  Packed documents: the tile's document (B == 1; past the last tile
  // the CTA exits before it allocates anything).
  int qt, b, kbase, t_end;
  if constexpr (VAR) {
    if (warp == 0) {
      SeqTile st{};
      const bool have = varlen_tile(p.cu, p.nseq, T_, static_cast<int>(blockIdx.x), st);
      if (lane == 0) seq = have ? st : SeqTile{0, 0, -1, 0, 0};
    }
    __syncthreads();
    if (seq.j < 0) return;
    qt = seq.j;
    b = 0;
    kbase = seq.start;
    t_end = seq.end;
  } else {
    qt = (T_ + kBT - 1) / kBT - 1 - static_cast<int>(blockIdx.x);  // heaviest tiles first
    b = bh / p.HQ;
    kbase = 0;
    t_end = T_;
  }
  const int t0 = kbase + qt * kBT;
  const int nk = qt + 1;  // causal: key tiles 0..qt
  WaitCtx wc{p.status, &bars.abort_flag};

  if (threadIdx.x == 0) {
    bars.abort_flag = 0;
    mbar_init(&bars.q_full, 1);
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&bars.k_full[i], 1);
      mbar_init(&bars.k_empty[i], 1);
      mbar_init(&bars.v_full[i], 1);
      mbar_init(&bars.v_empty[i], 1);
    }
    for (int i = 0; i < kSlots; ++i) {
      mbar_init(&bars.s_full[i], 1);
      mbar_init(&bars.s_free[i], 8);
    }
    mbar_init(&bars.p_full[0], 8);
    mbar_init(&bars.p_full[1], 8);
    mbar_init(&bars.o_full, 1);
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

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(&bars.q_full, L::Q_BYTES);
      for (int bx = 0; bx < NBOX; ++bx)
        tma_load_4d(smem + L::OFF_Q + bx * (kBT * CW * 2), &tmQ, &bars.q_full, bx * CW, hq, t0, b);
      int issued_k = 0, issued_v = 0;
      for (int j = 0; j < nk; ++j) {
        const int st = j % kStages;
        const uint32_t ph = (j / kStages) & 1;
        if (!mbar_wait(&bars.k_empty[st], ph ^ 1, wc)) break;
        mbar_arrive_expect_tx(&bars.k_full[st], L::K_BYTES);
        uint8_t* sk = smem + L::OFF_K + st * L::K_BYTES;
        for (int bx = 0; bx < NBOX; ++bx)
          tma_load_4d(sk + bx * (kBK * CW * 2), &tmK, &bars.k_full[st], bx * CW, h, kbase + j * kBK, b);
        issued_k = j + 1;
        if (!mbar_wait(&bars.v_empty[st], ph ^ 1, wc)) break;
        mbar_arrive_expect_tx(&bars.v_full[st], L::V_BYTES);
        uint8_t* sv = smem + L::OFF_V + st * L::V_BYTES;
        for (int bx = 0; bx < NVBOX; ++bx)
          tma_load_4d(sv + bx * (kBK * VCW * 2), &tmV, &bars.v_full[st], bx * VCW, h, kbase + j * kBK, b);
        issued_v = j + 1;
      }
      if (*wc.abort) {
        // drain: wait (bounded) for the most recent copies of each stage so no TMA write lands
        // in shared memory after the CTA retires.
        for (int j = (issued_k > kStages ? issued_k - kStages : 0); j < issued_k; ++j)
          mbar_drain(&bars.k_full[j % kStages], (j / kStages) & 1);
        for (int j = (issued_v > kStages ? issued_v - kStages : 0); j < issued_v; ++j)
          mbar_drain(&bars.v_full[j % kStages], (j / kStages) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    {  // warp-wide issue (every lane runs the loop; one elected lane issues)
      const uint32_t idesc_qk = umma_idesc_f16(128, kBK, kBF16, false, false);
      const uint32_t idesc_pv = umma_idesc_f16(128, DV, kBF16, false, true);
      // Descriptor bases (group 0, stage 0); every operand below is a compile-time or stage-multiple
      // offset from one of these, so no descriptor is rebuilt inside the loops.
      const uint64_t qd0 = kmajor_desc<CW>(smem_u32(smem + L::OFF_Q), 0, E, 0);
      const uint64_t kd0 = kmajor_desc<CW>(smem_u32(smem + L::OFF_K), 0, E, 0);
      const uint64_t vd0 = mnmajor_desc<VCW>(smem_u32(smem + L::OFF_V), 0, 0);
      bool ok = mbar_wait_w(&bars.q_full, 0, wc);
      // O += P_i V_i with P_i read from TMEM slot `sl`; V_i is in stage `vst` (use parity `vpar`)
      auto issue_pv = [&](int i, int vst, uint32_t vpar, int sl) -> bool {
        if (!mbar_wait_w(&bars.p_full[i & 1], (i >> 1) & 1, wc)) return false;
        if (!mbar_wait_w(&bars.v_full[vst], vpar, wc)) return false;
        tc_fence_after();
        const uint64_t vd = vd0 + desc_units(static_cast<uint32_t>(vst) * L::V_BYTES);
        const uint32_t pa = tbase + static_cast<uint32_t>(sl) * 128u;
        const uint32_t acc0 = i > 0 ? 1u : 0u;
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)
          umma_ts_w(tbase + kOCol, pa + packed_col(kk), vd + mnstep<VCW>(kk), idesc_pv, kk > 0 ? 1u : acc0);
        umma_commit_w(&bars.v_empty[vst]);
        return true;
      };
      // Score part u (u = j*NP + pp) goes to slot u % kSlots; the counters below carry the slot,
      // the key stage j % kStages and the parities of their current uses.
      int slot = 0, st = 0;
      uint32_t slot_par = 0, st_par = 0;
      // key tile whose P*V chain is not issued yet: its slot, V stage and stage parity
      int pend = -1, pend_slot = 0, pend_st = 0;
      uint32_t pend_par = 0;
      for (int j = 0; ok && j < nk; ++j) {
        if (!mbar_wait_w(&bars.k_full[st], st_par, wc)) {
          ok = false;
          break;
        }
        const uint64_t kd = kd0 + desc_units(static_cast<uint32_t>(st) * L::K_BYTES);
        int last_slot = 0;
#pragma unroll
        for (int pp = 0; pp < NP; ++pp) {
          // The previous tile's P occupies the slot of its last part, (j*NP - 1) % kSlots, which
          // part pp of this tile reaches first at pp = kSlots - 1: its P*V chain is issued before.
          if (pp == kSlots - 1 && pend >= 0) {
            if (!issue_pv(pend, pend_st, pend_par, pend_slot)) {
              ok = false;
              break;
            }
            pend = -1;
          }
          if (!mbar_wait_w(&bars.s_free[slot], slot_par ^ 1, wc)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int ga = SUM ? pp / M : pp, gb = SUM ? pp % M : pp;  // constants once unrolled
          const uint64_t qd = qd0 + kmajor_goff<CW>(ga, E), kdp = kd + kmajor_goff<CW>(gb, E);
          const uint32_t sd = tbase + static_cast<uint32_t>(slot) * 128u;
#pragma unroll
          for (int kk = 0; kk < E / 16; ++kk)
            umma_ss_w(sd, qd + kstep<CW>(kk), kdp + kstep<CW>(kk), idesc_qk, kk > 0 ? 1u : 0u);
          umma_commit_w(&bars.s_full[slot]);
          last_slot = slot;
          if (++slot == kSlots) {
            slot = 0;
            slot_par ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_w(&bars.k_empty[st]);
        if (pend >= 0 && !issue_pv(pend, pend_st, pend_par, pend_slot)) {
          ok = false;
          break;
        }
        pend = j;
        pend_slot = last_slot;
        pend_st = st;
        pend_par = st_par;
        if (++st == kStages) {
          st = 0;
          st_par ^= 1;
        }
      }
      if (ok && pend >= 0) ok = issue_pv(pend, pend_st, pend_par, pend_slot);
      if (ok) umma_commit_w(&bars.o_full);
      // drain outstanding MMAs before the CTA can retire
      umma_commit_w(&bars.drain);
      mbar_drain(&bars.drain, 0);
    }
  } else {
    // ------------------------------------------------------------------ compute warpgroups
    const int cw = warp - kComputeWarp0;  // 0..7
    const int hc = cw >> 2;               // column half
    const int quarter = warp & 3;         // TMEM lane quarter
    const int row = quarter * 32 + lane;  // query row within the tile
    const int t = t0 + row;
    const uint32_t lane_addr = tbase + (static_cast<uint32_t>(quarter * 32) << 16);
    const float scale2 = p.scale * p.scale;
    float c_t = 0.f;
    const float* cbase = nullptr;
    if (DECAY) {
      cbase = p.c + static_cast<size_t>(b) * T_ * p.HQ + hq;
      c_t = (t < T_) ? cbase[static_cast<size_t>(t) * p.HQ] : 0.f;
    }
    float2 den2 = make_float2(0.f, 0.f);
    bool ok = true;
    int u = 0;
    for (int j = 0; j < nk && ok; ++j) {
      float2 acc[32];
      int slot = 0;
      float cpre[2] = {0.f, 0.f};  // decay: this lane's two key columns' c, loaded ahead of the parts
      if (DECAY) {
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          const int s0 = kbase + j * kBK + hc * 64 + h2 * 32 + lane;
          cpre[h2] = (s0 < T_) ? __ldg(cbase + static_cast<size_t>(s0) * p.HQ) : 0.f;
        }
      }
#pragma unroll
      for (int i = 0; i < 32; ++i) acc[i] = make_float2(0.f, 0.f);  // fma(s, s, 0) == s * s
      for (int pp = 0; pp < NP; ++pp, ++u) {
        slot = u % kSlots;
        if (!mbar_wait(&bars.s_full[slot], (u / kSlots) & 1, wc)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // both 32-column chunks in flight at once (one load latency per part), then the slot goes
        // back to the issuer before the squares are accumulated
        uint32_t r0[32], r1[32];
        const uint32_t a = lane_addr + slot * 128u + hc * 64u;
        tmem_ld32(a, r0);
        tmem_ld32(a + 32u, r1);
        tmem_wait_ld();
        if (pp < NP - 1) {  // the last part's slot receives P and is released after it
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars.s_free[slot]);
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float2 x0 = make_float2(__uint_as_float(r0[2 * i]), __uint_as_float(r0[2 * i + 1]));
          acc[i] = GRAM ? x0 : ffma2(x0, x0, acc[i]);  // Gram: A = S
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float2 x1 = make_float2(__uint_as_float(r1[2 * i]), __uint_as_float(r1[2 * i + 1]));
          acc[16 + i] = GRAM ? x1 : ffma2(x1, x1, acc[16 + i]);
        }
      }
      if (!ok) break;
      // A = scale^2 * acc, causal mask on the diagonal tile, optional decay; row sum; P -> TMEM.
      // For bf16 the scale^2 factor is left out of P and of the row sum: o = (P v) / den is
      // invariant under a common scale of P and den (bf16 has the fp32 exponent range, so the
      // unscaled P cannot overflow where the scaled one would not) and den is rescaled once in the
      // epilogue.  fp16 keeps the per-element scale so its overflow behaviour matches the
      // reference's cast of the scaled score to the value dtype.
      if (!kBF16) {
        const float2 sc2 = make_float2(scale2, scale2);
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = fmul2(acc[i], sc2);
      }
      const int s_base = kbase + j * kBK + hc * 64;
      if (j == qt) {  // diagonal tile: causal mask
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int s0 = s_base + 2 * i;
          if (s0 > t) acc[i].x = 0.f;
          if (s0 + 1 > t) acc[i].y = 0.f;
        }
      }
      if (DECAY) {
        // The 64 key columns' c values (strided by HQ in global memory) were loaded at the start of
        // the tile, one per lane for each half of 32.  Factored decay: with lo = the warp minimum of those 32 values, a row
        // with c_t <= lo has every c_t - c_s <= 0 and e = exp(c_t - lo) * exp(lo - c_s), both
        // factors <= 1 (no overflow; an underflow only flushes values below 1e-38), so the column
        // factors go to the warp's own 32 floats of den_x (the row-sum exchange, idle until the
        // epilogue; each warp writes only its slice there too) and each row takes one exponential.
        // If any row of the warp has c_t > lo, the warp takes exponentials per element, with c_s
        // from the lane that loaded it.
        float* fbuf = &bars.den_x[hc][quarter * 32];
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          const float cl = cpre[h2];
          float lo = cl;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
          if (!__any_sync(0xffffffffu, c_t > lo)) {
            fbuf[lane] = __expf(lo - cl);
            __syncwarp();
            const float rt = __expf(c_t - lo);
            const float2 rt2 = make_float2(rt, rt);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float4 f = *reinterpret_cast<const float4*>(fbuf + 4 * i);
              acc[h2 * 16 + 2 * i] = fmul2(acc[h2 * 16 + 2 * i], fmul2(rt2, make_float2(f.x, f.y)));
              acc[h2 * 16 + 2 * i + 1] = fmul2(acc[h2 * 16 + 2 * i + 1], fmul2(rt2, make_float2(f.z, f.w)));
            }
            __syncwarp();  // every lane has read the slice before it is rewritten
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float cs0 = __shfl_sync(0xffffffffu, cl, 2 * i);
              const float cs1 = __shfl_sync(0xffffffffu, cl, 2 * i + 1);
              acc[h2 * 16 + i].x *= __expf(fminf(c_t - cs0, 0.f));
              acc[h2 * 16 + i].y *= __expf(fminf(c_t - cs1, 0.f));
            }
          }
        }
      }
#pragma unroll
      for (int i = 0; i < 32; ++i) den2 = fadd2(den2, acc[i]);
      uint32_t w0[16], w1[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        w0[i] = pack2<T>(acc[i].x, acc[i].y);
        w1[i] = pack2<T>(acc[16 + i].x, acc[16 + i].y);
      }
      const uint32_t pa = lane_addr + slot * 128u + hc * 64u;
      tmem_st16(pa, w0);
      tmem_st16(pa + 16u, w1);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bars.p_full[j & 1]);
        mbar_arrive(&bars.s_free[slot]);
      }
    }
    // ------------------------------------------------------------------ epilogue
    const float den = den2.x + den2.y;
    bars.den_x[hc][row] = den;
    named_bar_sync(1, 256);
    const float den_all = (bars.den_x[0][row] + bars.den_x[1][row]) * (kBF16 ? scale2 : 1.f);
    if (ok && mbar_wait(&bars.o_full, 0, wc)) {
      tc_fence_after();
      // O holds sum_s P v with P unscaled for bf16, so divide by the unscaled row sum there
      const float den_o = kBF16 ? den_all / scale2 : den_all;
      const float inv = 1.f / (den_o > 0.f ? den_o : 1.f);
      constexpr int HALF = DV / 2;
      T* orow = static_cast<T*>(p.o) + ((static_cast<size_t>(b) * T_ + t) * p.HQ + hq) * DV + hc * HALF;
      const bool live = t < t_end;
#pragma unroll
      for (int c0 = 0; c0 < HALF; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(lane_addr + kOCol + hc * HALF + c0, r);
        tmem_wait_ld();
        if (live) {
#pragma unroll
          for (int v4 = 0; v4 < 4; ++v4) {
            uint4 w;
            w.x = pack2<T>(__uint_as_float(r[8 * v4 + 0]) * inv, __uint_as_float(r[8 * v4 + 1]) * inv);
            w.y = pack2<T>(__uint_as_float(r[8 * v4 + 2]) * inv, __uint_as_float(r[8 * v4 + 3]) * inv);
            w.z = pack2<T>(__uint_as_float(r[8 * v4 + 4]) * inv, __uint_as_float(r[8 * v4 + 5]) * inv);
            w.w = pack2<T>(__uint_as_float(r[8 * v4 + 6]) * inv, __uint_as_float(r[8 * v4 + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + c0 + 8 * v4) = w;
          }
        }
      }
      if (hc == 0 && live) p.den[(static_cast<size_t>(b) * T_ + t) * p.HQ + hq] = den_all;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tbase, 512);
}

template <typename T, int D, int DV, int M, bool SUM, bool DECAY, bool GRAM = false, bool VAR = false>
int launch_fwd(const AttnFwdParams& p, cudaStream_t st) {
  constexpr int E = D / M;
  constexpr int CW = ScoreBoxW<E, GRAM>::value;
  constexpr int VCW = DV < 64 ? DV : 64;
  CUtensorMap tq, tk, tv;
  int e = make_tm_tokens(&tq, p.q, p.B, p.T, p.HQ, D, CW);
  if (!e) e = make_tm_tokens(&tk, p.k, p.B, p.T, p.H, D, CW);
  if (!e) e = make_tm_tokens(&tv, p.v, p.B, p.T, p.H, DV, VCW);
  if (e) return e;
  const size_t smem = FwdSmem<D, DV>::TOTAL + 1024;
  auto kern = attn_fwd_tc<T, D, DV, M, SUM, DECAY, GRAM, VAR>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
    return KATA_ERR_CUDA;
  const int ntiles = VAR ? varlen_tile_bound(p.T, p.nseq) : (p.T + kBT - 1) / kBT;
  const dim3 grid(ntiles, p.B * p.HQ);
  kern<<<grid, kThreads, smem, st>>>(tq, tk, tv, p);
  return from_cuda(cudaGetLastError());
}

template <typename T, int D, int DV, int M>
int dispatch_variant(const AttnFwdParams& p, bool sum, cudaStream_t st) {
  const bool dec = p.c != nullptr;
  // packed documents (p.cu): the VAR instantiations
  if (sum) {
    // the reference pairs decay with the concat score only (kata/layer.py:187-193)
    if constexpr (M * M <= 16) {
      if (!dec)
        return p.cu ? launch_fwd<T, D, DV, M, true, false, false, true>(p, st) : launch_fwd<T, D, DV, M, true, false>(p, st);
    }
    return KATA_ERR_UNSUPPORTED;
  }
  if (p.cu)
    return dec ? launch_fwd<T, D, DV, M, false, true, false, true>(p, st) : launch_fwd<T, D, DV, M, false, false, false, true>(p, st);
  return dec ? launch_fwd<T, D, DV, M, false, true>(p, st) : launch_fwd<T, D, DV, M, false, false>(p, st);
}

template <typename T, int D, int DV>
int dispatch_m(const AttnFwdParams& p, bool sum, cudaStream_t st) {
  switch (p.M) {
    case 1: return dispatch_variant<T, D, DV, 1>(p, sum, st);
    case 2: return dispatch_variant<T, D, DV, 2>(p, sum, st);
    case 4: return dispatch_variant<T, D, DV, 4>(p, sum, st);
    default: break;
  }
  if constexpr (D / 8 >= 16) {
    if (p.M == 8) return dispatch_variant<T, D, DV, 8>(p, sum, st);
  }
  return KATA_ERR_UNSUPPORTED;
}

template <typename T>
int dispatch_dims(const AttnFwdParams& p, bool sum, cudaStream_t st) {
  if (p.D == 128 && p.Dv == 128) return dispatch_m<T, 128, 128>(p, sum, st);
  if (p.D == 64 && p.Dv == 64) return dispatch_m<T, 64, 64>(p, sum, st);
  if (p.D == 128 && p.Dv == 64) return dispatch_m<T, 128, 64>(p, sum, st);
  return KATA_ERR_UNSUPPORTED;
}

}  // namespace

bool tc_fwd_supported(int dtype, int D, int Dv, int M, bool sum) {
  if (dtype != KATA_DTYPE_BF16 && dtype != KATA_DTYPE_F16) return false;
  // (128, 64): the offset-gated heads of the 200M geometry (M groups of 16 padded to 32, v of 64)
  if (!((D == 64 && Dv == 64) || (D == 128 && Dv == 128) || (D == 128 && Dv == 64))) return false;
  if (!(M == 1 || M == 2 || M == 4 || M == 8) || D % M) return false;
  if ((D / M) % 16) return false;
  if (sum && M * M > 16) return false;
  return true;
}

bool tc_fwd_supports_decay(bool sum) { return !sum; }

int tc_attn_fwd(const AttnFwdParams& p, int dtype, bool sum, cudaStream_t st) {
  if (!tc_fwd_supported(dtype, p.D, p.Dv, p.M, sum)) return KATA_ERR_UNSUPPORTED;
  return dtype == KATA_DTYPE_BF16 ? dispatch_dims<__nv_bfloat16>(p, sum, st) : dispatch_dims<__half>(p, sum, st);
}

// Linear-score forward over bf16 Gram features: p.q, p.k hold phi (kGramFP columns), p.D = kGramFP,
// p.M = 1, p.scale = 1 (the scale is inside the features).
int tc_attn_fwd_gram(const AttnFwdParams& p, cudaStream_t st) {
  if (p.D != kGramFP || p.M != 1 || p.Dv != 64 || p.c) return KATA_ERR_UNSUPPORTED;
  return launch_fwd<__nv_bfloat16, kGramFP, 64, 1, false, false, true>(p, st);
}

}  // namespace kata
