// selftest.cu -- device check of the UMMA/TMA encodings used by the attention kernels.
//
// One CTA of 128 threads loads A and B with TMA (any of the 32/64/128-byte swizzles, K-major or
// MN-major), optionally restages A into tensor memory, runs K/16 tcgen05.mma steps into a TMEM
// accumulator and writes D = A * B^T back as fp32.  The host test compares against a plain GEMM.
#include "host_util.h"
#include "sm100.cuh"

namespace kata {
namespace {

struct SelftestParams {
  int M, N, K;
  int a_mn, b_mn, a_sw, b_sw, a_tmem;
  int lane_off;  // M == 64 only: TMEM lane offset of the accumulator (0 or 16)
  const __nv_bfloat16* A;  // for the a_tmem path (row-major M x K or K x M)
  float* D;
  int* status;
};

// Descriptor of a 16-row K-step for an operand laid out as TMA boxes of `cw` elements
// (cw*2 == swizzle bytes).  K-major: boxes tile K, each box holds `rows` rows.  MN-major: boxes
// tile the M/N extent, each box holds `krows` rows of K.
__device__ uint64_t operand_desc(uint32_t base, bool mn_major, int cw, int rows_or_krows, int kk) {
  const uint32_t rb = static_cast<uint32_t>(cw) * 2u;
  const int sw = static_cast<int>(rb);
  if (!mn_major) {
    const int k0 = kk * 16;
    const uint32_t box = static_cast<uint32_t>(k0 / cw);
    const uint32_t within = static_cast<uint32_t>(k0 % cw) * 2u;
    return umma_smem_desc(base + box * static_cast<uint32_t>(rows_or_krows) * rb + within, 16u, 8u * rb, sw);
  }
  const uint32_t box_stride = static_cast<uint32_t>(rows_or_krows) * rb;
  return umma_smem_desc(base + static_cast<uint32_t>(kk) * 16u * rb, box_stride, 8u * rb, sw);
}

__global__ void __launch_bounds__(128, 1)
    selftest_umma_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                         SelftestParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t bar_load, bar_mma;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  const int tid = threadIdx.x, warp = tid >> 5;
  WaitCtx wc{p.status, &abort_flag};

  const int cwA = p.a_sw / 2, cwB = p.b_sw / 2;
  const int a_bytes = p.M * p.K * 2, b_bytes = p.N * p.K * 2;
  uint8_t* sA = smem;
  uint8_t* sB = smem + ((a_bytes + 1023) & ~1023);

  if (tid == 0) {
    abort_flag = 0;
    mbar_init(&bar_load, 1);
    mbar_init(&bar_mma, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_base;

  if (tid == 0) {
    mbar_arrive_expect_tx(&bar_load, static_cast<uint32_t>((p.a_tmem ? 0 : a_bytes) + b_bytes));
    if (!p.a_tmem) {
      const int nboxA = p.a_mn ? p.M / cwA : p.K / cwA;
      const int rowsA = p.a_mn ? p.K : p.M;
      for (int b = 0; b < nboxA; ++b) tma_load_4d(sA + b * rowsA * p.a_sw, &tmA, &bar_load, b * cwA, 0, 0, 0);
    }
    const int nboxB = p.b_mn ? p.N / cwB : p.K / cwB;
    const int rowsB = p.b_mn ? p.K : p.N;
    for (int b = 0; b < nboxB; ++b) tma_load_4d(sB + b * rowsB * p.b_sw, &tmB, &bar_load, b * cwB, 0, 0, 0);
  }

  const uint32_t a_col = 256;  // TMEM column of the A operand when staged in tensor memory
  if (p.a_tmem) {
    // Each warp owns 32 TMEM lanes (rows); thread = row.  Column c holds A[row][2c], A[row][2c+1].
    const int row = tid;
    for (int k0 = 0; k0 < p.K; k0 += 32) {
      uint32_t r[16];
      for (int j = 0; j < 16; ++j) {
        const int k = k0 + 2 * j;
        float lo, hi;
        if (p.a_mn) {
          lo = __bfloat162float(p.A[static_cast<size_t>(k) * p.M + row]);
          hi = __bfloat162float(p.A[static_cast<size_t>(k + 1) * p.M + row]);
        } else {
          lo = __bfloat162float(p.A[static_cast<size_t>(row) * p.K + k]);
          hi = __bfloat162float(p.A[static_cast<size_t>(row) * p.K + k + 1]);
        }
        r[j] = pack2<__nv_bfloat16>(lo, hi);
      }
      tmem_st16(tbase + (static_cast<uint32_t>(warp * 32) << 16) + a_col + static_cast<uint32_t>(k0 / 2), r);
    }
    tmem_wait_st();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (tid == 0) {
    if (mbar_wait(&bar_load, 0, wc)) {
      tc_fence_after();
      const uint32_t idesc = umma_idesc_f16(p.M, p.N, true, p.a_tmem ? false : p.a_mn != 0, p.b_mn != 0);
      const uint32_t baseA = smem_u32(sA), baseB = smem_u32(sB);
      for (int kk = 0; kk < p.K / 16; ++kk) {
        const uint64_t bd = operand_desc(baseB, p.b_mn != 0, cwB, p.b_mn ? p.K : p.N, kk);
        if (p.a_tmem) {
          umma_ts(tbase, tbase + a_col + static_cast<uint32_t>(kk * 8), bd, idesc, kk > 0);
        } else {
          const uint64_t ad = operand_desc(baseA, p.a_mn != 0, cwA, p.a_mn ? p.K : p.M, kk);
          umma_ss(tbase + (static_cast<uint32_t>(p.lane_off) << 16), ad, bd, idesc, kk > 0);
        }
      }
      umma_commit(&bar_mma);
    }
  }
  __syncwarp();
  const bool ok = mbar_wait(&bar_mma, 0, wc);
  tc_fence_after();
  if (ok) {
    // M = 128: row = TMEM lane.  M = 64 (one CTA): row m sits in lane (m % 16) + 32 * (m / 16) +
    // lane_off, i.e. the first (or, with lane_off 16, the second) half of every warp's 32 lanes.
    const int lane = tid & 31;
    const bool mine = p.M == 128 || (lane & 16) == p.lane_off;
    const int row = p.M == 128 ? tid : warp * 16 + (lane & 15);
    for (int n0 = 0; n0 < p.N; n0 += 16) {
      uint32_t r[16];
      tmem_ld16(tbase + (static_cast<uint32_t>(warp * 32) << 16) + static_cast<uint32_t>(n0), r);
      tmem_wait_ld();
      if (mine)
        for (int j = 0; j < 16; ++j) p.D[static_cast<size_t>(row) * p.N + n0 + j] = __uint_as_float(r[j]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, 512);
}


// CTA-pair check: D (256 x N) = A * B^T through one M = 256 cta_group::2 MMA chain.  Cluster of two
// CTAs; rank r loads rows [128 r, 128 r + 128) of A (or, MN-major, that column range of the stored
// K x M matrix) and half of B: rows [N/2 r, N/2 (r + 1)) of a K-major B, or that column range of an
// MN-major one, each into its own shared memory at the same offset.  Both loads complete on the
// leader's mbarrier; the leader issues the chain and the commit signals both CTAs; each CTA writes
// its 128 rows of D from its own tensor memory.  a_tmem stages each CTA's A rows in its TMEM.
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(128, 1)
    selftest_umma_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                              SelftestParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t bar_load, bar_mma;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  const int tid = threadIdx.x, warp = tid >> 5;
  const uint32_t rank = cluster_rank();
  WaitCtx wc{p.status, &abort_flag};

  const int cwA = p.a_sw / 2, cwB = p.b_sw / 2;
  const int NH = p.N / 2;
  const int a_bytes = 128 * p.K * 2, b_bytes = NH * p.K * 2;
  uint8_t* sA = smem;
  uint8_t* sB = smem + ((a_bytes + 1023) & ~1023);

  if (tid == 0) {
    abort_flag = 0;
    mbar_init(&bar_load, 1);
    mbar_init(&bar_mma, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc2(&tmem_base, 512);
    tmem_relinquish2();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tbase = tmem_base;
  const uint32_t lead_load = mapa_shared(smem_u32(&bar_load), 0);

  if (tid == 0) {
    if (rank == 0) mbar_arrive_expect_tx(&bar_load, static_cast<uint32_t>(2 * ((p.a_tmem ? 0 : a_bytes) + b_bytes)));
    if (!p.a_tmem) {
      if (p.a_mn) {  // stored K x 256: this CTA's 128 columns, boxes of cwA columns x K rows
        for (int b = 0; b < 128 / cwA; ++b)
          tma_load_4d_pair(sA + b * p.K * p.a_sw, &tmA, lead_load, 128 * static_cast<int>(rank) + b * cwA, 0, 0, 0);
      } else {  // stored 256 x K: this CTA's 128 rows, boxes of cwA columns x 128 rows
        for (int b = 0; b < p.K / cwA; ++b)
          tma_load_4d_pair(sA + b * 128 * p.a_sw, &tmA, lead_load, b * cwA, 128 * static_cast<int>(rank), 0, 0);
      }
    }
    if (p.b_mn) {  // stored K x N: this CTA's N/2 columns
      for (int b = 0; b < NH / cwB; ++b)
        tma_load_4d_pair(sB + b * p.K * p.b_sw, &tmB, lead_load, NH * static_cast<int>(rank) + b * cwB, 0, 0, 0);
    } else {  // stored N x K: this CTA's N/2 rows
      for (int b = 0; b < p.K / cwB; ++b)
        tma_load_4d_pair(sB + b * NH * p.b_sw, &tmB, lead_load, b * cwB, NH * static_cast<int>(rank), 0, 0);
    }
  }
  const uint32_t a_col = 256;
  if (p.a_tmem) {
    const int row = 128 * static_cast<int>(rank) + tid;
    for (int k0 = 0; k0 < p.K; k0 += 32) {
      uint32_t r[16];
      for (int j = 0; j < 16; ++j) {
        const int k = k0 + 2 * j;
        const float lo = __bfloat162float(p.A[static_cast<size_t>(row) * p.K + k]);
        const float hi = __bfloat162float(p.A[static_cast<size_t>(row) * p.K + k + 1]);
        r[j] = pack2<__nv_bfloat16>(lo, hi);
      }
      tmem_st16(tbase + (static_cast<uint32_t>(warp * 32) << 16) + a_col + static_cast<uint32_t>(k0 / 2), r);
    }
    tmem_wait_st();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' TMEM A rows are stored
  tc_fence_after();

  if (rank == 0 && warp == 0) {
    const bool ok = mbar_wait_w(&bar_load, 0, wc);
    if (ok) {
      tc_fence_after();
      const uint32_t idesc = umma_idesc_f16(256, p.N, true, p.a_tmem ? false : p.a_mn != 0, p.b_mn != 0);
      const uint32_t baseA = smem_u32(sA), baseB = smem_u32(sB);
      for (int kk = 0; kk < p.K / 16; ++kk) {
        const uint64_t bd = operand_desc(baseB, p.b_mn != 0, cwB, p.b_mn ? p.K : NH, kk);
        if (p.a_tmem) {
          umma2_ts_w(tbase, tbase + a_col + static_cast<uint32_t>(kk * 8), bd, idesc, kk > 0);
        } else {
          const uint64_t ad = operand_desc(baseA, p.a_mn != 0, cwA, p.a_mn ? p.K : 128, kk);
          umma2_ss_w(tbase, ad, bd, idesc, kk > 0);
        }
      }
    }
    umma2_commit_both_w(&bar_mma);  // on the abort path too: the follower's wait then ends
  }
  __syncwarp();
  const bool ok = mbar_wait(&bar_mma, 0, wc);
  tc_fence_after();
  if (ok) {
    const int row = 128 * static_cast<int>(rank) + tid;
    for (int n0 = 0; n0 < p.N; n0 += 16) {
      uint32_t r[16];
      tmem_ld16(tbase + (static_cast<uint32_t>(warp * 32) << 16) + static_cast<uint32_t>(n0), r);
      tmem_wait_ld();
      for (int j = 0; j < 16; ++j) p.D[static_cast<size_t>(row) * p.N + n0 + j] = __uint_as_float(r[j]);
    }
  }
  tc_fence_before();
  cluster_sync();
  if (warp == 0) tmem_dealloc2(tbase, 512);
}

}  // namespace
}  // namespace kata

namespace {
int selftest_launch(const void* A, const void* B, float* D, int M, int N, int K, int a_mn, int b_mn, int a_sw,
                    int b_sw, int a_tmem, int lane_off, kata_stream_t stream);
}  // namespace

extern "C" int kata_selftest_umma(const void* A, const void* B, float* D, int M, int N, int K, int a_mn, int b_mn,
                                  int a_sw, int b_sw, int a_tmem, kata_stream_t stream) {
  if (M != 128) return KATA_ERR_SHAPE;
  return selftest_launch(A, B, D, M, N, K, a_mn, b_mn, a_sw, b_sw, a_tmem, 0, stream);
}

extern "C" int kata_selftest_umma_m64(const void* A, const void* B, float* D, int N, int K, int a_mn, int b_mn,
                                      int lane_off, kata_stream_t stream) {
  if (lane_off != 0 && lane_off != 16) return KATA_ERR_INVALID;
  return selftest_launch(A, B, D, 64, N, K, a_mn, b_mn, 128, 128, 0, lane_off, stream);
}

extern "C" int kata_selftest_umma_pair(const void* A, const void* B, float* D, int N, int K, int a_mn, int b_mn,
                                       int a_sw, int b_sw, int a_tmem, kata_stream_t stream) {
  using namespace kata;
  if (!A || !B || !D) return KATA_ERR_INVALID;
  auto sw_ok = [](int s) { return s == 32 || s == 64 || s == 128; };
  if (N < 32 || N > 256 || N % 32 || K < 16 || K > 256 || K % 16 || !sw_ok(a_sw) || !sw_ok(b_sw) ||
      (a_tmem && a_mn))
    return KATA_ERR_SHAPE;
  const int cwA = a_sw / 2, cwB = b_sw / 2;
  if ((a_mn ? 128 : K) % cwA || (b_mn ? N / 2 : K) % cwB) return KATA_ERR_SHAPE;
  const int M = 256;
  CUtensorMap tmA, tmB;
  {
    const uint64_t cols = a_mn ? M : K, rows = a_mn ? K : M;
    const uint64_t dims[4] = {cols, rows, 1, 1};
    const uint64_t strides[3] = {cols * 2, cols * rows * 2, cols * rows * 2};
    const uint32_t box[4] = {static_cast<uint32_t>(cwA), static_cast<uint32_t>(a_mn ? K : 128), 1, 1};
    int e = encode_tmap_16bit(&tmA, A, 4, dims, strides, box, a_sw);
    if (e) return e;
  }
  {
    const uint64_t cols = b_mn ? N : K, rows = b_mn ? K : N;
    const uint64_t dims[4] = {cols, rows, 1, 1};
    const uint64_t strides[3] = {cols * 2, cols * rows * 2, cols * rows * 2};
    const uint32_t box[4] = {static_cast<uint32_t>(cwB), static_cast<uint32_t>(b_mn ? K : N / 2), 1, 1};
    int e = encode_tmap_16bit(&tmB, B, 4, dims, strides, box, b_sw);
    if (e) return e;
  }
  SelftestParams p{M, N, K, a_mn, b_mn, a_sw, b_sw, a_tmem, 0, static_cast<const __nv_bfloat16*>(A), D, nullptr};
  const size_t smem = ((static_cast<size_t>(128) * K * 2 + 1023) & ~size_t(1023)) + static_cast<size_t>(N / 2) * K * 2 + 1024;
  cudaError_t ce = cudaFuncSetAttribute(selftest_umma_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(smem));
  if (ce != cudaSuccess) return KATA_ERR_CUDA;
  selftest_umma_pair_kernel<<<2, 128, smem, reinterpret_cast<cudaStream_t>(stream)>>>(tmA, tmB, p);
  return from_cuda(cudaGetLastError());
}

namespace {
int selftest_launch(const void* A, const void* B, float* D, int M, int N, int K, int a_mn, int b_mn, int a_sw,
                    int b_sw, int a_tmem, int lane_off, kata_stream_t stream) {
  using namespace kata;
  if (!A || !B || !D) return KATA_ERR_INVALID;
  auto sw_ok = [](int s) { return s == 32 || s == 64 || s == 128; };
  if ((M != 128 && M != 64) || (M == 64 && a_tmem) || N < 16 || N > 256 || N % 16 || K < 16 || K > 256 ||
      K % 16 || !sw_ok(a_sw) || !sw_ok(b_sw))
    return KATA_ERR_SHAPE;
  const int cwA = a_sw / 2, cwB = b_sw / 2;
  if ((a_mn ? M : K) % cwA || (b_mn ? N : K) % cwB) return KATA_ERR_SHAPE;

  CUtensorMap tmA, tmB;
  // A: rows x cols row-major; box = (cw cols, all rows).
  {
    const uint64_t cols = a_mn ? M : K, rows = a_mn ? K : M;
    const uint64_t dims[4] = {cols, rows, 1, 1};
    const uint64_t strides[3] = {cols * 2, cols * rows * 2, cols * rows * 2};
    const uint32_t box[4] = {static_cast<uint32_t>(cwA), static_cast<uint32_t>(rows), 1, 1};
    int e = encode_tmap_16bit(&tmA, A, 4, dims, strides, box, a_sw);
    if (e) return e;
  }
  {
    const uint64_t cols = b_mn ? N : K, rows = b_mn ? K : N;
    const uint64_t dims[4] = {cols, rows, 1, 1};
    const uint64_t strides[3] = {cols * 2, cols * rows * 2, cols * rows * 2};
    const uint32_t box[4] = {static_cast<uint32_t>(cwB), static_cast<uint32_t>(rows), 1, 1};
    int e = encode_tmap_16bit(&tmB, B, 4, dims, strides, box, b_sw);
    if (e) return e;
  }
  SelftestParams p{M, N, K, a_mn, b_mn, a_sw, b_sw, a_tmem, lane_off, static_cast<const __nv_bfloat16*>(A), D,
                   nullptr};
  const size_t smem = ((static_cast<size_t>(M) * K * 2 + 1023) & ~size_t(1023)) + static_cast<size_t>(N) * K * 2 + 1024;
  cudaError_t ce = cudaFuncSetAttribute(selftest_umma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(smem));
  if (ce != cudaSuccess) return KATA_ERR_CUDA;
  selftest_umma_kernel<<<1, 128, smem, reinterpret_cast<cudaStream_t>(stream)>>>(tmA, tmB, p);
  return from_cuda(cudaGetLastError());
}
}  // namespace
