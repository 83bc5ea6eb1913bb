// tc64.cuh -- 64 x 64 tile machinery for the chunked (64-token) tensor-core kernels: 16-bit tiles of
// 64 rows x 128 bytes in shared memory with the 128-byte swizzle, M = 64 tcgen05.mma chains into
// tensor memory, and the row <-> TMEM-lane mapping of an M = 64 accumulator (row m in lane
// (m % 16) + 32 (m / 16), plus 16 for a second copy issued at lane offset 16).  Shared by the gated
// delta rule (gdn_tc.cu) and the SPD delta-rule scans (delta_tc.cu).
#pragma once
#include <type_traits>

#include "attn_common.cuh"
#include "sm100.cuh"

namespace kata {
namespace tc64 {

constexpr uint32_t TB = 8192;  // a 64 x 64 16-bit tile: rows of 128 B, 128-byte swizzle

__device__ __forceinline__ uint8_t* align1k(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~static_cast<uintptr_t>(1023));
}

__device__ __forceinline__ uint32_t toff(int r, int c) { return swz_offset(r, c * 2, 128); }

// K-major operand: tile rows are the M (or N) index, the 64 columns of a row are K.
__device__ __forceinline__ uint64_t kdesc(const void* t) { return umma_smem_desc(smem_u32(t), 16, 1024, 128); }
// MN-major operand: tile rows are the K index, the 64 columns of a row are M (or N).
__device__ __forceinline__ uint64_t mdesc(const void* t) { return umma_smem_desc(smem_u32(t), TB, 1024, 128); }

// D (64 x 64, fp32, TMEM) (+)= A (64 x 64) B (64 x 64); issued by one thread, four K steps of 16.
template <bool BF, bool AMN, bool BMN>
__device__ __forceinline__ void mma64(uint32_t d, const void* a, const void* b, bool acc) {
  constexpr uint32_t idesc = umma_idesc_f16(64, 64, BF, AMN, BMN);
  const uint64_t ad = AMN ? mdesc(a) : kdesc(a);
  const uint64_t bd = BMN ? mdesc(b) : kdesc(b);
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    // K step: 32 bytes along a K-major row, or 16 rows (2048 bytes) of an MN-major tile
    const uint64_t ao = AMN ? static_cast<uint64_t>(kk * 128) : static_cast<uint64_t>(kk * 2);
    const uint64_t bo = BMN ? static_cast<uint64_t>(kk * 128) : static_cast<uint64_t>(kk * 2);
    umma_ss(d, ad + ao, bd + bo, idesc, (acc || kk > 0) ? 1u : 0u);
  }
}

// Row of the M = 64 accumulators this thread reads: slot = chunk (lane half), row = tile row.
struct RowMap {
  int slot, row;
  uint32_t lane;  // (32 * warp) << 16: the warp's TMEM lane base
};
__device__ __forceinline__ RowMap rowmap() {
  const int w = threadIdx.x >> 5, ln = threadIdx.x & 31;
  return {ln >> 4, w * 16 + (ln & 15), static_cast<uint32_t>(32 * w) << 16};
}

// Bounded wait on the CTA's MMA barrier; false (uniformly) when some thread timed out.
__device__ __forceinline__ bool wait_mma(uint64_t* bar, uint32_t& phase, volatile int* abort) {
  WaitCtx wc{nullptr, abort};
  const bool ok = mbar_wait(bar, phase, wc);
  phase ^= 1u;
  const bool fail = __syncthreads_or(!ok);
  tc_fence_after();
  return !fail;
}

template <typename T>
constexpr bool is_bf16() {
  return std::is_same<T, __nv_bfloat16>::value;
}

// tcgen05.ld / st take one TMEM address for the whole warp, so a lane half cannot name its own
// columns: the warp loads 32 columns and each lane half keeps its 16 (h = lane >> 4).
__device__ __forceinline__ void ld_quarter(uint32_t taddr, int h, float (&x)[16]) {
  uint32_t a[32];
  tmem_ld32(taddr, a);
  tmem_wait_ld();
#pragma unroll
  for (int j = 0; j < 16; ++j) x[j] = __uint_as_float(h ? a[16 + j] : a[j]);
}
// 16 values into row r, columns [c0, c0 + 16) of a tile (c0 a multiple of 8).
template <typename T>
__device__ __forceinline__ void st_row16(uint8_t* tile, int r, int c0, const float (&x)[16]) {
  const uint32_t base = smem_u32(tile);
#pragma unroll
  for (int c = 0; c < 2; ++c)
    st_shared_v4(base + toff(r, c0 + 8 * c), pack2<T>(x[8 * c], x[8 * c + 1]), pack2<T>(x[8 * c + 2], x[8 * c + 3]),
                 pack2<T>(x[8 * c + 4], x[8 * c + 5]), pack2<T>(x[8 * c + 6], x[8 * c + 7]));
}

// 16 bytes (8 16-bit values) at row r, column c (a multiple of 8) of a tile.
__device__ __forceinline__ void st_shared_v4_at(uint8_t* tile, int r, int c, uint32_t a, uint32_t b, uint32_t c2,
                                                uint32_t d) {
  st_shared_v4(smem_u32(tile) + toff(r, c), a, b, c2, d);
}
__device__ __forceinline__ void zero_tile(uint8_t* tile) {
  const uint32_t base = smem_u32(tile);
  for (int i = threadIdx.x; i < static_cast<int>(TB / 16); i += blockDim.x) st_shared_v4(base + 16 * i, 0u, 0u, 0u, 0u);
}
// The same MMA into lane offsets 0 and 16 (both lane halves of every warp receive all 64 rows).
template <bool BF, bool AMN, bool BMN>
__device__ __forceinline__ void mma64x2(uint32_t d, const void* a, const void* b, bool acc) {
  mma64<BF, AMN, BMN>(d, a, b, acc);
  mma64<BF, AMN, BMN>(d + (16u << 16), a, b, acc);
}

// Async 16-byte copy global -> shared (src-size 0 zero-fills), as in the fp32 scans; the
// copies of one thread complete in commit-group order.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(pred ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src, bool pred) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(dst), "l"(src), "r"(pred ? 4 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

}  // namespace tc64
}  // namespace kata
