// attn_tc_common.cuh -- tile geometry, UMMA descriptor helpers and tensor-map construction
// shared by the tcgen05 forward and backward attention kernels.
//
// Shared-memory tile layout.  A [128 rows][W cols] 16-bit tile is stored as W/CW TMA boxes of
// [128 rows][CW cols], each box dense with CW*2-byte rows and the matching 32/64/128-byte swizzle
// (CW = min(group width, 64)).  For the score operands the box width equals the group width E
// (or 64 when E >= 64), so every group g of q/k is a whole number of boxes: its K-major slices
// (score MMAs) and its MN-major slices (gradient MMAs) are both canonical UMMA layouts.
#pragma once
#include "attn_common.cuh"
#include "host_util.h"
#include "sm100.cuh"

namespace kata {

constexpr int kTile = 128;  // rows of every q/k/v/dO tile (= UMMA M)

// K-major descriptor of K-step kk (16 elements) inside columns [g*E, (g+1)*E) of a tile stored as
// boxes of CW columns, 128 rows each.
template <int CW>
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int g, int E, int kk) {
  const int col = g * E + kk * 16;
  const uint32_t box = static_cast<uint32_t>(col / CW);
  const uint32_t within = static_cast<uint32_t>(col % CW) * 2u;
  return umma_smem_desc(base + box * (kTile * CW * 2u) + within, 16u, 8u * CW * 2u, CW * 2);
}

// Descriptor increment (in 16-byte units, added to the start-address field) from K-step 0 to K-step
// kk of a K-major operand stored as boxes of CW columns: 16 elements = 32 bytes per step, and a new
// box every CW elements.  Compile-time after unrolling; the start address never carries out of
// its 14-bit field because shared-memory addresses are below 256 KB.
template <int CW>
__device__ __forceinline__ constexpr uint64_t kstep(int kk) {
  return static_cast<uint64_t>(((kk * 16 / CW) * (kTile * CW * 2) + (kk * 16 % CW) * 2) >> 4);
}
// Same for an MN-major operand: each K-step is 16 rows of CW*2 bytes.
template <int CW>
__device__ __forceinline__ constexpr uint64_t mnstep(int kk) {
  return static_cast<uint64_t>((kk * 16 * CW * 2) >> 4);
}

// MN-major descriptor of K-step kk (16 rows of the tile) for the N extent starting at box
// `box0` of a tile stored as boxes of CW columns (the N extent may span several boxes, LBO apart).
template <int CW>
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t base, int box0, int kk) {
  const uint32_t box_bytes = kTile * CW * 2u;
  return umma_smem_desc(base + static_cast<uint32_t>(box0) * box_bytes + static_cast<uint32_t>(kk) * 16u * (CW * 2u),
                        box_bytes, 8u * CW * 2u, CW * 2);
}

// Descriptor arithmetic without rebuilding descriptors.  The start-address field holds the byte
// address >> 4 in the low bits, so moving an operand by a multiple of 16 bytes is a plain add of
// (bytes >> 4) to the descriptor (no carry out of the 14-bit field: shared-memory addresses stay
// below 256 KB).  The MMA issuer is one thread whose every integer op is on the critical path of
// the tensor pipe (a descriptor rebuilt per chain costs more issue time than a 128x128x16 MMA
// takes to execute), so the issue loops use a base descriptor plus these compile-time offsets.
__host__ __device__ constexpr uint64_t desc_units(uint32_t bytes) { return static_cast<uint64_t>(bytes >> 4); }
// Offset of K-major group g (columns [g*E, (g+1)*E)) from group 0 of the same tile.
template <int CW>
__host__ __device__ constexpr uint64_t kmajor_goff(int g, int E) {
  return desc_units(static_cast<uint32_t>((g * E / CW) * (kTile * CW * 2) + (g * E % CW) * 2));
}
// Offset of the MN-major N extent starting at box `box0` from box 0 of the same tile.
template <int CW>
__host__ __device__ constexpr uint64_t mnmajor_boff(int box0) {
  return desc_units(static_cast<uint32_t>(box0 * kTile * CW * 2));
}

// K-major descriptor of K-step kk of a [128][128] 16-bit tile written by threads as two
// 128B-swizzled boxes of 64 columns (P / dA tiles).
__device__ __forceinline__ uint64_t kmajor128_desc(uint32_t base, int kk) {
  return umma_smem_desc(base + static_cast<uint32_t>(kk >> 2) * 16384u + static_cast<uint32_t>(kk & 3) * 32u, 16u,
                        1024u, 128);
}

// Thread-side store of 8 consecutive 16-bit values (one 16-byte chunk) of row `row`, columns
// [col0, col0+8) of a [128][128] tile stored as two 128B-swizzled boxes of 64 columns.
__device__ __forceinline__ void st_tile128(uint32_t base, int row, int col0, uint32_t w0, uint32_t w1, uint32_t w2,
                                           uint32_t w3) {
  const uint32_t box = static_cast<uint32_t>(col0 >> 6);
  const uint32_t byte = static_cast<uint32_t>(col0 & 63) * 2u;
  st_shared_v4(base + box * 16384u + swz_offset(static_cast<uint32_t>(row), byte, 128), w0, w1, w2, w3);
}

// TMEM column (relative to a 128-column slot) of K-step kk of a packed 16-bit A operand written
// by the two column halves of the compute warpgroups: each half stores its 64 values as 32
// packed words at the start of its own 64-column half, i.e. slot columns [0,32) and [64,96).
__device__ __forceinline__ uint32_t packed_col(int kk) {
  return static_cast<uint32_t>(8 * kk + (kk >= 4 ? 32 : 0));
}

// Tensor map over a time-major (B, T, heads, W) 16-bit tensor with boxes [cw cols][1][128 rows][1].
inline int make_tm_tokens(CUtensorMap* tm, const void* base, int B, int T, int heads, int W, int cw) {
  const uint64_t es = 2;
  const uint64_t dims[4] = {static_cast<uint64_t>(W), static_cast<uint64_t>(heads), static_cast<uint64_t>(T),
                            static_cast<uint64_t>(B)};
  const uint64_t str[3] = {W * es, W * es * heads, W * es * heads * T};
  const uint32_t box[4] = {static_cast<uint32_t>(cw), 1, kTile, 1};
  return encode_tmap_16bit(tm, base, 4, dims, str, box, cw * 2);
}

template <int W>
struct BoxW {
  static constexpr int value = W < 64 ? W : 64;
};

// Packed documents (cu_seqlens): every document is cut into its own 128-row tiles, and the tiles of
// all documents are numbered in document order.  Tile `tile` -> its document's first and one-past-
// last row, the tile's index j inside the document, the document's tile count and the number of
// the document's first tile.  The whole warp calls it with the same arguments (a 32-wide scan over
// the documents: running maximum of the offsets, tile counts, an inclusive prefix sum by shuffles,
// a ballot for the owner); false past the last tile.  Zero-length documents own no tile.  The
// offsets are normalised on the fly: each is clamped to [0, T] and raised to the largest offset
// before it, so the documents come out disjoint, ordered and inside [0, T] whatever the array holds
// (a valid array is unchanged) and every tile, row and vector index stays in bounds.
struct SeqTile {
  int start, end, j, ntiles, base;
};
__device__ __forceinline__ bool varlen_tile(const int* cu, int nseq, int T, int tile, SeqTile& out) {
  const int lane = threadIdx.x & 31;
  int base = 0;                       // tiles of the documents before this group of 32
  int carry = min(max(cu[0], 0), T);  // largest offset so far
  for (int n0 = 0; n0 < nseq; n0 += 32) {
    const int n = n0 + lane;
    int e = n < nseq ? min(max(cu[n + 1], 0), T) : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {  // inclusive running maximum over the lanes
      const int v = __shfl_up_sync(0xffffffffu, e, o);
      if (lane >= o) e = max(e, v);
    }
    e = max(e, carry);
    int s = __shfl_up_sync(0xffffffffu, e, 1);
    if (lane == 0) s = carry;
    const int nt = n < nseq ? (e - s + kTile - 1) / kTile : 0;
    int incl = nt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    const int excl = incl - nt;
    const unsigned own = __ballot_sync(0xffffffffu, nt > 0 && tile >= base + excl && tile < base + incl);
    if (own) {
      const int src = __ffs(own) - 1;
      out.start = __shfl_sync(0xffffffffu, s, src);
      out.end = __shfl_sync(0xffffffffu, e, src);
      out.ntiles = __shfl_sync(0xffffffffu, nt, src);
      out.base = base + __shfl_sync(0xffffffffu, excl, src);
      out.j = tile - out.base;
      return true;
    }
    base += __shfl_sync(0xffffffffu, incl, 31);
    carry = __shfl_sync(0xffffffffu, e, 31);
  }
  return false;
}
// Upper bound on the tiles of T packed rows in nseq documents (each document wastes < 1 tile).
__host__ __device__ inline int varlen_tile_bound(int T, int nseq) { return (T + kTile - 1) / kTile + nseq; }

// Sum score on Gram features.  With groups of E = 16 (D = 16 M) the sum score is a linear score
//   A[t,s] = scale^2 sum_{a,b} (q_a . k_b)^2 = scale^2 <G(q_t), G(k_s)>_F = <phi(q_t), phi(k_s)>,
//   G(x) = sum_a x_a x_a^T (16 x 16, symmetric),  phi(x)_(e,f) = scale c_ef G(x)_ef  (e <= f,
//   c_ee = 1, c_ef = sqrt 2),
// over kGramF = 136 features, stored as kGramFP = 144 columns (zero-padded to a whole number of
// 16-column MMA K-steps).  The tensor-core kernels run it as M = 1 with D = kGramFP, no squaring
// (GRAM), and the feature tiles in 32-byte-swizzled boxes of 16 columns.
constexpr int kGramE = 16;
constexpr int kGramF = kGramE * (kGramE + 1) / 2;
constexpr int kGramFP = 144;
template <int E, bool GRAM>
struct ScoreBoxW {
  static constexpr int value = GRAM ? 16 : BoxW<E>::value;
};

}  // namespace kata
