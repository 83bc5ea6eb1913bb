// attn_gram.cu -- the sum score on Gram features: feature map, its adjoint, and the forward /
// backward around the linear-score tensor-core kernels (GRAM mode of attn_tc_fwd.cu / attn_tc_bwd.cu).
//
// The sum score (kata/kernels/parallel_kata.py:202-345; backward kata/parallel_kata_attn.py:579-653
// and kata/kernels/parallel_kata_sum.py) with M groups of E = D / M,
//   A[t,s] = scale^2 sum_{a,b} (q_a[t] . k_b[s])^2 = scale^2 tr(G(q_t) G(k_s)),  G(x) = sum_a x_a x_a^T,
// is a linear score over the E (E + 1) / 2 entries of the symmetric E x E matrix G:
//   A[t,s] = <phi(q_t), phi(k_s)>,  phi(x)_(e,f) = scale c_ef G(x)_ef,  e <= f,  c_ee = 1, c_ef = sqrt 2.
// For E = 16 (M = 4 at D = 64, M = 8 at D = 128) that is 136 features (144 stored columns): one
// K = 144 MMA per 128 x 128 score tile and no per-element squares, where the parts form runs M^2
// K = 16 MMAs and M^2 squares per score element.  The backward maps d phi back to the inputs:
//   dx_a = scale Dsym dphi x_a,  Dsym_gg = 2 dphi_(g,g),  Dsym_gh = sqrt 2 dphi_(min(g,h), max(g,h)).
// The features are bf16 (8-bit mantissa, like the MMA operands of the parts form); a feature sum
// carries off-diagonal terms of either sign, so A near 0 can round to a tiny negative value where
// the parts form's sum of squares cannot.
#include "attn_common.cuh"
#include "attn_tc_common.cuh"
#include "attn_gram.h"

namespace kata {
int tc_attn_fwd_gram(const AttnFwdParams& p, cudaStream_t st);
int tc_attn_bwd_gram(const AttnBwdParams& p, cudaStream_t st);

namespace {

constexpr float kSqrt2 = 1.4142135623730951f;
constexpr int kPhiThreads = 128;

struct PhiJob {
  const __nv_bfloat16* x;  // (rows, D)
  __nv_bfloat16* phi;      // (rows, kGramFP)
  long long rows;
};

__device__ __forceinline__ void unpack8(uint4 u, float* v) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
__device__ __forceinline__ uint4 pack8(const float (&v)[8]) {
  uint4 u;
  u.x = pack2<__nv_bfloat16>(v[0], v[1]);
  u.y = pack2<__nv_bfloat16>(v[2], v[3]);
  u.z = pack2<__nv_bfloat16>(v[4], v[5]);
  u.w = pack2<__nv_bfloat16>(v[6], v[7]);
  return u;
}

// Feature index of (e, g), e <= g, e-major over the upper triangle of the 16 x 16 Gram matrix.
__host__ __device__ constexpr int gram_index(int e, int g) { return e * kGramE - e * (e - 1) / 2 + (g - e); }

// phi for up to two row sets (blockIdx.y): one thread per row, the row's D values in registers and
// the 136 features formed with compile-time indices (fully unrolled, M products each), stored as
// 17 16-byte vectors plus one of zero padding.  HBM-bound: 2 D bytes read, 288 written per row.
template <int M>
__global__ void __launch_bounds__(kPhiThreads) gram_phi_kernel(PhiJob j0, PhiJob j1, float scale) {
  constexpr int D = kGramE * M;
  const PhiJob j = blockIdx.y ? j1 : j0;
  const long long row = static_cast<long long>(blockIdx.x) * kPhiThreads + threadIdx.x;
  if (row >= j.rows) return;
  float x[D];
  const uint4* src = reinterpret_cast<const uint4*>(j.x + row * D);
#pragma unroll
  for (int c = 0; c < D / 8; ++c) unpack8(__ldg(src + c), x + 8 * c);
  uint4* dst = reinterpret_cast<uint4*>(j.phi + row * kGramFP);
  float out[8];
#pragma unroll
  for (int e = 0; e < kGramE; ++e) {
#pragma unroll
    for (int g = e; g < kGramE; ++g) {
      float s = 0.f;
#pragma unroll
      for (int a = 0; a < M; ++a) s = fmaf(x[a * kGramE + e], x[a * kGramE + g], s);
      const int f = gram_index(e, g);
      out[f & 7] = s * (e == g ? scale : scale * kSqrt2);
      if ((f & 7) == 7) dst[f >> 3] = pack8(out);
    }
  }
  static_assert(kGramF == 17 * 8 && kGramFP == 18 * 8, "136 features in 17 vectors, one of padding");
  dst[17] = make_uint4(0u, 0u, 0u, 0u);
}

struct PhiBwdJob {
  const __nv_bfloat16* dphi;  // (rows, kGramFP)
  const __nv_bfloat16* x;     // (rows, D)
  __nv_bfloat16* dx;          // (rows, D)
  long long rows;
};

// bf16 value i of a row held as packed pairs
__device__ __forceinline__ float bf_at(const uint32_t* w, int i) {
  return __uint_as_float((i & 1) ? (w[i >> 1] & 0xffff0000u) : (w[i >> 1] << 16));
}

// dx for up to two row sets (blockIdx.y): one thread per (row, group a), M consecutive threads per
// row.  dx_a[g] = scale (2 dphi_gg x_a[g] + sqrt 2 sum_{h != g} dphi_(g,h) x_a[h])
//              = sqrt 2 scale (sum_{h != g} dphi_(g,h) x_a[h] + sqrt 2 dphi_gg x_a[g]),
// with the row's d phi kept as 68 packed bf16 pairs in registers (compile-time indices).
template <int M>
__global__ void __launch_bounds__(kPhiThreads) gram_phi_bwd_kernel(PhiBwdJob j0, PhiBwdJob j1, float scale) {
  constexpr int D = kGramE * M;
  const PhiBwdJob j = blockIdx.y ? j1 : j0;
  const long long t = static_cast<long long>(blockIdx.x) * kPhiThreads + threadIdx.x;
  const long long row = t / M;
  const int a = static_cast<int>(t % M);
  if (row >= j.rows) return;
  uint32_t w[kGramF / 2];
  const uint4* dsrc = reinterpret_cast<const uint4*>(j.dphi + row * kGramFP);
#pragma unroll
  for (int c = 0; c < kGramF / 8; ++c) {
    const uint4 u = __ldg(dsrc + c);
    w[4 * c] = u.x;
    w[4 * c + 1] = u.y;
    w[4 * c + 2] = u.z;
    w[4 * c + 3] = u.w;
  }
  float x[kGramE];
  const uint4* xsrc = reinterpret_cast<const uint4*>(j.x + row * D + a * kGramE);
  unpack8(__ldg(xsrc), x);
  unpack8(__ldg(xsrc + 1), x + 8);
  const float sc = kSqrt2 * scale;
  float out[kGramE];
#pragma unroll
  for (int g = 0; g < kGramE; ++g) {
    float s = kSqrt2 * bf_at(w, gram_index(g, g)) * x[g];
#pragma unroll
    for (int h = 0; h < kGramE; ++h)
      if (h != g) s = fmaf(bf_at(w, h < g ? gram_index(h, g) : gram_index(g, h)), x[h], s);
    out[g] = s * sc;
  }
  uint4* dst = reinterpret_cast<uint4*>(j.dx + row * D + a * kGramE);
  float o8[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) o8[i] = out[i];
  dst[0] = pack8(o8);
#pragma unroll
  for (int i = 0; i < 8; ++i) o8[i] = out[8 + i];
  dst[1] = pack8(o8);
}

size_t al256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }
size_t phi_bytes(long long rows) { return al256(static_cast<size_t>(rows) * kGramFP * 2); }

int launch_phi(PhiJob j0, PhiJob j1, int D, float scale, cudaStream_t st) {
  const long long rmax = j0.rows > j1.rows ? j0.rows : j1.rows;
  const long long nb = (rmax + kPhiThreads - 1) / kPhiThreads;
  if (nb > 0x7fffffffll) return KATA_ERR_SHAPE;
  const dim3 grid(static_cast<unsigned>(nb), j1.rows > 0 ? 2 : 1);
  if (D == 64)
    gram_phi_kernel<4><<<grid, kPhiThreads, 0, st>>>(j0, j1, scale);
  else if (D == 128)
    gram_phi_kernel<8><<<grid, kPhiThreads, 0, st>>>(j0, j1, scale);
  else
    return KATA_ERR_UNSUPPORTED;
  return from_cuda(cudaGetLastError());
}

int launch_phi_bwd(PhiBwdJob j0, PhiBwdJob j1, int D, float scale, cudaStream_t st) {
  const long long rmax = j0.rows > j1.rows ? j0.rows : j1.rows;
  const int M = D / kGramE;
  const long long nb = (rmax * M + kPhiThreads - 1) / kPhiThreads;
  if (nb > 0x7fffffffll) return KATA_ERR_SHAPE;
  const dim3 grid(static_cast<unsigned>(nb), j1.rows > 0 ? 2 : 1);
  if (D == 64)
    gram_phi_bwd_kernel<4><<<grid, kPhiThreads, 0, st>>>(j0, j1, scale);
  else if (D == 128)
    gram_phi_bwd_kernel<8><<<grid, kPhiThreads, 0, st>>>(j0, j1, scale);
  else
    return KATA_ERR_UNSUPPORTED;
  return from_cuda(cudaGetLastError());
}

}  // namespace

bool gram_supported(int dtype, int D, int Dv, int M, int score, bool decay) {
  return dtype == KATA_DTYPE_BF16 && score == KATA_SCORE_SUM && !decay && M >= 1 && D == kGramE * M &&
         (D == 64 || D == 128) && Dv == 64;
}

size_t gram_fwd_workspace_bytes(int B, int T, int H, int HQ) {
  return phi_bytes(static_cast<long long>(B) * T * HQ) + phi_bytes(static_cast<long long>(B) * T * H);
}

size_t gram_bwd_workspace_bytes(int B, int T, int H, int HQ) { return 2 * gram_fwd_workspace_bytes(B, T, H, HQ); }

int gram_attn_fwd(const AttnFwdParams& p, void* ws, cudaStream_t st) {
  const long long rq = static_cast<long long>(p.B) * p.T * p.HQ, rk = static_cast<long long>(p.B) * p.T * p.H;
  auto* pq = static_cast<__nv_bfloat16*>(ws);
  auto* pk = reinterpret_cast<__nv_bfloat16*>(static_cast<uint8_t*>(ws) + phi_bytes(rq));
  int e = launch_phi(PhiJob{static_cast<const __nv_bfloat16*>(p.q), pq, rq},
                     PhiJob{static_cast<const __nv_bfloat16*>(p.k), pk, rk}, p.D, p.scale, st);
  if (e) return e;
  AttnFwdParams g = p;
  g.q = pq;
  g.k = pk;
  g.D = kGramFP;
  g.M = 1;
  g.scale = 1.f;
  return tc_attn_fwd_gram(g, st);
}

int gram_attn_bwd(const AttnBwdParams& p, void* ws, cudaStream_t st) {
  const long long rq = static_cast<long long>(p.B) * p.T * p.HQ, rk = static_cast<long long>(p.B) * p.T * p.H;
  uint8_t* w = static_cast<uint8_t*>(ws);
  auto* pq = reinterpret_cast<__nv_bfloat16*>(w);
  auto* pk = reinterpret_cast<__nv_bfloat16*>(w + phi_bytes(rq));
  auto* dpq = reinterpret_cast<__nv_bfloat16*>(w + phi_bytes(rq) + phi_bytes(rk));
  auto* dpk = reinterpret_cast<__nv_bfloat16*>(w + 2 * phi_bytes(rq) + phi_bytes(rk));
  // q and k the same tensor (the delta rule's erase-term backward, q := k): one feature map
  const bool same = p.q == p.k && p.HQ == p.H;
  const auto* xq = static_cast<const __nv_bfloat16*>(p.q);
  const auto* xk = static_cast<const __nv_bfloat16*>(p.k);
  int e = KATA_OK;
  if (p.phases != 2) {  // a dk/dv-only call reads the features of the dq pass on this workspace
    e = same ? launch_phi(PhiJob{xk, pk, rk}, PhiJob{nullptr, nullptr, 0}, p.D, p.scale, st)
             : launch_phi(PhiJob{xq, pq, rq}, PhiJob{xk, pk, rk}, p.D, p.scale, st);
    if (e) return e;
  }
  AttnBwdParams g = p;
  g.q = same ? pk : pq;
  g.k = pk;
  g.dq = dpq;
  g.dk = dpk;
  g.D = kGramFP;
  g.M = 1;
  g.scale = 1.f;
  if ((e = tc_attn_bwd_gram(g, st))) return e;
  const PhiBwdJob jq{dpq, xq, static_cast<__nv_bfloat16*>(p.dq), rq};
  const PhiBwdJob jk{dpk, xk, static_cast<__nv_bfloat16*>(p.dk), rk};
  const PhiBwdJob none{nullptr, nullptr, nullptr, 0};
  if (p.phases == 1) return launch_phi_bwd(jq, none, p.D, p.scale, st);
  if (p.phases == 2) return launch_phi_bwd(jk, none, p.D, p.scale, st);
  return launch_phi_bwd(jq, jk, p.D, p.scale, st);
}

}  // namespace kata
