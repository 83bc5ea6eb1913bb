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
constexpr int kPhiRows = 16;                      // rows per block of the feature map
constexpr int kPhiChunks = kGramFP / 8;           // 18 chunks of 8 features per row
constexpr int kPhiThreads = kPhiRows * kPhiChunks;  // 288
constexpr int kMaxD = 128;

struct PhiJob {
  const __nv_bfloat16* x;  // (rows, D)
  __nv_bfloat16* phi;      // (rows, kGramFP)
  long long rows;
};

// Feature index f (e-major over e <= g) -> (e, g); 255 marks the zero padding past kGramF.
__device__ __forceinline__ void gram_pair(int f, unsigned char& e_out, unsigned char& g_out) {
  if (f >= kGramF) {
    e_out = g_out = 255;
    return;
  }
  int e = 0;
  while (f >= kGramE - e) {
    f -= kGramE - e;
    ++e;
  }
  e_out = static_cast<unsigned char>(e);
  g_out = static_cast<unsigned char>(e + f);
}

__device__ __forceinline__ void unpack8(uint4 u, float (&v)[8]) {
  const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __bfloat162float(h[i]);
}
__device__ __forceinline__ uint4 pack8(const float (&v)[8]) {
  uint4 u;
  u.x = pack2<__nv_bfloat16>(v[0], v[1]);
  u.y = pack2<__nv_bfloat16>(v[2], v[3]);
  u.z = pack2<__nv_bfloat16>(v[4], v[5]);
  u.w = pack2<__nv_bfloat16>(v[6], v[7]);
  return u;
}

// phi for up to two row sets (blockIdx.y), 16 rows per block: the rows are staged in shared memory,
// then thread (row, chunk) forms 8 features (M products each) and stores them as one 16-byte vector,
// so consecutive threads write consecutive 16 bytes of the (rows, 144) output.
__global__ void __launch_bounds__(kPhiThreads) gram_phi_kernel(PhiJob j0, PhiJob j1, int D, float scale) {
  const PhiJob j = blockIdx.y ? j1 : j0;
  __shared__ float xs[kPhiRows][kMaxD + 1];
  __shared__ unsigned char pe[kGramFP], pg[kGramFP];
  const int tid = threadIdx.x;
  if (tid < kGramFP) gram_pair(tid, pe[tid], pg[tid]);
  const long long r0 = static_cast<long long>(blockIdx.x) * kPhiRows;
  if (r0 >= j.rows) return;  // uniform over the block
  const int nv = D / 8;
  for (int i = tid; i < kPhiRows * nv; i += kPhiThreads) {
    const int r = i / nv, c = i % nv;
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (r0 + r < j.rows) unpack8(*reinterpret_cast<const uint4*>(j.x + (r0 + r) * D + c * 8), v);
#pragma unroll
    for (int e = 0; e < 8; ++e) xs[r][c * 8 + e] = v[e];
  }
  __syncthreads();
  const int r = tid / kPhiChunks, c = tid % kPhiChunks;
  if (r0 + r >= j.rows) return;
  const int M = D / kGramE;
  float out[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int f = c * 8 + i;
    float s = 0.f;
    if (pe[f] != 255) {
      const int e = pe[f], g = pg[f];
      for (int a = 0; a < M; ++a) s = fmaf(xs[r][a * kGramE + e], xs[r][a * kGramE + g], s);
      s *= e == g ? scale : scale * kSqrt2;
    }
    out[i] = s;
  }
  *reinterpret_cast<uint4*>(j.phi + (r0 + r) * kGramFP + c * 8) = pack8(out);
}

struct PhiBwdJob {
  const __nv_bfloat16* dphi;  // (rows, kGramFP)
  const __nv_bfloat16* x;     // (rows, D)
  __nv_bfloat16* dx;          // (rows, D)
  long long rows;
};

constexpr int kPbThreads = 256;

// dx for up to two row sets (blockIdx.y): 256 / (D / 8) rows per block staged in shared memory
// (d phi and x as fp32); thread (row, chunk) forms 8 outputs of one group a, each a 16-term
// product of a row of scale * Dsym with x_a, and stores them as one 16-byte vector.
__global__ void __launch_bounds__(kPbThreads) gram_phi_bwd_kernel(PhiBwdJob j0, PhiBwdJob j1, int D, float scale) {
  const PhiBwdJob j = blockIdx.y ? j1 : j0;
  constexpr int kRowsMax = kPbThreads / 8;  // D = 64
  __shared__ float ds[kRowsMax][kGramFP + 1];
  __shared__ float xs[kRowsMax][kMaxD + 1];
  __shared__ unsigned char gi[kGramE * kGramE];
  __shared__ float gc[kGramE * kGramE];
  const int tid = threadIdx.x;
  {  // (g, h) -> feature index of (min, max) and the coefficient of Dsym (scale folded in)
    const int g = tid / kGramE, h = tid % kGramE;
    const int e = g < h ? g : h, f = g < h ? h : g;
    gi[tid] = static_cast<unsigned char>(e * kGramE - e * (e - 1) / 2 + (f - e));
    gc[tid] = g == h ? 2.f * scale : kSqrt2 * scale;
  }
  const int cpr = D / 8;  // chunks (threads) per row
  const int rpb = kPbThreads / cpr;
  const long long r0 = static_cast<long long>(blockIdx.x) * rpb;
  if (r0 >= j.rows) return;  // uniform over the block
  for (int i = tid; i < rpb * kPhiChunks; i += kPbThreads) {
    const int r = i / kPhiChunks, c = i % kPhiChunks;
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (r0 + r < j.rows) unpack8(*reinterpret_cast<const uint4*>(j.dphi + (r0 + r) * kGramFP + c * 8), v);
#pragma unroll
    for (int e = 0; e < 8; ++e) ds[r][c * 8 + e] = v[e];
  }
  for (int i = tid; i < rpb * cpr; i += kPbThreads) {
    const int r = i / cpr, c = i % cpr;
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (r0 + r < j.rows) unpack8(*reinterpret_cast<const uint4*>(j.x + (r0 + r) * D + c * 8), v);
#pragma unroll
    for (int e = 0; e < 8; ++e) xs[r][c * 8 + e] = v[e];
  }
  __syncthreads();
  const int r = tid / cpr, c = tid % cpr;
  if (r0 + r >= j.rows) return;
  const int a = (c * 8) / kGramE, g0 = (c * 8) % kGramE;
  float xa[kGramE];
#pragma unroll
  for (int h = 0; h < kGramE; ++h) xa[h] = xs[r][a * kGramE + h];
  float out[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int g = g0 + i;
    float s = 0.f;
#pragma unroll
    for (int h = 0; h < kGramE; ++h) s = fmaf(gc[g * kGramE + h] * ds[r][gi[g * kGramE + h]], xa[h], s);
    out[i] = s;
  }
  *reinterpret_cast<uint4*>(j.dx + (r0 + r) * D + c * 8) = pack8(out);
}

size_t al256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }
size_t phi_bytes(long long rows) { return al256(static_cast<size_t>(rows) * kGramFP * 2); }

int launch_phi(PhiJob j0, PhiJob j1, int D, float scale, cudaStream_t st) {
  const long long rmax = j0.rows > j1.rows ? j0.rows : j1.rows;
  const long long nb = (rmax + kPhiRows - 1) / kPhiRows;
  if (nb > 0x7fffffffll) return KATA_ERR_SHAPE;
  gram_phi_kernel<<<dim3(static_cast<unsigned>(nb), j1.rows > 0 ? 2 : 1), kPhiThreads, 0, st>>>(j0, j1, D, scale);
  return from_cuda(cudaGetLastError());
}

int launch_phi_bwd(PhiBwdJob j0, PhiBwdJob j1, int D, float scale, cudaStream_t st) {
  const long long rmax = j0.rows > j1.rows ? j0.rows : j1.rows;
  const int rpb = kPbThreads / (D / 8);
  const long long nb = (rmax + rpb - 1) / rpb;
  if (nb > 0x7fffffffll) return KATA_ERR_SHAPE;
  gram_phi_bwd_kernel<<<dim3(static_cast<unsigned>(nb), j1.rows > 0 ? 2 : 1), kPbThreads, 0, st>>>(j0, j1, D, scale);
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
