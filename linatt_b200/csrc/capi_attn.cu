// capi_attn.cu -- C-ABI entry points for causal KATA-SPD attention: argument validation and
// dispatch between the tcgen05 tensor-core kernels (parts form, or the sum score on Gram features)
// and the fp32-exact SIMT kernels.
#include "attn_common.cuh"
#include "attn_gram.h"
#include "attn_internal.h"
#include "host_util.h"

namespace kata {
bool simt_supported(int D, int Dv, int M, bool sum);
int simt_attn_fwd(const AttnFwdParams& p, int dtype, bool sum, cudaStream_t st);
int simt_attn_bwd(const AttnBwdParams& p, int dtype, bool sum, cudaStream_t st);
bool tc_fwd_supported(int dtype, int D, int Dv, int M, bool sum);
bool tc_bwd_supported(int dtype, int D, int Dv, int M, bool sum);
int tc_attn_fwd(const AttnFwdParams& p, int dtype, bool sum, cudaStream_t st);
int tc_attn_bwd(const AttnBwdParams& p, int dtype, bool sum, cudaStream_t st);
size_t tc_bwd_workspace_bytes(int B, int T, int HQ, bool decay, int nseq);
}  // namespace kata

using namespace kata;

namespace {

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_common(int dtype, int B, int T, int H, int HQ, int D, int Dv, int M, int score) {
  if (dtype != KATA_DTYPE_F32 && dtype != KATA_DTYPE_BF16 && dtype != KATA_DTYPE_F16) return KATA_ERR_DTYPE;
  if (B < 1 || T < 1 || H < 1 || HQ < 1 || D < 1 || Dv < 1 || M < 1) return KATA_ERR_SHAPE;
  if (HQ % H != 0 || D % M != 0) return KATA_ERR_SHAPE;
  if (score != KATA_SCORE_CONCAT && score != KATA_SCORE_SUM) return KATA_ERR_INVALID;
  if (static_cast<long long>(B) * T * HQ * (D > Dv ? D : Dv) >= (1ll << 40)) return KATA_ERR_SHAPE;
  return KATA_OK;
}

size_t al256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// Gram form wanted for these arguments (AUTO or TC_GRAM on a problem it covers)
bool gram_wanted(int algo, int dtype, int D, int Dv, int M, int score, bool decay) {
  return (algo == KATA_ALGO_AUTO || algo == KATA_ALGO_TC_GRAM) && gram_supported(dtype, D, Dv, M, score, decay);
}

// Packed documents: B = 1, at least one document, the tensor-core parts form (16-bit); KATA_OK
// when cu_seqlens is not given.
int varlen_check(const int* cu, int nseq, int B, int dtype, int algo) {
  if (!cu) return KATA_OK;
  if (B != 1 || nseq < 1) return KATA_ERR_SHAPE;
  if (dtype == KATA_DTYPE_F32 || algo == KATA_ALGO_SIMT || algo == KATA_ALGO_TC_GRAM) return KATA_ERR_UNSUPPORTED;
  return KATA_OK;
}

// Chooses the kernel family of the parts form: 1 = tensor cores, 2 = SIMT, or a negative error.
int choose_algo(int algo, bool tc_ok, bool simt_ok, int dtype) {
  if (algo == KATA_ALGO_TC) return tc_ok ? 1 : KATA_ERR_UNSUPPORTED;
  if (algo == KATA_ALGO_SIMT) return simt_ok ? 2 : KATA_ERR_UNSUPPORTED;
  if (algo != KATA_ALGO_AUTO) return KATA_ERR_INVALID;
  if (dtype != KATA_DTYPE_F32 && tc_ok) return 1;
  return simt_ok ? 2 : KATA_ERR_UNSUPPORTED;
}

}  // namespace

extern "C" size_t kata_attn_fwd_workspace_bytes(const kata_attn_fwd_args* a) {
  if (!a || check_common(a->dtype, a->B, a->T, a->H, a->HQ, a->D, a->Dv, a->M, a->score)) return 0;
  if (a->cu_seqlens || !gram_wanted(a->algo, a->dtype, a->D, a->Dv, a->M, a->score, a->c != nullptr)) return 0;
  return gram_fwd_workspace_bytes(a->B, a->T, a->H, a->HQ);
}

extern "C" int kata_attn_fwd(const kata_attn_fwd_args* a, kata_stream_t stream) {
  if (!a) return KATA_ERR_INVALID;
  int e = check_common(a->dtype, a->B, a->T, a->H, a->HQ, a->D, a->Dv, a->M, a->score);
  if (e) return e;
  if (!a->q || !a->k || !a->v || !a->o || !a->den) return KATA_ERR_INVALID;
  if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) || !aligned16(a->o)) return KATA_ERR_ALIGN;
  if ((e = varlen_check(a->cu_seqlens, a->num_seqs, a->B, a->dtype, a->algo))) return e;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (!a->cu_seqlens && gram_wanted(a->algo, a->dtype, a->D, a->Dv, a->M, a->score, a->c != nullptr)) {
    const size_t need = gram_fwd_workspace_bytes(a->B, a->T, a->H, a->HQ);
    const bool have = a->workspace && a->workspace_bytes >= need;
    if (a->algo == KATA_ALGO_TC_GRAM && !have) return KATA_ERR_WORKSPACE;
    if (have) {
      if (!aligned16(a->workspace)) return KATA_ERR_ALIGN;
      AttnFwdParams p{a->q, a->k, a->v, a->c, a->o, a->den, a->status, a->B, a->T, a->H, a->HQ, a->D, a->Dv, a->M,
                      a->HQ / a->H, a->scale, nullptr, 0};
      return gram_attn_fwd(p, a->workspace, st);
    }
  } else if (a->algo == KATA_ALGO_TC_GRAM) {
    return KATA_ERR_UNSUPPORTED;
  }
  const bool sum = a->score == KATA_SCORE_SUM;
  const bool tc_ok = tc_fwd_supported(a->dtype, a->D, a->Dv, a->M, sum) && !(a->c && sum);
  const int alg = choose_algo(a->algo, tc_ok, !a->cu_seqlens && simt_supported(a->D, a->Dv, a->M, sum), a->dtype);
  if (alg < 0) return alg;
  AttnFwdParams p{a->q, a->k, a->v, a->c, a->o, a->den, a->status, a->B, a->T, a->H, a->HQ, a->D, a->Dv, a->M,
                  a->HQ / a->H, a->scale, a->cu_seqlens, a->cu_seqlens ? a->num_seqs : 0};
  return alg == 1 ? tc_attn_fwd(p, a->dtype, sum, st) : simt_attn_fwd(p, a->dtype, sum, st);
}

extern "C" int kata_attn_algo(const kata_attn_fwd_args* a) {
  if (!a) return KATA_ERR_INVALID;
  int e = check_common(a->dtype, a->B, a->T, a->H, a->HQ, a->D, a->Dv, a->M, a->score);
  if (e) return e;
  if ((e = varlen_check(a->cu_seqlens, a->num_seqs, a->B, a->dtype, a->algo))) return e;
  if (!a->cu_seqlens && gram_wanted(a->algo, a->dtype, a->D, a->Dv, a->M, a->score, a->c != nullptr))
    return KATA_ALGO_TC_GRAM;
  if (a->algo == KATA_ALGO_TC_GRAM) return KATA_ERR_UNSUPPORTED;
  const bool sum = a->score == KATA_SCORE_SUM;
  const bool tc_ok = tc_fwd_supported(a->dtype, a->D, a->Dv, a->M, sum) &&
                     tc_bwd_supported(a->dtype, a->D, a->Dv, a->M, sum) && !(a->c && sum);
  const int alg = choose_algo(a->algo, tc_ok, !a->cu_seqlens && simt_supported(a->D, a->Dv, a->M, sum), a->dtype);
  if (alg < 0) return alg;
  return alg == 1 ? KATA_ALGO_TC : KATA_ALGO_SIMT;
}

size_t kata::attn_bwd_min_workspace_bytes(const kata_attn_bwd_args* a) {
  if (!a || a->B < 1 || a->T < 1 || a->HQ < 1) return 0;
  // fp32 delta = <o, dO> per (b, t, hq), plus 1/den and delta/den in a padded head-major layout
  // for the tensor-core key-tile kernel, and with decay (c given) a head-major copy of c (the SIMT
  // kernels use the first part only); TC_GRAM adds the features and their gradients
  const size_t base = tc_bwd_workspace_bytes(a->B, a->T, a->HQ, a->c != nullptr, a->cu_seqlens ? a->num_seqs : 0);
  if (a->algo != KATA_ALGO_TC_GRAM || a->H < 1) return base;
  return al256(base) + gram_bwd_workspace_bytes(a->B, a->T, a->H, a->HQ);
}

extern "C" size_t kata_attn_bwd_workspace_bytes(const kata_attn_bwd_args* a) {
  if (!a || a->B < 1 || a->T < 1 || a->HQ < 1) return 0;
  const size_t base = tc_bwd_workspace_bytes(a->B, a->T, a->HQ, a->c != nullptr, a->cu_seqlens ? a->num_seqs : 0);
  if (a->cu_seqlens || a->H < 1 || check_common(a->dtype, a->B, a->T, a->H, a->HQ, a->D, a->Dv, a->M, a->score) ||
      !gram_wanted(a->algo, a->dtype, a->D, a->Dv, a->M, a->score, a->c != nullptr))
    return base;
  return al256(base) + gram_bwd_workspace_bytes(a->B, a->T, a->H, a->HQ);
}

int kata::attn_bwd_impl(const kata_attn_bwd_args* a, const float* delta_in, kata_stream_t stream) {
  if (!a) return KATA_ERR_INVALID;
  int e = check_common(a->dtype, a->B, a->T, a->H, a->HQ, a->D, a->Dv, a->M, a->score);
  if (e) return e;
  if (!a->q || !a->k || !a->v || (!a->o && !delta_in) || !a->den || !a->dout || !a->dq || !a->dk || !a->dv)
    return KATA_ERR_INVALID;
  if (a->c && !a->dc) return KATA_ERR_INVALID;
  if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) || !aligned16(a->o) || !aligned16(a->dout) ||
      !aligned16(a->dq) || !aligned16(a->dk) || !aligned16(a->dv))
    return KATA_ERR_ALIGN;
  if (a->phases < 0 || a->phases > 2) return KATA_ERR_INVALID;
  if ((e = varlen_check(a->cu_seqlens, a->num_seqs, a->B, a->dtype, a->algo))) return e;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int nseq = a->cu_seqlens ? a->num_seqs : 0;
  AttnBwdParams p{a->q,  a->k,  a->v,  a->o,  a->den, a->dout, a->c,  a->dq, a->dk,           a->dv,
                  a->dc, static_cast<float*>(a->workspace), a->status, a->B, a->T, a->H, a->HQ, a->D, a->Dv, a->M,
                  a->HQ / a->H, a->scale, a->phases, delta_in, a->cu_seqlens, nseq};
  const size_t base = tc_bwd_workspace_bytes(a->B, a->T, a->HQ, a->c != nullptr, nseq);
  if (!a->cu_seqlens && gram_wanted(a->algo, a->dtype, a->D, a->Dv, a->M, a->score, a->c != nullptr)) {
    const size_t need = al256(base) + gram_bwd_workspace_bytes(a->B, a->T, a->H, a->HQ);
    const bool have = a->workspace && a->workspace_bytes >= need;
    if (a->algo == KATA_ALGO_TC_GRAM && !have) return KATA_ERR_WORKSPACE;
    if (have) {
      if (!aligned16(a->workspace)) return KATA_ERR_ALIGN;
      return gram_attn_bwd(p, static_cast<uint8_t*>(a->workspace) + al256(base), st);
    }
  } else if (a->algo == KATA_ALGO_TC_GRAM) {
    return KATA_ERR_UNSUPPORTED;
  }
  if (base && (!a->workspace || a->workspace_bytes < base)) return KATA_ERR_WORKSPACE;
  const bool sum = a->score == KATA_SCORE_SUM;
  const bool tc_ok = tc_bwd_supported(a->dtype, a->D, a->Dv, a->M, sum) && !(a->c && sum);
  const int alg = choose_algo(a->algo, tc_ok, !a->cu_seqlens && simt_supported(a->D, a->Dv, a->M, sum), a->dtype);
  if (alg < 0) return alg;
  return alg == 1 ? tc_attn_bwd(p, a->dtype, sum, st) : simt_attn_bwd(p, a->dtype, sum, st);
}

extern "C" int kata_attn_bwd(const kata_attn_bwd_args* a, kata_stream_t stream) {
  return kata::attn_bwd_impl(a, nullptr, stream);
}
