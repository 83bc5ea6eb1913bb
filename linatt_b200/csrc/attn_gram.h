// attn_gram.h -- the sum score on Gram features (attn_gram.cu), for the C-ABI entry points.
#pragma once
#include <cstddef>

#include "attn_common.cuh"

namespace kata {
// bf16 sum score with groups of 16 (D = 16 M, D in {64, 128}), Dv = 64, no decay
bool gram_supported(int dtype, int D, int Dv, int M, int score, bool decay);
// bf16 features of q and k (forward); features and their gradients (backward, on top of the
// parts-form workspace)
size_t gram_fwd_workspace_bytes(int B, int T, int H, int HQ);
size_t gram_bwd_workspace_bytes(int B, int T, int H, int HQ);
// p as for the parts form (q, k of width D, the caller's scale); ws 16-byte aligned
int gram_attn_fwd(const AttnFwdParams& p, void* ws, cudaStream_t st);
int gram_attn_bwd(const AttnBwdParams& p, void* ws, cudaStream_t st);
}  // namespace kata
