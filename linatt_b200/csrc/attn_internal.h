// attn_internal.h -- attention entry points for other parts of this library (not exported).
#pragma once
#include "kata_b200.h"

namespace kata {
// kata_attn_bwd with the per-row delta_t (B,T,HQ fp32) supplied by the caller instead of
// <o_t, dO_t>; args->o is then not read and may be null.  delta_in == null: kata_attn_bwd.
int attn_bwd_impl(const kata_attn_bwd_args* a, const float* delta_in, kata_stream_t stream);
// Smallest workspace kata_attn_bwd accepts for these arguments: the parts-form size, or for
// algo == KATA_ALGO_TC_GRAM the Gram-form size (AUTO takes the Gram form only when given
// kata_attn_bwd_workspace_bytes(), which includes it).
size_t attn_bwd_min_workspace_bytes(const kata_attn_bwd_args* a);
}  // namespace kata
