// attn_internal.h -- attention entry points for other parts of this library (not exported).
#pragma once
#include "kata_b200.h"

namespace kata {
// kata_attn_bwd with the per-row delta_t (B,T,HQ fp32) supplied by the caller instead of
// <o_t, dO_t>; args->o is then not read and may be null.  delta_in == null: kata_attn_bwd.
int attn_bwd_impl(const kata_attn_bwd_args* a, const float* delta_in, kata_stream_t stream);
}  // namespace kata
