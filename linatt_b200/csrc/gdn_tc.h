// gdn_tc.h -- the tensor-core (tcgen05) gated delta rule for bf16 / fp16 inputs (gdn_tc.cu), called by
// the C-ABI entry points in gdn.cu when they choose that kernel family.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

#include "kata_b200.h"

namespace kata {
size_t gdn_tc_fwd_workspace_bytes(int B, int T, int HV, int NC);
size_t gdn_tc_bwd_workspace_bytes(int B, int T, int HV, int NC, bool reuse);
int gdn_tc_fwd(const kata_gdn_fwd_args* a, cudaStream_t st);
int gdn_tc_bwd(const kata_gdn_bwd_args* a, cudaStream_t st);
}  // namespace kata
