// attn_tc_bwd.cu -- tcgen05 tensor-core backward of causal KATA-SPD attention (bf16 / fp16).
#include "attn_common.cuh"
#include "host_util.h"

namespace kata {

bool tc_bwd_supported(int dtype, int D, int Dv, int M, bool sum) {
  (void)dtype; (void)D; (void)Dv; (void)M; (void)sum;
  return false;
}

int tc_attn_bwd(const AttnBwdParams& p, int dtype, bool sum, cudaStream_t st) {
  (void)p; (void)dtype; (void)sum; (void)st;
  return KATA_ERR_UNSUPPORTED;
}

}  // namespace kata
