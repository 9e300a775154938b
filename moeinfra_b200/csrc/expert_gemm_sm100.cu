// Grouped NF4 expert GEMM (tcgen05) -- placeholder until the kernel lands.
#include "common.cuh"

namespace moe {
int launch_grouped_gemm_experts(const moe_nf4_expert_t*, int, const int32_t*, const uint16_t*,
                                int64_t, int, int, uint16_t*, uint16_t*, cudaStream_t) {
  return MOE_ERR_UNSUPPORTED;
}
}  // namespace moe
