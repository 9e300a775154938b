// Status strings, build identification and the launch counter of the C ABI.
#include <atomic>

#include "common.cuh"

namespace moe {
namespace {
std::atomic<unsigned long long> g_launches{0};
}
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
}  // namespace moe

extern "C" uint64_t moe_launch_count(void) {
  return moe::g_launches.load(std::memory_order_relaxed);
}

extern "C" const char* moe_status_string(int status) {
  switch (status) {
    case MOE_OK: return "ok";
    case MOE_ERR_INVALID_ARG: return "invalid argument";
    case MOE_ERR_UNSUPPORTED: return "unsupported shape or configuration";
    case MOE_ERR_CUDA: return "CUDA launch or runtime error";
    case MOE_ERR_WORKSPACE: return "workspace missing or too small";
    case MOE_ERR_ALIGNMENT: return "pointer not 16-byte aligned";
    case MOE_ERR_TIMEOUT: return "device wait timed out";
    default: return "unknown status";
  }
}

extern "C" const char* moe_version(void) { return "moe_b200 sm_100a 0.1"; }

namespace moe {
// Set to 1 by any kernel whose bounded wait timed out; read and cleared by
// moe_take_device_error().
__device__ int g_wait_error = 0;
}  // namespace moe

namespace moe {
int gemm_take_error(int* value);    // expert_gemm_sm100.cu
int decode_take_error(int* value);  // expert_decode.cu
}

extern "C" int moe_take_device_error(int* value) {
  if (!value) return MOE_ERR_INVALID_ARG;
  int gemm = 0;
  if (moe::gemm_take_error(&gemm) != MOE_OK) return MOE_ERR_CUDA;
  int decode = 0;
  if (moe::decode_take_error(&decode) != MOE_OK) return MOE_ERR_CUDA;
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, moe::g_wait_error, sizeof(int)) != cudaSuccess) return MOE_ERR_CUDA;
  const int zero = 0;
  if (cudaMemcpyToSymbol(moe::g_wait_error, &zero, sizeof(int)) != cudaSuccess) return MOE_ERR_CUDA;
  *value = v | gemm | decode;
  return MOE_OK;
}
