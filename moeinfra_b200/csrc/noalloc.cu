// moe_layer_forward_noalloc: moe_layer_forward with its scratch taken from a
// file-scope device array instead of a caller-provided workspace.
//
// The array is a module global: each device gets its own copy when the
// library's module is loaded on that device, and its address is looked up once
// per device with cudaGetSymbolAddress and cached.  The lookup may load the
// module, so the first call on a device belongs before any stream capture.
// One array per device means calls that overlap on one device (different
// streams, or host threads, without ordering between them) race on it.
// Nothing in it has to start at zero: every scratch byte the layer reads
// (expert offsets, sorted pairs, SwiGLU activations, split-K partials) is
// written earlier in the same call.
#include <mutex>

#include "common.cuh"

namespace moe {
bool decode_supported(int hidden, int inter);  // expert_decode.cu
size_t layer_workspace_bytes(int64_t T, int hidden, int inter, int E, int k,
                             bool split_k);  // layer.cu

namespace {

constexpr size_t kNoAllocScratch = MOE_NOALLOC_SCRATCH_BYTES;
__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratch];

std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return MOE_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return MOE_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess) return MOE_ERR_CUDA;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return MOE_OK;
}

}  // namespace
}  // namespace moe

extern "C" int moe_layer_forward_noalloc(const uint16_t* h, const uint16_t* wg,
                                         const moe_nf4_expert_t* experts, int E, int k, int64_t T,
                                         int hidden, int inter, uint16_t* out, int64_t* indices,
                                         float* weights, void* stream) {
  using namespace moe;
  // The same argument checks as moe_layer_forward, before the size check, so
  // a bad call reports what is wrong with it rather than a size.
  if (T < 0 || E < 1 || E > MOE_MAX_EXPERTS || k < 1 || k > E || k > 8) return MOE_ERR_INVALID_ARG;
  if (!decode_supported(hidden, inter)) return MOE_ERR_UNSUPPORTED;
  if (T == 0) return MOE_OK;
  // The layer's optional split-K partials are used only when they fit too.
  if (layer_workspace_bytes(T, hidden, inter, E, k, false) > kNoAllocScratch)
    return MOE_ERR_WORKSPACE;
  void* scratch = nullptr;
  const int st = scratch_address(&scratch);
  if (st != MOE_OK) return st;
  return moe_layer_forward(h, wg, experts, E, k, T, hidden, inter, out, indices, weights, scratch,
                           kNoAllocScratch, stream);
}
