// Fused top-k router: gate GEMV + fp32 softmax + top-k + renormalise.
//
// Reference: ExpertRouter.route_with_logits (engine/router.py:65-94):
//   logits = F.linear(h, Wg)          fp16 out, fp32 accumulation  (:66-69)
//   p = softmax(logits.float(), -1)                                  (:81-84)
//   w, idx = topk(p, k)                                              (:86-90)
//   w /= w.sum(-1, keepdim=True)                                     (:92)
//
// Few tokens: one CTA of 32 warps per token (warps split experts and H, so
// every load of the row is in flight at once); many tokens: one warp per token.  Lane j (< E) owns
// expert j after the dot-product reduction.  The softmax follows the operation order of torch's CUDA warp
// softmax for a last dimension <= 32: butterfly max and butterfly sum over
// next_pow2(E) lanes (offsets W/2 .. 1), exp(l - max), then e / sum, so the
// fp32 probabilities are reproduced operation for operation.
#include "common.cuh"
#include "router_device.cuh"

namespace moe {
namespace {

using namespace route;

constexpr int kRouterWarps = 8;

// Many tokens: one warp per token.
template <int EMAX>
__global__ void __launch_bounds__(kRouterWarps * 32) k_router_topk(
    const uint4* __restrict__ h, const uint4* __restrict__ wg, int64_t T, int H, int E, int W,
    int k, uint16_t* __restrict__ logits, float* __restrict__ weights,
    int64_t* __restrict__ indices) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t t = blockIdx.x * (int64_t)kRouterWarps + (threadIdx.x >> 5);
  if (t >= T) return;
  const int nvec = H >> 3;  // 8 fp16 per 16-byte vector
  FF acc[EMAX];
#pragma unroll
  for (int e = 0; e < EMAX; ++e) acc[e] = FF{0.f, 0.f};
  gate_dots<EMAX>(h + t * nvec, wg, nvec, E, lane, 32, acc);
  double mine = 0.0;
#pragma unroll
  for (int e = 0; e < EMAX; ++e) {
    if (e < E) {
      const FF s = warp_sum_ff(acc[e]);
      if (lane == e) mine = ff_value(s);
    }
  }
  finish_token(mine, lane, E, W, k, t, logits, weights, indices);
}

// Few tokens: one CTA of 32 warps per token (route_token_cta).
__global__ void __launch_bounds__(kCtaWarps * 32) k_router_topk_cta(
    const uint4* __restrict__ h, const uint4* __restrict__ wg, int64_t T, int H, int E, int W,
    int k, uint16_t* __restrict__ logits, float* __restrict__ weights,
    int64_t* __restrict__ indices) {
  pdl_trigger();
  pdl_wait();
  __shared__ FF s_part[kCtaWarps];
  route_token_cta(h, wg, blockIdx.x, H, E, W, k, logits, weights, indices, s_part);
}

__global__ void __launch_bounds__(kRouterWarps * 32) k_router_from_logits(
    const uint16_t* __restrict__ logits, int64_t T, int E, int W, int k,
    float* __restrict__ weights, int64_t* __restrict__ indices) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t t = blockIdx.x * (int64_t)kRouterWarps + (threadIdx.x >> 5);
  if (t >= T) return;
  float l = (lane < E) ? h2f(logits[t * E + lane]) : 0.0f;
  float p = softmax_lane(l, lane, E, W);
  topk_renorm(p, lane, E, W, k, t, weights, indices);
}

int next_pow2(int v) {
  int w = 1;
  while (w < v) w <<= 1;
  return w;
}

}  // namespace
}  // namespace moe

extern "C" int moe_router_topk(const uint16_t* h, const uint16_t* wg, int64_t T, int H, int E,
                               int k, uint16_t* logits, float* weights, int64_t* indices,
                               void* stream) {
  using namespace moe;
  if (T < 0 || H <= 0 || (H & 7) || E < 1 || E > 32 || k < 1 || k > E) return MOE_ERR_INVALID_ARG;
  if (T == 0) return MOE_OK;
  if (!h || !wg || !weights || !indices) return MOE_ERR_INVALID_ARG;
  if (!aligned16(h) || !aligned16(wg)) return MOE_ERR_ALIGNMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint4* h4 = reinterpret_cast<const uint4*>(h);
  const uint4* w4 = reinterpret_cast<const uint4*>(wg);
  const int W = next_pow2(E);
  // Code size matters (each token runs the unrolled body once): instantiate
  // for the expert-count bound that covers E.
  cudaError_t st = cudaSuccess;
  if (T <= 2 * sm_count()) {
    const int grid = static_cast<int>(T);
    st = launch_pdl(k_router_topk_cta, grid, kCtaWarps * 32, 0, s, h4, w4, T, H, E, W, k, logits,
                    weights, indices);
  } else {
    const int grid = static_cast<int>(ceil_div(T, kRouterWarps));
    if (E <= 8) st = launch_pdl(k_router_topk<8>, grid, kRouterWarps * 32, 0, s, h4, w4, T, H, E, W, k, logits, weights, indices);
    else if (E <= 16) st = launch_pdl(k_router_topk<16>, grid, kRouterWarps * 32, 0, s, h4, w4, T, H, E, W, k, logits, weights, indices);
    else st = launch_pdl(k_router_topk<32>, grid, kRouterWarps * 32, 0, s, h4, w4, T, H, E, W, k, logits, weights, indices);
  }
  if (st != cudaSuccess) return MOE_ERR_CUDA;
  MOE_CHECK_LAUNCH();
  return MOE_OK;
}

extern "C" int moe_router_topk_from_logits(const uint16_t* logits, int64_t T, int E, int k,
                                           float* weights, int64_t* indices, void* stream) {
  using namespace moe;
  if (T < 0 || E < 1 || E > 32 || k < 1 || k > E) return MOE_ERR_INVALID_ARG;
  if (T == 0) return MOE_OK;
  if (!logits || !weights || !indices) return MOE_ERR_INVALID_ARG;
  int grid = static_cast<int>(ceil_div(T, kRouterWarps));
  cudaError_t st = launch_pdl(k_router_from_logits, grid, kRouterWarps * 32, 0, static_cast<cudaStream_t>(stream), 
      logits, T, E, next_pow2(E), k, weights, indices);
  if (st != cudaSuccess) return MOE_ERR_CUDA;
  MOE_CHECK_LAUNCH();
  return MOE_OK;
}
