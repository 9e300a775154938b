// Fused top-k router: gate GEMV + fp32 softmax + top-k + renormalise.
//
// Reference: ExpertRouter.route_with_logits (engine/router.py:65-94):
//   logits = F.linear(h, Wg)          fp16 out, fp32 accumulation  (:66-69)
//   p = softmax(logits.float(), -1)                                  (:81-84)
//   w, idx = topk(p, k)                                              (:86-90)
//   w /= w.sum(-1, keepdim=True)                                     (:92)
//
// One warp per token.  Lane j (< E) owns expert j after the dot-product
// reduction.  The softmax follows the operation order of torch's CUDA warp
// softmax for a last dimension <= 32: butterfly max and butterfly sum over
// next_pow2(E) lanes (offsets W/2 .. 1), exp(l - max), then e / sum, so the
// fp32 probabilities are reproduced operation for operation.
#include "common.cuh"

namespace moe {
namespace {

constexpr int kRouterWarps = 8;

__device__ __forceinline__ void topk_renorm(float p, int lane, int E, int W, int k, int64_t t,
                                            float* __restrict__ weights,
                                            int64_t* __restrict__ indices) {
  // Iterative arg-max: larger probability wins; exact ties go to the lower
  // expert index.  Lanes >= E never win (p = -1 sentinel; probabilities >= 0).
  float cand = (lane < E) ? p : -1.0f;
  float sel_sum = 0.0f;
  float my_sel = -1.0f;  // selected probability held by output lane j
  int my_idx = 0;
#pragma unroll 1
  for (int j = 0; j < k; ++j) {
    float bv = cand;
    int bi = lane;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    // Renormaliser accumulates in selection order (sum over the k outputs).
    sel_sum = (j == 0) ? bv : __fadd_rn(sel_sum, bv);
    if (lane == j) {
      my_sel = bv;
      my_idx = bi;
    }
    if (lane == bi) cand = -1.0f;
  }
  if (lane < k) {
    weights[t * k + lane] = __fdiv_rn(my_sel, sel_sum);
    indices[t * k + lane] = static_cast<int64_t>(my_idx);
  }
  (void)W;
}

__device__ __forceinline__ float softmax_lane(float logit, int lane, int E, int W) {
  float v = (lane < E) ? logit : -INFINITY;
  float m = v;
  for (int o = W >> 1; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float e = (lane < E) ? expf(__fsub_rn(v, m)) : 0.0f;
  float s = e;
  for (int o = W >> 1; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
  return __fdiv_rn(e, s);
}

__global__ void __launch_bounds__(kRouterWarps * 32) k_router_topk(
    const uint4* __restrict__ h, const uint4* __restrict__ wg, int64_t T, int H, int E, int W,
    int k, uint16_t* __restrict__ logits, float* __restrict__ weights,
    int64_t* __restrict__ indices) {
  const int lane = threadIdx.x & 31;
  const int64_t t = blockIdx.x * (int64_t)kRouterWarps + (threadIdx.x >> 5);
  if (t >= T) return;
  const int nvec = H >> 3;  // 8 fp16 per 16-byte vector
  float acc[32];
#pragma unroll
  for (int e = 0; e < 32; ++e) acc[e] = 0.0f;
  const uint4* hrow = h + t * nvec;
  for (int v = lane; v < nvec; v += 32) {
    uint4 hv = hrow[v];
    const __half2* hh = reinterpret_cast<const __half2*>(&hv);
    float2 x0 = __half22float2(hh[0]), x1 = __half22float2(hh[1]);
    float2 x2 = __half22float2(hh[2]), x3 = __half22float2(hh[3]);
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      if (e < E) {
        uint4 wv = __ldg(wg + (int64_t)e * nvec + v);
        const __half2* ww = reinterpret_cast<const __half2*>(&wv);
        float2 w0 = __half22float2(ww[0]), w1 = __half22float2(ww[1]);
        float2 w2 = __half22float2(ww[2]), w3 = __half22float2(ww[3]);
        float a = acc[e];
        a = fmaf(x0.x, w0.x, a); a = fmaf(x0.y, w0.y, a);
        a = fmaf(x1.x, w1.x, a); a = fmaf(x1.y, w1.y, a);
        a = fmaf(x2.x, w2.x, a); a = fmaf(x2.y, w2.y, a);
        a = fmaf(x3.x, w3.x, a); a = fmaf(x3.y, w3.y, a);
        acc[e] = a;
      }
    }
  }
  float mine = 0.0f;
#pragma unroll
  for (int e = 0; e < 32; ++e) {
    if (e < E) {
      float s = warp_sum(acc[e]);
      if (lane == e) mine = s;
    }
  }
  // Round once to fp16 (F.linear output dtype), then softmax on float(logit).
  uint16_t l16 = f2h(mine);
  if (logits != nullptr && lane < E) logits[t * E + lane] = l16;
  float p = softmax_lane(h2f(l16), lane, E, W);
  topk_renorm(p, lane, E, W, k, t, weights, indices);
}

__global__ void __launch_bounds__(kRouterWarps * 32) k_router_from_logits(
    const uint16_t* __restrict__ logits, int64_t T, int E, int W, int k,
    float* __restrict__ weights, int64_t* __restrict__ indices) {
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
  int grid = static_cast<int>(ceil_div(T, kRouterWarps));
  k_router_topk<<<grid, kRouterWarps * 32, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint4*>(h), reinterpret_cast<const uint4*>(wg), T, H, E,
      next_pow2(E), k, logits, weights, indices);
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
  k_router_from_logits<<<grid, kRouterWarps * 32, 0, static_cast<cudaStream_t>(stream)>>>(
      logits, T, E, next_pow2(E), k, weights, indices);
  MOE_CHECK_LAUNCH();
  return MOE_OK;
}
