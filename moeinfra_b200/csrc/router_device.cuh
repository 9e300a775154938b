// Router arithmetic shared by the router kernels and the fused 1-token
// decode layer: exact gate dot products (double-float sums of exact fp16
// products, rounded once to fp16), torch's warp softmax operation order, and
// top-k with torch's tie order.  See router.cu for the reference lines.
#pragma once
#include "common.cuh"

namespace moe {
namespace route {

__device__ __forceinline__ void topk_renorm(float p, int lane, int E, int W, int k, int64_t t,
                                            float* __restrict__ weights,
                                            int64_t* __restrict__ indices) {
  // Iterative arg-max: larger probability wins; among exact ties the lower
  // expert index is selected first.  Lanes >= E never win (p = -1 sentinel;
  // probabilities are >= 0).
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
  // The selected set takes the lower expert indices among equal probabilities;
  // torch's CUDA topk then lists equal values in descending index order.
  // Reverse each run of equal selected values to match (runs are contiguous:
  // the selection order is descending in value).
  int rs = lane, re = lane;
  for (int m = 0; m < k; ++m) {
    const float vm = __shfl_sync(0xffffffffu, my_sel, m);
    if (lane < k && vm == my_sel) {
      rs = min(rs, m);
      re = max(re, m);
    }
  }
  const int src = (lane < k) ? rs + re - lane : lane;
  const float out_sel = __shfl_sync(0xffffffffu, my_sel, src);
  const int out_idx = __shfl_sync(0xffffffffu, my_idx, src);
  if (lane < k) {
    weights[t * k + lane] = __fdiv_rn(out_sel, sel_sum);
    indices[t * k + lane] = static_cast<int64_t>(out_idx);
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

// Dot products of one token against the E gate rows over the vector range
// [v_begin, v_end) handled by this lane (stride `stride` vectors of 8 fp16).
// Float-float accumulator: value = hi + lo, updated with the error-free
// TwoSum, so a 4096-term sum of exact fp16 x fp16 products keeps ~48 bits.
struct FF {
  float hi, lo;
};
__device__ __forceinline__ void ff_add(FF& a, float p) {
  const float s = __fadd_rn(a.hi, p);
  const float bp = __fsub_rn(s, a.hi);
  const float err = __fadd_rn(__fsub_rn(a.hi, __fsub_rn(s, bp)), __fsub_rn(p, bp));
  a.hi = s;
  a.lo = __fadd_rn(a.lo, err);
}
__device__ __forceinline__ void ff_merge(FF& a, const FF& b) {
  ff_add(a, b.hi);
  a.lo = __fadd_rn(a.lo, b.lo);
}
__device__ __forceinline__ double ff_value(const FF& a) { return (double)a.hi + (double)a.lo; }

// fp16 x fp16 products are exact in fp32; they are summed in float-float and
// rounded once to fp16, which gives the correctly rounded logit.
template <int EMAX>
__device__ __forceinline__ void gate_dots(const uint4* __restrict__ hrow, const uint4* __restrict__ wg,
                                          int nvec, int E, int v_begin, int stride,
                                          FF (&acc)[EMAX]) {
#pragma unroll 1
  for (int v = v_begin; v < nvec; v += stride) {
    uint4 hv = hrow[v];
    const __half2* hh = reinterpret_cast<const __half2*>(&hv);
    float2 x0 = __half22float2(hh[0]), x1 = __half22float2(hh[1]);
    float2 x2 = __half22float2(hh[2]), x3 = __half22float2(hh[3]);
#pragma unroll
    for (int e = 0; e < EMAX; ++e) {
      if (e < E) {
        uint4 wv = __ldg(wg + (int64_t)e * nvec + v);
        const __half2* ww = reinterpret_cast<const __half2*>(&wv);
        float2 w0 = __half22float2(ww[0]), w1 = __half22float2(ww[1]);
        float2 w2 = __half22float2(ww[2]), w3 = __half22float2(ww[3]);
        FF a = acc[e];
        ff_add(a, __fmul_rn(x0.x, w0.x)); ff_add(a, __fmul_rn(x0.y, w0.y));
        ff_add(a, __fmul_rn(x1.x, w1.x)); ff_add(a, __fmul_rn(x1.y, w1.y));
        ff_add(a, __fmul_rn(x2.x, w2.x)); ff_add(a, __fmul_rn(x2.y, w2.y));
        ff_add(a, __fmul_rn(x3.x, w3.x)); ff_add(a, __fmul_rn(x3.y, w3.y));
        acc[e] = a;
      }
    }
  }
}

__device__ __forceinline__ FF warp_sum_ff(FF v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    FF w;
    w.hi = __shfl_xor_sync(0xffffffffu, v.hi, o);
    w.lo = __shfl_xor_sync(0xffffffffu, v.lo, o);
    ff_merge(v, w);
  }
  return v;
}

__device__ __forceinline__ void finish_token(double logit, int lane, int E, int W, int k,
                                             int64_t t, uint16_t* __restrict__ logits,
                                             float* __restrict__ weights,
                                             int64_t* __restrict__ indices) {
  // Round once to fp16 (F.linear output dtype), then softmax on float(logit).
  uint16_t l16 = __half_as_ushort(__double2half(logit));
  if (logits != nullptr && lane < E) logits[t * E + lane] = l16;
  float p = softmax_lane(h2f(l16), lane, E, W);
  topk_renorm(p, lane, E, W, k, t, weights, indices);
}

// Few tokens: one CTA of kCtaWarps warps per token.  Warp w takes expert
// w % E and range w / E of the row's 16-byte vectors (kCtaWarps / E ranges),
// issues its loads ahead of the arithmetic, and sums exactly in double-float;
// the ranges meet in shared memory (`s_part`, kCtaWarps entries) in a fixed
// order.  The fp16 logit is the correctly rounded sum, as in the many-token
// kernel.  Every thread of the CTA calls it (one barrier inside); warp 0
// writes token t's outputs.
constexpr int kCtaWarps = 32;
constexpr int kCtaUnroll = 4;

__device__ __forceinline__ void route_token_cta(const uint4* __restrict__ h,
                                                const uint4* __restrict__ wg, int64_t t, int H,
                                                int E, int W, int k, uint16_t* __restrict__ logits,
                                                float* __restrict__ weights,
                                                int64_t* __restrict__ indices, FF* s_part) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nvec = H >> 3;
  const int groups = kCtaWarps / E;  // >= 1 for E <= 32
  if (warp < groups * E) {
    const int e = warp % E, r = warp / E;
    const int v0 = static_cast<int>((int64_t)nvec * r / groups);
    const int v1 = static_cast<int>((int64_t)nvec * (r + 1) / groups);
    const uint4* hrow = h + t * nvec;
    const uint4* wrow = wg + (int64_t)e * nvec;
    FF acc{0.f, 0.f};
    for (int vb = v0 + lane; vb < v1; vb += 32 * kCtaUnroll) {
      uint4 hv[kCtaUnroll], wv[kCtaUnroll];
#pragma unroll
      for (int u = 0; u < kCtaUnroll; ++u) {
        const int v = vb + u * 32;
        hv[u] = v < v1 ? hrow[v] : make_uint4(0, 0, 0, 0);
        wv[u] = v < v1 ? __ldg(wrow + v) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < kCtaUnroll; ++u) {
        const __half2* hh = reinterpret_cast<const __half2*>(&hv[u]);
        const __half2* ww = reinterpret_cast<const __half2*>(&wv[u]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 x = __half22float2(hh[q]), y = __half22float2(ww[q]);
          ff_add(acc, __fmul_rn(x.x, y.x));
          ff_add(acc, __fmul_rn(x.y, y.y));
        }
      }
    }
    const FF tot = warp_sum_ff(acc);
    if (lane == 0) s_part[warp] = tot;
  }
  __syncthreads();
  if (warp == 0) {
    double mine = 0.0;
    if (lane < E) {
      FF tot = s_part[lane];
      for (int r = 1; r < groups; ++r) ff_merge(tot, s_part[r * E + lane]);
      mine = ff_value(tot);
    }
    finish_token(mine, lane, E, W, k, t, logits, weights, indices);
  }
}

}  // namespace route
}  // namespace moe
