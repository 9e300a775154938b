// Token permute (stable counting sort by expert), row gather, and the
// weighted combine in ascending expert order.
//
// Reference: MoELayer._forward_tokens (model/moe_layer.py:147-191):
//   output = zeros_like(h)                                        (:147)
//   for e in sorted(unique(idx)):                                 (:150-153,:172)
//     mask = any(idx == e, -1); token_w = sum(w * (idx == e), -1) (:174-183)
//     output[mask] += expert(h[mask]) * token_w[mask, None]       (:185-191)
// The in-place add on the fp16 output computes in fp32 and rounds to fp16
// once per expert, in ascending expert id; h[mask] is in ascending token order.
#include "common.cuh"

namespace moe {
namespace {

constexpr int kPermThreads = 1024;

__global__ void __launch_bounds__(kPermThreads) k_permute(
    const int64_t* __restrict__ indices, const float* __restrict__ weights, int64_t T, int k,
    int E, int32_t* __restrict__ expert_offsets, int32_t* __restrict__ pair_token,
    float* __restrict__ pair_weight, int32_t* __restrict__ pair_slot, int32_t* __restrict__ zero,
    int nzero) {
  pdl_trigger();
  pdl_wait();
  // Completion counters of the expert launch that follows (after the wait:
  // the previous user of these words has finished).
  for (int i = threadIdx.x; i < nzero; i += kPermThreads) zero[i] = 0;
  __shared__ int s_count[32];
  __shared__ int s_off[33];
  __shared__ int s_run[32];
  __shared__ int s_wcnt[32][32];  // [warp][expert]
  __shared__ int s_wpre[32][32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t P = T * k;
  if (tid < 32) {
    s_count[tid] = 0;
    s_run[tid] = 0;
  }
  __syncthreads();
  for (int64_t p = tid; p < P; p += kPermThreads) {
    int64_t e = indices[p];
    if (e >= 0 && e < E) atomicAdd(&s_count[e], 1);
  }
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int e = 0; e < E; ++e) {
      s_off[e] = acc;
      acc += s_count[e];
    }
    s_off[E] = acc;
  }
  __syncthreads();
  if (tid <= E) expert_offsets[tid] = s_off[tid];
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int64_t base = 0; base < P; base += kPermThreads) {
    s_wcnt[warp][lane] = 0;
    __syncthreads();
    const int64_t p = base + tid;
    int e = -1;
    if (p < P) {
      int64_t ev = indices[p];
      e = (ev >= 0 && ev < E) ? static_cast<int>(ev) : -1;
    }
    const unsigned same = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(same & lt_mask);
    if (e >= 0 && rank == 0) s_wcnt[warp][e] = __popc(same);
    __syncthreads();
    {  // thread (w = warp, e = lane): exclusive prefix over earlier warps
      int acc = 0;
      for (int w = 0; w < warp; ++w) acc += s_wcnt[w][lane];
      s_wpre[warp][lane] = acc;
    }
    __syncthreads();
    if (e >= 0) {
      const int pos = s_off[e] + s_run[e] + s_wpre[warp][e] + rank;
      pair_token[pos] = static_cast<int32_t>(p / k);
      pair_weight[pos] = weights[p];
      pair_slot[p] = pos;
    } else if (p < P) {
      pair_slot[p] = -1;
    }
    __syncthreads();
    if (tid < E) {
      int tot = 0;
      for (int w = 0; w < 32; ++w) tot += s_wcnt[w][tid];
      s_run[tid] += tot;
    }
    __syncthreads();
  }
}

__global__ void k_gather_rows(const uint4* __restrict__ in, const int32_t* __restrict__ index,
                              int64_t n, int vec_per_row, uint4* __restrict__ out) {
  const int64_t total = n * vec_per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / vec_per_row, v = i - r * vec_per_row;
    out[i] = in[(int64_t)index[r] * vec_per_row + v];
  }
}

// Source of one expert-output element: fp16 rows, or S fp32 split-K partials
// laid out [slot][S][width] that are summed in split order and rounded once.
struct YHalf {
  const uint16_t* y;
  __device__ __forceinline__ float get(int64_t slot, int c, int width) const {
    return h2f(y[slot * width + c]);
  }
};
struct YPartials {
  const float* part;
  int S;
  __device__ __forceinline__ float get(int64_t slot, int c, int width) const {
    const float* p = part + slot * (int64_t)S * width + c;
    float s = p[0];
    for (int i = 1; i < S; ++i) s = __fadd_rn(s, p[(int64_t)i * width]);
    return h2f(f2h(s));
  }
};

MOE_DEFINE_ERROR_WORD()

// wait_flags (peer-memory exchange): every CTA first waits (bounded) until all
// wait_G flags reach *wait_seq, i.e. every owner's results have landed.
template <class Y>
__global__ void k_combine(Y ysrc, const int32_t* __restrict__ pair_slot,
                          const int64_t* __restrict__ indices, const float* __restrict__ weights,
                          int64_t T, int k, int width, uint16_t* __restrict__ out,
                          const int32_t* wait_flags, int wait_G, const int32_t* wait_seq,
                          uint64_t wait_ns) {
  pdl_trigger();
  pdl_wait();
  if (wait_flags) {
    if (threadIdx.x < wait_G && !wait_peer_flag(wait_flags, threadIdx.x, wait_seq, wait_ns))
      set_device_error(kErrWaitTimeout);
    __syncthreads();
  }
  const int64_t total = T * width;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / width;
    const int c = static_cast<int>(i - t * width);
    // The token's k experts in ascending id (each id appears at most once).
    int order[8];
    int n = 0;
    for (int j = 0; j < k && j < 8; ++j) {
      int pos = n;
      const int64_t ej = indices[t * k + j];
      while (pos > 0 && indices[t * k + order[pos - 1]] > ej) {
        order[pos] = order[pos - 1];
        --pos;
      }
      order[pos] = j;
      ++n;
    }
    float acc = 0.0f;  // output starts at +0 (zeros_like)
    for (int m = 0; m < n; ++m) {
      const int j = order[m];
      const int32_t slot = pair_slot[t * k + j];
      if (slot < 0) continue;
      const float prod = __fmul_rn(ysrc.get(slot, c, width), weights[t * k + j]);
      acc = h2f(f2h(__fadd_rn(acc, prod)));
    }
    out[i] = f2h(acc);
  }
}

int grid_for(int64_t work, int threads) {
  int64_t b = ceil_div(work, threads);
  int64_t cap = (int64_t)sm_count() * 8;
  return static_cast<int>(b < cap ? (b > 0 ? b : 1) : cap);
}

}  // namespace

int launch_combine_partials(const float* part, int S, const int32_t* pair_slot,
                            const int64_t* indices, const float* weights, int64_t T, int k,
                            int width, uint16_t* out, cudaStream_t s) {
  if (launch_pdl(k_combine<YPartials>, grid_for(T * width, 256), 256, 0, s, YPartials{part, S},
                 pair_slot, indices, weights, T, k, width, out,
                 static_cast<const int32_t*>(nullptr), 0, static_cast<const int32_t*>(nullptr),
                 uint64_t{0}) != cudaSuccess)
    return MOE_ERR_CUDA;
  MOE_CHECK_LAUNCH();
  return MOE_OK;
}

int launch_permute(const int64_t* indices, const float* weights, int64_t T, int k, int E,
                   int32_t* expert_offsets, int32_t* pair_token, float* pair_weight,
                   int32_t* pair_slot, int32_t* zero, int nzero, cudaStream_t s) {
  if (launch_pdl(k_permute, 1, kPermThreads, 0, s, indices, weights, T, k, E, expert_offsets,
                 pair_token, pair_weight, pair_slot, zero, nzero) != cudaSuccess)
    return MOE_ERR_CUDA;
  MOE_CHECK_LAUNCH();
  return MOE_OK;
}

int launch_gather_rows(const uint16_t* rows_in, const int32_t* index, int64_t n, int width,
                       uint16_t* rows_out, cudaStream_t s) {
  const int vpr = width / 8;
  k_gather_rows<<<grid_for(n * vpr, 256), 256, 0, s>>>(reinterpret_cast<const uint4*>(rows_in),
                                                       index, n, vpr,
                                                       reinterpret_cast<uint4*>(rows_out));
  MOE_CHECK_LAUNCH();
  return MOE_OK;
}

}  // namespace moe

extern "C" int moe_permute(const int64_t* indices, const float* weights, int64_t T, int k, int E,
                           int32_t* expert_offsets, int32_t* pair_token, float* pair_weight,
                           int32_t* pair_slot, void* stream) {
  if (T < 0 || k < 1 || E < 1 || E > 32 || T * k > (int64_t)1 << 30) return MOE_ERR_INVALID_ARG;
  if (!indices || !weights || !expert_offsets || !pair_token || !pair_weight || !pair_slot)
    return MOE_ERR_INVALID_ARG;
  return moe::launch_permute(indices, weights, T, k, E, expert_offsets, pair_token, pair_weight,
                             pair_slot, nullptr, 0, static_cast<cudaStream_t>(stream));
}

extern "C" int moe_gather_rows(const uint16_t* rows_in, const int32_t* index, int64_t n, int width,
                               uint16_t* rows_out, void* stream) {
  if (n < 0 || width <= 0 || (width & 7)) return MOE_ERR_INVALID_ARG;
  if (n == 0) return MOE_OK;
  if (!rows_in || !index || !rows_out) return MOE_ERR_INVALID_ARG;
  if (!moe::aligned16(rows_in) || !moe::aligned16(rows_out)) return MOE_ERR_ALIGNMENT;
  return moe::launch_gather_rows(rows_in, index, n, width, rows_out,
                                 static_cast<cudaStream_t>(stream));
}

namespace moe {
namespace {
int combine_half(const uint16_t* y_sorted, const int32_t* pair_slot, const int64_t* indices,
                 const float* weights, int64_t T, int k, int width, uint16_t* out,
                 const int32_t* flags, int G, const int32_t* seq, void* stream) {
  if (T < 0 || k < 1 || k > 8 || width <= 0) return MOE_ERR_INVALID_ARG;
  if (T == 0) return MOE_OK;
  if (!y_sorted || !pair_slot || !indices || !weights || !out) return MOE_ERR_INVALID_ARG;
  if (launch_pdl(k_combine<YHalf>, grid_for(T * width, 256), 256, 0,
                 static_cast<cudaStream_t>(stream), YHalf{y_sorted}, pair_slot, indices, weights,
                 T, k, width, out, flags, G, seq, wait_limit_ns()) != cudaSuccess)
    return MOE_ERR_CUDA;
  MOE_CHECK_LAUNCH();
  return MOE_OK;
}
}  // namespace
}  // namespace moe

extern "C" int moe_combine(const uint16_t* y_sorted, const int32_t* pair_slot,
                           const int64_t* indices, const float* weights, int64_t T, int k,
                           int width, uint16_t* out, void* stream) {
  return moe::combine_half(y_sorted, pair_slot, indices, weights, T, k, width, out, nullptr, 0,
                           nullptr, stream);
}

extern "C" int moe_combine_p2p(const uint16_t* y_back, const int32_t* pair_slot,
                               const int64_t* indices, const float* weights, int64_t T, int k,
                               int width, uint16_t* out, const int32_t* flags, int G,
                               const int32_t* seq, void* stream) {
  if (!flags || !seq || G < 1 || G > MOE_MAX_EXPERTS) return MOE_ERR_INVALID_ARG;
  return moe::combine_half(y_back, pair_slot, indices, weights, T, k, width, out, flags, G, seq,
                           stream);
}
