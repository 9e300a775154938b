// Decode-path SwiGLU experts on packed NF4 weights (few tokens per expert).
//
// Reference: ReconstructedNF4Expert.forward (transfer/nf4_reconstruct.py:152-155)
//   y = w2(silu(w1 x) * w3 x), each wN a bitsandbytes Linear4bit in fp16
//   compute (:94).  bitsandbytes' matmul_4bit takes the 4-bit GEMV for a
//   single input row and dequant(bf16)->fp16 GEMM otherwise; the kernels
//   below pick the same semantics per expert from its device-side token count:
//     1 token : w = fp16(fp16(code) * fp16(absmax)), acc += fp32(x)*fp32(w)
//     n > 1   : w = fp16(bf16(code * absmax)),       acc += fp32(x)*fp32(w)
//   and round each output once to fp16.
//
// Work split (HBM-bound streaming of packed rows):
//   gate_up : CTA item = (expert, 64 rows of W1 and W3); a warp owns whole
//             row pairs so SwiGLU is formed in registers; x of the expert's
//             tokens is staged once per item in shared memory.
//   down    : CTA item = (expert, K-split, 64 rows of W2); split-K over the
//             14336-long reduction for load balance; fp32 partials are summed
//             in split order by the combine kernel (deterministic).
// Each lane loads 16 packed bytes (32 weights) per 128-bit load.  Bytes are
// decoded through shared-memory tables indexed by the whole byte, replicated
// per bank so random bytes never conflict: lut16 (half2 of the two fp16
// codes, 32 KB) for the 1-token semantics, lut32 (float2 of the two fp32
// codes, 32 KB) for the multi-token semantics.
#include "common.cuh"

namespace moe {

struct ExpertTable {
  moe_nf4_expert_t e[MOE_MAX_EXPERTS];
};

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kRowsPerItem = 64;  // rows per CTA work item
constexpr int kMaxTok = 4;        // tokens per expert handled by this path
constexpr int kLut16Words = 256 * 32;
constexpr int kLut32Pairs = 256 * 16;

struct DecodeArgs {
  ExpertTable ex;
  int E;
  const int32_t* expert_offsets;  // [E+1] device
  const int32_t* pair_token;      // [P] token row in x for each sorted pair, or null (identity)
  const uint16_t* x;              // fp16 rows [*, H]
  uint16_t* h_sorted;             // fp16 [P, I]
  float* y_part;                  // fp32 [P][S][H]
  int H, I, S, split_chunks;
};

__device__ __forceinline__ void build_luts(const float* __restrict__ code, bool need16, bool need32,
                                           uint32_t* lut16, float2* lut32) {
  __shared__ float s_code[16];
  if (threadIdx.x < 16) s_code[threadIdx.x] = code[threadIdx.x];
  __syncthreads();
  if (need16) {
    for (int i = threadIdx.x; i < kLut16Words; i += blockDim.x) {
      const int v = i >> 5;
      __half2 h = __floats2half2_rn(s_code[v >> 4], s_code[v & 15]);
      lut16[i] = *reinterpret_cast<uint32_t*>(&h);
    }
  }
  if (need32) {
    for (int i = threadIdx.x; i < kLut32Pairs; i += blockDim.x) {
      const int v = i >> 4;
      lut32[i] = make_float2(s_code[v >> 4], s_code[v & 15]);
    }
  }
  __syncthreads();
}

// Swizzled shared layout of fp16 rows: chunk c (32 halves = 4 x 16 B) stores
// its logical 16-byte segment g at physical segment (g + (c >> 1)) & 3, so
// the 8 lanes of a 128-bit wavefront (chunks l, l+1, ...) hit distinct banks.
__device__ __forceinline__ int xs_index(int c, int g) { return c * 4 + ((g + (c >> 1)) & 3); }

// Dot products of one 16-byte packed chunk (32 weights) against n tokens.
template <bool kGemv>
__device__ __forceinline__ void chunk_dot(const uint4& qv, float absmax, const uint32_t* lut16_l,
                                          const float2* lut32_l, const uint4* xs, int xs_stride,
                                          int c, int n, float* acc) {
  const uint32_t w4[4] = {qv.x, qv.y, qv.z, qv.w};
  if (kGemv) {
    const __half a16 = __float2half_rn(absmax);
    const __half2 a2 = __halves2half2(a16, a16);
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const uint4 xv = xs[xs_index(c, g)];
      const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const uint32_t byte = (w4[g] >> (8 * b)) & 0xFFu;
        uint32_t cw = lut16_l[byte * 32];
        __half2 w = __hmul2(*reinterpret_cast<__half2*>(&cw), a2);
        const uint32_t wv = *reinterpret_cast<uint32_t*>(&w);
        acc[0] = fma_f16f16_f32(lo16(xw[b]), lo16(wv), acc[0]);
        acc[0] = fma_f16f16_f32(hi16(xw[b]), hi16(wv), acc[0]);
      }
    }
  } else {
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      uint4 xv[kMaxTok];
#pragma unroll
      for (int t = 0; t < kMaxTok; ++t)
        xv[t] = (t < n) ? xs[t * xs_stride + xs_index(c, g)] : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const uint32_t byte = (w4[g] >> (8 * b)) & 0xFFu;
        const float2 cc = lut32_l[byte * 16];
        const uint32_t wv = nf4_pair_multirow(cc.x, cc.y, absmax);
#pragma unroll
        for (int t = 0; t < kMaxTok; ++t) {
          if (t < n) {
            const uint32_t xw = (b == 0) ? xv[t].x : (b == 1) ? xv[t].y : (b == 2) ? xv[t].z : xv[t].w;
            acc[t] = fma_f16f16_f32(lo16(xw), lo16(wv), acc[t]);
            acc[t] = fma_f16f16_f32(hi16(xw), hi16(wv), acc[t]);
          }
        }
      }
    }
  }
}

// Shared prologue: per-expert counts, the active-expert list and the LUTs.
struct ActiveSet {
  int n_active;
  int first;
  bool any1, anyN;
};

__device__ __forceinline__ ActiveSet load_active(const DecodeArgs& a, int* s_off, int* s_active) {
  __shared__ int s_n;
  __shared__ int s_flags;
  if (threadIdx.x == 0) {
    int n = 0, flags = 0;
    for (int e = 0; e <= a.E; ++e) s_off[e] = a.expert_offsets[e];
    for (int e = 0; e < a.E; ++e) {
      const int cnt = s_off[e + 1] - s_off[e];
      if (cnt > 0) {
        s_active[n++] = e;
        flags |= (cnt == 1) ? 1 : 2;
      }
    }
    s_n = n;
    s_flags = flags;
  }
  __syncthreads();
  ActiveSet r;
  r.n_active = s_n;
  r.first = s_n > 0 ? s_active[0] : 0;
  r.any1 = (s_flags & 1) != 0;
  r.anyN = (s_flags & 2) != 0;
  return r;
}

__global__ void __launch_bounds__(kThreads) k_gate_up_decode(const __grid_constant__ DecodeArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  uint32_t* lut16 = reinterpret_cast<uint32_t*>(smem);
  float2* lut32 = reinterpret_cast<float2*>(smem + kLut16Words * 4);
  uint4* xs = reinterpret_cast<uint4*>(smem + kLut16Words * 4 + kLut32Pairs * 8);
  __shared__ int s_off[MOE_MAX_EXPERTS + 1];
  __shared__ int s_active[MOE_MAX_EXPERTS];

  const ActiveSet act = load_active(a, s_off, s_active);
  if (act.n_active == 0) return;
  build_luts(a.ex.e[act.first].w1.code, act.any1, act.anyN, lut16, lut32);

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t* lut16_l = lut16 + lane;
  const float2* lut32_l = lut32 + (lane & 15);
  const int items_per_expert = a.I / kRowsPerItem;
  const int total = act.n_active * items_per_expert;
  const int nchunks = a.H / 32;  // 16-byte chunks per row
  const int xs_stride = nchunks * 4;
  int staged = -1;

  for (int item = blockIdx.x; item < total; item += gridDim.x) {
    const int e = s_active[item / items_per_expert];
    const int rb = item % items_per_expert;
    const int base = s_off[e];
    const int n = s_off[e + 1] - base;
    if (e != staged) {
      __syncthreads();
      for (int i = threadIdx.x; i < n * nchunks * 4; i += kThreads) {
        const int t = i / (nchunks * 4), rem = i - t * nchunks * 4;
        const int c = rem >> 2, g = rem & 3;
        const int64_t row = a.pair_token ? a.pair_token[base + t] : (int64_t)(base + t);
        xs[t * xs_stride + xs_index(c, g)] =
            reinterpret_cast<const uint4*>(a.x + row * a.H)[c * 4 + g];
      }
      __syncthreads();
      staged = e;
    }
    const moe_nf4_matrix_t w1 = a.ex.e[e].w1, w3 = a.ex.e[e].w3;
    const int64_t row_bytes = a.H / 2;
    for (int rr = warp; rr < kRowsPerItem; rr += kWarps) {
      const int r = rb * kRowsPerItem + rr;
      float acc1[kMaxTok], acc3[kMaxTok];
#pragma unroll
      for (int t = 0; t < kMaxTok; ++t) acc1[t] = acc3[t] = 0.0f;
      const uint4* q1 = reinterpret_cast<const uint4*>(w1.q + r * row_bytes);
      const uint4* q3 = reinterpret_cast<const uint4*>(w3.q + r * row_bytes);
      const float* am1 = w1.absmax + (int64_t)r * (a.H / 64);
      const float* am3 = w3.absmax + (int64_t)r * (a.H / 64);
      for (int c = lane; c < nchunks; c += 32) {
        const uint4 v1 = __ldg(q1 + c), v3 = __ldg(q3 + c);
        const float s1 = __ldg(am1 + (c >> 1)), s3 = __ldg(am3 + (c >> 1));
        if (n == 1) {
          chunk_dot<true>(v1, s1, lut16_l, lut32_l, xs, xs_stride, c, 1, acc1);
          chunk_dot<true>(v3, s3, lut16_l, lut32_l, xs, xs_stride, c, 1, acc3);
        } else {
          chunk_dot<false>(v1, s1, lut16_l, lut32_l, xs, xs_stride, c, n, acc1);
          chunk_dot<false>(v3, s3, lut16_l, lut32_l, xs, xs_stride, c, n, acc3);
        }
      }
#pragma unroll
      for (int t = 0; t < kMaxTok; ++t) {
        if (t < n) {
          const float g = warp_sum(acc1[t]);
          const float u = warp_sum(acc3[t]);
          if (lane == 0) a.h_sorted[(int64_t)(base + t) * a.I + r] = swiglu_f16(f2h(g), f2h(u));
        }
      }
    }
  }
}

__global__ void __launch_bounds__(kThreads) k_down_decode(const __grid_constant__ DecodeArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  uint32_t* lut16 = reinterpret_cast<uint32_t*>(smem);
  float2* lut32 = reinterpret_cast<float2*>(smem + kLut16Words * 4);
  uint4* xs = reinterpret_cast<uint4*>(smem + kLut16Words * 4 + kLut32Pairs * 8);
  __shared__ int s_off[MOE_MAX_EXPERTS + 1];
  __shared__ int s_active[MOE_MAX_EXPERTS];

  const ActiveSet act = load_active(a, s_off, s_active);
  if (act.n_active == 0) return;
  build_luts(a.ex.e[act.first].w2.code, act.any1, act.anyN, lut16, lut32);

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t* lut16_l = lut16 + lane;
  const float2* lut32_l = lut32 + (lane & 15);
  const int row_blocks = a.H / kRowsPerItem;
  const int items_per_expert = a.S * row_blocks;
  const int total = act.n_active * items_per_expert;
  const int nchunks = a.I / 32;
  const int sc = a.split_chunks;
  const int xs_stride = sc * 4;
  int staged_e = -1, staged_s = -1;

  for (int item = blockIdx.x; item < total; item += gridDim.x) {
    const int e = s_active[item / items_per_expert];
    const int rem_item = item % items_per_expert;
    const int s = rem_item / row_blocks;
    const int rb = rem_item % row_blocks;
    const int base = s_off[e];
    const int n = s_off[e + 1] - base;
    const int c0 = s * sc;
    const int c1 = min(c0 + sc, nchunks);
    if (e != staged_e || s != staged_s) {
      __syncthreads();
      const int span = (c1 - c0) * 4;
      for (int i = threadIdx.x; i < n * span; i += kThreads) {
        const int t = i / span, rem = i - t * span;
        const int cl = rem >> 2, g = rem & 3;
        xs[t * xs_stride + xs_index(cl, g)] =
            reinterpret_cast<const uint4*>(a.h_sorted + (int64_t)(base + t) * a.I)[(c0 + cl) * 4 + g];
      }
      __syncthreads();
      staged_e = e;
      staged_s = s;
    }
    const moe_nf4_matrix_t w2 = a.ex.e[e].w2;
    const int64_t row_bytes = a.I / 2;
    for (int rr = warp; rr < kRowsPerItem; rr += kWarps) {
      const int r = rb * kRowsPerItem + rr;
      float acc[kMaxTok];
#pragma unroll
      for (int t = 0; t < kMaxTok; ++t) acc[t] = 0.0f;
      const uint4* q = reinterpret_cast<const uint4*>(w2.q + r * row_bytes);
      const float* am = w2.absmax + (int64_t)r * (a.I / 64);
      for (int c = c0 + lane; c < c1; c += 32) {
        const uint4 v = __ldg(q + c);
        const float sa = __ldg(am + (c >> 1));
        if (n == 1)
          chunk_dot<true>(v, sa, lut16_l, lut32_l, xs, xs_stride, c - c0, 1, acc);
        else
          chunk_dot<false>(v, sa, lut16_l, lut32_l, xs, xs_stride, c - c0, n, acc);
      }
#pragma unroll
      for (int t = 0; t < kMaxTok; ++t) {
        if (t < n) {
          const float y = warp_sum(acc[t]);
          if (lane == 0) a.y_part[((int64_t)(base + t) * a.S + s) * a.H + r] = y;
        }
      }
    }
  }
}

// y[slot] = fp16(sum over splits of y_part[slot][s]) (single-expert forward).
__global__ void k_reduce_partials(const float* __restrict__ part, int64_t P, int S, int width,
                                  uint16_t* __restrict__ y) {
  const int64_t total = P * width;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = i / width;
    const int c = static_cast<int>(i - p * width);
    const float* src = part + p * (int64_t)S * width + c;
    float s = src[0];
    for (int k = 1; k < S; ++k) s = __fadd_rn(s, src[(int64_t)k * width]);
    y[i] = f2h(s);
  }
}

__global__ void k_identity_offsets(int32_t* off, int n) {
  if (threadIdx.x == 0) {
    off[0] = 0;
    off[1] = n;
  }
}

}  // namespace

// Choose the K-split of the W2 reduction: splits of `split_chunks` 16-byte
// chunks, a multiple of 32 (one per lane) where the row allows.
void decode_split(int inter, int* S, int* split_chunks) {
  const int nchunks = inter / 32;
  int sc = 64;  // 2 chunks per lane
  if (nchunks <= sc) sc = nchunks;
  *split_chunks = sc;
  *S = static_cast<int>(ceil_div(nchunks, sc));
}

size_t decode_smem_bytes(int hidden, int inter, int split_chunks) {
  const size_t lut = (size_t)kLut16Words * 4 + (size_t)kLut32Pairs * 8;
  const size_t xs_gate = (size_t)kMaxTok * hidden * 2;
  const size_t xs_down = (size_t)kMaxTok * split_chunks * 64;
  (void)inter;
  return lut + (xs_gate > xs_down ? xs_gate : xs_down);
}

int decode_max_tokens() { return kMaxTok; }

int launch_decode_experts(const moe_nf4_expert_t* experts, int E, const int32_t* expert_offsets,
                          const int32_t* pair_token, const uint16_t* x, int hidden, int inter,
                          uint16_t* h_sorted, float* y_part, int S, int split_chunks,
                          cudaStream_t s) {
  if (E < 1 || E > MOE_MAX_EXPERTS) return MOE_ERR_INVALID_ARG;
  if (hidden % kRowsPerItem || inter % kRowsPerItem || hidden % 32 || inter % 32)
    return MOE_ERR_UNSUPPORTED;
  DecodeArgs a{};
  for (int e = 0; e < E; ++e) a.ex.e[e] = experts[e];
  a.E = E;
  a.expert_offsets = expert_offsets;
  a.pair_token = pair_token;
  a.x = x;
  a.h_sorted = h_sorted;
  a.y_part = y_part;
  a.H = hidden;
  a.I = inter;
  a.S = S;
  a.split_chunks = split_chunks;
  const size_t smem = decode_smem_bytes(hidden, inter, split_chunks);
  static bool attr_done = false;
  if (!attr_done) {
    cudaFuncSetAttribute(k_gate_up_decode, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
    cudaFuncSetAttribute(k_down_decode, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
    attr_done = true;
  }
  if (smem > 160 * 1024) return MOE_ERR_UNSUPPORTED;
  const int grid_cap = sm_count() * 2;
  const int gate_items = E * (inter / kRowsPerItem);
  const int down_items = E * S * (hidden / kRowsPerItem);
  k_gate_up_decode<<<gate_items < grid_cap ? gate_items : grid_cap, kThreads, smem, s>>>(a);
  MOE_CHECK_LAUNCH();
  k_down_decode<<<down_items < grid_cap ? down_items : grid_cap, kThreads, smem, s>>>(a);
  MOE_CHECK_LAUNCH();
  return MOE_OK;
}

int launch_reduce_partials(const float* part, int64_t P, int S, int width, uint16_t* y,
                           cudaStream_t s) {
  int64_t blocks = ceil_div(P * width, 256);
  int grid = static_cast<int>(blocks < sm_count() * 8 ? blocks : sm_count() * 8);
  k_reduce_partials<<<grid > 0 ? grid : 1, 256, 0, s>>>(part, P, S, width, y);
  MOE_CHECK_LAUNCH();
  return MOE_OK;
}

int launch_identity_offsets(int32_t* off, int n, cudaStream_t s) {
  k_identity_offsets<<<1, 32, 0, s>>>(off, n);
  MOE_CHECK_LAUNCH();
  return MOE_OK;
}

}  // namespace moe
