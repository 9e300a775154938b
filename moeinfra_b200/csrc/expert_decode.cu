// Decode-path SwiGLU experts (1..8 tokens per expert) on tile16 NF4 weights.
//
// Reference: ReconstructedNF4Expert.forward (transfer/nf4_reconstruct.py:152-155),
// y = w2(silu(w1 x) * w3 x) with three bitsandbytes Linear4bit layers in fp16
// compute (:94).  bitsandbytes takes its 4-bit GEMV for a single input row
// and dequant(bf16) -> fp16 GEMM otherwise; the kernels pick per expert from
// its device-side token count n:
//   n == 1 ("gemv"):  y_row += absmax_b * sum_{i in block b} fp16(code_i) * x_i
//                     (absmax in fp32 per 64-element block; bitsandbytes rounds
//                     fp16(code)*fp16(absmax) per weight instead);
//   n >= 2 ("multi"): w_i = fp16(bf16(code_i * absmax_b)), y = sum w_i x_i;
// exact fp16 products, fp32 accumulation, outputs rounded once to fp16.
//
// Design (HBM-bound streaming, no weight byte read twice):
//   * weights are in the tile16 layout (nf4_layout.cu): per 64-element block a
//     thread (g = lane/4, t = lane%4) loads 8 bytes of MMA row g and of row
//     g+8, and the warp's loads are 256 contiguous bytes; streaming loads go
//     straight to registers (weights never touch shared memory, which is kept
//     for the decode table);
//   * packed bytes index a shared-memory table placed at shared-window address
//     0x10000: entry (byte, lane) is the byte's two fp16 codes (32 bank
//     replicas) and, at +128, its two fp32 codes (16 replicas), so the address
//     is a single byte-permute of the packed word;
//   * the multiply-adds are m16n8k16 MMAs.  MMA j of a block takes bytes 2j,
//     2j+1 (elements 16t+4j..16t+4j+3) as virtual K columns 2t,2t+1 /
//     2t+8,2t+9, which makes the B fragment exactly the thread's own x words;
//     B column g carries token g (n > 1) or the single token (n == 1);
//   * 16 warps per CTA split K; their partials meet in shared memory in warp
//     order (deterministic).
//   gate_up: item = 8 rows; MMA rows 0..7 are W1 rows, 8..15 the same W3 rows,
//            so g and u of a (row, token) end up in one thread.
//   down   : item = (16 rows, K split s of 2048 elements); split partials go
//            to y_part[slot][S][H] and the combine kernel sums them in order.
#include "common.cuh"

namespace moe {
namespace {

constexpr int kWarpsK = 16;           // warps per CTA, each a K part
constexpr int kThreadsK = kWarpsK * 32;
constexpr int kMaxTok = 8;            // tokens per expert on this path
constexpr int kDownSlice = 2048;      // K elements per down split
constexpr uint32_t kLutWin = 0x10000;
constexpr int kDynSmem = 0x20000;     // dynamic allocation covering the window

struct DecodeArgs {
  ExpertTable ex;
  int E;
  const int32_t* expert_offsets;  // [E+1]
  const int32_t* pair_token;      // token row of each sorted pair (or null: identity)
  const uint16_t* x;              // fp16 input rows [*, H]
  uint16_t* h_sorted;             // fp16 [P, I]
  float* y_part;                  // fp32 [P][S][H]
  int H, I, S;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ float2 lds64f(uint32_t addr) {
  float2 v;
  asm volatile("ld.shared.v2.f32 {%0,%1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint2 ldg_stream64(const uint8_t* p) {
  return __ldcs(reinterpret_cast<const uint2*>(p));
}
// Hint: pull [p, p + bytes) into L2 (bytes a multiple of 16, p 16-byte aligned).
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Contiguous item range [begin, end) of this CTA (neighbouring items share
// tiles, so upcoming tiles are contiguous ranges worth prefetching).
__device__ __forceinline__ void cta_range(int total, int* begin, int* end) {
  const int64_t b = (int64_t)total * blockIdx.x / gridDim.x;
  const int64_t e = (int64_t)total * (blockIdx.x + 1) / gridDim.x;
  *begin = static_cast<int>(b);
  *end = static_cast<int>(e);
}

constexpr int kPrefetchItems = 4;  // L2 prefetch distance in items

template <int K>
__device__ __forceinline__ uint32_t perm_addr(uint32_t w, uint32_t base) {
  return __byte_perm(w, base, 0x7604u | (K << 4));
}

// A-fragment register (fp16 pair) of byte K of w.
template <bool kMulti, int K>
__device__ __forceinline__ uint32_t decode(uint32_t w, uint32_t base, float absmax) {
  if (kMulti) {
    const float2 c = lds64f(perm_addr<K>(w, base));
    return nf4_pair_multirow(c.x, c.y, absmax);
  } else {
    return lds32(perm_addr<K>(w, base));
  }
}

__device__ __forceinline__ void mma16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// One 64-element block into d (rows g, g+8; columns 2t, 2t+1).
template <bool kMulti>
__device__ __forceinline__ void block_mma(uint2 qa, uint2 qb, float sa, float sb, const uint32_t* xw,
                                          uint32_t base, float* d) {
  mma16816(d, decode<kMulti, 0>(qa.x, base, sa), decode<kMulti, 0>(qb.x, base, sb),
           decode<kMulti, 1>(qa.x, base, sa), decode<kMulti, 1>(qb.x, base, sb), xw[0], xw[1]);
  mma16816(d, decode<kMulti, 2>(qa.x, base, sa), decode<kMulti, 2>(qb.x, base, sb),
           decode<kMulti, 3>(qa.x, base, sa), decode<kMulti, 3>(qb.x, base, sb), xw[2], xw[3]);
  mma16816(d, decode<kMulti, 0>(qa.y, base, sa), decode<kMulti, 0>(qb.y, base, sb),
           decode<kMulti, 1>(qa.y, base, sa), decode<kMulti, 1>(qb.y, base, sb), xw[4], xw[5]);
  mma16816(d, decode<kMulti, 2>(qa.y, base, sa), decode<kMulti, 2>(qb.y, base, sb),
           decode<kMulti, 3>(qa.y, base, sa), decode<kMulti, 3>(qb.y, base, sb), xw[6], xw[7]);
}

__device__ __forceinline__ bool build_lut(const float* __restrict__ code, const void* dyn) {
  __shared__ float s_code[16];
  const uint32_t base = smem_u32(dyn);
  const bool ok = base <= kLutWin && base + kDynSmem >= kLutWin + 0x10000;
  if (threadIdx.x < 16) s_code[threadIdx.x] = code[threadIdx.x];
  __syncthreads();
  if (ok) {
    for (int i = threadIdx.x; i < 256 * 64; i += blockDim.x) {
      const int v = i >> 6, j = i & 63;
      uint32_t val;
      if (j < 32) {
        __half2 h = __floats2half2_rn(s_code[v >> 4], s_code[v & 15]);
        val = *reinterpret_cast<uint32_t*>(&h);
      } else {
        val = __float_as_uint((j & 1) ? s_code[v & 15] : s_code[v >> 4]);
      }
      asm volatile("st.shared.b32 [%0], %1;" ::"r"(kLutWin + v * 256 + j * 4), "r"(val));
    }
  }
  __syncthreads();
  return ok;
}

struct Active {
  int n;
  int first;
};

// Experts this launch serves: 1-token experts (!kMulti) or 2..8-token experts.
template <bool kMulti>
__device__ __forceinline__ Active load_active(const DecodeArgs& a, int* s_off, int* s_active) {
  __shared__ int s_n;
  if (threadIdx.x == 0) {
    int n = 0;
    for (int e = 0; e <= a.E; ++e) s_off[e] = a.expert_offsets[e];
    for (int e = 0; e < a.E; ++e) {
      const int cnt = s_off[e + 1] - s_off[e];
      if (kMulti ? (cnt > 1 && cnt <= kMaxTok) : (cnt == 1)) s_active[n++] = e;
    }
    s_n = n;
  }
  __syncthreads();
  return Active{s_n, s_n > 0 ? s_active[0] : 0};
}

// x words of this thread for blocks [blk0, blk0+NBW): elements blk*64+16t..+16
// of the token its B column carries (zeros past the expert's token count).
template <int NBW>
__device__ __forceinline__ void load_x(const uint16_t* row, bool valid, int blk0, int blk_end,
                                       int lane, uint32_t (*xr)[8]) {
  const int t = lane & 3;
#pragma unroll
  for (int kb = 0; kb < NBW; ++kb) {
    uint4 u0 = make_uint4(0, 0, 0, 0), u1 = u0;
    if (valid && blk0 + kb < blk_end) {
      const uint4* p = reinterpret_cast<const uint4*>(row + (blk0 + kb) * 64 + 16 * t);
      u0 = p[0];
      u1 = p[1];
    }
    xr[kb][0] = u0.x; xr[kb][1] = u0.y; xr[kb][2] = u0.z; xr[kb][3] = u0.w;
    xr[kb][4] = u1.x; xr[kb][5] = u1.y; xr[kb][6] = u1.z; xr[kb][7] = u1.w;
  }
}

// Items per reduction batch: one barrier per batch; partials of two batches
// live in the dynamic shared memory below the table window.
template <bool kMulti>
constexpr int batch_items() { return kMulti ? 2 : 4; }
template <bool kMulti>
constexpr int red_cols() { return kMulti ? kMaxTok : 1; }
template <bool kMulti>
constexpr int red_floats() { return 2 * batch_items<kMulti>() * kWarpsK * 16 * red_cols<kMulti>(); }

// Register-resident loads of one item (this warp's K part, rows g and g+8).
template <int NBW>
struct ItemLoads {
  uint2 qa[NBW], qb[NBW];
  float sa[NBW], sb[NBW];
};

// Loads of MMA rows A (tile row ra) and B (tile row rb_) of matrices ma / mb,
// blocks [blk0, blk0+NBW) of tile rb, skipping blocks >= blk_end.
template <int NBW>
__device__ __forceinline__ void load_item(ItemLoads<NBW>& L, const moe_nf4_matrix_t& ma, int ra,
                                          const moe_nf4_matrix_t& mb, int rb_, int rb, int nblk,
                                          int blk0, int blk_end, int t) {
#pragma unroll
  for (int kb = 0; kb < NBW; ++kb) {
    L.qa[kb] = L.qb[kb] = make_uint2(0x77777777u, 0x77777777u);  // NF4 code 7 == 0.0
    L.sa[kb] = L.sb[kb] = 0.f;
    if (blk0 + kb < blk_end) {
      const int64_t seg = ((int64_t)rb * nblk + blk0 + kb) * 16;
      L.qa[kb] = ldg_stream64(ma.q + (seg + ra) * 32 + t * 8);
      L.qb[kb] = ldg_stream64(mb.q + (seg + rb_) * 32 + t * 8);
      L.sa[kb] = __ldg(ma.absmax + seg + ra);
      L.sb[kb] = __ldg(mb.absmax + seg + rb_);
    }
  }
}

// acc[0..1] = MMA row A (columns 2t, 2t+1), acc[2..3] = MMA row B.
template <int NBW, bool kMulti>
__device__ __forceinline__ void compute_item(const ItemLoads<NBW>& L, const uint32_t (*xr)[8],
                                             uint32_t base, float* acc) {
  acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
#pragma unroll
  for (int kb = 0; kb < NBW; ++kb) {
    if (kMulti) {
      block_mma<true>(L.qa[kb], L.qb[kb], L.sa[kb], L.sb[kb], xr[kb], base, acc);
    } else {
      float d[4] = {0.f, 0.f, 0.f, 0.f};
      block_mma<false>(L.qa[kb], L.qb[kb], 0.f, 0.f, xr[kb], base, d);
      acc[0] = fmaf(L.sa[kb], d[0], acc[0]);
      acc[2] = fmaf(L.sb[kb], d[2], acc[2]);
    }
  }
}

template <bool kMulti>
__device__ __forceinline__ void stash(float* red, int slot, int warp, int g, int t, const float* acc) {
  constexpr int C = red_cols<kMulti>();
  float* p = red + ((slot * kWarpsK + warp) * 16) * C;
  if (kMulti) {
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      p[g * C + 2 * t + c] = acc[c];
      p[(g + 8) * C + 2 * t + c] = acc[2 + c];
    }
  } else if (t == 0) {
    p[g] = acc[0];
    p[g + 8] = acc[2];
  }
}

// Sum of the 16 warp partials (warp order) of (slot, row, column).
template <bool kMulti>
__device__ __forceinline__ float reduce_partials(const float* red, int slot, int row, int col) {
  constexpr int C = red_cols<kMulti>();
  const float* p = red + (slot * kWarpsK * 16 + row) * C + col;
  float s = p[0];
#pragma unroll
  for (int w = 1; w < kWarpsK; ++w) s = __fadd_rn(s, p[w * 16 * C]);
  return s;
}

// gate_up.  NBW = 64-element blocks per warp (16 warps split H).  Item = 8 rows
// of W1 and the same 8 rows of W3 (one MMA).
template <int NBW, bool kMulti>
__global__ void __launch_bounds__(kThreadsK, 1) k_gate_up_mma(const __grid_constant__ DecodeArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ int s_off[MOE_MAX_EXPERTS + 1];
  __shared__ int s_active[MOE_MAX_EXPERTS];
  constexpr int B = batch_items<kMulti>();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  Active act;
  float* red = nullptr;
  {
    act = load_active<kMulti>(a, s_off, s_active);
    if (act.n == 0) return;
    if (smem_u32(smem) + red_floats<kMulti>() * 4 > kLutWin) return;
    if (!build_lut(a.ex.e[act.first].w1.code, smem)) return;
    red = reinterpret_cast<float*>(smem);
  }
  const int H = a.H, I = a.I;
  const int nblk = H / 64;
  const int items_per_expert = I / 8;  // half tiles of 8 rows
  const int total = act.n * items_per_expert;
  int first, last;
  cta_range(total, &first, &last);
  const int my_items = last - first;
  const uint32_t base = kMulti ? (kLutWin | 128u | ((lane & 15) * 8)) : (kLutWin | (lane * 4));
  const int blk0 = warp * NBW;
  int staged = -1;
  uint32_t xr[NBW][8];
  ItemLoads<NBW> cur, nxt;

  auto item_of = [&](int i) { return first + i; };
  // One thread pulls the whole 16-row tile (W1, W3, both absmax) of an upcoming
  // item into L2 when that item starts a tile (or starts this CTA's range).
  auto prefetch = [&](int i) {
    if (threadIdx.x != 0 || i >= my_items) return;
    const int item = item_of(i);
    const int hi = item % items_per_expert;
    if ((hi & 1) && i != 0) return;
    const moe_nf4_expert_t& ex = a.ex.e[s_active[item / items_per_expert]];
    const int64_t tile = hi >> 1;
    const uint32_t qbytes = 16u * (H / 2), abytes = 16u * (H / 64) * 4u;
    prefetch_l2(ex.w1.q + tile * qbytes, qbytes);
    prefetch_l2(ex.w3.q + tile * qbytes, qbytes);
    prefetch_l2(ex.w1.absmax + tile * (abytes / 4), abytes);
    prefetch_l2(ex.w3.absmax + tile * (abytes / 4), abytes);
  };
  for (int i = 0; i < kPrefetchItems && i < my_items; ++i) prefetch(i);
  auto issue = [&](ItemLoads<NBW>& L, int i) {
    const int item = item_of(i);
    const moe_nf4_expert_t& ex = a.ex.e[s_active[item / items_per_expert]];
    const int hi = item % items_per_expert;
    const int rsub = (hi & 1) * 8 + g;
    load_item<NBW>(L, ex.w1, rsub, ex.w3, rsub, hi >> 1, nblk, blk0, nblk, t);
  };
  if (my_items > 0) issue(cur, 0);
  for (int i = 0; i < my_items; ++i) {
    prefetch(i + kPrefetchItems);
    if (i + 1 < my_items) issue(nxt, i + 1);
    const int item = item_of(i);
    const int e = s_active[item / items_per_expert];
    const int tok0 = s_off[e];
    const int n = s_off[e + 1] - tok0;
    if (e != staged) {
      const int tok = kMulti ? g : 0;
      const bool valid = tok < n;
      const int64_t xrow =
          valid ? (a.pair_token ? a.pair_token[tok0 + tok] : (int64_t)(tok0 + tok)) : 0;
      load_x<NBW>(a.x + xrow * H, valid, blk0, nblk, lane, xr);
      staged = e;
    }
    float acc[4];
    compute_item<NBW, kMulti>(cur, xr, base, acc);
    const int slot = (i / B) % 2 * B + i % B;
    stash<kMulti>(red, slot, warp, g, t, acc);
    if (i % B == B - 1 || i == my_items - 1) {
      __syncthreads();
      // Finalize the batch: items i0..i of this batch, 8 rows x tokens each.
      const int i0 = i - i % B;
      const int nb = i - i0 + 1;
      for (int job = threadIdx.x; job < nb * 8 * kMaxTok; job += blockDim.x) {
        const int bi = job / (8 * kMaxTok), rem = job % (8 * kMaxTok);
        const int rr = rem & 7, tok = rem >> 3;
        const int it2 = item_of(i0 + bi);
        const int e2 = s_active[it2 / items_per_expert];
        const int t0 = s_off[e2], n2 = s_off[e2 + 1] - t0;
        if (tok >= (kMulti ? n2 : 1)) continue;
        const int sl = ((i0 + bi) / B) % 2 * B + bi;
        const float gs = reduce_partials<kMulti>(red, sl, rr, kMulti ? tok : 0);
        const float us = reduce_partials<kMulti>(red, sl, rr + 8, kMulti ? tok : 0);
        const int hi = it2 % items_per_expert;
        const int r = (hi >> 1) * 16 + (hi & 1) * 8 + rr;
        a.h_sorted[(int64_t)(t0 + tok) * I + r] = swiglu_f16(f2h(gs), f2h(us));
      }
    }
    cur = nxt;
  }
}

// down.  NBW = 64-element blocks per warp of one 2048-element split.  Item =
// (split s, tile of 16 W2 rows).
template <int NBW, bool kMulti>
__global__ void __launch_bounds__(kThreadsK, 1) k_down_mma(const __grid_constant__ DecodeArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ int s_off[MOE_MAX_EXPERTS + 1];
  __shared__ int s_active[MOE_MAX_EXPERTS];
  constexpr int B = batch_items<kMulti>();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  Active act;
  float* red = nullptr;
  {
    act = load_active<kMulti>(a, s_off, s_active);
    if (act.n == 0) return;
    if (smem_u32(smem) + red_floats<kMulti>() * 4 > kLutWin) return;
    if (!build_lut(a.ex.e[act.first].w2.code, smem)) return;
    red = reinterpret_cast<float*>(smem);
  }
  const int H = a.H, I = a.I;
  const int nblk = I / 64;
  const int tiles = H / 16;
  const int items_per_expert = a.S * tiles;
  const int total = act.n * items_per_expert;
  int first, last;
  cta_range(total, &first, &last);
  const int my_items = last - first;
  const uint32_t base = kMulti ? (kLutWin | 128u | ((lane & 15) * 8)) : (kLutWin | (lane * 4));
  int staged_e = -1, staged_s = -1;
  uint32_t xr[NBW][8];
  ItemLoads<NBW> cur, nxt;

  auto item_of = [&](int i) { return first + i; };
  // One thread pulls an upcoming item's blocks (contiguous in tile16) into L2.
  auto prefetch = [&](int i) {
    if (threadIdx.x != 0 || i >= my_items) return;
    const int item = item_of(i);
    const moe_nf4_expert_t& ex = a.ex.e[s_active[item / items_per_expert]];
    const int rem = item % items_per_expert;
    const int s = rem / tiles, rb = rem % tiles;
    const int b0 = s * (kDownSlice / 64), b1 = min(b0 + kDownSlice / 64, nblk);
    const int64_t seg0 = ((int64_t)rb * nblk + b0) * 16;
    prefetch_l2(ex.w2.q + seg0 * 32, (uint32_t)(b1 - b0) * 512u);
    prefetch_l2(ex.w2.absmax + seg0, (uint32_t)(b1 - b0) * 64u);
  };
  for (int i = 0; i < kPrefetchItems && i < my_items; ++i) prefetch(i);
  auto issue = [&](ItemLoads<NBW>& L, int i) {
    const int item = item_of(i);
    const moe_nf4_expert_t& ex = a.ex.e[s_active[item / items_per_expert]];
    const int rem = item % items_per_expert;
    const int s = rem / tiles, rb = rem % tiles;
    const int b0 = s * (kDownSlice / 64) + warp * NBW;
    const int bend = min((s + 1) * (kDownSlice / 64), nblk);
    load_item<NBW>(L, ex.w2, g, ex.w2, g + 8, rb, nblk, b0, bend, t);
  };
  if (my_items > 0) issue(cur, 0);
  for (int i = 0; i < my_items; ++i) {
    prefetch(i + kPrefetchItems);
    if (i + 1 < my_items) issue(nxt, i + 1);
    const int item = item_of(i);
    const int e = s_active[item / items_per_expert];
    const int rem = item % items_per_expert;
    const int s = rem / tiles;
    const int tok0 = s_off[e];
    const int n = s_off[e + 1] - tok0;
    if (e != staged_e || s != staged_s) {
      const int blk0 = s * (kDownSlice / 64) + warp * NBW;
      const int blk_end = min((s + 1) * (kDownSlice / 64), nblk);
      const int tok = kMulti ? g : 0;
      const bool valid = tok < n;
      load_x<NBW>(a.h_sorted + (int64_t)(tok0 + (valid ? tok : 0)) * I, valid, blk0, blk_end,
                  lane, xr);
      staged_e = e;
      staged_s = s;
    }
    float acc[4];
    compute_item<NBW, kMulti>(cur, xr, base, acc);
    const int slot = (i / B) % 2 * B + i % B;
    stash<kMulti>(red, slot, warp, g, t, acc);
    if (i % B == B - 1 || i == my_items - 1) {
      __syncthreads();
      const int i0 = i - i % B;
      const int nb = i - i0 + 1;
      for (int job = threadIdx.x; job < nb * 16 * kMaxTok; job += blockDim.x) {
        const int bi = job / (16 * kMaxTok), rem2 = job % (16 * kMaxTok);
        const int rr = rem2 & 15, tok = rem2 >> 4;
        const int it2 = item_of(i0 + bi);
        const int e2 = s_active[it2 / items_per_expert];
        const int t0 = s_off[e2], n2 = s_off[e2 + 1] - t0;
        if (tok >= (kMulti ? n2 : 1)) continue;
        const int sl = ((i0 + bi) / B) % 2 * B + bi;
        const float ys = reduce_partials<kMulti>(red, sl, rr, kMulti ? tok : 0);
        const int r2 = it2 % items_per_expert;
        const int s2 = r2 / tiles, rb2 = r2 % tiles;
        a.y_part[((int64_t)(t0 + tok) * a.S + s2) * H + rb2 * 16 + rr] = ys;
      }
    }
    cur = nxt;
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

template <class K>
bool smem_attr(K kernel) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kDynSmem) ==
         cudaSuccess;
}

template <bool kMulti>
bool attrs() {
  return smem_attr(k_gate_up_mma<1, kMulti>) && smem_attr(k_gate_up_mma<2, kMulti>) &&
         smem_attr(k_gate_up_mma<4, kMulti>) && smem_attr(k_gate_up_mma<8, kMulti>) &&
         smem_attr(k_down_mma<kDownSlice / (64 * kWarpsK), kMulti>);
}

// Blocks per K part of the gate_up kernels: ceil(H / 64 / 16) rounded up to
// a power of two (parts past the row are idle).
int gate_nbw(int hidden) {
  const int need = static_cast<int>(ceil_div(hidden / 64, kWarpsK));
  return need <= 1 ? 1 : need <= 2 ? 2 : need <= 4 ? 4 : need <= 8 ? 8 : -1;
}

template <bool kMulti>
int launch_gate(const DecodeArgs& a, cudaStream_t s) {
  const int grid = sm_count();
  switch (gate_nbw(a.H)) {
    case 1: k_gate_up_mma<1, kMulti><<<grid, kThreadsK, kDynSmem, s>>>(a); break;
    case 2: k_gate_up_mma<2, kMulti><<<grid, kThreadsK, kDynSmem, s>>>(a); break;
    case 4: k_gate_up_mma<4, kMulti><<<grid, kThreadsK, kDynSmem, s>>>(a); break;
    case 8: k_gate_up_mma<8, kMulti><<<grid, kThreadsK, kDynSmem, s>>>(a); break;
    default: return MOE_ERR_UNSUPPORTED;
  }
  MOE_CHECK_LAUNCH();
  return MOE_OK;
}

template <bool kMulti>
int launch_down(const DecodeArgs& a, cudaStream_t s) {
  k_down_mma<kDownSlice / (64 * kWarpsK), kMulti><<<sm_count(), kThreadsK, kDynSmem, s>>>(a);
  MOE_CHECK_LAUNCH();
  return MOE_OK;
}

}  // namespace

// Shapes the decode kernels accept: H and I multiples of 64 (one absmax block)
// with H up to 8192.
bool decode_supported(int hidden, int inter) {
  return hidden > 0 && inter > 0 && hidden % 64 == 0 && inter % 64 == 0 && gate_nbw(hidden) > 0;
}

// Down-projection K splits of 2048 elements (the last may be partial).
int decode_splits(int inter) { return static_cast<int>(ceil_div(inter, kDownSlice)); }
int decode_max_tokens() { return kMaxTok; }

int launch_decode_experts(const moe_nf4_expert_t* experts, int E, const int32_t* expert_offsets,
                          const int32_t* pair_token, const uint16_t* x, int hidden, int inter,
                          uint16_t* h_sorted, float* y_part, int max_tokens_per_expert,
                          cudaStream_t s) {
  if (E < 1 || E > MOE_MAX_EXPERTS) return MOE_ERR_INVALID_ARG;
  if (!decode_supported(hidden, inter)) return MOE_ERR_UNSUPPORTED;
  static bool attr_ok = attrs<false>() && attrs<true>();
  if (!attr_ok) return MOE_ERR_CUDA;
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
  a.S = decode_splits(inter);
  const bool multi = max_tokens_per_expert > 1;
  int st = launch_gate<false>(a, s);
  if (st == MOE_OK && multi) st = launch_gate<true>(a, s);
  if (st == MOE_OK) st = launch_down<false>(a, s);
  if (st == MOE_OK && multi) st = launch_down<true>(a, s);
  return st;
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
