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
//   down   : item = (16 rows per tile, 2 tiles for 1-token experts; K split s
//            of 2048 elements); split partials go to y_part[slot][S][H] and
//            are summed in split order by the combine.
// Both phases run in one launch per layer and token kind (k_stage_mma): a
// CTA's down items wait (bounded) on per-split counters that the CTAs
// producing those h rows publish.  For a 1-token layer the same launch also
// routes the token (in every CTA) and the last CTA to finish each 32-row
// group of the output writes its weighted combine.
#include "common.cuh"
#include "router_device.cuh"

namespace moe {
namespace {

constexpr int kWarpsK = 16;           // warps per CTA, each a K part
constexpr int kThreadsK = kWarpsK * 32;
constexpr int kMaxTok = 8;            // tokens per expert on this path
static_assert(kMaxTok == MOE_DECODE_MAX_ROWS, "decode row bound of the public header");
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
  int* sync;                      // [MOE_MAX_EXPERTS][S] gate_up completion counters, zeroed
  int H, I, S;
  // Fused 1-token layer (route_wg != null): every CTA routes the token x[0]
  // itself; the last CTA to finish a row group writes its weighted combine.
  const uint16_t* route_wg;  // fp16 gate weights [E][H]
  int route_k;
  float* out_weights;        // [k] routing weights (written by CTA 0)
  int64_t* out_indices;      // [k] routed experts (written by CTA 0)
  uint16_t* out;             // [H] fp16 layer output
  int* rg_count;             // [H / 16] row-group completion counters, zeroed
  uint64_t wait_ns;          // limit of every bounded wait (moe_set_wait_limit_ns)
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
// The decode table is written once, before a barrier, and only read after it;
// the table reads and the MMAs are pure (non-volatile asm) so the compiler may
// interleave the blocks' table reads with the MMA chains.
__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ float2 lds64f(uint32_t addr) {
  float2 v;
  asm("ld.shared.v2.f32 {%0,%1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint2 ldg_stream64(const uint8_t* p) {
  return __ldcs(reinterpret_cast<const uint2*>(p));
}
// Hint: pull [p, p + bytes) into L2 (bytes a multiple of 16, p 16-byte
// aligned) when pred is set; a predicated instruction, not a branch.
__device__ __forceinline__ void prefetch_l2_if(bool pred, const void* p, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .pred q;\n\tsetp.ne.u32 q, %2, 0;\n\t"
      "@q cp.async.bulk.prefetch.L2.global [%0], %1;\n\t}" ::"l"(p),
      "r"(bytes), "r"((uint32_t)pred)
      : "memory");
}

// Contiguous item range [begin, end) of this CTA (neighbouring items share
// tiles, so upcoming tiles are contiguous ranges worth prefetching).
__device__ __forceinline__ void cta_range(int total, int* begin, int* end) {
  const int64_t b = (int64_t)total * blockIdx.x / gridDim.x;
  const int64_t e = (int64_t)total * (blockIdx.x + 1) / gridDim.x;
  *begin = static_cast<int>(b);
  *end = static_cast<int>(e);
}

// L2 prefetch distance in items (gate_up items are half tiles and prefetch
// whole tiles; down items are two tiles).
constexpr int kPrefetchGate = 2;
constexpr int kPrefetchDown = 2;

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
  asm(
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
    // Entry v: 32 words of the fp16 pair, then 16 fp32 pairs; 16-byte stores.
    for (int i = threadIdx.x; i < 256 * 16; i += blockDim.x) {
      const int v = i >> 4, q = i & 15;
      uint32_t w0, w1;
      if (q < 8) {
        __half2 h = __floats2half2_rn(s_code[v >> 4], s_code[v & 15]);
        w0 = w1 = *reinterpret_cast<uint32_t*>(&h);
      } else {
        w0 = __float_as_uint(s_code[v >> 4]);
        w1 = __float_as_uint(s_code[v & 15]);
      }
      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(kLutWin + v * 256 + q * 16),
                   "r"(w0), "r"(w1), "r"(w0), "r"(w1));
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
// of the token its B column carries (zeros past the expert's token count or
// past the row's last block).  kL2: rows written by other CTAs of the same
// launch, read through L2.
template <int NBW, bool kL2>
__device__ __forceinline__ void load_x(const uint16_t* row, bool valid, int blk0, int blk_end,
                                       int t, uint32_t (*xr)[8]) {
#pragma unroll
  for (int kb = 0; kb < NBW; ++kb) {
    uint4 u0 = make_uint4(0, 0, 0, 0), u1 = u0;
    if (valid && blk0 + kb < blk_end) {
      const uint4* p = reinterpret_cast<const uint4*>(row + (blk0 + kb) * 64 + 16 * t);
      if (kL2) {
        u0 = __ldcg(p);
        u1 = __ldcg(p + 1);
      } else {
        u0 = p[0];
        u1 = p[1];
      }
    }
    xr[kb][0] = u0.x; xr[kb][1] = u0.y; xr[kb][2] = u0.z; xr[kb][3] = u0.w;
    xr[kb][4] = u1.x; xr[kb][5] = u1.y; xr[kb][6] = u1.z; xr[kb][7] = u1.w;
  }
}

// Items per reduction batch (one barrier per batch); partials of two batches
// live in the dynamic shared memory below the table window.
template <bool kMulti>
constexpr int batch_items() { return kMulti ? 2 : 8; }
template <bool kMulti>
constexpr int red_cols() { return kMulti ? kMaxTok : 1; }
// Row tiles (16 rows) per down item: two for 1-token experts (an item then
// moves as many weight bytes as a gate_up item), one for 2..8 tokens (whose
// partials take 8 columns).
template <bool kMulti>
constexpr int down_tiles() { return kMulti ? 1 : 2; }
template <bool kMulti>
constexpr int red_floats() {
  return 2 * batch_items<kMulti>() * kWarpsK * 16 * down_tiles<kMulti>() * red_cols<kMulti>();
}

// Register-resident loads of one item: MMA rows g (qa) and g+8 (qb), blocks
// kb of this warp's K part, and the item's absmax.  kS = 0: sa[kb] / sb[kb]
// are the thread's own (rows g, g+8).  kS = 8 or 16 (cooperative): one load
// per lane, lane l holding block l / kS, row l % kS of the item's absmax
// chunk(s); threads fetch theirs with a shuffle (4x fewer load requests).
template <int NBW, int kS>
struct ItemLoads {
  uint2 qa[NBW], qb[NBW];
  float sa[kS ? 1 : NBW], sb[kS ? 1 : NBW];
};

// qa/qb: byte pointers of the thread's 8-byte segment of block 0 (rows g and
// g+8); consecutive blocks are 512 bytes apart.  Blocks with !valid(kb) read
// as code 7 (0.0).
template <int NBW, int kS, bool kFull>
__device__ __forceinline__ void load_codes(ItemLoads<NBW, kS>& L, const uint8_t* qa,
                                           const uint8_t* qb, int kb_valid) {
#pragma unroll
  for (int kb = 0; kb < NBW; ++kb) {
    if (kFull || kb < kb_valid) {
      L.qa[kb] = ldg_stream64(qa + kb * 512);
      L.qb[kb] = ldg_stream64(qb + kb * 512);
    } else {
      L.qa[kb] = L.qb[kb] = make_uint2(0x77777777u, 0x77777777u);  // NF4 code 7 == 0.0
    }
  }
}

// Per-thread absmax (kS = 0): blocks 16 floats apart; absmax 0 past the row.
template <int NBW, bool kFull>
__device__ __forceinline__ void load_abs_own(ItemLoads<NBW, 0>& L, const float* sa, const float* sb,
                                             int kb_valid) {
#pragma unroll
  for (int kb = 0; kb < NBW; ++kb) {
    const bool ok = kFull || kb < kb_valid;
    L.sa[kb] = ok ? __ldg(sa + kb * 16) : 0.f;
    L.sb[kb] = ok ? __ldg(sb + kb * 16) : 0.f;
  }
}

// absmax of block kb for the thread's rows g (a) and g+8 (b).
template <int NBW, int kS>
__device__ __forceinline__ void item_abs(const ItemLoads<NBW, kS>& L, int kb, int g, float& a,
                                         float& b) {
  if (kS == 0) {
    a = L.sa[kb];
    b = L.sb[kb];
  } else if (kS == 8) {  // gate_up: sa = W1 rows, sb = W3 rows of the 8-row item
    a = __shfl_sync(0xffffffffu, L.sa[0], kb * 8 + g);
    b = __shfl_sync(0xffffffffu, L.sb[0], kb * 8 + g);
  } else {  // down: sa = the 16 rows of the tile
    a = __shfl_sync(0xffffffffu, L.sa[0], kb * 16 + g);
    b = __shfl_sync(0xffffffffu, L.sa[0], kb * 16 + g + 8);
  }
}

// acc[0..1] = MMA row g (columns 2t, 2t+1), acc[2..3] = MMA row g+8.
template <int NBW, bool kMulti, int kS>
__device__ __forceinline__ void compute_item(const ItemLoads<NBW, kS>& L, const uint32_t (*xr)[8],
                                             uint32_t base, int g, float* acc) {
  acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
#pragma unroll
  for (int kb = 0; kb < NBW; ++kb) {
    float sa, sb;
    item_abs(L, kb, g, sa, sb);
    if (kMulti) {
      block_mma<true>(L.qa[kb], L.qb[kb], sa, sb, xr[kb], base, acc);
    } else {
      float d[4] = {0.f, 0.f, 0.f, 0.f};
      block_mma<false>(L.qa[kb], L.qb[kb], 0.f, 0.f, xr[kb], base, d);
      acc[0] = fmaf(sa, d[0], acc[0]);
      acc[2] = fmaf(sb, d[2], acc[2]);
    }
  }
}

// Partials of (slot, warp) take R rows x C columns; this MMA tile's rows
// start at row0.
template <bool kMulti, int R>
__device__ __forceinline__ void stash(float* red, int slot, int warp, int g, int t, const float* acc,
                                      int row0) {
  constexpr int C = red_cols<kMulti>();
  float* p = red + ((slot * kWarpsK + warp) * R + row0) * C;
  if (kMulti) {
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      p[g * C + 2 * t + c] = acc[c];
      p[(g + 8) * C + 2 * t + c] = acc[2 + c];
    }
  } else {
    // One token: every column of the MMA carries it, so the four t-lanes of a
    // row hold the same sum; all write it (same word, same value).
    p[g] = acc[0];
    p[g + 8] = acc[2];
  }
}

// Sum of the 16 warp partials (warp order) of (slot, row, column).
template <bool kMulti, int R>
__device__ __forceinline__ float reduce_partials(const float* red, int slot, int row, int col) {
  constexpr int C = red_cols<kMulti>();
  const float* p = red + (slot * kWarpsK * R + row) * C + col;
  float s = p[0];
#pragma unroll
  for (int w = 1; w < kWarpsK; ++w) s = __fadd_rn(s, p[w * R * C]);
  return s;
}

// Where a reduced item goes (written by warp 0 before the batch barrier).
struct SlotMeta {
  int tok0;  // first sorted pair of the item's expert
  int n;     // tokens of that expert
  int row;   // first output row of the item
  int s;     // down: K split
};

// Item order of a CTA: (active expert ai, index r within the expert), r
// fastest; advanced without division.
struct Cursor {
  int ai, r;
  __device__ __forceinline__ void next(int per) {
    if (++r == per) {
      r = 0;
      ++ai;
    }
  }
};

// ---------------------------------------------------------------------------
// Cross-CTA hand-off between the two phases of one launch.
//
// a.sync[ai * S + s] counts the gate_up items of active expert ai whose rows
// fall in down split s and whose h rows are written.  A CTA publishes its
// items once, after the barrier that follows its last stores (barrier, then
// one thread: release fence, atomic adds); a fence per batch would wait on
// the ring's loads in flight.  The down phase acquires the counter
// before it reads the split's h rows, which it reads through L2 (ld.cg).
// The counters are zeroed by the kernel that runs before each launch on the
// stream (permute / offsets) or by a memset.
MOE_DEFINE_ERROR_WORD()

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait until *p >= target; after limit_ns of %globaltimer it records
// the timeout in the device error word and returns (the launch's results are
// then invalid; moe_stream_check reports MOE_ERR_TIMEOUT).
__device__ __forceinline__ void wait_count(const int* p, int target, uint64_t limit_ns) {
  if (ld_acquire(p) >= target) return;
  const uint64_t t0 = globaltimer_ns();
  while (ld_acquire(p) < target) {
    if (globaltimer_ns() - t0 > limit_ns) {
      set_device_error(kErrWaitTimeout);
      return;
    }
    __nanosleep(256);
  }
}

// Release fence of the publishing thread (orders the CTA's stores, made
// visible to it by the preceding barrier, before the counter update).
__device__ __forceinline__ void fence_release_gpu() {
  asm volatile("fence.acq_rel.gpu;" ::: "memory");
}

// Adds the gate_up items [first, last) (per items per active expert, 256 per
// down split) to their (expert, split) counters.
__device__ __forceinline__ void publish_items(int* sync, int first, int last, int per, int S) {
  constexpr int kItemsPerSplit = kDownSlice / 8;
  fence_release_gpu();
  int i = first;
  while (i < last) {
    const int ai = i / per, r = i - ai * per;
    const int s = r / kItemsPerSplit;
    const int end = min(last, ai * per + min(per, (s + 1) * kItemsPerSplit));
    atomicAdd(sync + ai * S + s, end - i);
    i = end;
  }
}

// gate_up items of down split s (8 rows each).
__device__ __forceinline__ int split_items(int I, int s) {
  return min(kDownSlice, I - s * kDownSlice) / 8;
}

struct StageSmem {
  float* red;
  const int* s_off;
  const int* s_active;
  SlotMeta* s_meta;
  const int32_t* pair_token;  // token row of each sorted pair (null: identity)
};

// gate_up phase.  NBW = 64-element blocks per warp (16 warps split H).  Item =
// 8 rows of W1 and the same 8 rows of W3 (one MMA), r = 2*tile + half.
template <int NBW, bool kMulti, bool kFull>
__device__ __forceinline__ void gate_phase(const DecodeArgs& a, const Active& act,
                                           const StageSmem& sm) {
  constexpr int B = batch_items<kMulti>();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int H = a.H, I = a.I;
  const int nblk = H / 64;
  const int per = I / 8;
  int first, last;
  cta_range(act.n * per, &first, &last);
  const int my_items = last - first;
  if (my_items <= 0) return;
  float* red = sm.red;
  const int* s_off = sm.s_off;
  const int* s_active = sm.s_active;
  SlotMeta* s_meta = sm.s_meta;
  const uint32_t base = kMulti ? (kLutWin | 128u | ((lane & 15) * 8)) : (kLutWin | (lane * 4));
  const int blk0 = warp * NBW;
  const int kb_valid = nblk - blk0;  // blocks of this warp inside the row
  const uint32_t tile_q = nblk * 512u, tile_s = nblk * 16u;
  // Cooperative absmax while the item's chunks fit the warp (NBW <= 4).
  constexpr int kS = NBW <= 4 ? 8 : 0;
  const int thr_q = blk0 * 512 + g * 32 + t * 8;
  const int thr_s = kS ? blk0 * 16 + (lane >> 3) * 16 + (lane & 7) : blk0 * 16 + g;
  const bool abs_ok = kS == 0 || ((lane >> 3) < NBW && (kFull || (lane >> 3) < kb_valid));

  uint32_t xr[NBW][8];
  ItemLoads<NBW, kS> L0, L1;
  // Load cursor: the load expert's per-lane bases and the next item's offsets
  // in it, advanced without multiplies (half 0 -> 1: +256 / +8; next tile).
  Cursor ld{first / per, first % per};
  const uint8_t *q1, *q3;
  const float *s1, *s3;
  auto ld_expert = [&](int ai) {
    const moe_nf4_expert_t& ex = a.ex.e[s_active[ai]];
    q1 = ex.w1.q + thr_q;
    q3 = ex.w3.q + thr_q;
    s1 = ex.w1.absmax + thr_s;
    s3 = ex.w3.absmax + thr_s;
  };
  ld_expert(ld.ai);
  uint32_t qo = (ld.r >> 1) * tile_q + (ld.r & 1) * 256u;
  uint32_t so = (ld.r >> 1) * tile_s + (ld.r & 1) * 8u;

  auto issue = [&](ItemLoads<NBW, kS>& L) {
    load_codes<NBW, kS, kFull>(L, q1 + qo, q3 + qo, kb_valid);
    if constexpr (kS == 0) {
      load_abs_own<NBW, kFull>(L, s1 + so, s3 + so, kb_valid);
    } else {
      L.sa[0] = abs_ok ? __ldg(s1 + so) : 0.f;
      L.sb[0] = abs_ok ? __ldg(s3 + so) : 0.f;
    }
    if (++ld.r == per) {
      ld.r = 0;
      qo = so = 0;
      if (++ld.ai < act.n) ld_expert(ld.ai);
    } else {
      const bool odd = ld.r & 1;
      qo += odd ? 256u : tile_q - 256u;
      so += odd ? 8u : tile_s - 8u;
    }
  };
  // Warp 0 walks the prefetch cursor; its lane 0 pulls the whole 16-row tile
  // (W1, W3, both absmax) of an item kPrefetchGate ahead into L2 when that
  // item starts a tile, up to the CTA's last item (past it the tiles are the
  // next CTA's, long since streamed).
  Cursor pf = ld;
  int pf_i = first;
  auto prefetch = [&]() {
    if (pf_i++ < last && pf.ai < act.n && (pf.r & 1) == 0) {
      const moe_nf4_expert_t& ex = a.ex.e[s_active[pf.ai]];
      const uint32_t tile = pf.r >> 1;
      const uint32_t qbytes = 16u * (H / 2), abytes = 16u * (H / 64) * 4u;
      const bool p = lane == 0;
      prefetch_l2_if(p, ex.w1.q + (size_t)tile * qbytes, qbytes);
      prefetch_l2_if(p, ex.w3.q + (size_t)tile * qbytes, qbytes);
      prefetch_l2_if(p, ex.w1.absmax + (size_t)tile * (abytes / 4), abytes);
      prefetch_l2_if(p, ex.w3.absmax + (size_t)tile * (abytes / 4), abytes);
    }
    pf.next(per);
  };
  if (warp == 0)
    for (int i = 0; i < kPrefetchGate; ++i) prefetch();

  // Compute cursor and its expert's token range.
  Cursor cp = ld;
  int staged = -1, tok0 = 0, n = 0;
  auto body = [&](const ItemLoads<NBW, kS>& L, int i) {
    if (warp == 0) prefetch();
    if (cp.ai != staged) {
      const int e = s_active[cp.ai];
      tok0 = s_off[e];
      n = s_off[e + 1] - tok0;
      const int tok = kMulti ? g : 0;
      const bool valid = tok < n;
      const int64_t xrow =
          valid ? (sm.pair_token ? sm.pair_token[tok0 + tok] : (int64_t)(tok0 + tok)) : 0;
      load_x<NBW, false>(a.x + xrow * H, valid, blk0, nblk, t, xr);
      staged = cp.ai;
    }
    float acc[4];
    compute_item<NBW, kMulti, kS>(L, xr, base, g, acc);
    const int slot = ((i / B) & 1) * B + i % B;
    stash<kMulti, 16>(red, slot, warp, g, t, acc, 0);
    if (warp == 0) s_meta[slot] = SlotMeta{tok0, n, (cp.r >> 1) * 16 + (cp.r & 1) * 8, 0};
    cp.next(per);
    if (i % B == B - 1 || i == my_items - 1) {
      __syncthreads();
      // Finalize the batch: 8 rows x tokens of each of its items.
      const int i0 = i - i % B, sl0 = ((i0 / B) & 1) * B;
      const int jobs = (i - i0 + 1) * 8 * red_cols<kMulti>();
      for (int job = threadIdx.x; job < jobs; job += kThreadsK) {
        const int bi = job / (8 * red_cols<kMulti>()), rem = job % (8 * red_cols<kMulti>());
        const int rr = rem & 7, tk = rem >> 3;
        const SlotMeta m = s_meta[sl0 + bi];
        if (tk >= m.n) continue;
        const float gs = reduce_partials<kMulti, 16>(red, sl0 + bi, rr, tk);
        const float us = reduce_partials<kMulti, 16>(red, sl0 + bi, rr + 8, tk);
        a.h_sorted[(int64_t)(m.tok0 + tk) * I + m.row + rr] = swiglu_f16(f2h(gs), f2h(us));
      }
    }
  };

  issue(L0);
  for (int i = 0; i < my_items; i += 2) {
    if (i + 1 < my_items) issue(L1);
    body(L0, i);
    if (i + 1 >= my_items) break;
    if (i + 2 < my_items) issue(L0);
    body(L1, i + 1);
  }
  // Every h store of this CTA, and every warp's reads of the partial slots,
  // are done after this barrier; then the CTA's items are published per
  // (expert, split) counter.
  __syncthreads();
  if (threadIdx.x == 0) publish_items(a.sync, first, last, per, a.S);
}

// down phase.  NBW = 64-element blocks per warp of one 2048-element split.
// Item = (split s, group rg of kT consecutive 16-row W2 tiles), rg fastest:
// r = s * groups + rg.
template <int NBW, bool kMulti, bool kFull>
__device__ __forceinline__ void down_phase(const DecodeArgs& a, const Active& act,
                                           const StageSmem& sm) {
  constexpr int B = batch_items<kMulti>();
  constexpr int kT = down_tiles<kMulti>();
  constexpr int kRows = 16 * kT;
  constexpr int C = red_cols<kMulti>();
  constexpr int kSplitBlocks = kDownSlice / 64;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int H = a.H, I = a.I;
  const int nblk = I / 64;
  const int groups = H / kRows;
  const int per = a.S * groups;
  int first, last;
  cta_range(act.n * per, &first, &last);
  const int my_items = last - first;
  if (my_items <= 0) return;
  float* red = sm.red;
  const int* s_off = sm.s_off;
  const int* s_active = sm.s_active;
  SlotMeta* s_meta = sm.s_meta;
  const uint32_t base = kMulti ? (kLutWin | 128u | ((lane & 15) * 8)) : (kLutWin | (lane * 4));
  const int wblk = warp * NBW;  // this warp's first block within a split
  const uint32_t tile_q = nblk * 512u, tile_s = nblk * 16u;
  // Cooperative absmax: a tile's NBW blocks x 16 rows are contiguous floats.
  constexpr int kS = NBW <= 2 ? 16 : 0;
  const int thr_q = wblk * 512 + g * 32 + t * 8;
  const int thr_s = kS ? wblk * 16 + lane : wblk * 16 + g;

  uint32_t xr[NBW][8];
  ItemLoads<NBW, kS> L0[kT], L1[kT];
  // Load cursor (ai, s, rg), the load expert's per-lane bases and the item's
  // offsets in them (next group: + kT tiles; next split: its first block).
  int l_ai = first / per, l_r = first % per;
  int l_s = l_r / groups, l_rg = l_r % groups;
  const uint8_t* qb;
  const float* sb;
  auto ld_expert = [&](int ai) {
    const moe_nf4_expert_t& ex = a.ex.e[s_active[ai]];
    qb = ex.w2.q + thr_q;
    sb = ex.w2.absmax + thr_s;
  };
  ld_expert(l_ai);
  uint32_t qo = l_rg * kT * tile_q + l_s * (kSplitBlocks * 512u);
  uint32_t so = l_rg * kT * tile_s + l_s * (kSplitBlocks * 16u);
  int kb_valid = nblk - l_s * kSplitBlocks - wblk;
  const int c_first_ai = l_ai, c_first_s = l_s, c_first_rg = l_rg;

  auto issue = [&](ItemLoads<NBW, kS>* L) {
    const bool abs_ok = kFull || (lane >> 4) < kb_valid;
#pragma unroll
    for (int tt = 0; tt < kT; ++tt) {
      load_codes<NBW, kS, kFull>(L[tt], qb + qo + tt * tile_q, qb + qo + tt * tile_q + 256, kb_valid);
      if constexpr (kS == 0)
        load_abs_own<NBW, kFull>(L[tt], sb + so + tt * tile_s, sb + so + tt * tile_s + 8, kb_valid);
      else
        L[tt].sa[0] = abs_ok ? __ldg(sb + so + tt * tile_s) : 0.f;
    }
    if (++l_rg < groups) {
      qo += kT * tile_q;
      so += kT * tile_s;
    } else {
      l_rg = 0;
      if (++l_s == a.S) {
        l_s = 0;
        if (++l_ai < act.n) ld_expert(l_ai);
      }
      qo = l_s * (kSplitBlocks * 512u);
      so = l_s * (kSplitBlocks * 16u);
      kb_valid = nblk - l_s * kSplitBlocks - wblk;
    }
  };
  // Warp 0 walks the prefetch cursor; its lane 0 pulls an upcoming item's
  // blocks (contiguous in tile16) into L2, up to the CTA's last item.
  int p_ai = c_first_ai, p_s = c_first_s, p_rg = c_first_rg;
  int p_i = first;
  auto prefetch = [&]() {
    if (p_i++ < last && p_ai < act.n) {
      const moe_nf4_expert_t& ex = a.ex.e[s_active[p_ai]];
      const int b0 = p_s * kSplitBlocks, b1 = min(b0 + kSplitBlocks, nblk);
      const bool p = lane == 0;
#pragma unroll
      for (int tt = 0; tt < kT; ++tt) {
        const int64_t seg0 = ((int64_t)(p_rg * kT + tt) * nblk + b0) * 16;
        prefetch_l2_if(p, ex.w2.q + seg0 * 32, (uint32_t)(b1 - b0) * 512u);
        prefetch_l2_if(p, ex.w2.absmax + seg0, (uint32_t)(b1 - b0) * 64u);
      }
    }
    if (++p_rg == groups) {
      p_rg = 0;
      if (++p_s == a.S) {
        p_s = 0;
        ++p_ai;
      }
    }
  };
  if (warp == 0)
    for (int i = 0; i < kPrefetchDown; ++i) prefetch();

  // Compute cursor, its expert's token range and the staged (expert, split).
  int c_ai = c_first_ai, c_s = c_first_s, c_rg = c_first_rg;
  int staged_ai = -1, staged_s = -1, tok0 = 0, n = 0;
  auto body = [&](const ItemLoads<NBW, kS>* L, int i) {
    if (warp == 0) prefetch();
    if (c_ai != staged_ai || c_s != staged_s) {
      const int e = s_active[c_ai];
      tok0 = s_off[e];
      n = s_off[e + 1] - tok0;
      // h rows of this split come from other CTAs' gate_up items.
      wait_count(a.sync + c_ai * a.S + c_s, split_items(I, c_s), a.wait_ns);
      const int blk0 = c_s * kSplitBlocks + wblk;
      const int tok = kMulti ? g : 0;
      const bool valid = tok < n;
      load_x<NBW, true>(a.h_sorted + (int64_t)(tok0 + (valid ? tok : 0)) * I, valid, blk0, nblk, t,
                        xr);
      staged_ai = c_ai;
      staged_s = c_s;
    }
    const int slot = ((i / B) & 1) * B + i % B;
#pragma unroll
    for (int tt = 0; tt < kT; ++tt) {
      float acc[4];
      compute_item<NBW, kMulti, kS>(L[tt], xr, base, g, acc);
      stash<kMulti, kRows>(red, slot, warp, g, t, acc, tt * 16);
    }
    if (warp == 0) s_meta[slot] = SlotMeta{tok0, n, c_rg * kRows, c_s};
    if (++c_rg == groups) {
      c_rg = 0;
      if (++c_s == a.S) {
        c_s = 0;
        ++c_ai;
      }
    }
    if (i % B == B - 1 || i == my_items - 1) {
      __syncthreads();
      const int i0 = i - i % B, sl0 = ((i0 / B) & 1) * B;
      const int jobs = (i - i0 + 1) * kRows * C;
      for (int job = threadIdx.x; job < jobs; job += kThreadsK) {
        const int bi = job / (kRows * C), rem = job % (kRows * C);
        const int rr = rem % kRows, tk = rem / kRows;
        const SlotMeta m = s_meta[sl0 + bi];
        if (tk >= m.n) continue;
        const float ys = reduce_partials<kMulti, kRows>(red, sl0 + bi, rr, tk);
        a.y_part[((int64_t)(m.tok0 + tk) * a.S + m.s) * H + m.row + rr] = ys;
      }
    }
  };

  issue(L0);
  for (int i = 0; i < my_items; i += 2) {
    if (i + 1 < my_items) issue(L1);
    body(L0, i);
    if (i + 1 >= my_items) break;
    if (i + 2 < my_items) issue(L0);
    body(L1, i + 1);
  }
}

// ---------------------------------------------------------------------------
// Fused 1-token layer: routing in every CTA, combine by row-group last arrivers.

// Routing of the layer's single token, identical in every CTA.
struct RouteSmem {
  double part[kWarpsK * MOE_MAX_EXPERTS];
  float w[8];          // routing weights in top-k output order
  int64_t idx[8];      // routed experts in top-k output order
  float w_slot[8];     // weight of the pair at sorted position p (ascending expert id)
  int32_t zero_tok[8];  // every pair reads token row 0
};

// Routing split: thread i takes the row's 16-byte vectors i, i + 512, ... and
// accumulates every expert from each (one load of the token per CTA).  The
// weights of its first vector for experts < kRoutePre are loaded before the
// wait on the predecessor (the gate weights do not depend on it).
constexpr int kRoutePre = 8;
__device__ __forceinline__ void route_preload(const DecodeArgs& a, uint4 (&wpre)[kRoutePre]) {
  const int nvec = a.H >> 3, v = threadIdx.x;
  const uint4* wg = reinterpret_cast<const uint4*>(a.route_wg);
#pragma unroll
  for (int e = 0; e < kRoutePre; ++e)
    wpre[e] = (e < a.E && v < nvec) ? __ldg(wg + (int64_t)e * nvec + v) : make_uint4(0, 0, 0, 0);
}

// acc += sum of the 8 exact fp16 x fp16 products of one vector (FP64 FMA:
// each product is exact in double, each add rounds to 53 bits).
__device__ __forceinline__ void dot8_f64(double& acc, const double (&hd)[8], const uint4& wv) {
  const __half2* ww = reinterpret_cast<const __half2*>(&wv);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float2 y = __half22float2(ww[q]);
    acc = fma((double)y.x, hd[2 * q], acc);
    acc = fma((double)y.y, hd[2 * q + 1], acc);
  }
}

__device__ __forceinline__ double warp_sum_f64(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Logits as the FP64 sum of the exact fp16 products (each thread sums its
// vectors in ascending order, then lanes by butterfly, then warps in order),
// rounded once to fp16 -- the correctly rounded logit, as the router kernels
// and a float64 matmul give; softmax and top-k as the router kernels; then
// the counting sort of the k pairs by expert (offsets, active experts).  The
// code runs once per launch, so it is kept short (cold instruction fetch).
__device__ __forceinline__ Active route_token(const DecodeArgs& a, const uint4 (&wpre)[kRoutePre],
                                              int* s_off, int* s_active, RouteSmem& rs) {
  __shared__ int s_n;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int E = a.E, k = a.route_k, H = a.H;
  const int nvec = H >> 3;
  const uint4* hrow = reinterpret_cast<const uint4*>(a.x);
  const uint4* wg = reinterpret_cast<const uint4*>(a.route_wg);
  double acc[kRoutePre];
#pragma unroll
  for (int e = 0; e < kRoutePre; ++e) acc[e] = 0.0;
  double* part = rs.part;  // [kWarpsK][MOE_MAX_EXPERTS]
  for (int v = threadIdx.x; v < nvec; v += kThreadsK) {
    const uint4 hv = hrow[v];
    const __half2* hh = reinterpret_cast<const __half2*>(&hv);
    double hd[8];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 x = __half22float2(hh[q]);
      hd[2 * q] = x.x;
      hd[2 * q + 1] = x.y;
    }
    const bool first = v == threadIdx.x;
#pragma unroll
    for (int e = 0; e < kRoutePre; ++e)
      if (e < E) dot8_f64(acc[e], hd, first ? wpre[e] : __ldg(wg + (int64_t)e * nvec + v));
  }
  if (E <= kRoutePre) {
    // Transposed butterfly: each exchange halves the experts a lane keeps
    // (lane bit 4 -> experts 4..7 or 0..3, bit 3, bit 2), then two plain
    // steps; lane l ends with expert (l >> 2) & 7 summed over the warp.
    static_assert(kRoutePre == 8, "transposed reduction assumes 8 preloaded experts");
    const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
    double v4[4], v2[2];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const double send = b4 ? acc[q] : acc[q + 4];
      v4[q] = (b4 ? acc[q + 4] : acc[q]) + __shfl_xor_sync(0xffffffffu, send, 16);
    }
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const double send = b3 ? v4[q] : v4[q + 2];
      v2[q] = (b3 ? v4[q + 2] : v4[q]) + __shfl_xor_sync(0xffffffffu, send, 8);
    }
    double v1 = (b2 ? v2[1] : v2[0]) + __shfl_xor_sync(0xffffffffu, b2 ? v2[0] : v2[1], 4);
    v1 += __shfl_xor_sync(0xffffffffu, v1, 2);
    v1 += __shfl_xor_sync(0xffffffffu, v1, 1);
    const int e = (lane >> 2) & 7;
    if ((lane & 3) == 0 && e < E) part[warp * MOE_MAX_EXPERTS + e] = v1;
  }
#pragma unroll 1
  for (int e = E <= kRoutePre ? E : 0; e < E; ++e) {
    double tot = 0.0;
    if (e < kRoutePre) {
#pragma unroll
      for (int j = 0; j < kRoutePre; ++j)
        if (j == e) tot = acc[j];
    } else {  // experts past the preloaded ones: one more pass over the row
      double hd[8];
      for (int v = threadIdx.x; v < nvec; v += kThreadsK) {
        const uint4 hv = hrow[v];
        const __half2* hh = reinterpret_cast<const __half2*>(&hv);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 x = __half22float2(hh[q]);
          hd[2 * q] = x.x;
          hd[2 * q + 1] = x.y;
        }
        dot8_f64(tot, hd, __ldg(wg + (int64_t)e * nvec + v));
      }
    }
    tot = warp_sum_f64(tot);
    if (lane == 0) part[warp * MOE_MAX_EXPERTS + e] = tot;
  }
  __syncthreads();
  if (warp == 0) {
    int W = 1;
    while (W < E) W <<= 1;
    double mine = 0.0;
    if (E <= 8) {  // lanes e, e+8, e+16, e+24 take four warps each of expert e
      const int e = lane & 7, w0 = (lane >> 3) * (kWarpsK / 4);
      if (e < E)
#pragma unroll
        for (int w = 0; w < kWarpsK / 4; ++w) mine += rs.part[(w0 + w) * MOE_MAX_EXPERTS + e];
      mine += __shfl_xor_sync(0xffffffffu, mine, 8);
      mine += __shfl_xor_sync(0xffffffffu, mine, 16);
      if (lane >= E) mine = 0.0;
    } else if (lane < E) {
      for (int w = 0; w < kWarpsK; ++w) mine += rs.part[w * MOE_MAX_EXPERTS + lane];
    }
    route::finish_token(mine, lane, E, W, k, 0, nullptr, rs.w, rs.idx);
    __syncwarp();
    // Stable counting sort of the k pairs (distinct experts) by expert id.
    int cnt = 0;
    for (int j = 0; j < k; ++j) cnt += (lane < E && rs.idx[j] == lane) ? 1 : 0;
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 0) s_off[0] = 0;
    if (lane < E) s_off[lane + 1] = incl;
    const unsigned act = __ballot_sync(0xffffffffu, lane < E && cnt == 1);
    if (lane < E && cnt == 1) s_active[__popc(act & ((1u << lane) - 1u))] = lane;
    if (lane == 0) s_n = __popc(act);
    if (lane < 8) rs.zero_tok[lane] = 0;
    __syncwarp();
    if (lane < k) {
      rs.w_slot[s_off[rs.idx[lane]]] = rs.w[lane];
      if (blockIdx.x == 0) {
        a.out_weights[lane] = rs.w[lane];
        a.out_indices[lane] = rs.idx[lane];
      }
    }
  }
  __syncthreads();
  return Active{s_n, s_n > 0 ? s_active[0] : 0};
}

// After the down phase: publish this CTA's down items per row group; a CTA
// that completes a row group (every active expert and split) writes the
// layer output of those rows: y_e = fp16(sum over splits, in order), then
// out = fp16(out + y_e * w_e) over the token's experts in ascending id.
template <bool kMulti>
__device__ __forceinline__ void combine_rows(const DecodeArgs& a, const Active& act,
                                             const RouteSmem& rs) {
  constexpr int kRows = 16 * down_tiles<kMulti>();
  constexpr int kChunk = kThreadsK;
  __shared__ int s_won[kChunk];
  __shared__ int s_nwon;
  const int groups = a.H / kRows, per = a.S * groups;
  int first, last;
  cta_range(act.n * per, &first, &last);
  const int target = act.n * a.S;
  const int k = a.route_k, S = a.S, H = a.H;
  for (int c0 = first; c0 < last; c0 += kChunk) {
    if (threadIdx.x == 0) s_nwon = 0;
    __syncthreads();  // this CTA's y_part stores (and the previous chunk's reads) are done
    // One item per thread: release, count, and on the last count acquire.
    const int i = c0 + threadIdx.x;
    if (i < last) {
      const int rg = (i % per) % groups;
      fence_release_gpu();
      if (atomicAdd(a.rg_count + rg, 1) == target - 1) {
        fence_release_gpu();  // acquire side: the other CTAs' partials of this group
        s_won[atomicAdd(&s_nwon, 1)] = rg;
      }
    }
    __syncthreads();
    const int nw = s_nwon;
    for (int job = threadIdx.x; job < nw * kRows; job += blockDim.x) {
      const int c = s_won[job / kRows] * kRows + job % kRows;
      float acc = 0.f;
      for (int p = 0; p < k; ++p) {
        const float* src = a.y_part + (int64_t)p * S * H + c;
        float ys = __ldcg(src);
        for (int sp = 1; sp < S; ++sp) ys = __fadd_rn(ys, __ldcg(src + (int64_t)sp * H));
        acc = h2f(f2h(__fadd_rn(acc, __fmul_rn(h2f(f2h(ys)), rs.w_slot[p]))));
      }
      a.out[c] = f2h(acc);
    }
    __syncthreads();
  }
}

// The decode tables come from expert 0's codebooks (w1 for gate_up, w2 for
// down); CTA 0 checks that every active expert carries the same ones and
// flags the launch otherwise (moe_stream_check: MOE_ERR_CODEBOOK).
__device__ __forceinline__ void check_codebooks(const DecodeArgs& a, const Active& act,
                                                const int* s_active) {
  if (blockIdx.x != 0) return;
  const int i = threadIdx.x;
  if (i < act.n * 3) {
    const moe_nf4_expert_t& ex = a.ex.e[s_active[i / 3]];
    const int m = i % 3;
    const float* c = m == 0 ? ex.w1.code : m == 1 ? ex.w3.code : ex.w2.code;
    const float* ref = m == 2 ? a.ex.e[0].w2.code : a.ex.e[0].w1.code;
    if (!same_code16(c, ref)) set_device_error(kErrCodebook);
  }
}

// One launch per layer for the experts of one kind (1 token or 2..8 tokens):
// every CTA runs its share of the gate_up items, then its share of the down
// items; a down split starts as soon as the gate_up items it reads are
// published, with its weight loads and L2 prefetches already in flight.  The
// grid is one CTA per SM and every gate_up item is done before its CTA waits
// on anything, so the waits end once all CTAs are resident.
template <int NBW, bool kMulti, bool kFullG, bool kFullD>
__global__ void __launch_bounds__(kThreadsK, 1) k_stage_mma(const __grid_constant__ DecodeArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ int s_off[MOE_MAX_EXPERTS + 1];
  __shared__ int s_active[MOE_MAX_EXPERTS];
  __shared__ SlotMeta s_meta[2 * batch_items<kMulti>()];
  // The decode table depends only on the weights' codebook (one per launch).
  // The 1-token launch, first in a layer, builds it before waiting for the
  // kernel that produced its inputs; the 2..8-token launch follows a
  // full-grid kernel (nothing to overlap) and first checks it has work.
  __shared__ RouteSmem s_route;
  pdl_trigger();
  const bool routed = !kMulti && a.route_wg != nullptr;
  uint4 wpre[kRoutePre];
  if (routed) route_preload(a, wpre);
  const bool room = smem_u32(smem) + red_floats<kMulti>() * 4 <= kLutWin;
  bool lut_ok = !kMulti && room && build_lut(a.ex.e[0].w1.code, smem);
  pdl_wait();
  const Active act = routed ? route_token(a, wpre, s_off, s_active, s_route)
                            : load_active<kMulti>(a, s_off, s_active);
  if (act.n == 0) return;
  check_codebooks(a, act, s_active);
  if (kMulti) lut_ok = room && build_lut(a.ex.e[0].w1.code, smem);
  if (!lut_ok) return;
  const StageSmem sm{reinterpret_cast<float*>(smem), s_off, s_active, s_meta,
                     routed ? s_route.zero_tok : a.pair_token};
  gate_phase<NBW, kMulti, kFullG>(a, act, sm);
  if (!same_code16(a.ex.e[0].w1.code, a.ex.e[0].w2.code)) {
    __syncthreads();
    build_lut(a.ex.e[0].w2.code, smem);
  }
  down_phase<kDownSlice / (64 * kWarpsK), kMulti, kFullD>(a, act, sm);
  if (routed) combine_rows<kMulti>(a, act, s_route);
}

// y[slot] = fp16(sum over splits of y_part[slot][s]) (single-expert forward).
__global__ void k_reduce_partials(const float* __restrict__ part, int64_t P, int S, int width,
                                  uint16_t* __restrict__ y) {
  pdl_trigger();
  pdl_wait();
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

// Offsets of one expert holding all n rows; also zeroes the decode launch's
// completion counters.
__global__ void k_identity_offsets(int32_t* off, int n, int32_t* zero, int nzero) {
  if (threadIdx.x == 0) {
    off[0] = 0;
    off[1] = n;
  }
  for (int i = threadIdx.x; i < nzero; i += blockDim.x) zero[i] = 0;
}

// Zeroes the decode launch's completion counters (after the predecessor).
__global__ void k_zero_words(int32_t* p, int n) {
  pdl_trigger();
  pdl_wait();
  for (int i = threadIdx.x; i < n; i += blockDim.x) p[i] = 0;
}

template <class K>
bool smem_attr(K kernel) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kDynSmem) ==
         cudaSuccess;
}

template <int NBW, bool kMulti>
bool attrs_nbw() {
  return smem_attr(k_stage_mma<NBW, kMulti, true, true>) &&
         smem_attr(k_stage_mma<NBW, kMulti, true, false>) &&
         smem_attr(k_stage_mma<NBW, kMulti, false, true>) &&
         smem_attr(k_stage_mma<NBW, kMulti, false, false>);
}
template <bool kMulti>
bool attrs() {
  return attrs_nbw<1, kMulti>() && attrs_nbw<2, kMulti>() && attrs_nbw<4, kMulti>() &&
         attrs_nbw<8, kMulti>();
}
bool decode_attrs() { return attrs<false>() && attrs<true>(); }

// Blocks per K part of the gate_up phase: ceil(H / 64 / 16) rounded up to a
// power of two (parts past the row are idle).
int gate_nbw(int hidden) {
  const int need = static_cast<int>(ceil_div(hidden / 64, kWarpsK));
  return need <= 1 ? 1 : need <= 2 ? 2 : need <= 4 ? 4 : need <= 8 ? 8 : -1;
}

template <int NBW, bool kMulti>
cudaError_t launch_stage_nbw(const DecodeArgs& a, cudaStream_t s) {
  const bool full_g = a.H / 64 == NBW * kWarpsK;
  const bool full_d = (a.I / 64) % (kDownSlice / 64) == 0;
  auto k = full_g ? (full_d ? k_stage_mma<NBW, kMulti, true, true> : k_stage_mma<NBW, kMulti, true, false>)
                  : (full_d ? k_stage_mma<NBW, kMulti, false, true>
                            : k_stage_mma<NBW, kMulti, false, false>);
  // One CTA per SM (the CTA takes the whole register file), so the grid is
  // resident as soon as the predecessor's CTAs leave; the predecessor never
  // waits on this kernel and the successor starts only after every CTA here
  // has run its trigger.  A co-resident (cooperative) launch would also hold
  // when other streams occupy SMs, but it forgoes the programmatic overlap
  // (about 3 us per layer); the cross-CTA waits are bounded either way.
  return launch_pdl(k, sm_count(), kThreadsK, kDynSmem, s, a);
}

template <bool kMulti>
int launch_stage(const DecodeArgs& a, cudaStream_t s) {
  cudaError_t st;
  switch (gate_nbw(a.H)) {
    case 1: st = launch_stage_nbw<1, kMulti>(a, s); break;
    case 2: st = launch_stage_nbw<2, kMulti>(a, s); break;
    case 4: st = launch_stage_nbw<4, kMulti>(a, s); break;
    case 8: st = launch_stage_nbw<8, kMulti>(a, s); break;
    default: return MOE_ERR_UNSUPPORTED;
  }
  if (st != cudaSuccess) return MOE_ERR_CUDA;
  MOE_CHECK_LAUNCH();
  return MOE_OK;
}

}  // namespace

// Shapes the decode kernels accept: H and I multiples of 64 (one absmax block)
// with H up to 8192.
bool decode_supported(int hidden, int inter) {
  return hidden > 0 && inter > 0 && hidden % 64 == 0 && inter % 64 == 0 && gate_nbw(hidden) > 0 &&
         (int64_t)hidden * inter / 2 < ((int64_t)1 << 31);  // 32-bit offsets within a matrix
}

// Down-projection K splits of 2048 elements (the last may be partial).
int decode_splits(int inter) { return static_cast<int>(ceil_div(inter, kDownSlice)); }
int decode_max_tokens() { return kMaxTok; }
// Completion counters the decode launches need (zeroed before each layer).
int decode_sync_words(int inter) { return 2 * MOE_MAX_EXPERTS * decode_splits(inter); }

int launch_decode_experts(const moe_nf4_expert_t* experts, int E, const int32_t* expert_offsets,
                          const int32_t* pair_token, const uint16_t* x, int hidden, int inter,
                          uint16_t* h_sorted, float* y_part, int32_t* sync,
                          int max_tokens_per_expert, cudaStream_t s) {
  if (E < 1 || E > MOE_MAX_EXPERTS || !sync) return MOE_ERR_INVALID_ARG;
  if (!decode_supported(hidden, inter)) return MOE_ERR_UNSUPPORTED;
  if (!once_per_device(reinterpret_cast<const void*>(&decode_attrs), &decode_attrs))
    return MOE_ERR_CUDA;
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
  a.sync = sync;
  a.wait_ns = wait_limit_ns();
  int st = launch_stage<false>(a, s);
  if (st == MOE_OK && max_tokens_per_expert > 1) {
    a.sync = sync + MOE_MAX_EXPERTS * a.S;
    st = launch_stage<true>(a, s);
  }
  return st;
}

// One launch for a 1-token layer: routing, gate_up, down and the weighted
// combine (the permute of one token is a sort of its k distinct experts).
int launch_decode_layer1(const moe_nf4_expert_t* experts, int E, int k, const uint16_t* h,
                         const uint16_t* wg, int hidden, int inter, uint16_t* h_sorted,
                         float* y_part, int32_t* sync, int32_t* rg_count, uint16_t* out,
                         int64_t* indices, float* weights, cudaStream_t s) {
  if (E < 1 || E > MOE_MAX_EXPERTS || E > kWarpsK || k < 1 || k > 8 || k > E || !sync ||
      !rg_count)
    return MOE_ERR_INVALID_ARG;
  if (!decode_supported(hidden, inter)) return MOE_ERR_UNSUPPORTED;
  if (!once_per_device(reinterpret_cast<const void*>(&decode_attrs), &decode_attrs))
    return MOE_ERR_CUDA;
  DecodeArgs a{};
  for (int e = 0; e < E; ++e) a.ex.e[e] = experts[e];
  a.E = E;
  a.x = h;
  a.h_sorted = h_sorted;
  a.y_part = y_part;
  a.H = hidden;
  a.I = inter;
  a.S = decode_splits(inter);
  a.sync = sync;
  a.route_wg = wg;
  a.route_k = k;
  a.out_weights = weights;
  a.out_indices = indices;
  a.out = out;
  a.rg_count = rg_count;
  a.wait_ns = wait_limit_ns();
  return launch_stage<false>(a, s);
}

int launch_reduce_partials(const float* part, int64_t P, int S, int width, uint16_t* y,
                           cudaStream_t s) {
  int64_t blocks = ceil_div(P * width, 256);
  int grid = static_cast<int>(blocks < sm_count() * 8 ? blocks : sm_count() * 8);
  if (launch_pdl(k_reduce_partials, grid > 0 ? grid : 1, 256, 0, s, part, P, S, width, y) !=
      cudaSuccess)
    return MOE_ERR_CUDA;
  MOE_CHECK_LAUNCH();
  return MOE_OK;
}

int launch_zero_words(int32_t* p, int n, cudaStream_t s) {
  if (launch_pdl(k_zero_words, 1, 256, 0, s, p, n) != cudaSuccess) return MOE_ERR_CUDA;
  MOE_CHECK_LAUNCH();
  return MOE_OK;
}

int launch_identity_offsets(int32_t* off, int n, int32_t* zero, int nzero, cudaStream_t s) {
  k_identity_offsets<<<1, 256, 0, s>>>(off, n, zero, nzero);
  MOE_CHECK_LAUNCH();
  return MOE_OK;
}

}  // namespace moe
