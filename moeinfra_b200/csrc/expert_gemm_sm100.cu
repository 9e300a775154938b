// Grouped NF4 expert GEMM on the 5th-generation tensor cores (tcgen05 + TMEM),
// for experts with more than 8 tokens (prefill and large decode batches).
//
// Reference: ReconstructedNF4Expert.forward (transfer/nf4_reconstruct.py:152-155)
// on n > 1 tokens, where bitsandbytes dequantizes each NF4 weight to bf16
// (nf4_reconstruct.py:12) and casts it to the fp16 compute dtype (:94) before an
// fp16 GEMM with fp32 accumulation:  w = fp16(bf16(code * absmax)).
//
// One launch per projection; a persistent CTA per SM walks tiles of
// (expert, 128 weight rows, up to kTileN tokens of that expert):
//   gate_up: D1 = W1 . X^T and D3 = W3 . X^T in TMEM (2 x kTileN fp32 columns),
//            epilogue h = fp16(silu(fp16(D1)) * fp16(D3)) -> h_sorted [P, I];
//   down   : D = W2 . H^T (kTileN columns), epilogue y = fp16(D) -> y_sorted [P, H].
// Two configurations: wide (prefill: 256-token tiles, 8 dequant warps) and
// narrow (decode batches of at most ~64 tokens per expert: 64-token tiles, 16
// dequant warps).  Warp roles (DQ dequant warps + 2):
//   warps 0..DQ-1  dequantize the 128 x 64 weight tile of each K step (one
//              NF4 block per row; warp w takes rows 32*(w%4).., byte part w/4)
//              either into shared memory in the UMMA K-major 128-byte swizzled
//              layout (wide gate_up) or into tensor memory with tcgen05.st
//              (narrow tiles, wide down), then run the epilogue (TMEM ->
//              registers -> global);
//   warp DQ    lane 0 loads the token tile of each K step with TMA (no
//              multicast; rows past the tensor read as zeros);
//   warp DQ+1  lane 0 issues tcgen05.mma (kind::f16, M = 128, N = tokens
//              rounded up to 16, K = 16 per instruction; A from shared or
//              tensor memory) and commits stages.
// Stage barriers: a_full (DQ dequant warps), b_full (TMA bytes), empty (MMA
// commit); accumulator barriers acc_full (MMA commit) and acc_empty (DQ
// epilogue warps).  Every wait is bounded: on timeout the GEMM error word is
// set, the waiting role stops, and before exit the CTA waits (bounded) for its
// issued copies and MMAs, then frees its TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"

namespace moe {

// Narrow (split bf16) tiles when the experts average at most 32 tokens.
bool gemm_narrow(int64_t P, int E) { return P <= (int64_t)32 * E; }

namespace {

constexpr int kBM = 128;           // weight rows per tile (UMMA M)
constexpr int kBK = 64;            // K per stage: one NF4 block
constexpr int kMaxN = 256;         // tokens per tile (UMMA N, max)
constexpr int kBoxRows = 64;       // token rows per TMA box
// Dequant warps per CTA: 8 for wide and narrow tiles.  Warp w takes rows
// 32*(w%4).. and part w/4 of the row's 32 packed bytes: a thread loads 16
// bytes of a row per K step (lanes 32 bytes apart).  Narrow tiles are bound
// by the L1 load/store data pipe, and 16 warps with 8-byte loads cost it more
// wavefronts per byte (569 -> 522 us per bs64 layer going from 16 to 8).
template <int DQ>
constexpr int threads_for() { return (DQ + 2) * 32; }
constexpr uint32_t kATile = kBM * kBK * 2;         // 16 KB fp16, swizzled
constexpr uint32_t kBBox = kBoxRows * kBK * 2;      // 8 KB
constexpr uint32_t kLutBytes = 256 * 16 * 8;        // byte -> (code hi, code lo), 16 replicas
// Narrow tiles: the table (32 replicas, 64 KB) sits at shared-window address
// 0x10000, entry (byte v, lane l) at 0x10000 | v << 8 | l * 8, so one byte
// permute of the packed word forms the address.
constexpr uint32_t kLutWin = 0x10000;
MOE_DEFINE_ERROR_WORD()

// kNarrow: tiles of at most 32 tokens.  Their weights are decoded straight to
// bf16: fp16(bf16(code * absmax)) -- the reference's multi-row weight -- equals
// bf16(code * absmax) exactly, so the MMA takes A as bf16 and skips the fp16
// widening (4 instead of 7 instructions per packed byte).  The tokens then go
// in as bf16 too, each fp16 row x split into two bf16 rows hi = bf16(x),
// lo = bf16(x - hi) (exact: an fp16 significand has 11 bits, hi takes 8, the
// remainder at most 3), and the epilogue adds the two accumulator columns of a
// token: every product is exact and accumulates in fp32, as in the fp16 GEMM.
// The split rows (2 x 32 per tile) fill one TMA box, as 64 fp16 rows did.
// Narrow tiles, and the down projection of wide ones, keep the dequantized
// weights (A) in tensor memory: the dequant threads (one weight row each)
// write them with tcgen05.st and the MMA reads A from TMEM, so A never crosses
// shared memory (its shared-memory traffic bounded both).  TMEM columns:
// accumulators (W1 at 0, W3 at kTileN), then the A stages, 32 columns per
// matrix and stage.  Wide gate_up keeps A in shared memory: its two 256-column
// accumulators fill TMEM.
template <bool kGate, bool kNarrow>
struct Cfg {
  static constexpr int kMats = kGate ? 2 : 1;
  static constexpr bool kSplit = kNarrow;                 // tokens as bf16 hi/lo rows
  static constexpr int kTileN = kNarrow ? kBoxRows / 2 : kMaxN;  // tokens per tile
  static constexpr int kBRows = kSplit ? 2 * kTileN : kTileN;    // B rows per tile
  static constexpr bool kATmem = kNarrow || !kGate;
  static constexpr int kStages = kNarrow ? (kGate ? 6 : 7) : (kGate ? 3 : 6);
  // K steps of packed codes in flight per dequant thread.
  static constexpr int kPrefetch = kNarrow ? (kGate ? 6 : 8) : 4;
  static constexpr uint32_t kAStage = kATmem ? 0 : kMats * kATile;  // A bytes in a smem stage
  static constexpr uint32_t kStage = kAStage + (uint32_t)kBRows * kBK * 2;
  static constexpr uint32_t kDCol3 = kNarrow ? kBRows : 256;       // W3 accumulator column
  static constexpr uint32_t kACol = kATmem ? kMats * kBRows : 0;  // first A column
  static constexpr uint32_t kTmemCols = 512;
  static constexpr bool kLutWindow = kNarrow;
  // Wide: stages, table, alignment slack.  Narrow: everything below the
  // window (stages) plus the window itself.
  static constexpr uint32_t kSmem =
      kLutWindow ? 2 * kLutWin : kStages * kStage + kLutBytes + 1024;
  static_assert(!kLutWindow || kStages * kStage + 8192 <= kLutWin, "stages below the table");
  static_assert(!kATmem || kACol + kStages * kMats * 32 <= kTmemCols, "TMEM columns");
};

struct GemmArgs {
  ExpertTable ex;
  int E;
  const int32_t* offsets;  // [E+1] rows of each expert in the token matrix
  int K;                   // reduction length (H for gate_up, I for down)
  int rows;                // output rows per expert (I for gate_up, H for down)
  uint16_t* out;           // [P, rows] fp16
  uint64_t wait_ns;        // limit of every bounded wait (moe_set_wait_limit_ns)
  // Split-K: ksplit > 1 splits every tile's K blocks into ksplit chunks, one
  // work unit each; a unit writes its fp32 accumulators to
  // part[((chunk * P + pair) * mats + m) * rows + row] and k_splitk_reduce
  // applies the epilogue to their in-order sum.
  int ksplit;
  float* part;
};

// ---- PTX wrappers ----------------------------------------------------------

__device__ __forceinline__ uint32_t saddr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
// One try: the thread may be suspended in hardware (up to the hint, 10 ms)
// until the phase completes, so a waiting thread takes no issue slots from
// the warps sharing its scheduler.
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(10000000u)
      : "memory");
  return ok != 0;
}
// Waits for the phase of `parity`; false (error word set) after limit_ns of
// %globaltimer.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try(bar, parity)) {
    if (globaltimer_ns() - t0 > limit_ns) {
      set_device_error(kErrWaitTimeout);
      return false;
    }
  }
  return true;
}
// Warp-uniform wait: lane 0 waits, the result is broadcast (all lanes of a
// warp then take the same path through warp-collective tcgen05 instructions).
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
  int ok = 0;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, limit_ns) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  __syncwarp();
  return ok != 0;
}
// Byte `shift/8` of w -> fp16 pair (element 2j low) of fp16(bf16(code * absmax)):
// table address from the byte, the byte's two fp32 codes, one packed multiply,
// bf16 rounding, then the exact widening to fp16 (the reference's multi-row
// weight).  One PTX block so the sequence stays nine instructions.
__device__ __forceinline__ uint32_t decode_byte(uint32_t w, uint32_t shift, uint32_t lut_lane,
                                                uint64_t am2) {
  uint32_t out;
  asm("{\n .reg .b32 v, ad, lo, hi, bf;\n .reg .b64 c, p;\n"
      " bfe.u32 v, %1, %2, 8;\n"
      " mad.lo.u32 ad, v, 128, %3;\n"
      " ld.shared.b64 c, [ad];\n"
      " mul.rn.f32x2 p, c, %4;\n"
      " mov.b64 {lo, hi}, p;\n"
      " cvt.rn.bf16x2.f32 bf, hi, lo;\n"
      " and.b32 hi, bf, 0xFFFF0000;\n"
      " shl.b32 lo, bf, 16;\n"
      " cvt.rn.f16x2.f32 %0, hi, lo;\n}\n"
      : "=r"(out)
      : "r"(w), "r"(shift), "r"(lut_lane), "l"(am2));
  return out;
}
// The same for the windowed table: the address is one byte permute.
template <int K>
__device__ __forceinline__ uint32_t decode_byte_w(uint32_t w, uint32_t lut_lane, uint64_t am2) {
  uint32_t out;
  asm("{\n .reg .b32 ad, lo, hi, bf;\n .reg .b64 c, p;\n"
      " prmt.b32 ad, %1, %2, %3;\n"
      " ld.shared.b64 c, [ad];\n"
      " mul.rn.f32x2 p, c, %4;\n"
      " mov.b64 {lo, hi}, p;\n"
      " cvt.rn.bf16x2.f32 bf, hi, lo;\n"
      " and.b32 hi, bf, 0xFFFF0000;\n"
      " shl.b32 lo, bf, 16;\n"
      " cvt.rn.f16x2.f32 %0, hi, lo;\n}\n"
      : "=r"(out)
      : "r"(w), "r"(lut_lane), "n"(0x7604 | (K << 4)), "l"(am2));
  return out;
}
// Byte K of w -> bf16 pair (element 2j low) of bf16(code * absmax): table
// address, the two fp32 codes, one packed multiply, one packed rounding.
template <int K>
__device__ __forceinline__ uint32_t decode_byte_bf16(uint32_t w, uint32_t lut_lane, uint64_t am2) {
  uint32_t out;
  asm("{\n .reg .b32 ad, lo, hi;\n .reg .b64 c, p;\n"
      " prmt.b32 ad, %1, %2, %3;\n"
      " ld.shared.b64 c, [ad];\n"
      " mul.rn.f32x2 p, c, %4;\n"
      " mov.b64 {lo, hi}, p;\n"
      " cvt.rn.bf16x2.f32 %0, hi, lo;\n}\n"
      : "=r"(out)
      : "r"(w), "r"(lut_lane), "n"(0x7604 | (K << 4)), "l"(am2));
  return out;
}
// fp16 value -> its exact bf16 hi/lo pair (hi = bf16(v), lo = bf16(v - hi)).
__device__ __forceinline__ void split_bf16(float v, uint16_t* hi, uint16_t* lo) {
  const __nv_bfloat16 h = __float2bfloat16_rn(v);
  *hi = __bfloat16_as_ushort(h);
  *lo = __bfloat16_as_ushort(__float2bfloat16_rn(__fsub_rn(v, __bfloat162float(h))));
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
// 2-D TMA load of one box into this CTA's shared memory (no multicast).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, "
      "{%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}
// D[tmem] (+)= A[smem desc] . B[smem desc]^T, kind::f16 (fp16 x fp16 -> fp32).
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
  const uint32_t z = 0;
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(
          d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z)
      : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// D[tmem] (+)= A[tmem] . B[smem desc]^T, kind::f16: A is 128 lanes (rows) x 8
// columns (16 fp16 of K, the lower K index in the lower half of a column).
__device__ __forceinline__ void tc_mma_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  const uint32_t z = 0;
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(
          d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z)
      : "memory");
}
// Each thread of the warp writes 8 (16) consecutive columns of its own lane.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (rows are 128 bytes = 64 fp16 of K).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  return (uint64_t)((addr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor: fp32 accumulate, fp16 (or bf16) A and B, both
// K-major, M=128, N.
__device__ __forceinline__ uint32_t instr_desc(int n, bool bf16) {
  const uint32_t ab = bf16 ? ((1u << 7) | (1u << 10)) : 0u;
  return (1u << 4) | ab | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
}

// Tile t of this launch -> expert e, first weight row m0, first token n0, tokens nt.
struct Tile {
  int e, m0, n0, nt;
};
template <int kTileN>
__device__ __forceinline__ Tile tile_of(int t, const int* s_base, const int* s_off, int E,
                                        int mtiles) {
  int e = 0;
  while (e + 1 < E && s_base[e + 1] <= t) ++e;
  const int local = t - s_base[e];
  const int n_e = s_off[e + 1] - s_off[e];
  const int nch = (n_e + kTileN - 1) / kTileN;
  const int m = local / nch, c = local - m * nch;
  const int n0 = c * kTileN;
  const int nt = min(kTileN, n_e - n0);
  return Tile{e, m * kBM, n0, nt};
}

template <bool kGate, int kDqWarps, bool kNarrowCfg>
__global__ void __launch_bounds__(threads_for<kDqWarps>(), 1)
    k_grouped_gemm(const __grid_constant__ GemmArgs a, const __grid_constant__ CUtensorMap tmap) {
  using C = Cfg<kGate, kNarrowCfg>;
  constexpr int kPrefetch = C::kPrefetch;
  constexpr int kThreads = threads_for<kDqWarps>();
  constexpr int kParts = kDqWarps / 4;  // parts of a row's 32 packed bytes
  constexpr int kWords = 8 / kParts;    // 4-byte words of codes per thread per K step
  constexpr int NS = C::kStages;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ __align__(8) unsigned long long s_afull[NS], s_bfull[NS], s_empty[NS];
  __shared__ __align__(8) unsigned long long s_accfull, s_accempty, s_drain;
  __shared__ uint32_t s_tmem;
  __shared__ int s_off[MOE_MAX_EXPERTS + 1];
  __shared__ int s_base[MOE_MAX_EXPERTS + 1];
  __shared__ float s_code[16];
  __shared__ volatile int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t raw = saddr(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;  // stages: 1024-aligned (swizzle atoms)
  const uint32_t lut = C::kLutWindow ? kLutWin : base + NS * C::kStage;
  const int mtiles = a.rows / kBM;
  const int nblk = a.K / kBK;
  if (C::kLutWindow && (base + NS * C::kStage > kLutWin || raw + C::kSmem < 2 * kLutWin)) {
    if (threadIdx.x == 0) set_device_error(kErrSmemLayout);  // shared-memory layout not as planned
    return;
  }

  if (threadIdx.x == 0) {
    int acc = 0;
    for (int e = 0; e <= a.E; ++e) s_off[e] = a.offsets[e];
    for (int e = 0; e < a.E; ++e) {
      s_base[e] = acc;
      const int n = s_off[e + 1] - s_off[e];
      acc += n > 0 ? mtiles * ((n + C::kTileN - 1) / C::kTileN) : 0;
    }
    s_base[a.E] = acc;
    s_abort = 0;
    for (int s = 0; s < NS; ++s) {
      mbar_init(saddr(&s_afull[s]), kDqWarps);
      mbar_init(saddr(&s_bfull[s]), 1);
      mbar_init(saddr(&s_empty[s]), 1);
    }
    mbar_init(saddr(&s_accfull), 1);
    mbar_init(saddr(&s_accempty), kDqWarps);
    mbar_init(saddr(&s_drain), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (threadIdx.x < 16) s_code[threadIdx.x] = (kGate ? a.ex.e[0].w1.code : a.ex.e[0].w2.code)[threadIdx.x];
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     saddr(&s_tmem)),
                 "r"(C::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  __syncthreads();
  // Byte -> (fp32 code of the high nibble, of the low nibble); 16 replicas so
  // the 16 lanes of a half-warp read disjoint banks.
  if (C::kLutWindow) {
    for (int i = threadIdx.x; i < 256 * 32; i += kThreads) {
      const int v = i >> 5;
      float2 c = make_float2(s_code[v >> 4], s_code[v & 15]);
      asm volatile("st.shared.v2.f32 [%0], {%1, %2};" ::"r"(kLutWin + i * 8), "f"(c.x), "f"(c.y)
                   : "memory");
    }
  } else {
    for (int i = threadIdx.x; i < 256 * 16; i += kThreads) {
      const int v = i >> 4;
      float2 c = make_float2(s_code[v >> 4], s_code[v & 15]);
      asm volatile("st.shared.v2.f32 [%0], {%1, %2};" ::"r"(lut + i * 8), "f"(c.x), "f"(c.y)
                   : "memory");
    }
  }
  // The decode table comes from expert 0's codebook; CTA 0 flags a launch whose
  // experts with tokens carry another one (moe_stream_check: MOE_ERR_CODEBOOK).
  if (blockIdx.x == 0 && threadIdx.x < a.E * C::kMats && s_off[threadIdx.x / C::kMats + 1] >
                                                           s_off[threadIdx.x / C::kMats]) {
    const moe_nf4_expert_t& ex = a.ex.e[threadIdx.x / C::kMats];
    const float* c = kGate ? ((threadIdx.x % C::kMats) ? ex.w3.code : ex.w1.code) : ex.w2.code;
    if (!same_code16(c, kGate ? a.ex.e[0].w1.code : a.ex.e[0].w2.code))
      set_device_error(kErrCodebook);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  const int ks = a.ksplit;
  const int total = s_base[a.E] * ks;
  const int kchunk = (nblk + ks - 1) / ks;  // K blocks per split-K unit

  if (warp < kDqWarps) {
    // ---------------- dequant producers + epilogue ----------------
    const int part = warp / 4, rw = warp % 4;
    const int i = rw * 32 + lane;  // tile row (also TMEM lane)
    const uint32_t lut_lane = C::kLutWindow ? (kLutWin | (lane * 8)) : lut + (lane & 15) * 8;
    uint32_t g = 0, it = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++it) {
      const int kc = t % ks;
      const Tile tl = tile_of<C::kTileN>(t / ks, s_base, s_off, a.E, mtiles);
      const int kb_lo = kc * kchunk, kb_hi = min(nblk, kb_lo + kchunk);
      const moe_nf4_expert_t& ex = a.ex.e[tl.e];
      const moe_nf4_matrix_t* mats[2] = {kGate ? &ex.w1 : &ex.w2, &ex.w3};
      const int R = tl.m0 + i;
      const int64_t rowseg = (int64_t)(R >> 4) * nblk * 16 + (R & 15);
      // This thread's 4*kWords bytes of block 0 and its absmax; block kb is 512
      // bytes (16 floats) further on in tile16.
      const uint8_t* qp[C::kMats];
      const float* ap[C::kMats];
#pragma unroll
      for (int m = 0; m < C::kMats; ++m) {
        qp[m] = mats[m]->q + rowseg * 32 + part * (4 * kWords);
        ap[m] = mats[m]->absmax + rowseg;
      }
      // Packed codes and absmax of K steps kb .. kb+kPrefetch-1 in flight in
      // registers while step kb is decoded.
      uint32_t qv[kPrefetch][C::kMats][kWords];
      float av[kPrefetch][C::kMats];
      auto load = [&](int kb, uint32_t (*q)[kWords], float* am) {
        if (kb < kb_hi) {
#pragma unroll
          for (int m = 0; m < C::kMats; ++m) {
            const uint8_t* src = qp[m] + (int64_t)kb * 512;
            if constexpr (kWords == 4) {
              const uint4 v = __ldg(reinterpret_cast<const uint4*>(src));
              q[m][0] = v.x; q[m][1] = v.y; q[m][2] = v.z; q[m][3] = v.w;
            } else {
              const uint2 v = __ldg(reinterpret_cast<const uint2*>(src));
              q[m][0] = v.x; q[m][1] = v.y;
            }
            am[m] = __ldg(ap[m] + (int64_t)kb * 16);
          }
        }
      };
#pragma unroll
      for (int d = 0; d < kPrefetch; ++d) load(kb_lo + d, qv[d], av[d]);
      bool stop = false;
      for (int kb0 = kb_lo; kb0 < kb_hi && !stop; kb0 += kPrefetch) {
#pragma unroll
        for (int d = 0; d < kPrefetch; ++d) {
          const int kb = kb0 + d;
          if (kb >= kb_hi) break;
          const int s = g % NS;
          stop = __shfl_sync(0xffffffffu, s_abort, 0) != 0 ||
                 !warp_wait(saddr(&s_empty[s]), ((g / NS) & 1) ^ 1, a.wait_ns);
          if (stop) {
            s_abort = 1;
            break;
          }
          const uint32_t stage = base + s * C::kStage;
          if constexpr (C::kATmem) tc_fence_after();  // the MMA that read this stage is done
#pragma unroll
          for (int m = 0; m < C::kMats; ++m) {
            const uint32_t amb = __float_as_uint(av[d][m]);
            const uint64_t am2 = (static_cast<uint64_t>(amb) << 32) | amb;
            if constexpr (C::kATmem) {
              uint32_t h[kWords * 4];
#pragma unroll
              for (int cc = 0; cc < kWords; ++cc) {
                if constexpr (C::kSplit) {
                  h[cc * 4 + 0] = decode_byte_bf16<0>(qv[d][m][cc], lut_lane, am2);
                  h[cc * 4 + 1] = decode_byte_bf16<1>(qv[d][m][cc], lut_lane, am2);
                  h[cc * 4 + 2] = decode_byte_bf16<2>(qv[d][m][cc], lut_lane, am2);
                  h[cc * 4 + 3] = decode_byte_bf16<3>(qv[d][m][cc], lut_lane, am2);
                } else if constexpr (C::kLutWindow) {
                  h[cc * 4 + 0] = decode_byte_w<0>(qv[d][m][cc], lut_lane, am2);
                  h[cc * 4 + 1] = decode_byte_w<1>(qv[d][m][cc], lut_lane, am2);
                  h[cc * 4 + 2] = decode_byte_w<2>(qv[d][m][cc], lut_lane, am2);
                  h[cc * 4 + 3] = decode_byte_w<3>(qv[d][m][cc], lut_lane, am2);
                } else {
#pragma unroll
                  for (int b = 0; b < 4; ++b)
                    h[cc * 4 + b] = decode_byte(qv[d][m][cc], 8 * b, lut_lane, am2);
                }
              }
              const uint32_t ta = tmem + ((uint32_t)(rw * 32) << 16) + C::kACol +
                                  (s * C::kMats + m) * 32 + part * (kWords * 4);
              if constexpr (kWords == 2)
                tmem_st8(ta, h);
              else
                tmem_st16(ta, h);
            } else {
              const uint32_t arow = stage + m * kATile + (i >> 3) * 1024 + (i & 7) * 128;
#pragma unroll
              for (int cc = 0; cc < kWords; ++cc) {
                uint32_t h[4];
#pragma unroll
                for (int b = 0; b < 4; ++b) h[b] = decode_byte(qv[d][m][cc], 8 * b, lut_lane, am2);
                const int chunk = part * kWords + cc;
                asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(
                                 arow + ((chunk ^ (i & 7)) << 4)),
                             "r"(h[0]), "r"(h[1]), "r"(h[2]), "r"(h[3])
                             : "memory");
              }
            }
          }
          if constexpr (C::kATmem) {
            tmem_wait_st();
            tc_fence_before();
          } else {
            fence_proxy_async();
          }
          __syncwarp();
          if ((threadIdx.x & 31) == 0) mbar_arrive(saddr(&s_afull[s]));
          ++g;
          load(kb + kPrefetch, qv[d], av[d]);
        }
      }
      if (stop) break;
      // Epilogue: this warp reads TMEM lanes 32*rw.. ; column chunks of 16,
      // alternating between the two byte halves' warps.
      if (!warp_wait(saddr(&s_accfull), it & 1, a.wait_ns)) {
        s_abort = 1;
        break;
      }
      tc_fence_after();
      constexpr int kTokPerChunk = C::kSplit ? 8 : 16;  // a 16-column chunk
      const int nchunk = (tl.nt + kTokPerChunk - 1) / kTokPerChunk;
      const uint32_t lane_addr = tmem + ((uint32_t)(rw * 32) << 16);
      for (int ch = part; ch < nchunk; ch += kParts) {
        uint32_t d1[16], d3[16];
        tmem_ld16(lane_addr + ch * 16, d1);
        if (kGate) tmem_ld16(lane_addr + C::kDCol3 + ch * 16, d3);
        tmem_wait_ld();
        const int row = tl.m0 + i;
#pragma unroll
        for (int j = 0; j < kTokPerChunk; ++j) {
          const int n = ch * kTokPerChunk + j;
          if (n < tl.nt) {
            const int64_t p = s_off[tl.e] + tl.n0 + n;
            float g, u = 0.f;
            if constexpr (C::kSplit) {  // token n's hi and lo columns
              g = __fadd_rn(__uint_as_float(d1[2 * j]), __uint_as_float(d1[2 * j + 1]));
              if (kGate) u = __fadd_rn(__uint_as_float(d3[2 * j]), __uint_as_float(d3[2 * j + 1]));
            } else {
              g = __uint_as_float(d1[j]);
              if (kGate) u = __uint_as_float(d3[j]);
            }
            if (ks > 1) {  // split-K unit: fp32 partials, epilogue after the sum
              float* pp = a.part + ((int64_t)(kc * s_off[a.E] + p) * C::kMats) * a.rows + row;
              pp[0] = g;
              if (kGate) pp[a.rows] = u;
            } else if (kGate) {
              const uint16_t o = swiglu_f16(f2h(g), f2h(u));
              if constexpr (C::kSplit) {  // h feeds the down projection as hi/lo rows
                uint16_t hi, lo;
                split_bf16(h2f(o), &hi, &lo);
                a.out[(2 * p) * a.rows + row] = hi;
                a.out[(2 * p + 1) * a.rows + row] = lo;
              } else {
                a.out[p * a.rows + row] = o;
              }
            } else {
              a.out[p * a.rows + row] = f2h(g);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(saddr(&s_accempty));
    }
  } else if (warp == kDqWarps) {
    // ---------------- TMA producer of the token tiles ----------------
    if (lane == 0) {
      uint32_t g = 0;
      for (int t = blockIdx.x; t < total && !s_abort; t += gridDim.x) {
        const int kc = t % ks;
        const Tile tl = tile_of<C::kTileN>(t / ks, s_base, s_off, a.E, mtiles);
        const int kb_lo = kc * kchunk, kb_hi = min(nblk, kb_lo + kchunk);
        const int brows = C::kSplit ? 2 * tl.nt : tl.nt;
        const int nbox = (brows + kBoxRows - 1) / kBoxRows;
        const int row0 = (C::kSplit ? 2 : 1) * (s_off[tl.e] + tl.n0);
        for (int kb = kb_lo; kb < kb_hi; ++kb, ++g) {
          const int s = g % NS;
          if (!s_abort && !mbar_wait(saddr(&s_empty[s]), ((g / NS) & 1) ^ 1, a.wait_ns)) s_abort = 1;
          if (s_abort) break;
          const uint32_t bar = saddr(&s_bfull[s]);
          const uint32_t bt = base + s * C::kStage + C::kAStage;
          mbar_expect_tx(bar, nbox * kBBox);
          for (int bx = 0; bx < nbox; ++bx)
            tma_load_2d(bt + bx * kBBox, &tmap, bar, kb * kBK, row0 + bx * kBoxRows);
        }
      }
      // Copies issued into stages never consumed (timeout): let them land.
      if (s_abort)
        for (uint32_t j = g > (uint32_t)NS ? g - NS : 0; j < g; ++j)
          mbar_wait(saddr(&s_bfull[j % NS]), (j / NS) & 1, a.wait_ns);
    }
  } else {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t g = 0, it = 0;
      bool issued_any = false;
      for (int t = blockIdx.x; t < total && !s_abort; t += gridDim.x, ++it) {
        const int kc = t % ks;
        const Tile tl = tile_of<C::kTileN>(t / ks, s_base, s_off, a.E, mtiles);
        const int kb_lo = kc * kchunk, kb_hi = min(nblk, kb_lo + kchunk);
        const int n = ((C::kSplit ? 2 * tl.nt : tl.nt) + 15) & ~15;
        const uint32_t idesc = instr_desc(n, C::kSplit);
        if (!mbar_wait(saddr(&s_accempty), (it & 1) ^ 1, a.wait_ns)) {
          s_abort = 1;
          break;
        }
        tc_fence_after();
        for (int kb = kb_lo; kb < kb_hi; ++kb, ++g) {
          const int s = g % NS;
          if (!mbar_wait(saddr(&s_afull[s]), (g / NS) & 1, a.wait_ns) ||
              !mbar_wait(saddr(&s_bfull[s]), (g / NS) & 1, a.wait_ns)) {
            s_abort = 1;
            break;
          }
          tc_fence_after();
          const uint32_t stage = base + s * C::kStage;
          const uint32_t bt = stage + C::kAStage;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
#pragma unroll
            for (int m = 0; m < C::kMats; ++m) {
              if constexpr (C::kATmem)
                tc_mma_ta(tmem + m * C::kDCol3, tmem + C::kACol + (s * C::kMats + m) * 32 + kk * 8,
                          smem_desc(bt + kk * 32), idesc, kb != kb_lo || kk != 0);
              else
                tc_mma(tmem + m * C::kDCol3, smem_desc(stage + m * kATile + kk * 32),
                       smem_desc(bt + kk * 32), idesc, kb != kb_lo || kk != 0);
            }
          }
          issued_any = true;
          tc_commit(saddr(&s_empty[s]));
        }
        if (s_abort) break;
        tc_commit(saddr(&s_accfull));
      }
      // After a timeout, wait (bounded) for the MMAs already issued.
      if (s_abort && issued_any) {
        tc_commit(saddr(&s_drain));
        mbar_wait(saddr(&s_drain), 0, a.wait_ns);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(C::kTmemCols)
                 : "memory");
  }
}

// ---- host side ----------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// Split-K epilogue: the ks fp32 partials of (pair p, row) summed in chunk
// order, then the tile epilogue -- gate_up: fp16 SwiGLU of the fp16-rounded
// sums (as bf16 hi/lo rows when `split_rows`, the narrow down projection's
// input); down: the fp16-rounded sum.  A thread takes 4 consecutive rows
// (rows are multiples of 128): 16-byte partial loads, 8-byte stores.
template <bool kGate>
__global__ void k_splitk_reduce(const float* __restrict__ part, int ks, int64_t P, int rows,
                                bool split_rows, uint16_t* __restrict__ out) {
  constexpr int kMats = kGate ? 2 : 1;
  const int r4 = rows / 4;
  const int64_t n = P * r4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = i / r4;
    const int row = static_cast<int>(i - p * r4) * 4;
    float4 g = make_float4(0.f, 0.f, 0.f, 0.f), u = g;
#pragma unroll 8
    for (int kc = 0; kc < ks; ++kc) {
      const float* pp = part + (((int64_t)kc * P + p) * kMats) * rows + row;
      const float4 a = __ldcs(reinterpret_cast<const float4*>(pp));
      if (kc == 0) {
        g = a;
      } else {
        g.x = __fadd_rn(g.x, a.x); g.y = __fadd_rn(g.y, a.y);
        g.z = __fadd_rn(g.z, a.z); g.w = __fadd_rn(g.w, a.w);
      }
      if (kGate) {
        const float4 b = __ldcs(reinterpret_cast<const float4*>(pp + rows));
        if (kc == 0) {
          u = b;
        } else {
          u.x = __fadd_rn(u.x, b.x); u.y = __fadd_rn(u.y, b.y);
          u.z = __fadd_rn(u.z, b.z); u.w = __fadd_rn(u.w, b.w);
        }
      }
    }
    const float gv[4] = {g.x, g.y, g.z, g.w}, uv[4] = {u.x, u.y, u.z, u.w};
    uint16_t o[4], lo[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      o[c] = kGate ? swiglu_f16(f2h(gv[c]), f2h(uv[c])) : f2h(gv[c]);
      if (kGate && split_rows) split_bf16(h2f(o[c]), &o[c], &lo[c]);
    }
    const uint2 ov = make_uint2(o[0] | (uint32_t)o[1] << 16, o[2] | (uint32_t)o[3] << 16);
    if (kGate && split_rows) {
      const uint2 lv = make_uint2(lo[0] | (uint32_t)lo[1] << 16, lo[2] | (uint32_t)lo[3] << 16);
      *reinterpret_cast<uint2*>(out + (2 * p) * rows + row) = ov;
      *reinterpret_cast<uint2*>(out + (2 * p + 1) * rows + row) = lv;
    } else {
      *reinterpret_cast<uint2*>(out + p * rows + row) = ov;
    }
  }
}

// fp16 rows [P, K] -> bf16 rows [2P, K]: row 2p = bf16(x_p), row 2p+1 = the
// exact remainder (the token operand of narrow tiles).
__global__ void k_split_rows(const uint16_t* __restrict__ x, int64_t n, int K,
                             uint16_t* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = i / K;
    const int c = static_cast<int>(i - p * K);
    uint16_t hi, lo;
    split_bf16(h2f(x[i]), &hi, &lo);
    out[(2 * p) * K + c] = hi;
    out[(2 * p + 1) * K + c] = lo;
  }
}

// Token matrix [rows_total, K] (fp16, or bf16 split rows), row-major: boxes of
// 64 rows x 64 K with the 128-byte swizzle the UMMA K-major descriptor expects.
bool make_token_map(CUtensorMap* map, const uint16_t* x, int64_t rows_total, int K, bool bf16) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows_total};
  const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  const cuuint32_t box[2] = {kBK, kBoxRows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
            const_cast<uint16_t*>(x), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool kGate, int DQ, bool kN>
bool gemm_attr() {
  return cudaFuncSetAttribute(k_grouped_gemm<kGate, DQ, kN>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                              Cfg<kGate, kN>::kSmem) == cudaSuccess;
}

template <bool kGate, int DQ, bool kN>
int launch_dq(const GemmArgs& a, const CUtensorMap& map, cudaStream_t s) {
  if (!once_per_device(reinterpret_cast<const void*>(&gemm_attr<kGate, DQ, kN>), &gemm_attr<kGate, DQ, kN>))
    return MOE_ERR_CUDA;
  k_grouped_gemm<kGate, DQ, kN><<<sm_count(), threads_for<DQ>(), Cfg<kGate, kN>::kSmem, s>>>(a, map);
  MOE_CHECK_LAUNCH();
  return MOE_OK;
}

// Narrow tiles (on average at most 32 tokens per expert): 32-token tiles of
// split bf16 rows (an expert with more tokens takes several), deeper pipeline.
// Wide tiles: 256-token fp16 tiles.  With
// a.ksplit > 1 the units write partials and k_splitk_reduce finishes.
template <bool kGate>
int launch_one(const GemmArgs& a, const uint16_t* x, int64_t P, bool narrow, cudaStream_t s) {
  CUtensorMap map;
  if (!make_token_map(&map, x, narrow ? 2 * P : P, a.K, narrow)) return MOE_ERR_CUDA;
  const int st = narrow ? launch_dq<kGate, 8, true>(a, map, s) : launch_dq<kGate, 8, false>(a, map, s);
  if (st != MOE_OK || a.ksplit == 1) return st;
  const int64_t n = P * (a.rows / 4);
  const int64_t blocks = ceil_div(n, 256);
  const int grid = static_cast<int>(blocks < sm_count() * 8 ? blocks : sm_count() * 8);
  k_splitk_reduce<kGate><<<grid, 256, 0, s>>>(a.part, a.ksplit, P, a.rows, narrow && kGate, a.out);
  MOE_CHECK_LAUNCH();
  return MOE_OK;
}

// Split-K factor of one projection on narrow tiles (rows x K weights, P token
// rows, E experts), 1 otherwise.  A projection with few row tiles leaves SMs
// idle (one expert's down projection: 32 tiles on 148 SMs; eight experts'
// down projection at bs64: 256 tiles, a second wave 40 SMs short); ks chunks
// of K per tile make ks x tiles units.  With several experts the per-expert
// token counts are on the device: the count assumes every expert active with
// one 32-token chunk.  Picks the ks <= 8 (chunks of at least 8 K blocks, fp32
// partials of at most kSplitKCap bytes) with the fewest waves per unit of
// work, each extra chunk charged 2 % (its partials and pipeline ramp).
constexpr size_t kSplitKCap = (size_t)16 << 20;
int gemm_ksplit(int64_t P, int E, int rows, int K, int mats) {
  if (!gemm_narrow(P, E)) return 1;
  const int64_t chunks = E == 1 ? ceil_div(P, Cfg<true, true>::kTileN) : (E < P ? E : P);
  const int64_t tiles = (int64_t)(rows / kBM) * chunks;
  const int nblk = K / kBK, sms = sm_count();
  int best = 1;
  double best_cost = 1e30;
  for (int ks = 1; ks <= 8 && (ks == 1 || nblk / ks >= 8); ++ks) {
    if (ks > 1 && (size_t)ks * P * mats * rows * sizeof(float) > kSplitKCap) break;
    const double cost = (double)ceil_div(tiles * ks, sms) / ks + 0.02 * (ks - 1);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = ks;
    }
  }
  return best;
}

}  // namespace


// fp32 partial floats a call's split-K units need (0: no split-K).
size_t gemm_splitk_floats(int64_t P, int E, int hidden, int inter) {
  const int kg = gemm_ksplit(P, E, inter, hidden, 2), kd = gemm_ksplit(P, E, hidden, inter, 1);
  const size_t g = kg > 1 ? (size_t)kg * P * 2 * inter : 0;
  const size_t d = kd > 1 ? (size_t)kd * P * hidden : 0;
  return g > d ? g : d;
}

// Shapes the tensor-core path accepts: weight rows (I and H) multiples of 128,
// K extents multiples of 64, K-major 16-byte-aligned operands.
bool gemm_supported(int hidden, int inter) {
  return hidden > 0 && inter > 0 && hidden % kBM == 0 && inter % kBM == 0 && hidden % kBK == 0 &&
         inter % kBK == 0;
}

// h_sorted: [P, inter] fp16 (wide) or [2P, inter] bf16 split rows (narrow);
// x_split: [2P, hidden] bf16, used (and required) only for narrow tiles;
// part: gemm_splitk_floats(P, E, hidden, inter) fp32 (null: no split-K).
int launch_grouped_gemm_experts(const moe_nf4_expert_t* experts, int E,
                                const int32_t* expert_offsets, const uint16_t* x_sorted,
                                int64_t P, int hidden, int inter, uint16_t* h_sorted,
                                uint16_t* y_sorted, uint16_t* x_split, float* part,
                                cudaStream_t s) {
  if (E < 1 || E > MOE_MAX_EXPERTS || P < 1) return MOE_ERR_INVALID_ARG;
  if (!gemm_supported(hidden, inter)) return MOE_ERR_UNSUPPORTED;
  if (P > INT32_MAX / 2) return MOE_ERR_UNSUPPORTED;
  if (!aligned16(x_sorted) || !aligned16(h_sorted) || !aligned16(y_sorted))
    return MOE_ERR_ALIGNMENT;
  for (int e = 0; e < E; ++e) {
    const moe_nf4_matrix_t* m[3] = {&experts[e].w1, &experts[e].w3, &experts[e].w2};
    for (auto* mm : m)
      if (!aligned16(mm->q) || (reinterpret_cast<uintptr_t>(mm->absmax) & 3)) return MOE_ERR_ALIGNMENT;
  }
  GemmArgs a{};
  for (int e = 0; e < E; ++e) a.ex.e[e] = experts[e];
  a.E = E;
  a.offsets = expert_offsets;
  a.K = hidden;
  a.rows = inter;
  a.out = h_sorted;
  a.wait_ns = wait_limit_ns();
  a.part = part;
  a.ksplit = part ? gemm_ksplit(P, E, inter, hidden, 2) : 1;
  const bool narrow = gemm_narrow(P, E);
  const uint16_t* x_in = x_sorted;
  if (narrow) {
    if (!x_split || !aligned16(x_split)) return MOE_ERR_WORKSPACE;
    const int64_t n = P * hidden;
    const int64_t blocks = ceil_div(n, 256);
    const int grid = static_cast<int>(blocks < sm_count() * 8 ? blocks : sm_count() * 8);
    k_split_rows<<<grid, 256, 0, s>>>(x_sorted, n, hidden, x_split);
    MOE_CHECK_LAUNCH();
    x_in = x_split;
  }
  int st = launch_one<true>(a, x_in, P, narrow, s);
  if (st != MOE_OK) return st;
  a.K = inter;
  a.rows = hidden;
  a.out = y_sorted;
  a.ksplit = part ? gemm_ksplit(P, E, hidden, inter, 1) : 1;
  return launch_one<false>(a, h_sorted, P, narrow, s);
}

}  // namespace moe
