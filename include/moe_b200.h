/*
 * moe_b200.h — C ABI of the B200-native MoEInfra quantized-expert hot path.
 *
 * Conventions (every entry point):
 *   - plain pointers and sizes; no torch or C++ types cross this boundary;
 *   - every device pointer is owned by the caller; the library never allocates
 *     device memory (scratch comes from a caller-provided, 16-byte-aligned
 *     workspace whose size the *_workspace_size functions report; an unaligned
 *     one returns MOE_ERR_ALIGNMENT);
 *   - all work is enqueued on the caller's stream (`stream` is a cudaStream_t
 *     passed as void*; NULL means the legacy default stream of the current
 *     device); call with the device that owns the stream and the pointers
 *     current (cudaSetDevice): a kernel launched on another device would
 *     dereference the pointers there;
 *   - the return value is a moe_status_t; nothing throws across the ABI;
 *     moe_status_string() turns it into text.
 *
 * Numeric formats follow the reference's NF4 expert store (per projection:
 * packed weight uint8 [out*in/2], element 2j in the HIGH nibble of byte j,
 * row-major over [out, in]; fp32 absmax [out*in/64]; fp32 codebook [16]).
 * fp16 and bf16 values are passed as uint16_t bit patterns.
 *
 * File:line citations refer to the reference project ParshwaPatel-07/MoEInfra.
 */
#ifndef MOE_B200_H
#define MOE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum moe_status {
  MOE_OK = 0,
  MOE_ERR_INVALID_ARG = 1,
  MOE_ERR_UNSUPPORTED = 2,
  MOE_ERR_CUDA = 3,
  MOE_ERR_WORKSPACE = 4,
  MOE_ERR_ALIGNMENT = 5,
  MOE_ERR_TIMEOUT = 6,
  MOE_ERR_CODEBOOK = 7
} moe_status_t;

#define MOE_MAX_EXPERTS 16
#define MOE_NF4_BLOCKSIZE 64
/* Rows an expert stage call (P) may have to run on the decode kernels. */
#define MOE_DECODE_MAX_ROWS 8

/* One resident NF4-quantized linear layer [rows=out, cols=in] in the tile16
 * device layout (see moe_nf4_tile16): rows % 16 == 0, cols % 64 == 0. */
typedef struct moe_nf4_matrix {
  const uint8_t* q;     /* packed codes, rows*cols/2 bytes, tile16, 16-byte aligned */
  const float* absmax;  /* fp32, rows*cols/64, tile16 order (already de-nested)    */
  const float* code;    /* fp32[16] codebook (the store's quant_map)               */
} moe_nf4_matrix_t;

/* One Mixtral SwiGLU expert: w1, w3 are [inter, hidden]; w2 is [hidden, inter]. */
typedef struct moe_nf4_expert {
  moe_nf4_matrix_t w1;
  moe_nf4_matrix_t w3;
  moe_nf4_matrix_t w2;
} moe_nf4_expert_t;

/* Text for a status code (static storage). */
const char* moe_status_string(int status);

/* Library build identifier (static storage). */
const char* moe_version(void);

/* Number of kernels this library has launched (or recorded into a stream
 * capture) in this process, counted on the host at each launch.  A CUDA-graph
 * replay re-runs the kernels captured without calling the library, so the
 * count taken around a capture is the kernel count of one replay. */
uint64_t moe_launch_count(void);

/* Reads and clears the device-side error words of the current device.
 * Kernels never trap; they record a problem found on the device as bits:
 *   1  a bounded wait (cross-CTA counter, mbarrier phase) ran out; the
 *      launch's outputs are invalid;
 *   2  the experts of one launch carry different NF4 codebooks (the kernels
 *      decode every expert with expert 0's w1 codebook for gate/up and its
 *      w2 codebook for down); the outputs are invalid;
 *   4  a kernel found its shared-memory layout not as planned and skipped.
 * Synchronous (device-to-host copies).  *value is 0 when nothing was set. */
int moe_take_device_error(int* value);

/* Synchronises `stream`, then turns the device error words into a status:
 * MOE_ERR_TIMEOUT (bit 1), MOE_ERR_CODEBOOK (bit 2), MOE_ERR_CUDA (bit 4 or a
 * CUDA error), else MOE_OK.  The words are cleared.  Call it at the points
 * where the caller synchronises anyway (end of a step, before reading
 * results back) to learn whether the launches since the last check were valid.
 * No counterpart in the reference (its library calls raise synchronously). */
int moe_stream_check(void* stream);

/* Limit of every bounded device wait, in nanoseconds of the GPU's global
 * timer (default 2 s; accepted range 1 us .. 60 s).  Launches read it when
 * they are enqueued (a captured CUDA graph keeps the value it was captured
 * with).  After the limit a wait gives up, sets error bit 1 and lets the
 * kernel run to its end, so a GPU is never held by a wait that cannot end. */
int moe_set_wait_limit_ns(uint64_t ns);
uint64_t moe_wait_limit_ns(void);

/* One bounded wait, on one thread, until the int at `flag` (device memory)
 * reaches `target`: the same acquire-poll-with-limit the layer kernels use
 * between CTAs.  A health check of the timeout path: with a flag nothing
 * sets, it gives up after moe_wait_limit_ns() and moe_stream_check() returns
 * MOE_ERR_TIMEOUT.  waited_ns (device int, may be NULL) receives the time
 * spent waiting. */
int moe_probe_wait(const int* flag, int target, int* waited_ns, void* stream);

/* ---------------------------------------------------------------------------
 * NF4 blockwise dequant to bf16, bit-exact:
 *   out[i] = bf16_rn(code[nib(i)] * absmax[i / blocksize])   (fp32 product)
 * Replaces bitsandbytes dequantize_4bit as reached from
 * transfer/nf4_reconstruct.py:45-54 (QuantState, dtype bf16 at :12).
 * numel must be even; blocksize a power of two >= 32.
 */
int moe_nf4_dequant(const uint8_t* q, const float* absmax, const float* code,
                    int64_t numel, int blocksize, uint16_t* out_bf16,
                    void* stream);

/* ---------------------------------------------------------------------------
 * Store layout -> tile16 device layout (exact permutation of bytes and words).
 * Store: row-major [rows, cols], element 2j in the high nibble of byte j, one
 * absmax per 64 consecutive elements of a row.  tile16: for row tile rb (16
 * rows) and 64-element block kb, the 16 rows' 32-byte block segments are
 * contiguous:
 *   q_out byte   ((rb*(cols/64) + kb)*16 + r)*32 + j = q row 16rb+r, block kb, byte j
 *   absmax_out   ((rb*(cols/64) + kb)*16 + r)        = absmax row 16rb+r, block kb
 * Used when an expert becomes GPU-resident (the reference's reconstruct step,
 * transfer/nf4_reconstruct.py:117-150).  rows % 16 == 0, cols % 64 == 0.
 */
int moe_nf4_tile16(const uint8_t* q, const float* absmax, int64_t rows,
                   int64_t cols, uint8_t* q_out, float* absmax_out,
                   void* stream);

/* bf16(code * absmax) of a tile16 matrix, written row-major [rows, cols];
 * bit-exact with moe_nf4_dequant on the store layout. */
int moe_nf4_dequant_tile16(const uint8_t* q, const float* absmax,
                           const float* code, int64_t rows, int64_t cols,
                           uint16_t* out_bf16, void* stream);

/* ---------------------------------------------------------------------------
 * Rebuild fp32 absmax from its double quantization (nested QuantState,
 * transfer/nf4_reconstruct.py:17-38, blocksize 256 at :13):
 *   out[b] = fp32(fp32(code2[qabs[b]] * absmax2[b / blocksize2]) + offset)
 */
int moe_nf4_nested_absmax(const uint8_t* qabs, const float* absmax2,
                          const float* code2, float offset, int64_t nblocks,
                          int blocksize2, float* out_absmax, void* stream);

/* ---------------------------------------------------------------------------
 * Fused top-k router: logits = fp16(h . Wg^T) (fp32 accumulation), fp32
 * softmax over E, top-k, renormalised over the k chosen.
 * Replaces ExpertRouter.logits/route_with_logits (engine/router.py:50-94).
 *   h      fp16 [T, H]      wg   fp16 [E, H]
 *   logits fp16 [T, E] (may be NULL)
 *   weights fp32 [T, k]     indices int64 [T, k] (descending probability;
 *   exact ties resolved toward the lower expert index)
 * Limits: 1 <= E <= 32, 1 <= k <= E, H % 8 == 0.
 */
int moe_router_topk(const uint16_t* h, const uint16_t* wg, int64_t T, int H,
                    int E, int k, uint16_t* logits, float* weights,
                    int64_t* indices, void* stream);

/* Softmax/top-k/renormalise stage alone, from fp16 logits [T, E]
 * (engine/router.py:81-92). */
int moe_router_topk_from_logits(const uint16_t* logits, int64_t T, int E,
                                int k, float* weights, int64_t* indices,
                                void* stream);

/* ---------------------------------------------------------------------------
 * SwiGLU expert on n fp16 tokens: y = w2(silu(w1 x) * w3 x)
 * Replaces ReconstructedNF4Expert.forward (transfer/nf4_reconstruct.py:152-155)
 * with the bitsandbytes Linear4bit path it reaches: n == 1 uses the 4-bit
 * GEMV semantics (fp16(fp16(code)*fp16(absmax)) weights), n > 1 the
 * dequant-to-bf16-then-fp16-GEMM semantics.
 *   x fp16 [n, hidden]  ->  y fp16 [n, hidden]; weights in tile16 layout.
 * Requires hidden % 64 == 0 (<= 8192) and inter % 64 == 0.
 * For 9..32 tokens a projection with few 128-row tiles splits its K blocks
 * over several work units (fp32 partials in the workspace, summed in order by
 * a second kernel), so one expert keeps every SM streaming; the workspace
 * size then depends on the current device's SM count: size and call on the
 * same device.
 */
size_t moe_expert_workspace_size(int64_t n, int hidden, int inter);
int moe_expert_forward(const moe_nf4_expert_t* expert, const uint16_t* x,
                       int64_t n, int hidden, int inter, uint16_t* y,
                       void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Codebooks.  moe_expert_forward, moe_experts_forward, moe_layer_forward and
 * moe_layer_forward_noalloc decode every expert of one call with expert 0's
 * codebooks (w1's for w1 and w3, w2's for w2).  All experts of one call must
 * carry equal codebook values (every NF4 store made by the reference's
 * quantizer does: the standard NF4 table).  A call whose experts differ is
 * detected on the device: its outputs are invalid and moe_stream_check()
 * returns MOE_ERR_CODEBOOK.
 *
 * ---------------------------------------------------------------------------
 * One sparse-MoE layer: router -> permute -> experts -> weighted combine,
 * with no host synchronisation.  Replaces MoELayer._forward_tokens
 * (model/moe_layer.py:117-211) for GPU-resident experts: routing
 * (:143), per-expert masked dispatch in ascending expert id (:150-186) and
 * output[mask] += y * w with one fp16 rounding per expert (:187-191).
 *   h fp16 [T, hidden], wg fp16 [E, hidden], experts[E] (host array)
 *   out fp16 [T, hidden]; indices int64 [T, k] and weights fp32 [T, k]
 *   receive the routing (both required).
 * The workspace needs no initialisation (the layer zeroes the counters it
 * keeps there); calls sharing a workspace must be ordered on the device.
 * For 9 or more tokens on narrow tiles (at most 32 per expert) the size
 * reported includes split-K partials for projections with few row tiles; a
 * smaller workspace that still holds everything else runs without them.
 * T == 1 runs as two launches: the counters, then one kernel that routes,
 * runs both projections and combines.  That kernel's CTAs (one per SM) wait
 * on one another's progress, so it needs the whole GPU's SMs; every such wait
 * is bounded, and a timeout sets the word read by moe_take_device_error.
 */
size_t moe_layer_workspace_size(int64_t T, int hidden, int inter, int E, int k);
int moe_layer_forward(const uint16_t* h, const uint16_t* wg,
                      const moe_nf4_expert_t* experts, int E, int k, int64_t T,
                      int hidden, int inter, uint16_t* out, int64_t* indices,
                      float* weights, void* workspace, size_t workspace_bytes,
                      void* stream);

/* ---------------------------------------------------------------------------
 * moe_layer_forward without a workspace argument.  No counterpart in the
 * reference (its layer allocates through PyTorch on every call).
 *
 * For callers that cannot hand the library device memory per call: C or FFI
 * hosts that bind only plain pointers and have no device allocator of their
 * own (a ctypes/cgo stub), and serving loops that must not allocate in the
 * steady state (cudaMalloc synchronises the device, and an allocator that
 * grows mid-step stalls the step).  Scratch comes from a file-scope device
 * array of MOE_NOALLOC_SCRATCH_BYTES (4 MiB) per device: enough for
 * T*k <= 16 routed pairs at Mixtral shapes (hidden 4096, inter 14336), i.e.
 * decode batches up to 8 tokens with top-2.  A call whose workspace need
 * (without the optional split-K partials, which moe_layer_forward uses only
 * when its workspace holds them) exceeds it returns MOE_ERR_WORKSPACE and
 * does nothing.  The array's address is looked up (cudaGetSymbolAddress) on the
 * first call on each device and cached; make that first call before any
 * stream capture on the device.  The scratch used is the CURRENT device's
 * (cudaGetDevice), which must be the device `stream` belongs to; the cached
 * address is invalid after cudaDeviceReset on that device.  Calls that overlap
 * on one device (other streams or host threads without ordering) race on the
 * one array: serialise them.  Nothing in the array needs to start at zero.
 * Same results as moe_layer_forward; like it, a wait that timed out or a
 * codebook mismatch is only visible through moe_stream_check() /
 * moe_take_device_error(), which callers must poll at their sync points.
 */
#define MOE_NOALLOC_SCRATCH_BYTES ((size_t)4 << 20)
int moe_layer_forward_noalloc(const uint16_t* h, const uint16_t* wg,
                              const moe_nf4_expert_t* experts, int E, int k,
                              int64_t T, int hidden, int inter, uint16_t* out,
                              int64_t* indices, float* weights, void* stream);

/* ---------------------------------------------------------------------------
 * Expert stage alone: SwiGLU experts on rows already grouped by expert (the
 * rows of expert e are [expert_offsets[e], expert_offsets[e+1]) of x_sorted,
 * device int32 [E+1]); y_sorted fp16 [P, hidden] in the same order.  Used after
 * an expert-parallel dispatch and to time the expert kernels alone.  Same
 * per-expert semantics as moe_expert_forward.
 */
size_t moe_experts_workspace_size(int64_t P, int hidden, int inter);
int moe_experts_forward(const moe_nf4_expert_t* experts, int E,
                        const int32_t* expert_offsets, const uint16_t* x_sorted,
                        int64_t P, int hidden, int inter, uint16_t* y_sorted,
                        void* workspace, size_t workspace_bytes, void* stream);

/* moe_experts_forward for a decode batch (P <= MOE_DECODE_MAX_ROWS; more returns
 * MOE_ERR_UNSUPPORTED) stopped before its last step: y_part fp32
 * [P, S, hidden] receives the down projection's S = moe_expert_splits(inter)
 * K-split partials of every row (rows of no expert are left as they were);
 * fp16(in-order sum over S) of a row is moe_experts_forward's output row.
 * For a consumer that sums them itself (moe_ep_return_partials_p2p), one
 * launch fewer.  Same workspace as moe_experts_forward.  counters: null, or
 * moe_experts_counter_words(inter) int32 that an earlier kernel on the stream
 * zeroed (moe_ep_front_p2p can), which spares the zeroing launch; the call
 * leaves them non-zero.  moe_expert_splits: S for `inter` (2048-element K
 * splits); both return -1 for an unsupported size. */
int moe_expert_splits(int inter);
int moe_experts_counter_words(int inter);
int moe_experts_forward_partials(const moe_nf4_expert_t* experts, int E,
                                 const int32_t* expert_offsets, const uint16_t* x_sorted,
                                 int64_t P, int hidden, int inter, float* y_part,
                                 int32_t* counters, void* workspace, size_t workspace_bytes,
                                 void* stream);

/* ---------------------------------------------------------------------------
 * Building blocks of moe_layer_forward, exported for tests and for the
 * expert-parallel path (dispatch/combine around an all-to-all).
 *
 * moe_permute: stable counting sort of the T*k (token, slot) pairs by expert.
 *   expert_offsets int32 [E+1]; pair_token int32 [T*k] (token of each sorted
 *   pair, ascending token order within an expert); pair_weight fp32 [T*k];
 *   pair_slot int32 [T*k] (sorted position of pair t*k+j).
 * (model/moe_layer.py:172-185: mask = any(idx == e), h[mask] in token order.)
 */
int moe_permute(const int64_t* indices, const float* weights, int64_t T, int k,
                int E, int32_t* expert_offsets, int32_t* pair_token,
                float* pair_weight, int32_t* pair_slot, void* stream);

/* rows_out[i] = rows_in[index[i]] for fp16 rows of width `width`. */
int moe_gather_rows(const uint16_t* rows_in, const int32_t* index, int64_t n,
                    int width, uint16_t* rows_out, void* stream);

/* Weighted combine in ascending expert order, one fp16 rounding per expert
 * (model/moe_layer.py:187-191):
 *   out[t] = fp16(out[t] + fp32(y[pair_slot[t*k+j]]) * w[t,j]) for the token's
 *   experts in ascending id, starting from out[t] = 0. */
int moe_combine(const uint16_t* y_sorted, const int32_t* pair_slot,
                const int64_t* indices, const float* weights, int64_t T, int k,
                int width, uint16_t* out, void* stream);

/* ---------------------------------------------------------------------------
 * Expert-parallel token exchange (one process per GPU; the caller runs the two
 * all-to-alls, e.g. NCCL, between these steps).  G ranks, E experts, rank r
 * owns experts [r*E/G, (r+1)*E/G).  Buffers are capacity-padded so both
 * all-to-alls use equal splits and nothing needs a host synchronisation:
 * cap >= tokens per rank * min(k, E/G) rows per (source, destination) pair.
 * Replaces nothing in the reference (single-GPU); it feeds the same per-expert
 * semantics (model/moe_layer.py:150-191) from tokens of every rank.
 *
 * moe_ep_dispatch (source; after moe_permute):
 *   send_rows fp16 [G*(cap+1), hidden]: chunk r holds send_rows[r*(cap+1)+i] =
 *   h[pair_token[off[r*E/G]+i]], and its last row (the header) carries rank r's
 *   E/G expert counts as int32 in its first bytes, so one all-to-all of rows
 *   also delivers the counts;
 *   send_counts int32 [E] (optional, may be NULL): the same counts, compact;
 *   pair_slot_ep int32 [T*k]: row of pair t*k+j in the returned buffer
 * moe_ep_receive (owner; after the all-to-all of rows):
 *   x_sorted fp16 [G*cap, hidden] grouped by local expert (then source rank),
 *   local_offsets int32 [E/G + 1], recv_counts int32 [E] (output: the counts
 *   read from the headers, compact); feed x_sorted and local_offsets to
 *   moe_experts_forward with P = G*cap.
 * moe_ep_return (owner): y_back fp16 [G*cap, hidden]: y_back[s*cap+i] =
 *   y_sorted[row of (s, i)], given the recv_counts moe_ep_receive wrote; after
 *   the all-to-all back, moe_combine(y_back, pair_slot_ep, ...) on the source.
 * Limits: E % G == 0, E <= 32, hidden % 8 == 0, 2*hidden >= 4*E/G.
 */
int moe_ep_dispatch(const uint16_t* h, const int32_t* expert_offsets,
                    const int32_t* pair_token, const int32_t* pair_slot, int64_t T,
                    int k, int E, int G, int cap, int hidden, uint16_t* send_rows,
                    int32_t* send_counts, int32_t* pair_slot_ep, void* stream);
int moe_ep_receive(const uint16_t* recv_rows, int32_t* recv_counts, int E,
                   int G, int cap, int hidden, uint16_t* x_sorted,
                   int32_t* local_offsets, void* stream);
int moe_ep_return(const uint16_t* y_sorted, const int32_t* recv_counts, int E,
                  int G, int cap, int hidden, uint16_t* y_back, void* stream);

/* ---------------------------------------------------------------------------
 * Expert-parallel exchange over peer memory (NVLink), in place of the two
 * all-to-alls.  No counterpart in the reference (single-GPU).  Each rank owns,
 * per exchange, a receive region laid out as the all-to-all would deliver it
 * (G chunks, chunk s from source rank s) and an int32 flag per source, both
 * mapped into every peer (e.g. CUDA IPC); peer_* are device arrays [G] of
 * those addresses (uint64).  seq and done are this rank's own device ints
 * for the exchange (both start at 0; done returns to 0 after every call).
 *
 * moe_ep_dispatch_p2p: moe_ep_dispatch that stores chunk r (cap rows + the
 *   count header row, cap + 1 rows) straight into rank r's receive region at
 *   chunk `rank`; when every CTA has stored, the launch bumps *seq and
 *   release-stores it into flag `rank` of every peer.
 * moe_ep_wait_p2p: bounded wait until all G of this rank's flags reach its
 *   *seq (the value its own send of the same exchange produced); then
 *   moe_ep_receive / moe_combine read the region with the ordinary kernels.
 *   A wait that runs out sets error bit 1 (moe_stream_check: MOE_ERR_TIMEOUT).
 * moe_ep_return_p2p: moe_ep_return that stores the rows for source s straight
 *   into s's return region (G chunks of cap rows) at chunk `rank`, then
 *   signals like the dispatch.
 * moe_ep_receive_p2p / moe_combine_p2p: moe_ep_receive / moe_combine with
 *   that wait inside the kernel (every CTA waits, bounded, on the G flags
 *   before it reads the region): one launch each instead of two.
 * moe_ep_front_p2p: the router (moe_router_topk), moe_permute and
 *   moe_ep_dispatch_p2p in one launch, for 0 <= T <= the GPU's SM count
 *   (more returns MOE_ERR_UNSUPPORTED): one CTA routes each token with the
 *   router kernel's arithmetic, the CTAs meet at a grid barrier on `bar`
 *   (two int32 of this rank, zero before first use; left consistent by every
 *   call), then each stores its token's row into the owners' regions at the
 *   sorted position moe_permute gives it.  Outputs weights fp32 / indices
 *   int64 [T, k] (the router's) and pair_slot_ep [T*k] (moe_ep_dispatch's),
 *   bit-identical to the three calls it replaces.  k <= 8.  It also zeroes
 *   n_zero int32 at zero_words (the counters of the expert stage that
 *   follows; may be 0 / null).  After a timeout the exchange state (flags,
 *   counters, barrier) is undefined: recreate the regions.
 * moe_ep_return_partials_p2p: moe_ep_return_p2p that reads the fp32 split
 *   partials of moe_experts_forward_partials (S splits) and stores
 *   fp16(in-order sum) -- the rows moe_experts_forward would have produced.
 * Calls of one exchange must not overlap; give every layer its own regions.
 */
int moe_ep_dispatch_p2p(const uint16_t* h, const int32_t* expert_offsets,
                        const int32_t* pair_token, const int32_t* pair_slot, int64_t T,
                        int k, int E, int G, int rank, int cap, int hidden,
                        const uint64_t* peer_recv, const uint64_t* peer_flags,
                        int32_t* seq, int32_t* done, int32_t* pair_slot_ep, void* stream);
int moe_ep_return_p2p(const uint16_t* y_sorted, const int32_t* recv_counts, int E, int G,
                      int rank, int cap, int hidden, const uint64_t* peer_back,
                      const uint64_t* peer_flags, int32_t* seq, int32_t* done, void* stream);
int moe_ep_wait_p2p(const int32_t* flags, int G, const int32_t* seq, void* stream);
int moe_ep_receive_p2p(const uint16_t* recv_rows, int32_t* recv_counts, int E, int G,
                       int cap, int hidden, uint16_t* x_sorted, int32_t* local_offsets,
                       const int32_t* flags, const int32_t* seq, void* stream);
int moe_combine_p2p(const uint16_t* y_back, const int32_t* pair_slot, const int64_t* indices,
                    const float* weights, int64_t T, int k, int width, uint16_t* out,
                    const int32_t* flags, int G, const int32_t* seq, void* stream);
int moe_ep_front_p2p(const uint16_t* h, const uint16_t* wg, int64_t T, int E, int k, int G,
                     int rank, int cap, int hidden, const uint64_t* peer_recv,
                     const uint64_t* peer_flags, int32_t* seq, int32_t* done, int32_t* bar,
                     float* weights, int64_t* indices, int32_t* pair_slot_ep,
                     int32_t* zero_words, int n_zero, void* stream);
int moe_ep_return_partials_p2p(const float* y_part, int S, const int32_t* recv_counts, int E,
                               int G, int rank, int cap, int hidden,
                               const uint64_t* peer_back, const uint64_t* peer_flags,
                               int32_t* seq, int32_t* done, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MOE_B200_H */
