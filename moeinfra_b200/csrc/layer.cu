// Host orchestration of the fused MoE layer and of the single-expert forward.
//
// moe_layer_forward replaces MoELayer._forward_tokens (model/moe_layer.py:117-211)
// for GPU-resident experts: one routing pass (:143), per-expert dispatch in
// ascending expert id over the tokens routed to it (:150-186) and the weighted
// fp16 combine (:187-191) -- as a fixed launch sequence on one stream with no
// device->host synchronisation (the reference syncs on unique().tolist(),
// :150-153).  Every buffer comes from the caller's workspace.
#include "common.cuh"

namespace moe {

// expert_decode.cu
bool decode_supported(int hidden, int inter);
int decode_splits(int inter);
int decode_max_tokens();
int launch_decode_experts(const moe_nf4_expert_t* experts, int E, const int32_t* expert_offsets,
                          const int32_t* pair_token, const uint16_t* x, int hidden, int inter,
                          uint16_t* h_sorted, float* y_part, int32_t* sync,
                          int max_tokens_per_expert, cudaStream_t s);
int decode_sync_words(int inter);
int launch_zero_words(int32_t* p, int n, cudaStream_t s);
int launch_decode_layer1(const moe_nf4_expert_t* experts, int E, int k, const uint16_t* h,
                         const uint16_t* wg, int hidden, int inter, uint16_t* h_sorted,
                         float* y_part, int32_t* sync, int32_t* rg_count, uint16_t* out,
                         int64_t* indices, float* weights, cudaStream_t s);
int launch_reduce_partials(const float* part, int64_t P, int S, int width, uint16_t* y,
                           cudaStream_t s);
int launch_identity_offsets(int32_t* off, int n, int32_t* zero, int nzero, cudaStream_t s);
// permute.cu
int launch_permute(const int64_t* indices, const float* weights, int64_t T, int k, int E,
                   int32_t* expert_offsets, int32_t* pair_token, float* pair_weight,
                   int32_t* pair_slot, int32_t* zero, int nzero, cudaStream_t s);
int launch_combine_partials(const float* part, int S, const int32_t* pair_slot,
                            const int64_t* indices, const float* weights, int64_t T, int k,
                            int width, uint16_t* out, cudaStream_t s);
// expert_gemm_sm100.cu
int launch_grouped_gemm_experts(const moe_nf4_expert_t* experts, int E,
                                const int32_t* expert_offsets, const uint16_t* x_sorted,
                                int64_t P, int hidden, int inter, uint16_t* h_sorted,
                                uint16_t* y_sorted, uint16_t* x_split, float* part,
                                cudaStream_t s);
bool gemm_narrow(int64_t P, int E);
size_t gemm_splitk_floats(int64_t P, int E, int hidden, int inter);

namespace {

constexpr size_t kAlign = 256;
size_t align_up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

// Sequential carve-out of the caller's workspace.
struct Carver {
  unsigned char* base;
  size_t used = 0;
  template <class T>
  T* take(size_t count) {
    T* p = reinterpret_cast<T*>(base ? base + used : nullptr);
    used += align_up(count * sizeof(T));
    return p;
  }
};

bool use_decode_path(int64_t T) { return T <= decode_max_tokens(); }

struct LayerBufs {
  int32_t* offsets;
  int32_t* pair_token;
  float* pair_weight;
  int32_t* pair_slot;
  uint16_t* h_sorted;
  float* y_part;      // decode path
  int32_t* sync;       // decode path: completion counters (gate_up splits, then row groups)
  uint16_t* x_sorted;  // grouped-GEMM path
  uint16_t* y_sorted;  // grouped-GEMM path
  uint16_t* x_split;   // grouped-GEMM path, narrow tiles: tokens as bf16 hi/lo rows
  float* part;         // grouped-GEMM path: split-K partials (null: none)
};

// The narrow grouped GEMM keeps the SwiGLU activations as bf16 hi/lo row pairs
// (two rows per token-expert pair) and needs the tokens split the same way.
// A call of P pairs can take narrow tiles only if P <= 32 x MOE_MAX_EXPERTS.
bool may_be_narrow(int64_t P) { return P <= (int64_t)32 * MOE_MAX_EXPERTS; }

// split_k: room for the grouped GEMM's split-K partials (the size the
// workspace query reports); a call whose workspace is smaller runs without.
size_t carve_layer(unsigned char* ws, int64_t T, int hidden, int inter, int E, int k,
                   LayerBufs* b, bool split_k = true) {
  Carver c{ws};
  const int64_t P = T * k;
  b->offsets = c.take<int32_t>(E + 1);
  b->pair_token = c.take<int32_t>(P);
  b->pair_weight = c.take<float>(P);
  b->pair_slot = c.take<int32_t>(P);
  const bool narrow = !use_decode_path(T) && gemm_narrow(P, E);
  b->h_sorted = c.take<uint16_t>((size_t)(narrow ? 2 * P : P) * inter);
  b->x_split = nullptr;
  if (use_decode_path(T)) {
    b->y_part = c.take<float>((size_t)P * decode_splits(inter) * hidden);
    b->sync = c.take<int32_t>(decode_sync_words(inter) + hidden / 16);
    b->x_sorted = b->y_sorted = nullptr;
  } else {
    b->y_part = nullptr;
    b->sync = nullptr;
    b->x_sorted = c.take<uint16_t>((size_t)P * hidden);
    b->y_sorted = c.take<uint16_t>((size_t)P * hidden);
    if (narrow) b->x_split = c.take<uint16_t>((size_t)2 * P * hidden);
  }
  const size_t part = use_decode_path(T) || !split_k ? 0 : gemm_splitk_floats(P, E, hidden, inter);
  b->part = part ? c.take<float>(part) : nullptr;
  return c.used;
}

bool shapes_ok(int hidden, int inter) { return decode_supported(hidden, inter); }

bool experts_aligned(const moe_nf4_expert_t* ex, int E) {
  for (int e = 0; e < E; ++e) {
    const moe_nf4_matrix_t* m[3] = {&ex[e].w1, &ex[e].w3, &ex[e].w2};
    for (auto* mm : m) {
      if (!mm->q || !mm->absmax || !mm->code) return false;
      if (!aligned16(mm->q) || (reinterpret_cast<uintptr_t>(mm->absmax) & 3)) return false;
    }
  }
  return true;
}

}  // namespace
}  // namespace moe

namespace moe {
// Workspace bytes of a layer call, with or without the split-K partials.
size_t layer_workspace_bytes(int64_t T, int hidden, int inter, int E, int k, bool split_k) {
  LayerBufs b;
  if (T < 0 || E < 1 || k < 1) return 0;
  return carve_layer(nullptr, T, hidden, inter, E, k, &b, split_k);
}
}  // namespace moe

extern "C" size_t moe_layer_workspace_size(int64_t T, int hidden, int inter, int E, int k) {
  moe::LayerBufs b;
  if (T < 0 || E < 1 || k < 1) return 0;
  return moe::carve_layer(nullptr, T, hidden, inter, E, k, &b);
}

extern "C" int moe_layer_forward(const uint16_t* h, const uint16_t* wg,
                                 const moe_nf4_expert_t* experts, int E, int k, int64_t T,
                                 int hidden, int inter, uint16_t* out, int64_t* indices,
                                 float* weights, void* workspace, size_t workspace_bytes,
                                 void* stream) {
  using namespace moe;
  if (T < 0 || E < 1 || E > MOE_MAX_EXPERTS || k < 1 || k > E || k > 8) return MOE_ERR_INVALID_ARG;
  if (!shapes_ok(hidden, inter)) return MOE_ERR_UNSUPPORTED;
  if (T == 0) return MOE_OK;
  if (!h || !wg || !experts || !out || !indices || !weights) return MOE_ERR_INVALID_ARG;
  if (!experts_aligned(experts, E) || !aligned16(h) || !aligned16(out)) return MOE_ERR_ALIGNMENT;
  LayerBufs b;
  const bool split_k = workspace_bytes >= carve_layer(nullptr, T, hidden, inter, E, k, &b);
  const size_t need = carve_layer(static_cast<unsigned char*>(workspace), T, hidden, inter, E, k,
                                  &b, split_k);
  if (!workspace || workspace_bytes < need) return MOE_ERR_WORKSPACE;
  if (!aligned16(workspace)) return MOE_ERR_ALIGNMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (T == 1 && E <= MOE_MAX_EXPERTS) {
    // One token: counters zeroed, then a single launch (route, experts, combine).
    const int words = decode_sync_words(inter);
    int st = launch_zero_words(b.sync, words + hidden / 16, s);
    if (st != MOE_OK) return st;
    return launch_decode_layer1(experts, E, k, h, wg, hidden, inter, b.h_sorted, b.y_part, b.sync,
                                b.sync + words, out, indices, weights, s);
  }
  int st = moe_router_topk(h, wg, T, hidden, E, k, nullptr, weights, indices, s);
  if (st != MOE_OK) return st;
  st = launch_permute(indices, weights, T, k, E, b.offsets, b.pair_token, b.pair_weight,
                      b.pair_slot, b.sync, b.sync ? decode_sync_words(inter) : 0, s);
  if (st != MOE_OK) return st;
  const int64_t P = T * k;
  if (use_decode_path(T)) {
    st = launch_decode_experts(experts, E, b.offsets, b.pair_token, h, hidden, inter, b.h_sorted,
                               b.y_part, b.sync, static_cast<int>(T), s);
    if (st != MOE_OK) return st;
    return launch_combine_partials(b.y_part, decode_splits(inter), b.pair_slot, indices, weights,
                                   T, k, hidden, out, s);
  }
  st = moe_gather_rows(h, b.pair_token, P, hidden, b.x_sorted, s);
  if (st != MOE_OK) return st;
  st = launch_grouped_gemm_experts(experts, E, b.offsets, b.x_sorted, P, hidden, inter, b.h_sorted,
                                   b.y_sorted, b.x_split, b.part, s);
  if (st != MOE_OK) return st;
  return moe_combine(b.y_sorted, b.pair_slot, indices, weights, T, k, hidden, out, s);
}

namespace moe {
namespace {
struct ExpertBufs {
  int32_t* offsets;
  uint16_t* h;
  float* y_part;
  int32_t* sync;
  uint16_t* x_split;
  float* part;  // split-K partials of the tensor-core path (null: none)
};
size_t carve_expert(unsigned char* ws, int64_t n, int hidden, int inter, ExpertBufs* b) {
  Carver c{ws};
  b->offsets = c.take<int32_t>(2);
  const bool narrow = !use_decode_path(n) && gemm_narrow(n, 1);
  b->h = c.take<uint16_t>((size_t)(narrow ? 2 * n : n) * inter);
  b->x_split = narrow ? c.take<uint16_t>((size_t)2 * n * hidden) : nullptr;
  const size_t part = use_decode_path(n) ? 0 : gemm_splitk_floats(n, 1, hidden, inter);
  b->part = part ? c.take<float>(part) : nullptr;
  if (use_decode_path(n)) {
    b->y_part = c.take<float>((size_t)n * decode_splits(inter) * hidden);
    b->sync = c.take<int32_t>(decode_sync_words(inter));
  } else {
    b->y_part = nullptr;
    b->sync = nullptr;
  }
  return c.used;
}
}  // namespace
}  // namespace moe

extern "C" size_t moe_expert_workspace_size(int64_t n, int hidden, int inter) {
  moe::ExpertBufs b;
  if (n < 0) return 0;
  return moe::carve_expert(nullptr, n, hidden, inter, &b);
}

extern "C" int moe_expert_forward(const moe_nf4_expert_t* expert, const uint16_t* x, int64_t n,
                                  int hidden, int inter, uint16_t* y, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  using namespace moe;
  if (n < 0) return MOE_ERR_INVALID_ARG;
  if (!shapes_ok(hidden, inter)) return MOE_ERR_UNSUPPORTED;
  if (n == 0) return MOE_OK;
  if (!expert || !x || !y) return MOE_ERR_INVALID_ARG;
  if (!experts_aligned(expert, 1) || !aligned16(x) || !aligned16(y)) return MOE_ERR_ALIGNMENT;
  if (n > (int64_t)1 << 30) return MOE_ERR_INVALID_ARG;
  ExpertBufs b;
  const size_t need = carve_expert(static_cast<unsigned char*>(workspace), n, hidden, inter, &b);
  if (!workspace || workspace_bytes < need) return MOE_ERR_WORKSPACE;
  if (!aligned16(workspace)) return MOE_ERR_ALIGNMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int st = launch_identity_offsets(b.offsets, static_cast<int>(n), b.sync,
                                   b.sync ? decode_sync_words(inter) : 0, s);
  if (st != MOE_OK) return st;
  if (use_decode_path(n)) {
    st = launch_decode_experts(expert, 1, b.offsets, nullptr, x, hidden, inter, b.h, b.y_part,
                               b.sync, static_cast<int>(n), s);
    if (st != MOE_OK) return st;
    return launch_reduce_partials(b.y_part, n, decode_splits(inter), hidden, y, s);
  }
  return launch_grouped_gemm_experts(expert, 1, b.offsets, x, n, hidden, inter, b.h, y, b.x_split,
                                     b.part, s);
}

// ---------------------------------------------------------------------------
// Expert stage alone: experts applied to already-permuted rows (the tokens of
// expert e are rows [offsets[e], offsets[e+1]) of x_sorted), y_sorted fp16.
namespace moe {
namespace {
struct StageBufs {
  uint16_t* h;
  float* y_part;
  int32_t* sync;
  uint16_t* x_split;
};
// The expert count is not known when the workspace is sized: room for narrow
// tiles is reserved whenever P pairs could take them.
size_t carve_stage(unsigned char* ws, int64_t P, int hidden, int inter, StageBufs* b) {
  Carver c{ws};
  const bool split = !use_decode_path(P) && may_be_narrow(P);
  b->h = c.take<uint16_t>((size_t)(split ? 2 * P : P) * inter);
  b->x_split = split ? c.take<uint16_t>((size_t)2 * P * hidden) : nullptr;
  b->y_part = use_decode_path(P) ? c.take<float>((size_t)P * decode_splits(inter) * hidden) : nullptr;
  b->sync = use_decode_path(P) ? c.take<int32_t>(decode_sync_words(inter)) : nullptr;
  return c.used;
}
}  // namespace
}  // namespace moe

extern "C" size_t moe_experts_workspace_size(int64_t P, int hidden, int inter) {
  moe::StageBufs b;
  if (P < 0) return 0;
  return moe::carve_stage(nullptr, P, hidden, inter, &b);
}

extern "C" int moe_experts_forward(const moe_nf4_expert_t* experts, int E,
                                   const int32_t* expert_offsets, const uint16_t* x_sorted,
                                   int64_t P, int hidden, int inter, uint16_t* y_sorted,
                                   void* workspace, size_t workspace_bytes, void* stream) {
  using namespace moe;
  if (P < 0 || E < 1 || E > MOE_MAX_EXPERTS) return MOE_ERR_INVALID_ARG;
  if (!shapes_ok(hidden, inter)) return MOE_ERR_UNSUPPORTED;
  if (P == 0) return MOE_OK;
  if (!experts || !expert_offsets || !x_sorted || !y_sorted) return MOE_ERR_INVALID_ARG;
  if (!experts_aligned(experts, E) || !aligned16(x_sorted) || !aligned16(y_sorted))
    return MOE_ERR_ALIGNMENT;
  StageBufs b;
  const size_t need = carve_stage(static_cast<unsigned char*>(workspace), P, hidden, inter, &b);
  if (!workspace || workspace_bytes < need) return MOE_ERR_WORKSPACE;
  if (!aligned16(workspace)) return MOE_ERR_ALIGNMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (use_decode_path(P)) {
    int st = launch_zero_words(b.sync, decode_sync_words(inter), s);
    if (st != MOE_OK) return st;
    st = launch_decode_experts(experts, E, expert_offsets, nullptr, x_sorted, hidden, inter,
                                   b.h, b.y_part, b.sync, static_cast<int>(P), s);
    if (st != MOE_OK) return st;
    return launch_reduce_partials(b.y_part, P, decode_splits(inter), hidden, y_sorted, s);
  }
  return launch_grouped_gemm_experts(experts, E, expert_offsets, x_sorted, P, hidden, inter, b.h,
                                     y_sorted, b.x_split, nullptr, s);
}

extern "C" int moe_expert_splits(int inter) {
  return inter > 0 && inter % 64 == 0 ? moe::decode_splits(inter) : -1;
}

extern "C" int moe_experts_counter_words(int inter) {
  return inter > 0 && inter % 64 == 0 ? moe::decode_sync_words(inter) : -1;
}

extern "C" int moe_experts_forward_partials(const moe_nf4_expert_t* experts, int E,
                                            const int32_t* expert_offsets,
                                            const uint16_t* x_sorted, int64_t P, int hidden,
                                            int inter, float* y_part, int32_t* counters,
                                            void* workspace, size_t workspace_bytes,
                                            void* stream) {
  using namespace moe;
  if (P < 0 || E < 1 || E > MOE_MAX_EXPERTS) return MOE_ERR_INVALID_ARG;
  if (!shapes_ok(hidden, inter) || !use_decode_path(P)) return MOE_ERR_UNSUPPORTED;
  if (P == 0) return MOE_OK;
  if (!experts || !expert_offsets || !x_sorted || !y_part) return MOE_ERR_INVALID_ARG;
  if (!experts_aligned(experts, E) || !aligned16(x_sorted) || !aligned16(y_part))
    return MOE_ERR_ALIGNMENT;
  StageBufs b;
  const size_t need = carve_stage(static_cast<unsigned char*>(workspace), P, hidden, inter, &b);
  if (!workspace || workspace_bytes < need) return MOE_ERR_WORKSPACE;
  if (!aligned16(workspace)) return MOE_ERR_ALIGNMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Caller-zeroed counters (e.g. by moe_ep_front_p2p) spare the zeroing launch.
  int32_t* sync = counters ? counters : b.sync;
  if (!counters) {
    const int st = launch_zero_words(b.sync, decode_sync_words(inter), s);
    if (st != MOE_OK) return st;
  }
  return launch_decode_experts(experts, E, expert_offsets, nullptr, x_sorted, hidden, inter, b.h,
                               y_part, sync, static_cast<int>(P), s);
}
