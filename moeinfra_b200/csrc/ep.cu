// Expert-parallel token exchange: the pack / receive / return steps around the
// two NCCL all-to-alls of an expert-parallel MoE layer.
//
// G ranks, E experts, El = E / G local experts: rank r owns experts
// [r*El, (r+1)*El).  Every buffer exchanged is capacity-padded, so the
// all-to-alls use equal splits and no step needs a host synchronisation:
//   cap = max tokens per rank * min(k, El) rows per (source, destination) pair.
//
// Source rank, after the router and moe_permute (pairs sorted by expert):
//   send_rows[r*cap + i]  = h[pair_token[offsets[r*El] + i]],  i < n_r
//   send_counts[r*El + j] = tokens of expert r*El + j
//   pair_slot_ep[q]       = r*cap + pair_slot[q] - offsets[r*El]   (r = owner)
// Destination rank, after the all-to-all (recv[s*cap + i] came from rank s):
//   x_sorted rows ordered by (local expert j, source s, i); local_offsets[j]
//   the first row of expert j -- the grouped layout the expert kernels read.
// Return: y_back[s*cap + i] = y_sorted[row of (s, i)], sent back by a second
// all-to-all, after which y_back on the source is addressed by pair_slot_ep
// and moe_combine applies the reference's ordered fp16 combine
// (model/moe_layer.py:187-191) unchanged.
#include "common.cuh"
#include "router_device.cuh"

namespace moe {
namespace {

MOE_DEFINE_ERROR_WORD()

constexpr int kEpMaxExperts = 32;
constexpr int kEpThreads = 256;

int grid_rows(int64_t work) {
  int64_t b = ceil_div(work, kEpThreads);
  int64_t cap = (int64_t)sm_count() * 8;
  return static_cast<int>(b < 1 ? 1 : (b < cap ? b : cap));
}

__global__ void __launch_bounds__(kEpThreads) k_ep_dispatch(
    const uint4* __restrict__ h, const int32_t* __restrict__ offsets,
    const int32_t* __restrict__ pair_token, const int32_t* __restrict__ pair_slot, int64_t P,
    int E, int El, int G, int cap, int vpr, uint4* __restrict__ send,
    int32_t* __restrict__ send_counts, int32_t* __restrict__ pair_slot_ep) {
  __shared__ int s_off[kEpMaxExperts + 1];
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x <= E) s_off[threadIdx.x] = offsets[threadIdx.x];
  __syncthreads();
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  // Header row (last row of each destination's chunk): that destination's El
  // expert counts as int32 in its first bytes; the optional compact copy too.
  if (tid < E) {
    const int r = static_cast<int>(tid) / El, j = static_cast<int>(tid) - r * El;
    const int c = s_off[tid + 1] - s_off[tid];
    reinterpret_cast<int32_t*>(send + ((int64_t)r * (cap + 1) + cap) * vpr)[j] = c;
    if (send_counts) send_counts[tid] = c;
  }
  for (int64_t q = tid; q < P; q += stride) {
    const int p = pair_slot[q];
    int e = 0;
    while (e + 1 < E && s_off[e + 1] <= p) ++e;
    const int r = e / El;
    pair_slot_ep[q] = r * cap + (p - s_off[r * El]);
  }
  const int64_t total = (int64_t)G * cap * vpr;
  for (int64_t v = tid; v < total; v += stride) {
    const int64_t row = v / vpr;
    const int c = static_cast<int>(v - row * vpr);
    const int r = static_cast<int>(row / cap), i = static_cast<int>(row - (int64_t)r * cap);
    const int p = s_off[r * El] + i;
    if (p < s_off[(r + 1) * El])
      send[(row + r) * vpr + c] = h[(int64_t)pair_token[p] * vpr + c];  // chunk stride cap + 1
  }
}

// Per-(source, local expert) bases of the receive layout, in shared memory.
struct RecvPlan {
  int n[kEpMaxExperts];         // rows from source s (clamped to cap)
  int src_base[kEpMaxExperts];  // [s*El + j]: first row of expert j within source s's chunk
  int dst_base[kEpMaxExperts];  // [s*El + j]: first x_sorted row of (j, s)
  int cnt[kEpMaxExperts];
  int local_off[kEpMaxExperts + 1];
};

// counts of source s, local expert j at counts[s * stride + j].
__device__ void build_plan(const int32_t* __restrict__ counts, int64_t stride, int El, int G,
                           int cap, RecvPlan& pl) {
  if (threadIdx.x == 0) {
    // Counts come from peers; clamp so that no source exceeds its cap rows and
    // every derived row index stays inside the G*cap-row buffers.
    for (int s = 0; s < G; ++s) {
      int acc = 0;
      for (int j = 0; j < El; ++j) {
        int c = counts[s * stride + j];
        c = c < 0 ? 0 : (c > cap - acc ? cap - acc : c);
        pl.cnt[s * El + j] = c;
        pl.src_base[s * El + j] = acc;
        acc += c;
      }
      pl.n[s] = acc;
    }
    int acc = 0;
    for (int j = 0; j < El; ++j) {
      pl.local_off[j] = acc;
      for (int s = 0; s < G; ++s) {
        pl.dst_base[s * El + j] = acc;
        acc += pl.cnt[s * El + j];
      }
    }
    pl.local_off[El] = acc;
  }
  __syncthreads();
}

// x_sorted row of received row (s, i), or -1 for a padding row.
__device__ __forceinline__ int64_t recv_dst(const RecvPlan& pl, int El, int s, int i) {
  if (i >= pl.n[s]) return -1;
  int j = 0;
  while (j + 1 < El && pl.src_base[s * El + j + 1] <= i) ++j;
  return pl.dst_base[s * El + j] + (i - pl.src_base[s * El + j]);
}

// kReceive: `in` is the received buffer (G chunks of cap + 1 rows, counts in
// each chunk's header row); writes x_sorted, local offsets and the compact
// counts.  Otherwise: `counts` is that compact copy and `in` is y_sorted.
// wait_flags (peer-memory exchange): every CTA first waits (bounded) until
// all G flags reach *wait_seq, i.e. every source's rows have landed.
template <bool kReceive>
__global__ void __launch_bounds__(kEpThreads) k_ep_move(
    const uint4* __restrict__ in, int32_t* __restrict__ counts, int El, int G, int cap,
    int vpr, uint4* __restrict__ out, int32_t* __restrict__ local_offsets,
    const int32_t* wait_flags, const int32_t* wait_seq, uint64_t wait_ns) {
  __shared__ RecvPlan pl;
  pdl_trigger();
  pdl_wait();
  if (wait_flags) {
    if (threadIdx.x < G && !wait_peer_flag(wait_flags, threadIdx.x, wait_seq, wait_ns))
      set_device_error(kErrWaitTimeout);
    __syncthreads();
  }
  if (kReceive)
    build_plan(reinterpret_cast<const int32_t*>(in + (int64_t)cap * vpr),
               (int64_t)(cap + 1) * vpr * 4, El, G, cap, pl);
  else
    build_plan(counts, El, El, G, cap, pl);
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (kReceive && tid <= El) local_offsets[tid] = pl.local_off[tid];
  if (kReceive && tid < El * G) counts[tid] = pl.cnt[tid];
  const int64_t total = (int64_t)G * cap * vpr;
  const int64_t rows_out = (int64_t)G * cap;
  for (int64_t v = tid; v < total; v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = v / vpr;  // (s, i) in the exchanged layout
    const int c = static_cast<int>(v - row * vpr);
    const int s = static_cast<int>(row / cap), i = static_cast<int>(row - (int64_t)s * cap);
    const int64_t dst = recv_dst(pl, El, s, i);
    if (dst < 0 || dst >= rows_out) continue;
    if (kReceive)
      out[dst * vpr + c] = in[(row + s) * vpr + c];  // chunk stride cap + 1
    else
      out[row * vpr + c] = in[dst * vpr + c];
  }
}

// ---------------------------------------------------------------------------
// Exchange over peer memory (NVLink), no collective library.  Every rank owns,
// per exchange, a receive region of G chunks (one per source rank, the layout
// the all-to-all would deliver) and G flags, mapped into its peers' address
// spaces.  A sender stores its chunk for rank r straight into r's region at
// chunk `rank`; when every CTA of the launch has stored (system-scope fence,
// then a CTA completion count), the last CTA bumps this exchange's local
// sequence number and, after one system-scope fence, stores it into flag
// `rank` of every peer (fence then relaxed store: a release pattern).  The
// receiver waits (bounded) until all G flags reach its own sequence number
// (each rank sends once and receives once per exchange, so the numbers agree)
// and then reads its region with the ordinary receive / combine kernels.

__device__ __forceinline__ void signal_peers(const uint64_t* __restrict__ peer_flags, int G,
                                             int rank, int32_t* seq, int32_t* done) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    if (atomicAdd(done, 1) == static_cast<int>(gridDim.x) - 1) {
      // This one system-scope fence orders every CTA's rows (published
      // through `done`) before all G flag stores, which are therefore plain
      // relaxed stores issued back to back: a release store per flag would
      // fence again and wait for the previous flag's NVLink round trip.
      __threadfence_system();
      const int s = *reinterpret_cast<volatile int32_t*>(seq) + 1;
      *reinterpret_cast<volatile int32_t*>(seq) = s;
      for (int r = 0; r < G; ++r) {
        int32_t* f = reinterpret_cast<int32_t*>(peer_flags[r]) + rank;
        asm volatile("st.relaxed.sys.global.b32 [%0], %1;" ::"l"(f), "r"(s) : "memory");
      }
      *reinterpret_cast<volatile int32_t*>(done) = 0;
    }
  }
}

__global__ void __launch_bounds__(kEpThreads) k_ep_dispatch_p2p(
    const uint4* __restrict__ h, const int32_t* __restrict__ offsets,
    const int32_t* __restrict__ pair_token, const int32_t* __restrict__ pair_slot, int64_t P,
    int E, int El, int G, int rank, int cap, int vpr, const uint64_t* __restrict__ peer_recv,
    const uint64_t* __restrict__ peer_flags, int32_t* seq, int32_t* done,
    int32_t* __restrict__ pair_slot_ep) {
  __shared__ int s_off[kEpMaxExperts + 1];
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x <= E) s_off[threadIdx.x] = offsets[threadIdx.x];
  __syncthreads();
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t chunk = (int64_t)(cap + 1) * vpr;  // one source's chunk in a receive region
  if (tid < E) {  // header row of the chunk for rank r: r's expert counts from this rank
    const int r = static_cast<int>(tid) / El, j = static_cast<int>(tid) - r * El;
    uint4* dst = reinterpret_cast<uint4*>(peer_recv[r]) + rank * chunk + (int64_t)cap * vpr;
    reinterpret_cast<int32_t*>(dst)[j] = s_off[tid + 1] - s_off[tid];
  }
  for (int64_t q = tid; q < P; q += stride) {
    const int p = pair_slot[q];
    int e = 0;
    while (e + 1 < E && s_off[e + 1] <= p) ++e;
    const int r = e / El;
    pair_slot_ep[q] = r * cap + (p - s_off[r * El]);
  }
  const int64_t total = (int64_t)G * cap * vpr;
  for (int64_t v = tid; v < total; v += stride) {
    const int64_t row = v / vpr;
    const int c = static_cast<int>(v - row * vpr);
    const int r = static_cast<int>(row / cap), i = static_cast<int>(row - (int64_t)r * cap);
    const int p = s_off[r * El] + i;
    if (p < s_off[(r + 1) * El]) {
      uint4* dst = reinterpret_cast<uint4*>(peer_recv[r]) + rank * chunk + (int64_t)i * vpr;
      dst[c] = h[(int64_t)pair_token[p] * vpr + c];
    }
  }
  signal_peers(peer_flags, G, rank, seq, done);
}

// Grid-wide meeting point of the n CTAs of one launch (all resident): a
// sense-reversing barrier on bar[0] (arrivals) and bar[1] (generation), so it
// needs no reset between launches of any size.  Bounded: false (and the
// device error bit) when the others did not arrive within limit_ns.
__device__ bool grid_meet(int32_t* bar, int n, uint64_t limit_ns) {
  __shared__ int s_ok;
  __syncthreads();
  if (threadIdx.x == 0) {
    volatile int32_t* gen = bar + 1;
    const int g = *gen;  // read before arriving: it cannot move until this CTA arrives
    __threadfence();     // orders the read and publishes this CTA's writes
    bool ok = true;
    if (atomicAdd(bar, 1) == n - 1) {
      *reinterpret_cast<volatile int32_t*>(bar) = 0;
      __threadfence();
      atomicExch(bar + 1, g + 1);
    } else {
      const uint64_t t0 = globaltimer_ns();
      int v;
      for (;;) {
        asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(bar + 1) : "memory");
        if (v != g) break;
        if (globaltimer_ns() - t0 > limit_ns) {
          ok = false;
          break;
        }
        __nanosleep(100);
      }
    }
    __threadfence();
    if (!ok) set_device_error(kErrWaitTimeout);
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

// The front of the expert-parallel layer for a decode batch in one launch:
// the router, moe_permute and k_ep_dispatch_p2p fused.  CTA t routes token t
// (route_token_cta: the router kernel's arithmetic, so weights and indices are
// the router's bit for bit), the CTAs meet, then each places its token's k
// pairs where the expert-sorted order puts them (pairs of earlier tokens of
// the same expert come first, as in the stable sort of moe_permute) and stores
// the token's row into each owner's receive region; CTA 0 writes the count
// headers (and zeroes `nzero` words for the expert stage that follows) and
// the last CTA to finish signals the peers.  T <= the SM count (every CTA
// resident); T == 0 launches one CTA that only signals.
__global__ void __launch_bounds__(route::kCtaWarps * 32) k_ep_front_p2p(
    const uint4* __restrict__ h, const uint4* __restrict__ wg, int T, int H, int E, int W,
    int k, int El, int G, int rank, int cap, int vpr, const uint64_t* __restrict__ peer_recv,
    const uint64_t* __restrict__ peer_flags, int32_t* seq, int32_t* done, int32_t* bar,
    float* weights, int64_t* indices, int32_t* __restrict__ pair_slot_ep, int32_t* zero,
    int nzero, uint64_t wait_ns) {
  __shared__ route::FF s_part[route::kCtaWarps];
  __shared__ int s_total[kEpMaxExperts], s_before[kEpMaxExperts], s_off[kEpMaxExperts + 1];
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  // The expert stage's completion counters (zeroed here, after the wait: their
  // previous user finished before the predecessor did).
  if (t == 0)
    for (int i = threadIdx.x; i < nzero; i += blockDim.x) zero[i] = 0;
  if (t < T) route::route_token_cta(h, wg, t, H, E, W, k, nullptr, weights, indices, s_part);
  if (threadIdx.x < E) {
    s_total[threadIdx.x] = 0;
    s_before[threadIdx.x] = 0;
  }
  if (!grid_meet(bar, gridDim.x, wait_ns)) return;  // the peers' waits run out too (bounded)
  // Every token's experts, written by the other CTAs above (read through L2).
  const int P = T * k;
  const long long* idx = reinterpret_cast<const long long*>(indices);
  for (int p = threadIdx.x; p < P; p += blockDim.x) {
    const long long e = __ldcg(idx + p);
    if (e >= 0 && e < E) {
      atomicAdd(&s_total[e], 1);
      if (p < t * k) atomicAdd(&s_before[e], 1);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int e = 0; e < E; ++e) {
      s_off[e] = acc;
      acc += s_total[e];
    }
    s_off[E] = acc;
  }
  __syncthreads();
  const int64_t chunk = (int64_t)(cap + 1) * vpr;  // one source's chunk in a receive region
  if (t == 0 && threadIdx.x < E) {  // header row of the chunk for rank r: r's expert counts
    const int r = threadIdx.x / El, j = threadIdx.x - r * El;
    uint4* dst = reinterpret_cast<uint4*>(peer_recv[r]) + rank * chunk + (int64_t)cap * vpr;
    reinterpret_cast<int32_t*>(dst)[j] = s_total[threadIdx.x];
  }
  if (t < T) {
    // Pair (t, j) of expert e sits at s_off[e] + s_before[e] in the sorted
    // order (a token's k experts are distinct); rank r = e / El receives it at
    // row i of this rank's chunk.
    if (threadIdx.x < k) {
      const long long e = __ldcg(idx + (int64_t)t * k + threadIdx.x);
      int32_t slot = -1;
      if (e >= 0 && e < E) {
        const int r = static_cast<int>(e) / El;
        slot = r * cap + (s_off[e] + s_before[e] - s_off[r * El]);
      }
      pair_slot_ep[(int64_t)t * k + threadIdx.x] = slot;
    }
    for (int v = threadIdx.x; v < k * vpr; v += blockDim.x) {
      const int j = v / vpr, c = v - j * vpr;
      const long long e = __ldcg(idx + (int64_t)t * k + j);
      if (e < 0 || e >= E) continue;
      const int r = static_cast<int>(e) / El;
      const int i = s_off[e] + s_before[e] - s_off[r * El];
      if (i >= cap) continue;
      uint4* dst = reinterpret_cast<uint4*>(peer_recv[r]) + rank * chunk + (int64_t)i * vpr;
      dst[c] = h[(int64_t)t * vpr + c];
    }
  }
  signal_peers(peer_flags, G, rank, seq, done);
}

// Owner side of the return: y rows of source s go to s's return region, chunk
// `rank`, at the row the source's combine expects (pair_slot_ep layout).
__global__ void __launch_bounds__(kEpThreads) k_ep_return_p2p(
    const uint4* __restrict__ y_sorted, const int32_t* __restrict__ counts, int El, int G,
    int rank, int cap, int vpr, const uint64_t* __restrict__ peer_back,
    const uint64_t* __restrict__ peer_flags, int32_t* seq, int32_t* done) {
  __shared__ RecvPlan pl;
  pdl_trigger();
  pdl_wait();
  build_plan(counts, El, El, G, cap, pl);
  const int64_t total = (int64_t)G * cap * vpr;
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < total;
       v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = v / vpr;
    const int c = static_cast<int>(v - row * vpr);
    const int s = static_cast<int>(row / cap), i = static_cast<int>(row - (int64_t)s * cap);
    const int64_t src = recv_dst(pl, El, s, i);
    if (src < 0 || src >= (int64_t)G * cap) continue;
    uint4* dst = reinterpret_cast<uint4*>(peer_back[s]) + ((int64_t)rank * cap + i) * vpr;
    dst[c] = y_sorted[src * vpr + c];
  }
  signal_peers(peer_flags, G, rank, seq, done);
}

// k_ep_return_p2p from the expert stage's fp32 split partials ([row][S][H]):
// each value is the in-order sum over the S splits rounded once to fp16, the
// arithmetic of the partials reduce that moe_experts_forward ends with, so the
// rows stored into the peers are the same bits.
__global__ void __launch_bounds__(kEpThreads) k_ep_return_partials_p2p(
    const float* __restrict__ part, int S, const int32_t* __restrict__ counts, int El, int G,
    int rank, int cap, int vpr, const uint64_t* __restrict__ peer_back,
    const uint64_t* __restrict__ peer_flags, int32_t* seq, int32_t* done) {
  __shared__ RecvPlan pl;
  pdl_trigger();
  pdl_wait();
  build_plan(counts, El, El, G, cap, pl);
  const int64_t total = (int64_t)G * cap * vpr;
  const int64_t width = (int64_t)vpr * 8;
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < total;
       v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = v / vpr;
    const int c = static_cast<int>(v - row * vpr);
    const int s = static_cast<int>(row / cap), i = static_cast<int>(row - (int64_t)s * cap);
    const int64_t src = recv_dst(pl, El, s, i);
    if (src < 0 || src >= (int64_t)G * cap) continue;
    const float4* p = reinterpret_cast<const float4*>(part + src * S * width + (int64_t)c * 8);
    float4 a = __ldcs(p), b = __ldcs(p + 1);
    for (int k = 1; k < S; ++k) {
      const float4 x = __ldcs(p + k * (width / 4)), y = __ldcs(p + k * (width / 4) + 1);
      a.x = __fadd_rn(a.x, x.x); a.y = __fadd_rn(a.y, x.y);
      a.z = __fadd_rn(a.z, x.z); a.w = __fadd_rn(a.w, x.w);
      b.x = __fadd_rn(b.x, y.x); b.y = __fadd_rn(b.y, y.y);
      b.z = __fadd_rn(b.z, y.z); b.w = __fadd_rn(b.w, y.w);
    }
    uint4 o;
    o.x = (uint32_t)f2h(a.x) | ((uint32_t)f2h(a.y) << 16);
    o.y = (uint32_t)f2h(a.z) | ((uint32_t)f2h(a.w) << 16);
    o.z = (uint32_t)f2h(b.x) | ((uint32_t)f2h(b.y) << 16);
    o.w = (uint32_t)f2h(b.z) | ((uint32_t)f2h(b.w) << 16);
    uint4* dst = reinterpret_cast<uint4*>(peer_back[s]) + ((int64_t)rank * cap + i) * vpr;
    dst[c] = o;
  }
  signal_peers(peer_flags, G, rank, seq, done);
}

// Bounded wait until every source's flag reaches this rank's sequence number.
__global__ void k_ep_wait(const int32_t* flags, int G, const int32_t* seq, uint64_t limit_ns) {
  pdl_trigger();
  pdl_wait();
  const int s = threadIdx.x;
  if (s < G && !wait_peer_flag(flags, s, seq, limit_ns)) set_device_error(kErrWaitTimeout);
}

// The header row must hold E/G int32 counts: hidden * 2 >= 4 * E / G.
bool ep_args_ok(int E, int G, int cap, int hidden) {
  return G >= 1 && E >= G && E <= kEpMaxExperts && E % G == 0 && cap >= 1 && hidden > 0 &&
         hidden % 8 == 0 && hidden * 2 >= 4 * (E / G);
}

}  // namespace
}  // namespace moe

extern "C" int moe_ep_dispatch(const uint16_t* h, const int32_t* expert_offsets,
                               const int32_t* pair_token, const int32_t* pair_slot, int64_t T,
                               int k, int E, int G, int cap, int hidden, uint16_t* send_rows,
                               int32_t* send_counts, int32_t* pair_slot_ep, void* stream) {
  using namespace moe;
  if (T < 0 || k < 1 || !ep_args_ok(E, G, cap, hidden)) return MOE_ERR_INVALID_ARG;
  const int El = E / G;
  if (T * (k < El ? k : El) > cap) return MOE_ERR_INVALID_ARG;
  if (!expert_offsets || !send_rows) return MOE_ERR_INVALID_ARG;
  if (T > 0 && (!h || !pair_token || !pair_slot || !pair_slot_ep)) return MOE_ERR_INVALID_ARG;
  if ((T > 0 && !aligned16(h)) || !aligned16(send_rows)) return MOE_ERR_ALIGNMENT;
  const int vpr = hidden / 8;
  if (launch_pdl(k_ep_dispatch, grid_rows((int64_t)G * cap * vpr), kEpThreads, 0,
                 static_cast<cudaStream_t>(stream), reinterpret_cast<const uint4*>(h),
                 expert_offsets, pair_token, pair_slot, T * k, E, El, G, cap, vpr,
                 reinterpret_cast<uint4*>(send_rows), send_counts, pair_slot_ep) != cudaSuccess)
    return MOE_ERR_CUDA;
  MOE_CHECK_LAUNCH();
  return MOE_OK;
}

namespace moe {
namespace {
int ep_receive(const uint16_t* recv_rows, int32_t* recv_counts, int E, int G, int cap, int hidden,
               uint16_t* x_sorted, int32_t* local_offsets, const int32_t* flags,
               const int32_t* seq, void* stream) {
  if (!ep_args_ok(E, G, cap, hidden)) return MOE_ERR_INVALID_ARG;
  if (!recv_rows || !recv_counts || !x_sorted || !local_offsets) return MOE_ERR_INVALID_ARG;
  if (!aligned16(recv_rows) || !aligned16(x_sorted)) return MOE_ERR_ALIGNMENT;
  const int vpr = hidden / 8;
  if (launch_pdl(k_ep_move<true>, grid_rows((int64_t)G * cap * vpr), kEpThreads, 0,
                 static_cast<cudaStream_t>(stream), reinterpret_cast<const uint4*>(recv_rows),
                 recv_counts, E / G, G, cap, vpr, reinterpret_cast<uint4*>(x_sorted),
                 local_offsets, flags, seq, wait_limit_ns()) != cudaSuccess)
    return MOE_ERR_CUDA;
  MOE_CHECK_LAUNCH();
  return MOE_OK;
}
}  // namespace
}  // namespace moe

extern "C" int moe_ep_receive(const uint16_t* recv_rows, int32_t* recv_counts, int E, int G,
                              int cap, int hidden, uint16_t* x_sorted, int32_t* local_offsets,
                              void* stream) {
  return moe::ep_receive(recv_rows, recv_counts, E, G, cap, hidden, x_sorted, local_offsets,
                         nullptr, nullptr, stream);
}

extern "C" int moe_ep_receive_p2p(const uint16_t* recv_rows, int32_t* recv_counts, int E, int G,
                                  int cap, int hidden, uint16_t* x_sorted,
                                  int32_t* local_offsets, const int32_t* flags,
                                  const int32_t* seq, void* stream) {
  if (!flags || !seq) return MOE_ERR_INVALID_ARG;
  return moe::ep_receive(recv_rows, recv_counts, E, G, cap, hidden, x_sorted, local_offsets,
                         flags, seq, stream);
}

extern "C" int moe_ep_return(const uint16_t* y_sorted, const int32_t* recv_counts, int E, int G,
                             int cap, int hidden, uint16_t* y_back, void* stream) {
  using namespace moe;
  if (!ep_args_ok(E, G, cap, hidden)) return MOE_ERR_INVALID_ARG;
  if (!y_sorted || !recv_counts || !y_back) return MOE_ERR_INVALID_ARG;
  if (!aligned16(y_sorted) || !aligned16(y_back)) return MOE_ERR_ALIGNMENT;
  const int vpr = hidden / 8;
  if (launch_pdl(k_ep_move<false>, grid_rows((int64_t)G * cap * vpr), kEpThreads, 0,
                 static_cast<cudaStream_t>(stream), reinterpret_cast<const uint4*>(y_sorted),
                 const_cast<int32_t*>(recv_counts), E / G, G, cap, vpr,
                 reinterpret_cast<uint4*>(y_back), static_cast<int32_t*>(nullptr),
                 static_cast<const int32_t*>(nullptr), static_cast<const int32_t*>(nullptr),
                 uint64_t{0}) != cudaSuccess)
    return MOE_ERR_CUDA;
  MOE_CHECK_LAUNCH();
  return MOE_OK;
}

extern "C" int moe_ep_dispatch_p2p(const uint16_t* h, const int32_t* expert_offsets,
                                   const int32_t* pair_token, const int32_t* pair_slot, int64_t T,
                                   int k, int E, int G, int rank, int cap, int hidden,
                                   const uint64_t* peer_recv, const uint64_t* peer_flags,
                                   int32_t* seq, int32_t* done, int32_t* pair_slot_ep,
                                   void* stream) {
  using namespace moe;
  if (T < 0 || k < 1 || !ep_args_ok(E, G, cap, hidden) || rank < 0 || rank >= G)
    return MOE_ERR_INVALID_ARG;
  const int El = E / G;
  if (T * (k < El ? k : El) > cap) return MOE_ERR_INVALID_ARG;
  if (!expert_offsets || !peer_recv || !peer_flags || !seq || !done) return MOE_ERR_INVALID_ARG;
  if (T > 0 && (!h || !pair_token || !pair_slot || !pair_slot_ep)) return MOE_ERR_INVALID_ARG;
  if (T > 0 && !aligned16(h)) return MOE_ERR_ALIGNMENT;
  const int vpr = hidden / 8;
  if (launch_pdl(k_ep_dispatch_p2p, grid_rows((int64_t)G * cap * vpr), kEpThreads, 0,
                 static_cast<cudaStream_t>(stream), reinterpret_cast<const uint4*>(h),
                 expert_offsets, pair_token, pair_slot, T * k, E, El, G, rank, cap, vpr,
                 peer_recv, peer_flags, seq, done, pair_slot_ep) != cudaSuccess)
    return MOE_ERR_CUDA;
  MOE_CHECK_LAUNCH();
  return MOE_OK;
}

extern "C" int moe_ep_front_p2p(const uint16_t* h, const uint16_t* wg, int64_t T, int E, int k,
                                int G, int rank, int cap, int hidden, const uint64_t* peer_recv,
                                const uint64_t* peer_flags, int32_t* seq, int32_t* done,
                                int32_t* bar, float* weights, int64_t* indices,
                                int32_t* pair_slot_ep, int32_t* zero_words, int n_zero,
                                void* stream) {
  using namespace moe;
  if (T < 0 || k < 1 || k > 8 || k > E || !ep_args_ok(E, G, cap, hidden) || rank < 0 ||
      rank >= G)
    return MOE_ERR_INVALID_ARG;
  const int El = E / G;
  if (T * (k < El ? k : El) > cap) return MOE_ERR_INVALID_ARG;
  if (T > sm_count()) return MOE_ERR_UNSUPPORTED;  // every CTA must be resident
  if (!peer_recv || !peer_flags || !seq || !done || !bar) return MOE_ERR_INVALID_ARG;
  if (n_zero < 0 || (n_zero > 0 && !zero_words)) return MOE_ERR_INVALID_ARG;
  if (T > 0 && (!h || !wg || !weights || !indices || !pair_slot_ep)) return MOE_ERR_INVALID_ARG;
  if (T > 0 && (!aligned16(h) || !aligned16(wg))) return MOE_ERR_ALIGNMENT;
  int W = 1;
  while (W < E) W <<= 1;
  const int grid = T > 0 ? static_cast<int>(T) : 1;
  if (launch_pdl(k_ep_front_p2p, grid, route::kCtaWarps * 32, 0,
                 static_cast<cudaStream_t>(stream), reinterpret_cast<const uint4*>(h),
                 reinterpret_cast<const uint4*>(wg), static_cast<int>(T), hidden, E, W, k, El, G,
                 rank, cap, hidden / 8, peer_recv, peer_flags, seq, done, bar, weights, indices,
                 pair_slot_ep, zero_words, n_zero, wait_limit_ns()) != cudaSuccess)
    return MOE_ERR_CUDA;
  MOE_CHECK_LAUNCH();
  return MOE_OK;
}

extern "C" int moe_ep_return_p2p(const uint16_t* y_sorted, const int32_t* recv_counts, int E,
                                 int G, int rank, int cap, int hidden, const uint64_t* peer_back,
                                 const uint64_t* peer_flags, int32_t* seq, int32_t* done,
                                 void* stream) {
  using namespace moe;
  if (!ep_args_ok(E, G, cap, hidden) || rank < 0 || rank >= G) return MOE_ERR_INVALID_ARG;
  if (!y_sorted || !recv_counts || !peer_back || !peer_flags || !seq || !done)
    return MOE_ERR_INVALID_ARG;
  if (!aligned16(y_sorted)) return MOE_ERR_ALIGNMENT;
  const int vpr = hidden / 8;
  if (launch_pdl(k_ep_return_p2p, grid_rows((int64_t)G * cap * vpr), kEpThreads, 0,
                 static_cast<cudaStream_t>(stream), reinterpret_cast<const uint4*>(y_sorted),
                 recv_counts, E / G, G, rank, cap, vpr, peer_back, peer_flags, seq,
                 done) != cudaSuccess)
    return MOE_ERR_CUDA;
  MOE_CHECK_LAUNCH();
  return MOE_OK;
}

extern "C" int moe_ep_return_partials_p2p(const float* y_part, int S, const int32_t* recv_counts,
                                          int E, int G, int rank, int cap, int hidden,
                                          const uint64_t* peer_back, const uint64_t* peer_flags,
                                          int32_t* seq, int32_t* done, void* stream) {
  using namespace moe;
  if (S < 1 || !ep_args_ok(E, G, cap, hidden) || rank < 0 || rank >= G)
    return MOE_ERR_INVALID_ARG;
  if (!y_part || !recv_counts || !peer_back || !peer_flags || !seq || !done)
    return MOE_ERR_INVALID_ARG;
  if (!aligned16(y_part)) return MOE_ERR_ALIGNMENT;
  const int vpr = hidden / 8;
  if (launch_pdl(k_ep_return_partials_p2p, grid_rows((int64_t)G * cap * vpr), kEpThreads, 0,
                 static_cast<cudaStream_t>(stream), y_part, S, recv_counts, E / G, G, rank, cap,
                 vpr, peer_back, peer_flags, seq, done) != cudaSuccess)
    return MOE_ERR_CUDA;
  MOE_CHECK_LAUNCH();
  return MOE_OK;
}

extern "C" int moe_ep_wait_p2p(const int32_t* flags, int G, const int32_t* seq, void* stream) {
  using namespace moe;
  if (!flags || !seq || G < 1 || G > kEpMaxExperts) return MOE_ERR_INVALID_ARG;
  if (launch_pdl(k_ep_wait, 1, 32, 0, static_cast<cudaStream_t>(stream), flags, G, seq,
                 wait_limit_ns()) != cudaSuccess)
    return MOE_ERR_CUDA;
  MOE_CHECK_LAUNCH();
  return MOE_OK;
}

