// Shared device/host helpers for the B200 MoE kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/moe_b200.h"

// Every kernel launch of the library is followed by this check; it also counts
// the launch (moe_launch_count), host side, so a CUDA-graph capture of a step
// reports how many kernels one replay runs.
#define MOE_CHECK_LAUNCH()                                   \
  do {                                                       \
    cudaError_t _e = cudaGetLastError();                     \
    if (_e != cudaSuccess) return MOE_ERR_CUDA;              \
    ::moe::note_launch();                                    \
  } while (0)

namespace moe {
void note_launch();

// Programmatic dependent launch.  Kernels of one decode layer (router,
// permute, expert GEMVs, combine) are launched with programmatic stream
// serialization: a kernel may start while its predecessor still runs, so its
// prologue (e.g. the decode table) overlaps the predecessor's tail.  Each such
// kernel lets its successor launch (pdl_trigger) and, before it reads anything
// an earlier kernel wrote -- and before it can finish -- waits for its
// predecessor to complete (pdl_wait; a no-op when launched normally).
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

constexpr int kWarp = 32;

// Expert descriptors passed by value as a kernel parameter.
struct ExpertTable {
  moe_nf4_expert_t e[MOE_MAX_EXPERTS];
};

__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Host-side state kept per CUDA device (the current device of the calling
// thread): SM count, one-time kernel attribute setup.  A process may drive
// several GPUs, so none of it is a process-wide single value.
constexpr int kMaxDevices = 64;
int current_device();  // cudaGetDevice(), or -1 on error / out of range
int sm_count();        // SMs of the current device (148 if it cannot be queried)
// Runs setup() once per (key, device) and remembers whether it succeeded.
bool once_per_device(const void* key, bool (*setup)());

// Bounded device waits.  Every spin (cross-CTA counters, mbarrier phases)
// gives up after the limit in nanoseconds of %globaltimer, sets a bit of the
// device error word and lets the kernel finish; the limit rides in each
// kernel's arguments (moe_set_wait_limit_ns) so a graph replays the value
// captured with it.
uint64_t wait_limit_ns();
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait of thread `s` until peer flag s reaches this rank's sequence
// number *seq (release-stored by the peer at system scope; read with
// acquire).  false once limit_ns of %globaltimer ran out.
__device__ __forceinline__ bool wait_peer_flag(const int32_t* flags, int s, const int32_t* seq,
                                               uint64_t limit_ns) {
  const int target = *reinterpret_cast<const volatile int32_t*>(seq);
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(flags + s) : "memory");
  if (v >= target) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    __nanosleep(64);  // short: the wait sits on the layer's critical path
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(flags + s) : "memory");
    if (v >= target) return true;
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
}
// Device error word bits (read and cleared by moe_take_device_error).
constexpr int kErrWaitTimeout = 1;    // a bounded wait ran out
constexpr int kErrCodebook = 2;       // experts of one launch carry different codebooks
constexpr int kErrSmemLayout = 4;     // shared-memory layout not as planned (launch skipped)

// Each translation unit whose kernels report errors owns one device word
// (device code is compiled per file, without relocatable linking, so a word
// cannot be shared across files); its host-side reader registers itself with
// moe_take_device_error, which ORs every word and clears it.
void register_error_reader(int (*reader)(int*));
#define MOE_DEFINE_ERROR_WORD()                                                          \
  namespace {                                                                            \
  __device__ int g_device_error = 0;                                                     \
  __device__ __forceinline__ void set_device_error(int bits) {                          \
    atomicOr(&g_device_error, bits);                                                     \
  }                                                                                      \
  int read_clear_error(int* value) {                                                     \
    int v = 0;                                                                           \
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return 1; \
    if (v != 0) {                                                                        \
      const int zero = 0;                                                                \
      if (cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)) != cudaSuccess) return 1; \
    }                                                                                    \
    *value = v;                                                                          \
    return 0;                                                                            \
  }                                                                                      \
  const bool g_error_reader_registered = (register_error_reader(&read_clear_error), true); \
  }

// True when the 16 fp32 codebook entries at a and b are equal.
__device__ __forceinline__ bool same_code16(const float* a, const float* b) {
  if (a == b) return true;
  bool same = true;
#pragma unroll
  for (int i = 0; i < 16; ++i) same &= __ldg(a + i) == __ldg(b + i);
  return same;
}

// fp16 <-> float on raw bit patterns.
__device__ __forceinline__ float h2f(uint16_t b) { return __half2float(__ushort_as_half(b)); }
__device__ __forceinline__ uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }

// acc += fp32(a) * fp32(b) for fp16 a, b: the product of two fp16 values is
// exact in fp32, so this is a single rounding of the sum (sm_100 mixed FMA).
__device__ __forceinline__ float fma_f16f16_f32(uint16_t a, uint16_t b, float acc) {
  float d;
  asm("fma.rn.f32.f16 %0, %1, %2, %3;" : "=f"(d) : "h"(a), "h"(b), "f"(acc));
  return d;
}

// Multirow (GEMM-path) weight: fp16(bf16_rn(code * absmax)), product in fp32.
// Returns the two fp16 weights of one packed byte as a half2 bit pattern
// (low half = element 2j, high half = element 2j+1).
__device__ __forceinline__ uint32_t nf4_pair_multirow(float c_even, float c_odd, float absmax) {
  float p0 = __fmul_rn(c_even, absmax);
  float p1 = __fmul_rn(c_odd, absmax);
  __nv_bfloat162 b = __floats2bfloat162_rn(p0, p1);  // .x = p0, .y = p1
  __half2 h = __floats2half2_rn(__bfloat162float(b.x), __bfloat162float(b.y));
  return *reinterpret_cast<uint32_t*>(&h);
}

// Split a half2 bit pattern into its two fp16 halves.
__device__ __forceinline__ uint16_t lo16(uint32_t v) { return static_cast<uint16_t>(v & 0xFFFFu); }
__device__ __forceinline__ uint16_t hi16(uint32_t v) { return static_cast<uint16_t>(v >> 16); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// torch F.silu on fp16 input: x / (1 + exp(-x)) in fp32, rounded to fp16;
// then (silu(g) * u) in fp32 rounded to fp16 (nf4_reconstruct.py:152-155).
__device__ __forceinline__ uint16_t swiglu_f16(uint16_t g16, uint16_t u16) {
  float g = h2f(g16);
  float s = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
  uint16_t s16 = f2h(s);
  return f2h(__fmul_rn(h2f(s16), h2f(u16)));
}

}  // namespace moe
