// Status strings, build identification, the launch counter, per-device host
// state and the device error words of the C ABI.
#include <atomic>
#include <map>
#include <mutex>
#include <utility>
#include <vector>

#include "common.cuh"

namespace moe {
namespace {
std::atomic<unsigned long long> g_launches{0};
std::atomic<uint64_t> g_wait_limit{2000000000ull};  // 2 s

std::mutex& state_mu() {
  static std::mutex mu;
  return mu;
}
std::vector<int (*)(int*)>& error_readers() {
  static std::vector<int (*)(int*)> readers;
  return readers;
}
}  // namespace

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

uint64_t wait_limit_ns() { return g_wait_limit.load(std::memory_order_relaxed); }

void register_error_reader(int (*reader)(int*)) {
  std::lock_guard<std::mutex> lock(state_mu());
  error_readers().push_back(reader);
}

int current_device() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -1;
  return dev;
}

int sm_count() {
  static std::atomic<int> counts[kMaxDevices] = {};
  const int dev = current_device();
  if (dev < 0) return 148;
  int n = counts[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    counts[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

bool once_per_device(const void* key, bool (*setup)()) {
  static std::map<std::pair<const void*, int>, bool> done;
  const int dev = current_device();
  if (dev < 0) return false;
  std::lock_guard<std::mutex> lock(state_mu());
  auto it = done.find({key, dev});
  if (it != done.end()) return it->second;
  const bool ok = setup();
  done[{key, dev}] = ok;
  return ok;
}

MOE_DEFINE_ERROR_WORD()

namespace {
// One bounded wait on a device flag: the same wait the layer kernels use
// between CTAs, exposed so its timeout path can be exercised without a fault.
__global__ void k_probe_wait(const int* flag, int target, uint64_t limit_ns, int* waited_ns) {
  const uint64_t t0 = globaltimer_ns();
  int v;
  for (;;) {
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if (v >= target) break;
    if (globaltimer_ns() - t0 > limit_ns) {
      set_device_error(kErrWaitTimeout);
      break;
    }
    __nanosleep(1000);
  }
  if (waited_ns) {
    const uint64_t dt = globaltimer_ns() - t0;
    *waited_ns = dt > 0x7fffffffull ? 0x7fffffff : static_cast<int>(dt);
  }
}
}  // namespace
}  // namespace moe

extern "C" uint64_t moe_launch_count(void) {
  return moe::g_launches.load(std::memory_order_relaxed);
}

extern "C" const char* moe_status_string(int status) {
  switch (status) {
    case MOE_OK: return "ok";
    case MOE_ERR_INVALID_ARG: return "invalid argument";
    case MOE_ERR_UNSUPPORTED: return "unsupported shape or configuration";
    case MOE_ERR_CUDA: return "CUDA launch or runtime error";
    case MOE_ERR_WORKSPACE: return "workspace missing or too small";
    case MOE_ERR_ALIGNMENT: return "pointer not 16-byte aligned";
    case MOE_ERR_TIMEOUT: return "device wait timed out";
    case MOE_ERR_CODEBOOK: return "experts of one launch carry different NF4 codebooks";
    default: return "unknown status";
  }
}

extern "C" const char* moe_version(void) { return "moe_b200 sm_100a 0.2"; }

extern "C" int moe_take_device_error(int* value) {
  if (!value) return MOE_ERR_INVALID_ARG;
  std::vector<int (*)(int*)> readers;
  {
    std::lock_guard<std::mutex> lock(moe::state_mu());
    readers = moe::error_readers();
  }
  int all = 0;
  for (auto* r : readers) {
    int v = 0;
    if (r(&v) != 0) return MOE_ERR_CUDA;
    all |= v;
  }
  *value = all;
  return MOE_OK;
}

extern "C" int moe_set_wait_limit_ns(uint64_t ns) {
  if (ns < 1000 || ns > 60ull * 1000000000ull) return MOE_ERR_INVALID_ARG;
  moe::g_wait_limit.store(ns, std::memory_order_relaxed);
  return MOE_OK;
}

extern "C" uint64_t moe_wait_limit_ns(void) { return moe::wait_limit_ns(); }

extern "C" int moe_stream_check(void* stream) {
  if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess) return MOE_ERR_CUDA;
  int v = 0;
  const int st = moe_take_device_error(&v);
  if (st != MOE_OK) return st;
  if (v & moe::kErrWaitTimeout) return MOE_ERR_TIMEOUT;
  if (v & moe::kErrCodebook) return MOE_ERR_CODEBOOK;
  if (v & moe::kErrSmemLayout) return MOE_ERR_CUDA;
  return MOE_OK;
}

extern "C" int moe_probe_wait(const int* flag, int target, int* waited_ns, void* stream) {
  if (!flag) return MOE_ERR_INVALID_ARG;
  moe::k_probe_wait<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(flag, target,
                                                                      moe::wait_limit_ns(),
                                                                      waited_ns);
  MOE_CHECK_LAUNCH();
  return MOE_OK;
}
