// Library-wide entry points of the C ABI: version, status text and the
// launch counter.  The op entry points live beside their kernels
// (rms_norm.cu, silu_mul.cu, rope_kv.cu).
#include <atomic>

#include "common.cuh"

namespace kani {
namespace {
std::atomic<uint64_t> g_launches{0};
std::atomic<long long> g_wait_limit{0};  // 0: the default bound of each kernel
}  // namespace

WaitBound wait_bound(long long default_cycles) {
  const long long c = g_wait_limit.load(std::memory_order_relaxed);
  if (c <= 0) return WaitBound{default_cycles, kWaitSuspendNs};
  return WaitBound{c, 0u};
}

namespace {
thread_local L2Prefetch t_l2_prefetch = {{nullptr, nullptr}, {0, 0}};
}  // namespace

L2Prefetch take_l2_prefetch() {
  const L2Prefetch pf = t_l2_prefetch;
  t_l2_prefetch = L2Prefetch{{nullptr, nullptr}, {0, 0}};
  return pf;
}

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int sm_count() {
  static std::atomic<int> cached[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int n = cached[dev].load(std::memory_order_relaxed);
  if (n > 0) return n;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  cached[dev].store(n, std::memory_order_relaxed);
  return n;
}

}  // namespace kani

extern "C" int kani_version(void) { return 100; }

extern "C" int kani_set_wait_limit(int64_t cycles) {
  if (cycles < 0) return KANI_ERR_INVALID_ARG;
  kani::g_wait_limit.store((long long)cycles, std::memory_order_relaxed);
  return KANI_OK;
}

extern "C" int kani_set_l2_prefetch(const void* ptr0, int64_t bytes0, const void* ptr1, int64_t bytes1) {
  if (bytes0 < 0 || bytes1 < 0 || (bytes0 > 0 && !ptr0) || (bytes1 > 0 && !ptr1)) return KANI_ERR_INVALID_ARG;
  if (bytes0 % 16 || bytes1 % 16 || (ptr0 && !kani::aligned16(ptr0)) || (ptr1 && !kani::aligned16(ptr1)))
    return KANI_ERR_UNSUPPORTED;
  kani::t_l2_prefetch = kani::L2Prefetch{{bytes0 ? ptr0 : nullptr, bytes1 ? ptr1 : nullptr},
                                         {(long long)bytes0, (long long)bytes1}};
  return KANI_OK;
}

extern "C" uint64_t kani_launch_count(void) {
  return kani::g_launches.load(std::memory_order_relaxed);
}

extern "C" const char* kani_status_string(int status) {
  switch (status) {
    case KANI_OK: return "ok";
    case KANI_ERR_INVALID_ARG: return "invalid argument (null pointer, negative size or stride)";
    case KANI_ERR_DTYPE: return "unsupported dtype code";
    case KANI_ERR_UNSUPPORTED: return "shape not supported by the kernels";
    default:
      if (status > 0) return cudaGetErrorString(static_cast<cudaError_t>(status));
      return "unknown status";
  }
}
