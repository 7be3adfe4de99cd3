// Library-wide entry points of the C ABI: version, status text and the
// launch counter.  The op entry points live beside their kernels
// (rms_norm.cu, silu_mul.cu, rope_kv.cu).
#include <atomic>

#include "common.cuh"

namespace kani {
namespace {
std::atomic<uint64_t> g_launches{0};
}  // namespace

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

}  // namespace kani

extern "C" int kani_version(void) { return 100; }

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
