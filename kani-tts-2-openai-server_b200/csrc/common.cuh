// Shared device helpers for the KaniTTS decode-path kernels (sm_100a).
//
// Every kernel in this library streams rows of bf16 / fp16 / fp32 data through
// 128-bit global loads and stores, does its arithmetic in fp32 and rounds once
// (round-to-nearest-even) to the storage type.  These helpers hold the 16-byte
// vector <-> fp32 conversions and the cache-hinted memory operations.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <utility>

#include "kani_b200.h"

namespace kani {

// ---------------------------------------------------------------- elements

template <typename T> struct Elem;

template <> struct Elem<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};

template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};

// Round an fp32 value to T and back (models the store/reload of an
// intermediate tensor of type T).
template <typename T>
__device__ __forceinline__ float round_to(float v) {
  return Elem<T>::to_f(Elem<T>::from_f(v));
}

// ------------------------------------------------------- 16-byte vectors

// Number of T elements in one 16-byte vector.
template <typename T> struct VecN { static constexpr int value = 16 / (int)sizeof(T); };

// Unpack 16 bytes holding VecN<T> elements into fp32.
template <typename T>
__device__ __forceinline__ void unpack16(const uint4& raw, float* f);

template <>
__device__ __forceinline__ void unpack16<float>(const uint4& raw, float* f) {
  f[0] = __uint_as_float(raw.x); f[1] = __uint_as_float(raw.y);
  f[2] = __uint_as_float(raw.z); f[3] = __uint_as_float(raw.w);
}

template <>
__device__ __forceinline__ void unpack16<__nv_bfloat16>(const uint4& raw, float* f) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    // bf16 -> fp32 is exact: the bf16 bits are the high half of the fp32.
    f[2 * i + 0] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

template <>
__device__ __forceinline__ void unpack16<__half>(const uint4& raw, float* f) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h2 = *reinterpret_cast<const __half2*>(&w[i]);
    float2 p = __half22float2(h2);
    f[2 * i + 0] = p.x;
    f[2 * i + 1] = p.y;
  }
}

// Pack VecN<T> fp32 values into 16 bytes of T (one RNE rounding each).
template <typename T>
__device__ __forceinline__ uint4 pack16(const float* f);

template <>
__device__ __forceinline__ uint4 pack16<float>(const float* f) {
  return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]),
                    __float_as_uint(f[2]), __float_as_uint(f[3]));
}

template <>
__device__ __forceinline__ uint4 pack16<__nv_bfloat16>(const float* f) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 b = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&b);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

template <>
__device__ __forceinline__ uint4 pack16<__half>(const float* f) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// ------------------------------------------------------ memory operations

// Plain coherent 128-bit load (safe when the same kernel later overwrites
// the location in place).
__device__ __forceinline__ uint4 ld16(const void* p) {
  return *reinterpret_cast<const uint4*>(p);
}

// Streaming 128-bit load for data read exactly once (evict-first in L1/L2).
__device__ __forceinline__ uint4 ld16_stream(const void* p) {
  return __ldcs(reinterpret_cast<const uint4*>(p));
}

// Read-only 128-bit load through the non-coherent path, for small tables
// (norm weights, frame table) that many threads re-read.
__device__ __forceinline__ uint4 ld16_ro(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

__device__ __forceinline__ void st16(void* p, const uint4& v) {
  *reinterpret_cast<uint4*>(p) = v;
}

// Load E weights of type W starting at element `off` and convert to fp32.
// E is the element count of one 16-byte vector of the row type, so the load
// is 8, 16 or 32 bytes wide; the caller guarantees matching alignment.
template <typename W, int E>
__device__ __forceinline__ void load_weights(const W* w, int64_t off, float* out) {
  constexpr int BYTES = E * (int)sizeof(W);
  static_assert(BYTES == 8 || BYTES == 16 || BYTES == 32, "weight vector width");
  const char* p = reinterpret_cast<const char*>(w + off);
  if constexpr (BYTES == 16) {
    uint4 raw = ld16_ro(p);
    unpack16<W>(raw, out);
  } else if constexpr (BYTES == 32) {
    uint4 a = ld16_ro(p), b = ld16_ro(p + 16);
    unpack16<W>(a, out);
    unpack16<W>(b, out + VecN<W>::value);
  } else {  // 8 bytes: E = 4 elements of a 2-byte type
    uint2 raw = __ldg(reinterpret_cast<const uint2*>(p));
    uint4 wide = make_uint4(raw.x, raw.y, 0u, 0u);
    float tmp[8];
    unpack16<W>(wide, tmp);
#pragma unroll
    for (int i = 0; i < 4; ++i) out[i] = tmp[i];
  }
}

// (g * sigmoid(g)) * u in fp32, the activation of the SwiGLU MLP (shared by the
// SiLU kernel and the GEMV epilogue so both round identically).  sigmoid from
// t = e^-|g| in (0, 1]: g / (1 + e^-g) is 1/(1+t) for g >= 0 and t/(1+t) for
// g < 0, so the divisor stays in [1, 2], where the fast divide is accurate.
// Below |g| ~ 87 the fast exponential flushes to zero while e^g is still
// representable, so that (rare) case takes the full-range expf.
__device__ __forceinline__ float silu_mul_f(float g, float u) {
  const float t = __expf(-fabsf(g));
  float sig = __fdividef(g >= 0.f ? 1.0f : t, 1.0f + t);
  if (t == 0.f && g < 0.f) sig = expf(g);
  return __fmul_rn(__fmul_rn(g, sig), u);
}

// ---------------------------------------------------------------- misc

__host__ __device__ __forceinline__ bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// Host-side launch accounting (number of kernels this library launched).
void note_launch();

// Streaming multiprocessors of the current device (queried once per device).
int sm_count();

// Bound of a kernel's on-chip waits (TMA mbarrier phases): clock64 cycles
// before the wait gives up and sets KANI_FLAG_TIMEOUT, and the suspend-time
// hint (ns) of each mbarrier.try_wait.  By default about 1 s with a 1 ms
// hint; kani_set_wait_limit(c) makes later launches give up after c cycles
// with no suspension, so a test can make a real wait run out while its copies
// still land.  Only a kernel's first wait on a stage takes the limit; the
// drain of copies still in flight keeps the default bound.
struct WaitBound {
  long long cycles;
  unsigned suspend_ns;
};
constexpr unsigned kWaitSuspendNs = 1000000u;
WaitBound wait_bound(long long default_cycles);

// Device ranges a decode launch prefetches into L2 as it starts: the weights
// of later launches, which do not depend on any earlier launch.  Set from the
// host with kani_set_l2_prefetch and taken (and cleared) by the next decode
// GEMV / head / reduce + add + RMSNorm / SiLU·mul entry point called on the
// same host thread.
struct L2Prefetch {
  const void* ptr[2];
  long long bytes[2];
};
L2Prefetch take_l2_prefetch();

// Thread 0 of each CTA issues its even share of the ranges (16-byte units,
// pieces of at most 64 KB) as cp.async.bulk.prefetch.L2: no data comes back
// to the SM, nothing waits on it, and it reads only memory that no launch
// writes, so it may run before griddepcontrol.wait.
__device__ __forceinline__ void l2_prefetch_share(const L2Prefetch& pf) {
  if (threadIdx.x != 0 || threadIdx.y != 0 || threadIdx.z != 0) return;
  const long long ncta = (long long)gridDim.x * gridDim.y * gridDim.z;
  const long long cta = blockIdx.x + (long long)gridDim.x * (blockIdx.y + (long long)gridDim.y * blockIdx.z);
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const long long units = pf.bytes[j] >> 4;
    if (pf.ptr[j] == nullptr || units <= 0) continue;
    const long long per = (units + ncta - 1) / ncta;
    const long long u0 = per * cta, u1 = u0 + per < units ? u0 + per : units;
    for (long long u = u0; u < u1; u += 4096) {
      const unsigned n = (unsigned)((u1 - u < 4096 ? u1 - u : 4096) * 16);
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(static_cast<const char*>(pf.ptr[j]) + u * 16),
                   "r"(n)
                   : "memory");
    }
  }
}

// Dispatch a runtime dtype code to a C++ type and invoke f.template
// operator()<T>().  Returns KANI_ERR_DTYPE for unknown codes.
template <typename F>
int dispatch_dtype(int32_t code, F&& f) {
  switch (code) {
    case KANI_DTYPE_F32: return f.template operator()<float>();
    case KANI_DTYPE_BF16: return f.template operator()<__nv_bfloat16>();
    case KANI_DTYPE_F16: return f.template operator()<__half>();
    default: return KANI_ERR_DTYPE;
  }
}

// Programmatic dependent launch.  A kernel launched with launch_pdl may start
// while the kernel before it in the stream is still finishing; it must call
// griddep_wait() before it touches global memory that kernel may have
// written (the wait returns once the earlier grid has completed and its
// writes are visible).  griddep_launch_dependents() lets the next launch's
// blocks be scheduled before this grid ends.  Both are no-ops when there is
// no programmatic dependency.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       Args&&... args) {
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
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// launch_pdl when `pdl`, else a plain launch of the same kernel.  The
// activation kernels between the decode step's GEMMs (add + RMSNorm, SiLU·mul,
// short conv, token RoPE) launch as programmatic dependents up to
// kPdlMaxRows rows: at 16 streams that measured 673 -> 657 us per step, while
// at 64 streams behind cuBLAS GEMMs the full bench measured 662-669 -> 678 us.
// Their kernels call griddep_wait() before any memory access either way.
constexpr int64_t kPdlMaxRows = 32;

template <typename... KArgs, typename... Args>
cudaError_t launch_maybe_pdl(bool pdl, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                             Args&&... args) {
  if (pdl) return launch_pdl(kern, grid, block, smem, s, std::forward<Args>(args)...);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  note_launch();
  return e == cudaSuccess ? KANI_OK : (int)e;
}

}  // namespace kani
