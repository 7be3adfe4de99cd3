// Shared pieces of the tensor-core (tcgen05) kernels: shared-memory matrix
// descriptors for the K-major 128-byte-swizzle operand layout, the kind::f16
// instruction descriptor, bounded mbarrier waits, TMA tile loads, tensor-memory
// allocation / loads, and the host-side tensor-map encoder (fetched from the
// driver through the runtime, so the library does not link the driver API).
#pragma once

#include <cuda.h>  // CUtensorMap and its encoder's types

#include <mutex>

#include "common.cuh"

namespace kani {
namespace tc {

constexpr int kM = 128;                       // MMA M: weight rows per CTA
constexpr int kKB = 64;                       // elements per K tile: one 128-byte swizzle row
constexpr uint32_t kATileBytes = kM * kKB * 2;  // one K tile of 128 weight rows
constexpr long long kWaitCycles = 2000000000LL;  // ~1 s

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// UMMA shared-memory descriptor for a K-major 128-byte-swizzle operand: start
// address >> 4, leading offset 1 (unused by this layout), stride offset
// 1024 bytes >> 4 (the next 8-row atom), version 1, layout type 2.  The tile
// base must be 1024-byte aligned; the 16-wide K steps of a tile start 32 bytes
// apart.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3fffu) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
         (2ull << 61);
}

// kind::f16 instruction descriptor: D fp32, A / B bf16 (1) or fp16 (0), both
// K-major, N >> 3 at bit 17, M >> 4 at bit 24.
template <typename T>
__device__ __forceinline__ uint32_t idesc_f16(int m, int n) {
  constexpr uint32_t ab = std::is_same_v<T, __nv_bfloat16> ? 1u : 0u;
  return (1u << 4) | (ab << 7) | (ab << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread
__device__ __forceinline__ void mma_f16(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate ? 1u : 0u)
      : "memory");
}

// arrive on an mbarrier once every MMA this thread issued so far has completed
__device__ __forceinline__ void commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void mbar_init(uint32_t bar) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(1000000u)
      : "memory");
  return ok != 0;
}

// bounded wait for the phase of the given parity; false after ~1 s
__device__ __forceinline__ bool wait(uint32_t bar, uint32_t parity) {
  if (try_wait(bar, parity)) return true;
  const long long start = clock64();
  while (!try_wait(bar, parity)) {
    if (clock64() - start > kWaitCycles) return false;
  }
  return true;
}

// 3-D TMA tile load {elements, row, tile} completing on an mbarrier; the
// innermost coordinate is 0 (16-byte aligned); rows past the tensor read as 0.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int row, int tile, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(row), "r"(tile), "r"(bar)
      : "memory");
}

// 5-D TMA tile load {elements, c1, c2, c3, c4}; innermost coordinate 0
__device__ __forceinline__ void tma_load_5d(uint32_t dst, const CUtensorMap* map, int c1, int c2, int c3, int c4,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5, "
      "%6}], [%7];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// tensor memory: one warp allocates / frees; the address lands in shared memory
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst_smem)),
               "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_free(uint32_t tmem, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(cols) : "memory");
}
__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 16 consecutive fp32 columns of this warp's 32 lanes (one lane each), waited on
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}

// fp32 bits rounded to nearest-even bf16 bits in integer arithmetic: the same
// bits as the hardware conversion (NaN -> the canonical 0x7fff)
__device__ __forceinline__ uint32_t bf16_rne_bits(uint32_t f) {
  if ((f & 0x7fffffffu) > 0x7f800000u) return 0x7fffu;
  return (f + 0x7fffu + ((f >> 16) & 1u)) >> 16;
}

// two fp32 values (as bits) rounded to T: a in the low half, b in the high half
template <typename T>
__device__ __forceinline__ uint32_t round_pair(uint32_t a, uint32_t b);
template <>
__device__ __forceinline__ uint32_t round_pair<__nv_bfloat16>(uint32_t a, uint32_t b) {
  return bf16_rne_bits(a) | (bf16_rne_bits(b) << 16);
}
template <>
__device__ __forceinline__ uint32_t round_pair<__half>(uint32_t a, uint32_t b) {
  const __half2 h = __floats2half2_rn(__uint_as_float(a), __uint_as_float(b));
  uint32_t u;
  memcpy(&u, &h, 4);
  return u;
}

// the fp32 value of 16-bit float bits
template <typename T>
__device__ __forceinline__ float from_bits16(uint32_t b);
template <>
__device__ __forceinline__ float from_bits16<__nv_bfloat16>(uint32_t b) {
  return __uint_as_float(b << 16);
}
template <>
__device__ __forceinline__ float from_bits16<__half>(uint32_t b) {
  return __half2float(__ushort_as_half((unsigned short)b));
}

// ------------------------------------------------------------------ host

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  });
  return fn;
}

// A tiled map of 16-bit elements with 128-byte swizzle, zero fill past the
// edges: dims[0] = 64 elements (128 bytes), strides[i] (bytes) for dims 1..rank-1.
inline bool encode_map(CUtensorMap* map, bool bf16, const void* base, int rank, const cuuint64_t* dims,
                       const cuuint64_t* strides, const cuuint32_t* box) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return false;
  const cuuint32_t estr[5] = {1u, 1u, 1u, 1u, 1u};
  return fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, (cuuint32_t)rank,
            const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Row-major [outer x inner] matrix viewed as {64 elements, outer rows, inner / 64
// tiles} (row stride, tile stride 128 B); box {64, box_rows, pz}.  One TMA load
// then brings pz consecutive 128-byte pieces of each row, which streams faster
// than boxes of single 128-byte rows.
inline bool encode_rows(CUtensorMap* map, bool bf16, const void* base, int64_t inner, int64_t outer,
                        int64_t row_stride, int box_rows, int pz) {
  const cuuint64_t dims[3] = {(cuuint64_t)kKB, (cuuint64_t)outer, (cuuint64_t)(inner / kKB)};
  const cuuint64_t strides[2] = {(cuuint64_t)row_stride * 2u, (cuuint64_t)kKB * 2u};
  const cuuint32_t box[3] = {(cuuint32_t)kKB, (cuuint32_t)box_rows, (cuuint32_t)pz};
  return encode_map(map, bf16, base, 3, dims, strides, box);
}

}  // namespace tc
}  // namespace kani
