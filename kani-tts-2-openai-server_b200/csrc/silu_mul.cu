// SiLU-gated activation y = silu(g) * u over rows of [g | u] (sm_100a).
//
// Reference: kani_tts/triton_kernels.py:67-105 — fp32 math
// (gate * sigmoid(gate)) * up, one rounding to the storage type.
//
// Launch shape: the output row is split into 16-byte column vectors; a 2-D
// grid gives each thread one column vector of RY consecutive rows, so every
// thread has 2*RY independent 16-byte loads in flight before it computes.
// grid.x covers the columns with a block width that divides the vector count
// when it can (n = 4608 bf16 -> 576 vectors = 3 x 192 threads); grid.y
// strides over row groups.  At one row (the decode step) the op spreads over
// grid.x CTAs instead of the reference's single program.  Inputs are read
// once, so they use evict-first loads; the output stays L2-resident for the
// down-projection GEMV that consumes it.
#include "common.cuh"

namespace kani {
namespace {

template <typename T, int RY>
__global__ void __launch_bounds__(256)
silu_mul_vec_kernel(const T* __restrict__ gu, int64_t in_stride, T* __restrict__ y,
                    int64_t out_stride, int64_t rows, int vpr, int64_t n) {
  constexpr int E = VecN<T>::value;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= vpr) return;
  const int64_t col = (int64_t)c * E;
  for (int64_t r0 = (int64_t)blockIdx.y * RY; r0 < rows; r0 += (int64_t)gridDim.y * RY) {
    uint4 g[RY], u[RY];
#pragma unroll
    for (int j = 0; j < RY; ++j) {
      if (r0 + j < rows) {
        const T* base = gu + (r0 + j) * in_stride + col;
        g[j] = ld16_stream(base);
        u[j] = ld16_stream(base + n);
      }
    }
#pragma unroll
    for (int j = 0; j < RY; ++j) {
      if (r0 + j < rows) {
        float gf[E], uf[E], o[E];
        unpack16<T>(g[j], gf);
        unpack16<T>(u[j], uf);
#pragma unroll
        for (int e = 0; e < E; ++e) o[e] = silu_mul_f(gf[e], uf[e]);
        st16(y + (r0 + j) * out_stride + col, pack16<T>(o));
      }
    }
  }
}

// Any n / alignment: one thread per output element of a row chunk.
template <typename T>
__global__ void __launch_bounds__(256)
silu_mul_generic_kernel(const T* __restrict__ gu, int64_t in_stride, T* __restrict__ y,
                        int64_t out_stride, int64_t rows, int64_t n) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= n) return;
  for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
    const T* row = gu + r * in_stride;
    const float g = Elem<T>::to_f(row[c]);
    const float u = Elem<T>::to_f(row[c + n]);
    y[r * out_stride + c] = Elem<T>::from_f(silu_mul_f(g, u));
  }
}

int pick_block_width(int vpr) {
  const int cand[] = {256, 192, 128, 96, 64};
  for (int b : cand)
    if (vpr % b == 0) return b;
  if (vpr < 64) return ((vpr + 31) / 32) * 32;
  return 128;
}

template <typename T>
int launch_silu(const void* gu, int64_t in_stride, void* y, int64_t out_stride, int64_t rows,
                int64_t n, cudaStream_t s) {
  constexpr int E = VecN<T>::value;
  const bool vec = (n % E) == 0 && aligned16(gu) && aligned16(y) && (in_stride % E) == 0 &&
                   (out_stride % E) == 0 && n / E <= 0x7fffffff;
  if (vec) {
    const int vpr = (int)(n / E);
    const int bx = pick_block_width(vpr);
    const unsigned gx = (unsigned)((vpr + bx - 1) / bx);
    constexpr int RY = 4;
    const int64_t groups = (rows + RY - 1) / RY;
    const unsigned gy = (unsigned)(groups < 65535 ? groups : 65535);
    if (rows >= RY) {
      silu_mul_vec_kernel<T, RY><<<dim3(gx, gy), bx, 0, s>>>(
          static_cast<const T*>(gu), in_stride, static_cast<T*>(y), out_stride, rows, vpr, n);
    } else {
      const unsigned gy1 = (unsigned)rows;
      silu_mul_vec_kernel<T, 1><<<dim3(gx, gy1), bx, 0, s>>>(
          static_cast<const T*>(gu), in_stride, static_cast<T*>(y), out_stride, rows, vpr, n);
    }
    return launch_status();
  }
  const int64_t gx64 = (n + 255) / 256;
  if (gx64 > 0x7fffffff) return KANI_ERR_UNSUPPORTED;
  const unsigned gy = (unsigned)(rows < 65535 ? rows : 65535);
  silu_mul_generic_kernel<T><<<dim3((unsigned)gx64, gy), 256, 0, s>>>(
      static_cast<const T*>(gu), in_stride, static_cast<T*>(y), out_stride, rows, n);
  return launch_status();
}

}  // namespace
}  // namespace kani

extern "C" int kani_silu_mul(int32_t dtype, const void* gate_up, int64_t in_row_stride, void* y,
                             int64_t out_row_stride, int64_t rows, int64_t n, void* stream) {
  if (rows < 0 || n < 0) return KANI_ERR_INVALID_ARG;
  if (rows == 0 || n == 0) return KANI_OK;
  if (gate_up == nullptr || y == nullptr) return KANI_ERR_INVALID_ARG;
  if (rows > 1 && (in_row_stride < 2 * n || out_row_stride < n)) return KANI_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return kani::dispatch_dtype(dtype, [&]<typename T>() {
    return kani::launch_silu<T>(gate_up, in_row_stride, y, out_row_stride, rows, n, s);
  });
}
