// SiLU-gated activation y = silu(g) * u over rows of [g | u] (sm_100a).
//
// Reference: kani_tts/triton_kernels.py:67-105 — fp32 math
// (gate * sigmoid(gate)) * up, one rounding to the storage type.
//
// Launch shapes (measured on B200 against the reference's one-program-per-row
// Triton kernel, bf16 [T, 2 x 4608]):
//   * T >= 2048: one 192-thread CTA per row; each thread loads all of its
//     16-byte gate and up vectors of that row (3 + 3 at n = 4608) before it
//     computes (T = 4096: 18.6 us, T = 32768: 128.5 us).
//   * shorter calls: a 2-D grid of 16-byte column vectors x rows, one row per
//     thread; the block narrows to 64 threads while the grid would leave SMs
//     idle (T = 512: 4.1 us; T = 64: 9 x 64 CTAs, 2.0 us; T = 1: 9 CTAs, 1.3
//     us, against the reference's single program).
// Inputs are read once; the output stays L2-resident for the down-projection
// GEMV that consumes it.
#include "common.cuh"

namespace kani {
namespace {

template <typename T, int RY>
__global__ void __launch_bounds__(256)
silu_mul_vec_kernel(const T* __restrict__ gu, int64_t in_stride, T* __restrict__ y,
                    int64_t out_stride, int64_t rows, int vpr, int64_t n, L2Prefetch pf) {
  constexpr int E = VecN<T>::value;
  l2_prefetch_share(pf);
  griddep_wait();  // launched as a programmatic dependent: the input comes from the launch before
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

// Long calls: one CTA per row (grid-stride), like one program per row, so a
// CTA reads one contiguous gate row and one up row; each thread issues all
// of its CV gate and CV up vectors before it computes.  Plain loads: here the
// evict-first hint measured slower (T = 4096: 18.6 against 19.3 us).
template <typename T, int CV>
__global__ void __launch_bounds__(192)
silu_mul_row_kernel(const T* __restrict__ gu, int64_t in_stride, T* __restrict__ y, int64_t out_stride,
                    int64_t rows, int vpr, int64_t n, L2Prefetch pf) {
  constexpr int E = VecN<T>::value;
  l2_prefetch_share(pf);
  griddep_wait();  // launched as a programmatic dependent: the input comes from the launch before
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const T* base = gu + r * in_stride;
    uint4 g[CV], u[CV];
#pragma unroll
    for (int j = 0; j < CV; ++j) {
      const int c = j * 192 + threadIdx.x;
      if (c < vpr) {
        g[j] = ld16(base + (int64_t)c * E);
        u[j] = ld16(base + n + (int64_t)c * E);
      }
    }
#pragma unroll
    for (int j = 0; j < CV; ++j) {
      const int c = j * 192 + threadIdx.x;
      if (c < vpr) {
        float gf[E], uf[E], o[E];
        unpack16<T>(g[j], gf);
        unpack16<T>(u[j], uf);
#pragma unroll
        for (int e = 0; e < E; ++e) o[e] = silu_mul_f(gf[e], uf[e]);
        st16(y + r * out_stride + (int64_t)c * E, pack16<T>(o));
      }
    }
  }
}

// Any n / alignment: one thread per output element of a row chunk.
template <typename T>
__global__ void __launch_bounds__(256)
silu_mul_generic_kernel(const T* __restrict__ gu, int64_t in_stride, T* __restrict__ y,
                        int64_t out_stride, int64_t rows, int64_t n, L2Prefetch pf) {
  l2_prefetch_share(pf);
  griddep_wait();  // launched as a programmatic dependent: the input comes from the launch before
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= n) return;
  for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
    const T* row = gu + r * in_stride;
    const float g = Elem<T>::to_f(row[c]);
    const float u = Elem<T>::to_f(row[c + n]);
    y[r * out_stride + c] = Elem<T>::from_f(silu_mul_f(g, u));
  }
}

constexpr int64_t kRowKernelMinRows = 2048;

int pick_block_width(int vpr) {
  const int cand[] = {256, 192, 128, 96, 64};
  for (int b : cand)
    if (vpr % b == 0) return b;
  if (vpr < 64) return ((vpr + 31) / 32) * 32;
  return 128;
}

template <typename T>
int launch_silu(const void* gu, int64_t in_stride, void* y, int64_t out_stride, int64_t rows,
                int64_t n, const L2Prefetch& pf, cudaStream_t s) {
  constexpr int E = VecN<T>::value;
  const bool vec = (n % E) == 0 && aligned16(gu) && aligned16(y) && (in_stride % E) == 0 &&
                   (out_stride % E) == 0 && n / E <= 0x7fffffff;
  if (vec) {
    const int vpr = (int)(n / E);
    const int cv = (vpr + 191) / 192;
    if (rows >= kRowKernelMinRows && cv <= 8) {
      const unsigned grid = (unsigned)(rows < 0x7fffffff ? rows : 0x7fffffff);
      auto go = [&](auto kern) {
        launch_maybe_pdl(rows <= kPdlMaxRows, kern, dim3(grid), dim3(192), 0, s, static_cast<const T*>(gu), in_stride, static_cast<T*>(y),
                   out_stride, rows, vpr, n, pf);
      };
      if (cv <= 2)      go(silu_mul_row_kernel<T, 2>);
      else if (cv <= 3) go(silu_mul_row_kernel<T, 3>);
      else if (cv <= 4) go(silu_mul_row_kernel<T, 4>);
      else if (cv <= 6) go(silu_mul_row_kernel<T, 6>);
      else              go(silu_mul_row_kernel<T, 8>);
      return launch_status();
    }
    // shorter calls: one row per thread, and narrower blocks while the grid
    // would leave SMs idle (T = 64: 9 x 64 CTAs of 64 threads)
    int bx = pick_block_width(vpr);
    unsigned gx = (unsigned)((vpr + bx - 1) / bx);
    const int64_t want = 2LL * sm_count();
    if ((int64_t)gx * rows < want && bx > 64) {
      bx = 64;
      gx = (unsigned)((vpr + bx - 1) / bx);
    }
    const unsigned gy = (unsigned)(rows < 65535 ? rows : 65535);
    launch_maybe_pdl(rows <= kPdlMaxRows, silu_mul_vec_kernel<T, 1>, dim3(gx, gy), dim3(bx), 0, s, static_cast<const T*>(gu), in_stride,
               static_cast<T*>(y), out_stride, rows, vpr, n, pf);
    return launch_status();
  }
  const int64_t gx64 = (n + 255) / 256;
  if (gx64 > 0x7fffffff) return KANI_ERR_UNSUPPORTED;
  const unsigned gy = (unsigned)(rows < 65535 ? rows : 65535);
  launch_maybe_pdl(rows <= kPdlMaxRows, silu_mul_generic_kernel<T>, dim3((unsigned)gx64, gy), dim3(256), 0, s, static_cast<const T*>(gu),
             in_stride, static_cast<T*>(y), out_stride, rows, n, pf);
  return launch_status();
}

}  // namespace
}  // namespace kani

extern "C" int kani_silu_mul(int32_t dtype, const void* gate_up, int64_t in_row_stride, void* y,
                             int64_t out_row_stride, int64_t rows, int64_t n, void* stream) {
  const kani::L2Prefetch pf = kani::take_l2_prefetch();
  if (rows < 0 || n < 0) return KANI_ERR_INVALID_ARG;
  if (rows == 0 || n == 0) return KANI_OK;
  if (gate_up == nullptr || y == nullptr) return KANI_ERR_INVALID_ARG;
  if (rows > 1 && (in_row_stride < 2 * n || out_row_stride < n)) return KANI_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return kani::dispatch_dtype(dtype, [&]<typename T>() {
    return kani::launch_silu<T>(gate_up, in_row_stride, y, out_row_stride, rows, n, pf, s);
  });
}
