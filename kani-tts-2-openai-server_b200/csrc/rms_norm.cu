// RMSNorm and residual-add + RMSNorm over the last dimension (sm_100a).
//
// Algorithm (reference: kani_tts/triton_kernels.py:17-35 for the norm; the
// residual add is the eager bf16 add of kani_tts/optimized_decode.py:252/277/283):
//   h   = round_T(x + r)                 (only with a residual; the eager add)
//   ss  = sum_i h_i^2                    (fp32)
//   rr  = 1 / sqrt(ss / n + eps)         (fp32, IEEE sqrt and divide)
//   y_i = round_T((h_i * rr) * w_i)      (fp32, one rounding)
//
// Layout: rows of n contiguous elements; rows addressed through row strides.
// Three launch shapes, chosen on the host:
//   * group path  — a power-of-two group of G <= 32 lanes owns one row and
//     keeps it in registers as up to 8 16-byte vectors per lane (rows up to
//     4 KB: bf16 n <= 2048, fp32 n <= 1024); the sum of squares is a
//     G-wide xor-shuffle tree.  n = 64 (per-head q/k norm) puts 4 rows in
//     one warp, n = 1024 bf16 gives one warp per row.
//   * block path  — one CTA of 256 threads per row, still in registers
//     (rows up to 32 KB), block reduction through shared memory.
//   * generic     — any n / alignment: one CTA per row, two passes with
//     scalar accesses.  The second pass re-reads h from residual_out (or x),
//     which each thread itself wrote or read in the first pass.
#include "common.cuh"

namespace kani {
namespace {

struct NormParams {
  const void* x;
  int64_t xs;
  const void* r;
  int64_t rs;
  const void* w;
  void* y;
  int64_t ys;
  void* h;
  int64_t hs;
  int64_t rows;
  int n;
  float eps;
};

__device__ __forceinline__ float rrms_of(float ss, int n, float eps) {
  return 1.0f / sqrtf(ss / (float)n + eps);
}

// --------------------------------------------------------------- group path
template <typename T, typename W, int V, bool RES>
__global__ void __launch_bounds__(128)
norm_group_kernel(NormParams p, int log2g) {
  griddep_launch_dependents();  // a dependent GEMV may start streaming its weights
  constexpr int E = VecN<T>::value;
  const int G = 1 << log2g;
  const int64_t gtid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t row = gtid >> log2g;
  const int lane = (int)(gtid & (G - 1));
  const int nvec = p.n / E;
  const bool active = row < p.rows;

  float h[V][E];
  float ss = 0.f;
  if (active) {
    const T* xr = static_cast<const T*>(p.x) + row * p.xs;
    const T* rr = RES ? static_cast<const T*>(p.r) + row * p.rs : nullptr;
    uint4 xv[V], rv[V];
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int vi = i * G + lane;
      if (vi < nvec) {
        xv[i] = ld16(xr + (int64_t)vi * E);
        if constexpr (RES) rv[i] = ld16(rr + (int64_t)vi * E);
      }
    }
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int vi = i * G + lane;
      if (vi < nvec) {
        unpack16<T>(xv[i], h[i]);
        if constexpr (RES) {
          float rf[E];
          unpack16<T>(rv[i], rf);
#pragma unroll
          for (int e = 0; e < E; ++e) h[i][e] = round_to<T>(__fadd_rn(h[i][e], rf[e]));
        }
#pragma unroll
        for (int e = 0; e < E; ++e) ss = fmaf(h[i][e], h[i][e], ss);
      }
    }
  }
  // every lane of the warp takes part, active or not (G is warp-uniform)
  for (int off = G >> 1; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if (!active) return;

  const float rr = rrms_of(ss, p.n, p.eps);
  T* yr = static_cast<T*>(p.y) + row * p.ys;
  T* hr = RES ? static_cast<T*>(p.h) + row * p.hs : nullptr;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int vi = i * G + lane;
    if (vi < nvec) {
      float wf[E], o[E];
      load_weights<W, E>(static_cast<const W*>(p.w), (int64_t)vi * E, wf);
#pragma unroll
      for (int e = 0; e < E; ++e) o[e] = __fmul_rn(__fmul_rn(h[i][e], rr), wf[e]);
      if constexpr (RES) st16(hr + (int64_t)vi * E, pack16<T>(h[i]));
      st16(yr + (int64_t)vi * E, pack16<T>(o));
    }
  }
}

// --------------------------------------------------------------- block path
template <int BT>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < BT / 32 ? red[lane] : 0.f;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (lane == 0) red[32] = v;
  }
  __syncthreads();
  v = red[32];
  __syncthreads();  // red is reused by the next row
  return v;
}

template <typename T, typename W, int V, bool RES, int BT>
__global__ void __launch_bounds__(BT)
norm_block_kernel(NormParams p) {
  griddep_launch_dependents();  // a dependent GEMV may start streaming its weights
  constexpr int E = VecN<T>::value;
  __shared__ float red[33];
  const int nvec = p.n / E;
  for (int64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
    const T* xr = static_cast<const T*>(p.x) + row * p.xs;
    const T* rr = RES ? static_cast<const T*>(p.r) + row * p.rs : nullptr;
    float h[V][E];
    uint4 xv[V], rv[V];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int vi = i * BT + threadIdx.x;
      if (vi < nvec) {
        xv[i] = ld16(xr + (int64_t)vi * E);
        if constexpr (RES) rv[i] = ld16(rr + (int64_t)vi * E);
      }
    }
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int vi = i * BT + threadIdx.x;
      if (vi < nvec) {
        unpack16<T>(xv[i], h[i]);
        if constexpr (RES) {
          float rf[E];
          unpack16<T>(rv[i], rf);
#pragma unroll
          for (int e = 0; e < E; ++e) h[i][e] = round_to<T>(__fadd_rn(h[i][e], rf[e]));
        }
#pragma unroll
        for (int e = 0; e < E; ++e) ss = fmaf(h[i][e], h[i][e], ss);
      }
    }
    ss = block_sum<BT>(ss, red);
    const float r = rrms_of(ss, p.n, p.eps);
    T* yr = static_cast<T*>(p.y) + row * p.ys;
    T* hr = RES ? static_cast<T*>(p.h) + row * p.hs : nullptr;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int vi = i * BT + threadIdx.x;
      if (vi < nvec) {
        float wf[E], o[E];
        load_weights<W, E>(static_cast<const W*>(p.w), (int64_t)vi * E, wf);
#pragma unroll
        for (int e = 0; e < E; ++e) o[e] = __fmul_rn(__fmul_rn(h[i][e], r), wf[e]);
        if constexpr (RES) st16(hr + (int64_t)vi * E, pack16<T>(h[i]));
        st16(yr + (int64_t)vi * E, pack16<T>(o));
      }
    }
  }
}

// ------------------------------------------------------------- generic path
template <typename T, typename W, bool RES>
__global__ void __launch_bounds__(256)
norm_generic_kernel(NormParams p) {
  griddep_launch_dependents();  // a dependent GEMV may start streaming its weights
  __shared__ float red[33];
  for (int64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
    const T* xr = static_cast<const T*>(p.x) + row * p.xs;
    const T* rr = RES ? static_cast<const T*>(p.r) + row * p.rs : nullptr;
    T* hr = RES ? static_cast<T*>(p.h) + row * p.hs : nullptr;
    T* yr = static_cast<T*>(p.y) + row * p.ys;
    float ss = 0.f;
    for (int i = threadIdx.x; i < p.n; i += 256) {
      float hv = Elem<T>::to_f(xr[i]);
      if constexpr (RES) {
        hv = round_to<T>(__fadd_rn(hv, Elem<T>::to_f(rr[i])));
        hr[i] = Elem<T>::from_f(hv);
      }
      ss = fmaf(hv, hv, ss);
    }
    ss = block_sum<256>(ss, red);
    const float r = rrms_of(ss, p.n, p.eps);
    const W* w = static_cast<const W*>(p.w);
    for (int i = threadIdx.x; i < p.n; i += 256) {
      const float hv = RES ? Elem<T>::to_f(hr[i]) : Elem<T>::to_f(xr[i]);
      yr[i] = Elem<T>::from_f(__fmul_rn(__fmul_rn(hv, r), Elem<W>::to_f(w[i])));
    }
  }
}

// ------------------------------------------------------------------ launch
constexpr int64_t kMaxGrid = 1 << 20;  // grid-stride cap for the row loops

template <typename T, typename W, bool RES>
int launch_norm(const NormParams& p, cudaStream_t s) {
  constexpr int E = VecN<T>::value;
  bool vec = (p.n % E) == 0 && aligned16(p.x) && aligned16(p.y) && aligned16(p.w) &&
             (p.xs % E) == 0 && (p.ys % E) == 0;
  if (RES) vec = vec && aligned16(p.r) && aligned16(p.h) && (p.rs % E) == 0 && (p.hs % E) == 0;
  const int nvec = p.n / E;

  if (vec && nvec <= 32 * 8) {
    int log2g = 0;
    while ((1 << log2g) < nvec && log2g < 5) ++log2g;
    const int G = 1 << log2g;
    const int per = (nvec + G - 1) / G;
    // 128-thread blocks, narrowed (down to one warp) while the grid would leave
    // SMs idle: 64 decode rows of 1024 take 64 one-warp CTAs instead of 16
    int bt = 128;
    const int64_t want = 2LL * sm_count();
    while (bt > 32 && (p.rows * G + bt - 1) / bt < want) bt >>= 1;
    const int rows_per_block = bt / G;
    const int64_t grid = (p.rows + rows_per_block - 1) / rows_per_block;
    if (grid > 0x7fffffff) return KANI_ERR_UNSUPPORTED;
    if (per <= 1)      norm_group_kernel<T, W, 1, RES><<<(unsigned)grid, bt, 0, s>>>(p, log2g);
    else if (per <= 2) norm_group_kernel<T, W, 2, RES><<<(unsigned)grid, bt, 0, s>>>(p, log2g);
    else if (per <= 4) norm_group_kernel<T, W, 4, RES><<<(unsigned)grid, bt, 0, s>>>(p, log2g);
    else               norm_group_kernel<T, W, 8, RES><<<(unsigned)grid, bt, 0, s>>>(p, log2g);
    return launch_status();
  }
  const unsigned grid = (unsigned)(p.rows < kMaxGrid ? p.rows : kMaxGrid);
  if (vec && nvec <= 256 * 8) {
    const int per = (nvec + 255) / 256;
    if (per <= 2)      norm_block_kernel<T, W, 2, RES, 256><<<grid, 256, 0, s>>>(p);
    else if (per <= 4) norm_block_kernel<T, W, 4, RES, 256><<<grid, 256, 0, s>>>(p);
    else               norm_block_kernel<T, W, 8, RES, 256><<<grid, 256, 0, s>>>(p);
    return launch_status();
  }
  norm_generic_kernel<T, W, RES><<<grid, 256, 0, s>>>(p);
  return launch_status();
}

template <bool RES>
int norm_entry(int32_t dtype, int32_t w_dtype, const NormParams& p, cudaStream_t s) {
  return dispatch_dtype(dtype, [&]<typename T>() {
    return dispatch_dtype(w_dtype, [&]<typename W>() { return launch_norm<T, W, RES>(p, s); });
  });
}

// A row view is usable when it has a base pointer and, for more than one row,
// a row stride of at least n elements.
bool bad_rows(const void* base, int64_t stride, int64_t n, int64_t rows) {
  return base == nullptr || (rows > 1 && stride < n);
}

}  // namespace
}  // namespace kani

using kani::NormParams;

extern "C" int kani_rms_norm(int32_t dtype, int32_t w_dtype, const void* x, int64_t x_row_stride,
                             const void* weight, void* y, int64_t y_row_stride, int64_t rows,
                             int64_t n, float eps, void* stream) {
  if (rows < 0 || n < 0 || n > 0x7fffffff) return KANI_ERR_INVALID_ARG;
  if (rows == 0 || n == 0) return KANI_OK;
  if (weight == nullptr || kani::bad_rows(x, x_row_stride, n, rows) ||
      kani::bad_rows(y, y_row_stride, n, rows))
    return KANI_ERR_INVALID_ARG;
  NormParams p{x, x_row_stride, nullptr, 0, weight, y, y_row_stride, nullptr, 0, rows, (int)n, eps};
  return kani::norm_entry<false>(dtype, w_dtype, p, static_cast<cudaStream_t>(stream));
}

extern "C" int kani_add_rms_norm(int32_t dtype, int32_t w_dtype, const void* x, int64_t x_row_stride,
                                 const void* residual, int64_t r_row_stride, const void* weight,
                                 void* y, int64_t y_row_stride, void* residual_out,
                                 int64_t h_row_stride, int64_t rows, int64_t n, float eps,
                                 void* stream) {
  if (rows < 0 || n < 0 || n > 0x7fffffff) return KANI_ERR_INVALID_ARG;
  if (rows == 0 || n == 0) return KANI_OK;
  if (weight == nullptr || kani::bad_rows(x, x_row_stride, n, rows) ||
      kani::bad_rows(residual, r_row_stride, n, rows) || kani::bad_rows(y, y_row_stride, n, rows) ||
      kani::bad_rows(residual_out, h_row_stride, n, rows))
    return KANI_ERR_INVALID_ARG;
  if (y == residual_out) return KANI_ERR_INVALID_ARG;
  NormParams p{x, x_row_stride, residual, r_row_stride, weight, y, y_row_stride,
               residual_out, h_row_stride, rows, (int)n, eps};
  return kani::norm_entry<true>(dtype, w_dtype, p, static_cast<cudaStream_t>(stream));
}
