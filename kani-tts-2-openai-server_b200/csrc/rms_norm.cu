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
  griddep_wait();               // launched as a programmatic dependent: the inputs come from the launch before
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
  griddep_wait();               // launched as a programmatic dependent: the inputs come from the launch before
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
  griddep_wait();               // launched as a programmatic dependent: the inputs come from the launch before
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
    if (per <= 1)      launch_maybe_pdl(p.rows <= kPdlMaxRows, norm_group_kernel<T, W, 1, RES>, dim3((unsigned)grid), dim3(bt), 0, s, p, log2g);
    else if (per <= 2) launch_maybe_pdl(p.rows <= kPdlMaxRows, norm_group_kernel<T, W, 2, RES>, dim3((unsigned)grid), dim3(bt), 0, s, p, log2g);
    else if (per <= 4) launch_maybe_pdl(p.rows <= kPdlMaxRows, norm_group_kernel<T, W, 4, RES>, dim3((unsigned)grid), dim3(bt), 0, s, p, log2g);
    else               launch_maybe_pdl(p.rows <= kPdlMaxRows, norm_group_kernel<T, W, 8, RES>, dim3((unsigned)grid), dim3(bt), 0, s, p, log2g);
    return launch_status();
  }
  const unsigned grid = (unsigned)(p.rows < kMaxGrid ? p.rows : kMaxGrid);
  if (vec && nvec <= 256 * 8) {
    const int per = (nvec + 255) / 256;
    if (per <= 2)      launch_maybe_pdl(p.rows <= kPdlMaxRows, norm_block_kernel<T, W, 2, RES, 256>, dim3(grid), dim3(256), 0, s, p);
    else if (per <= 4) launch_maybe_pdl(p.rows <= kPdlMaxRows, norm_block_kernel<T, W, 4, RES, 256>, dim3(grid), dim3(256), 0, s, p);
    else               launch_maybe_pdl(p.rows <= kPdlMaxRows, norm_block_kernel<T, W, 8, RES, 256>, dim3(grid), dim3(256), 0, s, p);
    return launch_status();
  }
  launch_maybe_pdl(p.rows <= kPdlMaxRows, norm_generic_kernel<T, W, RES>, dim3(grid), dim3(256), 0, s, p);
  return launch_status();
}

// ------------------------------------------- K-split partials + add + RMSNorm
// The projection before a residual add, computed as S fp32 partial products over
// slices of K (a batched GEMM with an fp32 output), is finished here:
//   d = round_T(p[0] + p[1] + ... + p[S-1])   (fp32, in split order: F.linear's
//                                              output, one rounding)
//   h = round_T(d + r), y = round_T((h * rr) * w)   (as kani_add_rms_norm)
// One CTA of 256 threads per row; a thread owns 4-element chunks c = tid,
// tid + 256, ... and issues every split's load of a chunk before it sums.
struct RedParams {
  const float* part;
  int64_t ps;  // elements between splits
  int64_t pr;  // elements between rows of one split
  int splits;
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
  L2Prefetch pf;  // later launches' weights, prefetched into L2 at entry
};

constexpr int kRedThreads = 256;

template <typename T>
__device__ __forceinline__ void ld4(const T* ptr, float* f) {
  if constexpr (sizeof(T) == 2) {
    const uint2 v = *reinterpret_cast<const uint2*>(ptr);
    const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) f[i] = Elem<T>::to_f(e[i]);
  } else {
    const float4 v = *reinterpret_cast<const float4*>(ptr);
    f[0] = v.x; f[1] = v.y; f[2] = v.z; f[3] = v.w;
  }
}

template <typename T>
__device__ __forceinline__ void st4(T* ptr, const float* f) {
  if constexpr (sizeof(T) == 2) {
    uint2 v;
    T* e = reinterpret_cast<T*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) e[i] = Elem<T>::from_f(f[i]);
    *reinterpret_cast<uint2*>(ptr) = v;
  } else {
    *reinterpret_cast<float4*>(ptr) = make_float4(f[0], f[1], f[2], f[3]);
  }
}

template <typename T, typename W, int V>
__global__ void __launch_bounds__(kRedThreads) reduce_add_norm_kernel(RedParams p) {
  griddep_launch_dependents();  // a dependent GEMV may start streaming its weights
  griddep_wait();               // launched as a programmatic dependent: the inputs come from the launch before
  l2_prefetch_share(p.pf);
  __shared__ float red[33];
  const int tid = threadIdx.x;
  for (int64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
    float h[V][4];
    float ss = 0.f;
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const int c = (v * kRedThreads + tid) * 4;
      if (c < p.n) {
        const float* src = p.part + row * p.pr + c;
        float acc[4];
        {
          const float4 a = *reinterpret_cast<const float4*>(src);
          acc[0] = a.x; acc[1] = a.y; acc[2] = a.z; acc[3] = a.w;
        }
#pragma unroll 4
        for (int sp = 1; sp < p.splits; ++sp) {
          const float4 a = *reinterpret_cast<const float4*>(src + sp * p.ps);
          acc[0] = __fadd_rn(acc[0], a.x);
          acc[1] = __fadd_rn(acc[1], a.y);
          acc[2] = __fadd_rn(acc[2], a.z);
          acc[3] = __fadd_rn(acc[3], a.w);
        }
        float rv[4];
        ld4<T>(static_cast<const T*>(p.r) + row * p.rs + c, rv);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          h[v][e] = round_to<T>(__fadd_rn(round_to<T>(acc[e]), rv[e]));
          ss = fmaf(h[v][e], h[v][e], ss);
        }
      }
    }
    ss = block_sum<kRedThreads>(ss, red);
    const float rr = rrms_of(ss, p.n, p.eps);
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const int c = (v * kRedThreads + tid) * 4;
      if (c < p.n) {
        float wf[4], o[4];
        ld4<W>(static_cast<const W*>(p.w) + c, wf);
#pragma unroll
        for (int e = 0; e < 4; ++e) o[e] = __fmul_rn(__fmul_rn(h[v][e], rr), wf[e]);
        st4<T>(static_cast<T*>(p.h) + row * p.hs + c, h[v]);
        st4<T>(static_cast<T*>(p.y) + row * p.ys + c, o);
      }
    }
  }
}

template <typename T, typename W>
int launch_reduce_norm(const RedParams& p, cudaStream_t s) {
  const unsigned grid = (unsigned)(p.rows < kMaxGrid ? p.rows : kMaxGrid);
  const int v = (p.n + 4 * kRedThreads - 1) / (4 * kRedThreads);
  if (v <= 1)      launch_maybe_pdl(p.rows <= kPdlMaxRows, reduce_add_norm_kernel<T, W, 1>, dim3(grid), dim3(kRedThreads), 0, s, p);
  else if (v <= 2) launch_maybe_pdl(p.rows <= kPdlMaxRows, reduce_add_norm_kernel<T, W, 2>, dim3(grid), dim3(kRedThreads), 0, s, p);
  else             launch_maybe_pdl(p.rows <= kPdlMaxRows, reduce_add_norm_kernel<T, W, 4>, dim3(grid), dim3(kRedThreads), 0, s, p);
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

extern "C" int kani_reduce_add_rms_norm(int32_t dtype, int32_t w_dtype, const float* partials, int64_t split_stride,
                                        int64_t partial_row_stride, int32_t splits, const void* residual,
                                        int64_t r_row_stride, const void* weight, void* y, int64_t y_row_stride,
                                        void* residual_out, int64_t h_row_stride, int64_t rows, int64_t n, float eps,
                                        void* stream) {
  const kani::L2Prefetch pf = kani::take_l2_prefetch();
  if (rows < 0 || n < 0 || splits < 1) return KANI_ERR_INVALID_ARG;
  if (rows == 0 || n == 0) return KANI_OK;
  if (!partials || !residual || !weight || !y || !residual_out) return KANI_ERR_INVALID_ARG;
  if (y == residual_out) return KANI_ERR_INVALID_ARG;
  if (rows > 1 && (partial_row_stride < n || r_row_stride < n || y_row_stride < n || h_row_stride < n))
    return KANI_ERR_INVALID_ARG;
  if (splits > 1) {  // the splits must not overlap: split-major or row-major blocks of partials
    const bool split_major = split_stride >= (rows - 1) * partial_row_stride + n;
    const bool row_major = split_stride >= n && partial_row_stride >= (splits - 1) * split_stride + n;
    if (!split_major && !row_major) return KANI_ERR_INVALID_ARG;
  }
  if (n % 4 != 0 || n > 4 * 4 * kani::kRedThreads) return KANI_ERR_UNSUPPORTED;
  if (!kani::aligned16(partials) || split_stride % 4 != 0 || partial_row_stride % 4 != 0 ||
      (reinterpret_cast<uintptr_t>(residual) | reinterpret_cast<uintptr_t>(y) |
       reinterpret_cast<uintptr_t>(residual_out) | reinterpret_cast<uintptr_t>(weight)) % 16 != 0 ||
      r_row_stride % 4 != 0 || y_row_stride % 4 != 0 || h_row_stride % 4 != 0)
    return KANI_ERR_UNSUPPORTED;
  kani::RedParams p{partials, split_stride, partial_row_stride, splits, residual, r_row_stride, weight, y,
                    y_row_stride, residual_out, h_row_stride, rows, (int)n, eps, pf};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return kani::dispatch_dtype(dtype, [&]<typename T>() {
    return kani::dispatch_dtype(w_dtype, [&]<typename W>() { return kani::launch_reduce_norm<T, W>(p, s); });
  });
}
