// Small-batch decode GEMV with its neighbours fused (sm_100a), for up to 8
// streams.
//
//   y[b, r] = round(sum_k a[b, k] * W[r, k])            (fp32 accumulation)
//
// The input a[b] is either x[b] itself, or (NORM) the RMSNorm of the residual
// stream, folded in front of the GEMV that consumes it:
//   h = round(x + residual)  (when a residual is given; h is written to
//                             residual_out by CTA 0 for the next layer)
//   a = round((h * rr) * w), rr = 1 / sqrt(sum h^2 / K + eps)
// — the arithmetic of kani_add_rms_norm / kani_rms_norm.  With SILU the
// weight holds 2N rows (gate rows, then up rows) and the epilogue is
//   y[b, r] = round(silu(round(g)) * round(u)),  g = acc row r, u = acc row N + r
// — F.linear(gate_up) followed by the fused SiLU·mul kernel, rounding for
// rounding.  kani_gemv_short_conv ends the in_proj GEMV with the LFM2 gated
// short-conv step instead (the B, C and x rows of a channel in one warp; the
// arithmetic of short_conv.cu, optimized_decode.py:256-277).  Reference: the decode step of kani_tts/optimized_decode.py:175-289
// (residual adds :252/:277/:283, norms :206/:280/:286, the QKV / in_proj /
// gate_up / down / o_proj / out_proj F.linear calls, the SiLU·mul of
// kani_tts/triton_kernels.py:67-105).  Merging norm + GEMV and GEMV + SiLU
// removes a launch each per use; at one token per stream every launch costs
// a few microseconds of latency, more than the bytes it moves.
//
// Layout: 256-thread CTAs; one warp per output row (SILU: per gate/up pair)
// streams the row with 16-byte evict-first loads (K / 256 loads in flight per
// lane); the B input rows sit in shared memory.  Every CTA recomputes the
// norm (a few KB from L2).  Launches use programmatic dependent launch: a
// warp issues its first row's weight loads before griddepcontrol.wait, so the
// weight stream of one launch overlaps the tail of the launch before it; all
// reads of activations and all writes come after the wait.
#include "common.cuh"

namespace kani {
namespace {

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kGemvMaxB = 8;

struct GemvParams {
  const void* x;
  int64_t x_stride;
  const void* res;
  int64_t res_stride;
  void* res_out;
  int64_t res_out_stride;
  const void* norm_w;
  float eps;
  const void* w;
  int64_t w_stride;
  int n, k, batch;
  void* y;
  int64_t y_stride;
  void* conv_state;  // EPI 2: [batch, n, kConvL] state, batch stride
  int64_t conv_state_stride;
  const void* conv_w;  // EPI 2: [n, kConvL]
};

constexpr int kConvL = 3;  // the LFM2 short-conv kernel length the fused epilogue serves

// EPI: 0 = store, 1 = SiLU·mul of the gate / up rows r and n + r,
//      2 = gated short-conv step of channel r over rows r (B), n + r (C), 2n + r (x)
template <typename T, int B, int CH, bool NORM, int EPI>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(GemvParams p) {
  constexpr int E = 8;
  constexpr int K = CH * 256;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ float s_part[kGemvWarps][B];
  T* as = reinterpret_cast<T*>(smem_raw);  // [B][K] GEMV input
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  // ---- the weights do not depend on earlier launches: start this warp's
  //      first row streaming before waiting for them (programmatic dependent
  //      launch), then let the next launch start its own weight stream
  const T* W = static_cast<const T*>(p.w);
  constexpr int NR = EPI == 0 ? 1 : (EPI == 1 ? 2 : 3);
  int r = blockIdx.x * kGemvWarps + warp;
  uint4 wv[NR][CH];
  auto load_row = [&](int row) {
#pragma unroll
    for (int q = 0; q < NR; ++q)
#pragma unroll
      for (int c = 0; c < CH; ++c)
        wv[q][c] = ld16_stream(W + (int64_t)(row + q * p.n) * p.w_stride + c * 256 + lane * E);
  };
  if (r < p.n) load_row(r);
  griddep_launch_dependents();
  griddep_wait();

  // ---- input rows (NORM: residual add + RMSNorm) into shared memory
  if constexpr (!NORM) {
    for (int v = tid; v < B * K / E; v += kGemvThreads) {
      const int b = v / (K / E), c = v % (K / E);
      uint4 x = make_uint4(0u, 0u, 0u, 0u);
      if (b < p.batch) x = ld16(static_cast<const T*>(p.x) + (int64_t)b * p.x_stride + c * E);
      reinterpret_cast<uint4*>(as)[v] = x;
    }
  } else {
    float ss[B];
#pragma unroll
    for (int b = 0; b < B; ++b) ss[b] = 0.f;
    for (int v = tid; v < B * K / E; v += kGemvThreads) {
      const int b = v / (K / E), c = v % (K / E);
      float h[E];
#pragma unroll
      for (int e = 0; e < E; ++e) h[e] = 0.f;
      if (b < p.batch) {
        unpack16<T>(ld16(static_cast<const T*>(p.x) + (int64_t)b * p.x_stride + c * E), h);
        if (p.res) {
          float rv[E];
          unpack16<T>(ld16(static_cast<const T*>(p.res) + (int64_t)b * p.res_stride + c * E), rv);
#pragma unroll
          for (int e = 0; e < E; ++e) h[e] = round_to<T>(__fadd_rn(h[e], rv[e]));
          if (p.res_out && blockIdx.x == 0)
            st16(static_cast<T*>(p.res_out) + (int64_t)b * p.res_out_stride + c * E, pack16<T>(h));
        }
      }
      float s = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) s = fmaf(h[e], h[e], s);
      // b is uniform over runs of K/E consecutive v, so accumulate per b
#pragma unroll
      for (int bb = 0; bb < B; ++bb)
        if (bb == b) ss[bb] += s;
      reinterpret_cast<uint4*>(as)[v] = pack16<T>(h);  // h (rounded), normalised below
    }
#pragma unroll
    for (int b = 0; b < B; ++b) {
      float s = ss[b];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) s_part[warp][b] = s;
    }
    __syncthreads();
    for (int v = tid; v < B * K / E; v += kGemvThreads) {
      const int b = v / (K / E), c = v % (K / E);
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < kGemvWarps; ++w) tot += s_part[w][b];
      const float rr = 1.0f / sqrtf(tot / (float)K + p.eps);
      float h[E], wf[E];
      unpack16<T>(reinterpret_cast<const uint4*>(as)[v], h);
      unpack16<T>(ld16_ro(static_cast<const T*>(p.norm_w) + c * E), wf);
#pragma unroll
      for (int e = 0; e < E; ++e) h[e] = __fmul_rn(__fmul_rn(h[e], rr), wf[e]);
      reinterpret_cast<uint4*>(as)[v] = pack16<T>(h);
    }
  }
  __syncthreads();

  // ---- one warp per output row (SILU: per gate/up pair); row r's weights
  //      are already in flight
  for (; r < p.n; r += gridDim.x * kGemvWarps) {
    if (r != blockIdx.x * kGemvWarps + warp) load_row(r);
    float acc[NR][B];
#pragma unroll
    for (int q = 0; q < NR; ++q)
#pragma unroll
      for (int b = 0; b < B; ++b) acc[q][b] = 0.f;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      float wf[NR][E];
#pragma unroll
      for (int q = 0; q < NR; ++q) unpack16<T>(wv[q][c], wf[q]);
#pragma unroll
      for (int b = 0; b < B; ++b) {
        float af[E];
        unpack16<T>(reinterpret_cast<const uint4*>(as + b * K + c * 256)[lane], af);
#pragma unroll
        for (int q = 0; q < NR; ++q)
#pragma unroll
          for (int e = 0; e < E; ++e) acc[q][b] = fmaf(wf[q][e], af[e], acc[q][b]);
      }
    }
#pragma unroll
    for (int q = 0; q < NR; ++q)
#pragma unroll
      for (int b = 0; b < B; ++b)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc[q][b] += __shfl_xor_sync(0xffffffffu, acc[q][b], o);
    // lane b stores stream b
#pragma unroll
    for (int b = 0; b < B; ++b) {
      if (lane == b && b < p.batch) {
        float v;
        if constexpr (EPI == 1) {
          v = silu_mul_f(round_to<T>(acc[0][b]), round_to<T>(acc[1][b]));
        } else if constexpr (EPI == 2) {
          // the in_proj output [Bg | C | x] of channel r, rounded as F.linear
          // stores it, then the step of short_conv.cu for this channel
          const float bg = round_to<T>(acc[0][b]), cg = round_to<T>(acc[1][b]), xg = round_to<T>(acc[2][b]);
          T* st = static_cast<T*>(p.conv_state) + (int64_t)b * p.conv_state_stride + (int64_t)r * kConvL;
          const T* cw = static_cast<const T*>(p.conv_w) + (int64_t)r * kConvL;
          float sv[kConvL];
#pragma unroll
          for (int i = 0; i + 1 < kConvL; ++i) sv[i] = Elem<T>::to_f(st[i + 1]);
          sv[kConvL - 1] = round_to<T>(__fmul_rn(bg, xg));
          float conv = 0.f;
#pragma unroll
          for (int i = 0; i < kConvL; ++i) {
            st[i] = Elem<T>::from_f(sv[i]);
            conv = __fadd_rn(conv, round_to<T>(__fmul_rn(sv[i], Elem<T>::to_f(cw[i]))));
          }
          v = __fmul_rn(cg, round_to<T>(conv));
        } else {
          v = acc[0][b];
        }
        static_cast<T*>(p.y)[(int64_t)b * p.y_stride + r] = Elem<T>::from_f(v);
      }
    }
  }
}

template <typename T, int B, int CH>
int launch_gemv_bk(const GemvParams& prm, bool norm, int epi, cudaStream_t s) {
  const size_t smem = (size_t)B * CH * 256 * sizeof(T);
  const int want = (prm.n + kGemvWarps - 1) / kGemvWarps;
  const int grid = want < 4096 ? want : 4096;
  auto go = [&](auto kern) -> int {
    if (smem > 48 * 1024) {
      const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return (int)e;
    }
    const cudaError_t e = launch_pdl(kern, dim3(grid), dim3(kGemvThreads), smem, s, prm);
    note_launch();
    return e == cudaSuccess ? KANI_OK : (int)e;
  };
  if (epi == 2) {  // the conv epilogue only follows the normed in_proj (K = hidden)
    if constexpr (CH == 4) return norm ? go(gemv_kernel<T, B, CH, true, 2>) : go(gemv_kernel<T, B, CH, false, 2>);
    return KANI_ERR_UNSUPPORTED;
  }
  if (norm) return epi ? go(gemv_kernel<T, B, CH, true, 1>) : go(gemv_kernel<T, B, CH, true, 0>);
  return epi ? go(gemv_kernel<T, B, CH, false, 1>) : go(gemv_kernel<T, B, CH, false, 0>);
}

template <typename T, int B>
int launch_gemv_b(const GemvParams& prm, bool norm, int epi, cudaStream_t s) {
  switch (prm.k) {
    case 1024: return launch_gemv_bk<T, B, 4>(prm, norm, epi, s);
    case 4608: return launch_gemv_bk<T, B, 18>(prm, norm, epi, s);
    default: return KANI_ERR_UNSUPPORTED;
  }
}

template <typename T>
int launch_gemv(const GemvParams& prm, bool norm, int epi, cudaStream_t s) {
  if (prm.batch <= 1) return launch_gemv_b<T, 1>(prm, norm, epi, s);
  if (prm.batch <= 2) return launch_gemv_b<T, 2>(prm, norm, epi, s);
  if (prm.batch <= 4) return launch_gemv_b<T, 4>(prm, norm, epi, s);
  return launch_gemv_b<T, 8>(prm, norm, epi, s);
}

// argument checks shared by both entry points
int check_gemv(int32_t dtype, const void* x, int64_t x_row_stride, const void* residual, int64_t residual_row_stride,
               void* residual_out, int64_t residual_out_row_stride, const void* norm_weight, const void* weight,
               int64_t weight_row_stride, int32_t n_out, int32_t k, int64_t batch, const void* y,
               int64_t y_row_stride) {
  if (!x || !weight || !y) return KANI_ERR_INVALID_ARG;
  if ((residual || residual_out) && !norm_weight) return KANI_ERR_INVALID_ARG;  // the add belongs to the norm
  if (residual_out && (residual_out == residual || residual_out == x)) return KANI_ERR_INVALID_ARG;
  if (batch > kGemvMaxB) return KANI_ERR_UNSUPPORTED;
  if (dtype != KANI_DTYPE_BF16 && dtype != KANI_DTYPE_F16)
    return dtype == KANI_DTYPE_F32 ? KANI_ERR_UNSUPPORTED : KANI_ERR_DTYPE;
  if (weight_row_stride < k || (batch > 1 && (x_row_stride < k || y_row_stride < n_out)) ||
      (residual && batch > 1 && residual_row_stride < k) || (residual_out && batch > 1 && residual_out_row_stride < k))
    return KANI_ERR_INVALID_ARG;
  if (!aligned16(x) || !aligned16(weight) || x_row_stride % 8 != 0 || weight_row_stride % 8 != 0 ||
      (residual && (!aligned16(residual) || residual_row_stride % 8 != 0)) ||
      (residual_out && (!aligned16(residual_out) || residual_out_row_stride % 8 != 0)) ||
      (norm_weight && !aligned16(norm_weight)))
    return KANI_ERR_UNSUPPORTED;
  return KANI_OK;
}

}  // namespace
}  // namespace kani

extern "C" int kani_gemv(int32_t dtype, const void* x, int64_t x_row_stride, const void* residual,
                         int64_t residual_row_stride, void* residual_out, int64_t residual_out_row_stride,
                         const void* norm_weight, float eps, const void* weight, int64_t weight_row_stride,
                         int32_t n_out, int32_t k, int64_t batch, int32_t silu_pairs, void* y, int64_t y_row_stride,
                         void* stream) {
  if (batch < 0 || n_out < 0 || k < 0) return KANI_ERR_INVALID_ARG;
  if (batch == 0 || n_out == 0) return KANI_OK;
  const int rc = kani::check_gemv(dtype, x, x_row_stride, residual, residual_row_stride, residual_out,
                                  residual_out_row_stride, norm_weight, weight, weight_row_stride, n_out, k, batch, y,
                                  y_row_stride);
  if (rc != KANI_OK) return rc;
  kani::GemvParams prm{x, x_row_stride, residual, residual_row_stride, residual_out, residual_out_row_stride,
                       norm_weight, eps, weight, weight_row_stride, n_out, k, (int)batch, y, y_row_stride,
                       nullptr, 0, nullptr};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool norm = norm_weight != nullptr;
  const int epi = silu_pairs != 0 ? 1 : 0;
  if (dtype == KANI_DTYPE_BF16) return kani::launch_gemv<__nv_bfloat16>(prm, norm, epi, s);
  return kani::launch_gemv<__half>(prm, norm, epi, s);
}

extern "C" int kani_gemv_short_conv(int32_t dtype, const void* x, int64_t x_row_stride, const void* residual,
                                    int64_t residual_row_stride, void* residual_out, int64_t residual_out_row_stride,
                                    const void* norm_weight, float eps, const void* in_proj_weight,
                                    int64_t weight_row_stride, int32_t hidden, int32_t k, int64_t batch,
                                    void* conv_state, int64_t conv_state_batch_stride, const void* conv_weight,
                                    int32_t kernel_len, void* y, int64_t y_row_stride, void* stream) {
  if (batch < 0 || hidden < 0 || k < 0) return KANI_ERR_INVALID_ARG;
  if (batch == 0 || hidden == 0) return KANI_OK;
  if (!conv_state || !conv_weight) return KANI_ERR_INVALID_ARG;
  if (kernel_len != kani::kConvL) return KANI_ERR_UNSUPPORTED;
  if (batch > 1 && conv_state_batch_stride < (int64_t)hidden * kernel_len) return KANI_ERR_INVALID_ARG;
  const int rc = kani::check_gemv(dtype, x, x_row_stride, residual, residual_row_stride, residual_out,
                                  residual_out_row_stride, norm_weight, in_proj_weight, weight_row_stride, hidden, k,
                                  batch, y, y_row_stride);
  if (rc != KANI_OK) return rc;
  kani::GemvParams prm{x, x_row_stride, residual, residual_row_stride, residual_out, residual_out_row_stride,
                       norm_weight, eps, in_proj_weight, weight_row_stride, hidden, k, (int)batch, y, y_row_stride,
                       conv_state, conv_state_batch_stride, conv_weight};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool norm = norm_weight != nullptr;
  if (dtype == KANI_DTYPE_BF16) return kani::launch_gemv<__nv_bfloat16>(prm, norm, 2, s);
  return kani::launch_gemv<__half>(prm, norm, 2, s);
}
