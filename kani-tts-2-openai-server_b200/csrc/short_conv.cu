// LFM2 gated short-convolution decode step (sm_100a).
//
// Reference: the eager composition of kani_tts/optimized_decode.py:256-277
// (same as the patched Lfm2ShortConv decode branch, kani_tts/core.py:308-328):
//     B, C, x = chunk(in_proj(h), 3)          (the caller passes in_proj(h))
//     Bx      = round(B * x)
//     state   = roll(state, -1); state[:, :, L-1] = Bx      (written back)
//     conv    = round(sum_i round(state[:, :, i] * w[:, i]))  (fp32 sum)
//     y       = round(C * conv)
// with every product rounded to the storage type as the eager bf16 ops do,
// so the result matches the eager composition bit for bit (the three-term
// sum is accumulated left to right in fp32, as torch.sum does).
//
// One thread per 8 channels of one stream: 16-byte loads of B, C and x, the
// channel's L state values and weights, one 16-byte store of y and the state
// write-back.  Replaces ~8 eager launches per conv layer with one.
#include "common.cuh"

namespace kani {
namespace {

constexpr int kMaxL = 8;

template <typename T, int L>
__global__ void __launch_bounds__(128)
short_conv_kernel(const T* __restrict__ bcx, int64_t bcx_stride, T* __restrict__ state,
                  int64_t state_stride, const T* __restrict__ w, T* __restrict__ y, int64_t y_stride,
                  int64_t batch, int hidden) {
  constexpr int E = VecN<T>::value;
  griddep_launch_dependents();  // a dependent GEMV may start streaming its weights
  griddep_wait();               // launched as a programmatic dependent: the inputs come from the launch before
  const int groups = hidden / E;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= batch * groups) return;
  const int64_t b = idx / groups;
  const int c0 = (int)(idx - b * groups) * E;
  const T* row = bcx + b * bcx_stride;
  float bg[E], cg[E], xg[E];
  unpack16<T>(ld16(row + c0), bg);
  unpack16<T>(ld16(row + hidden + c0), cg);
  unpack16<T>(ld16(row + 2 * hidden + c0), xg);
  // state and weights of these E channels: E*L contiguous elements each,
  // moved as 16-byte vectors when E*L*sizeof(T) is a multiple of 16
  constexpr int BYTES = E * L * (int)sizeof(T);
  constexpr bool VEC = BYTES % 16 == 0;
  T* st = state + b * state_stride + (int64_t)c0 * L;
  const T* wr = w + (int64_t)c0 * L;
  union Row {
    T e[E * L];
    uint4 v[VEC ? BYTES / 16 : 1];
  } sv, wv;
  if constexpr (VEC) {
#pragma unroll
    for (int i = 0; i < BYTES / 16; ++i) {
      sv.v[i] = ld16(st + i * (16 / (int)sizeof(T)));
      wv.v[i] = ld16_ro(wr + i * (16 / (int)sizeof(T)));
    }
  } else {
#pragma unroll
    for (int i = 0; i < E * L; ++i) {
      sv.e[i] = st[i];
      wv.e[i] = wr[i];
    }
  }
  float out[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const float bx = round_to<T>(__fmul_rn(bg[e], xg[e]));
    float s[L];
#pragma unroll
    for (int i = 0; i + 1 < L; ++i) s[i] = Elem<T>::to_f(sv.e[e * L + i + 1]);
    s[L - 1] = bx;
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < L; ++i) {
      sv.e[e * L + i] = Elem<T>::from_f(s[i]);
      acc = __fadd_rn(acc, round_to<T>(__fmul_rn(s[i], Elem<T>::to_f(wv.e[e * L + i]))));
    }
    out[e] = __fmul_rn(cg[e], round_to<T>(acc));
  }
  if constexpr (VEC) {
#pragma unroll
    for (int i = 0; i < BYTES / 16; ++i) st16(st + i * (16 / (int)sizeof(T)), sv.v[i]);
  } else {
#pragma unroll
    for (int i = 0; i < E * L; ++i) st[i] = sv.e[i];
  }
  st16(y + b * y_stride + c0, pack16<T>(out));
}

template <typename T>
int launch_conv(const void* bcx, int64_t bcx_stride, void* state, int64_t state_stride, const void* w,
                void* y, int64_t y_stride, int64_t batch, int hidden, int L, cudaStream_t s) {
  constexpr int E = VecN<T>::value;
  if (hidden % E != 0 || !aligned16(bcx) || !aligned16(y) || bcx_stride % E != 0 || y_stride % E != 0 ||
      !aligned16(state) || !aligned16(w) || (state_stride * (int64_t)sizeof(T)) % 16 != 0)
    return KANI_ERR_UNSUPPORTED;
  const int64_t threads = batch * (hidden / E);
  const int64_t grid = (threads + 127) / 128;
  if (grid > 0x7fffffff) return KANI_ERR_UNSUPPORTED;
  const T* bp = static_cast<const T*>(bcx);
  T* sp = static_cast<T*>(state);
  const T* wp = static_cast<const T*>(w);
  T* yp = static_cast<T*>(y);
  switch (L) {
    case 2: launch_maybe_pdl(batch <= kPdlMaxRows, short_conv_kernel<T, 2>, dim3((unsigned)grid), dim3(128), 0, s, bp, bcx_stride, sp, state_stride, wp, yp, y_stride, batch, hidden); break;
    case 3: launch_maybe_pdl(batch <= kPdlMaxRows, short_conv_kernel<T, 3>, dim3((unsigned)grid), dim3(128), 0, s, bp, bcx_stride, sp, state_stride, wp, yp, y_stride, batch, hidden); break;
    case 4: launch_maybe_pdl(batch <= kPdlMaxRows, short_conv_kernel<T, 4>, dim3((unsigned)grid), dim3(128), 0, s, bp, bcx_stride, sp, state_stride, wp, yp, y_stride, batch, hidden); break;
    default: return KANI_ERR_UNSUPPORTED;
  }
  return launch_status();
}

}  // namespace
}  // namespace kani

extern "C" int kani_short_conv_step(int32_t dtype, const void* bcx, int64_t bcx_row_stride, void* state,
                                    int64_t state_batch_stride, const void* conv_w, void* y,
                                    int64_t y_row_stride, int64_t batch, int32_t hidden, int32_t kernel_len,
                                    void* stream) {
  if (batch < 0 || hidden < 0 || kernel_len < 0) return KANI_ERR_INVALID_ARG;
  if (batch == 0 || hidden == 0) return KANI_OK;
  if (!bcx || !state || !conv_w || !y) return KANI_ERR_INVALID_ARG;
  if (kernel_len < 2 || kernel_len > kani::kMaxL) return KANI_ERR_UNSUPPORTED;
  if (batch > 1 && (bcx_row_stride < 3 * (int64_t)hidden || y_row_stride < hidden ||
                    state_batch_stride < (int64_t)hidden * kernel_len))
    return KANI_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return kani::dispatch_dtype(dtype, [&]<typename T>() {
    return kani::launch_conv<T>(bcx, bcx_row_stride, state, state_batch_stride, conv_w, y, y_row_stride, batch,
                                hidden, kernel_len, s);
  });
}
