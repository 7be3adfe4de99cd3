// The input prologue of the decode GEMVs and the fused head (sm_100a): the B
// input rows of a GEMV staged in shared memory, optionally as the residual
// add + RMSNorm of kani_add_rms_norm folded in front of it.  Included by
// gemv.cu and head_argmax.cu, so the projections and the head normalise
// with the same arithmetic.
#pragma once

#include "common.cuh"

namespace kani {
namespace {

// What the prologue reads: x (the GEMV input, or the residual-stream update
// with a norm), the residual it is added to, where the sum goes (CTA 0
// writes it; may be null), the norm weight (null: no norm) and eps.
struct NormIn {
  const void* x;
  int64_t x_stride;
  const void* res;
  int64_t res_stride;
  void* res_out;
  int64_t res_out_stride;
  const void* norm_w;
  float eps;
  int batch;
};

// The B GEMV input rows into shared memory (as, [B][K]); with NORM the
// residual add (h written to res_out by CTA 0) and the RMSNorm.  nw0 is the
// norm-weight chunk of this thread's first row chunk (v = tid), fetched by the
// caller before the programmatic-launch wait.  Ends with a barrier.
template <typename T, int B, int K, bool NORM, int NT>
__device__ __forceinline__ void stage_input(const NormIn& p, T* as, float (*s_part)[B], int tid, int lane,
                                            int warp, uint4 nw0) {
  constexpr int E = 8;
  if constexpr (!NORM) {
    for (int v = tid; v < B * K / E; v += NT) {
      const int b = v / (K / E), c = v % (K / E);
      uint4 x = make_uint4(0u, 0u, 0u, 0u);
      if (b < p.batch) x = ld16(static_cast<const T*>(p.x) + (int64_t)b * p.x_stride + c * E);
      reinterpret_cast<uint4*>(as)[v] = x;
    }
  } else {
    float ss[B];
#pragma unroll
    for (int b = 0; b < B; ++b) ss[b] = 0.f;
    for (int v = tid; v < B * K / E; v += NT) {
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
    for (int v = tid; v < B * K / E; v += NT) {
      const int b = v / (K / E), c = v % (K / E);
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < (NT / 32); ++w) tot += s_part[w][b];
      const float rr = 1.0f / sqrtf(tot / (float)K + p.eps);
      float h[E], wf[E];
      unpack16<T>(reinterpret_cast<const uint4*>(as)[v], h);
      unpack16<T>(v == tid ? nw0 : ld16_ro(static_cast<const T*>(p.norm_w) + c * E), wf);
#pragma unroll
      for (int e = 0; e < E; ++e) h[e] = __fmul_rn(__fmul_rn(h[e], rr), wf[e]);
      reinterpret_cast<uint4*>(as)[v] = pack16<T>(h);
    }
  }
  __syncthreads();

}

// The norm-weight chunk stage_input's thread `tid` applies first (a weight:
// fetched before the programmatic-launch wait, like the matrix rows).
template <typename T, int B, int K, bool NORM>
__device__ __forceinline__ uint4 first_norm_chunk(const NormIn& p, int tid) {
  if (!NORM || tid >= B * K / 8) return make_uint4(0u, 0u, 0u, 0u);
  return ld16_ro(static_cast<const T*>(p.norm_w) + (tid % (K / 8)) * 8);
}

}  // namespace
}  // namespace kani
