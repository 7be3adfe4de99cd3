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
#include "gemv_input.cuh"
#include "rope_core.cuh"

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
  L2Prefetch pf;       // later launches' weights, prefetched into L2 at entry
};

constexpr int kConvL = 3;  // the LFM2 short-conv kernel length the fused epilogue serves

// EPI: 0 = store, 1 = SiLU·mul of the gate / up rows r and n + r,
//      2 = gated short-conv step of channel r over rows r (B), n + r (C), 2n + r (x)
template <typename T, int B, int CH, bool NORM, int EPI, int NT = kGemvThreads>
__global__ void __launch_bounds__(NT) gemv_kernel(GemvParams p) {
  constexpr int NW = NT / 32;
  constexpr int E = 8;
  constexpr int K = CH * 256;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ float s_part[NW][B];
  T* as = reinterpret_cast<T*>(smem_raw);  // [B][K] GEMV input
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  // ---- the weights do not depend on earlier launches: start this warp's
  //      first row streaming before waiting for them (programmatic dependent
  //      launch), then let the next launch start its own weight stream
  const T* W = static_cast<const T*>(p.w);
  constexpr int NR = EPI == 0 ? 1 : (EPI == 1 ? 2 : 3);
  int r = blockIdx.x * NW + warp;
  uint4 wv[NR][CH];
  auto load_row = [&](int row) {
#pragma unroll
    for (int q = 0; q < NR; ++q)
#pragma unroll
      for (int c = 0; c < CH; ++c)
        wv[q][c] = ld16_stream(W + (int64_t)(row + q * p.n) * p.w_stride + c * 256 + lane * E);
  };
  if (r < p.n) load_row(r);
  const NormIn in{p.x, p.x_stride, p.res, p.res_stride, p.res_out, p.res_out_stride, p.norm_w, p.eps, p.batch};
  const uint4 nw0 = first_norm_chunk<T, B, K, NORM>(in, tid);
  // EPI 2: lane b's conv weights of the warp's first channel (before the wait)
  // and stream b's conv state of it (after the wait), fetched ahead of the dot
  // products instead of after them
  const int r_first = r;
  float cw0[kConvL] = {}, st0[kConvL] = {};
  if constexpr (EPI == 2) {
    if (r < p.n && lane < p.batch && lane < B) {
      const T* cw = static_cast<const T*>(p.conv_w) + (int64_t)r * kConvL;
#pragma unroll
      for (int i = 0; i < kConvL; ++i) cw0[i] = Elem<T>::to_f(cw[i]);
    }
  }
  l2_prefetch_share(p.pf);
  griddep_launch_dependents();
  griddep_wait();
  if constexpr (EPI == 2) {
    if (r < p.n && lane < p.batch && lane < B) {
      const T* st = static_cast<const T*>(p.conv_state) + (int64_t)lane * p.conv_state_stride + (int64_t)r * kConvL;
#pragma unroll
      for (int i = 0; i + 1 < kConvL; ++i) st0[i] = Elem<T>::to_f(st[i + 1]);
    }
  }

  stage_input<T, B, K, NORM, NT>(in, as, s_part, tid, lane, warp, nw0);

  // ---- one warp per output row (SILU: per gate/up pair); row r's weights
  //      are already in flight
  for (; r < p.n; r += gridDim.x * NW) {
    if (r != blockIdx.x * NW + warp) load_row(r);
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
          const bool pre = r == r_first;  // the first channel's state and weights are in registers
          float sv[kConvL], wc[kConvL];
#pragma unroll
          for (int i = 0; i + 1 < kConvL; ++i) sv[i] = pre ? st0[i] : Elem<T>::to_f(st[i + 1]);
#pragma unroll
          for (int i = 0; i < kConvL; ++i) wc[i] = pre ? cw0[i] : Elem<T>::to_f(cw[i]);
          sv[kConvL - 1] = round_to<T>(__fmul_rn(bg, xg));
          float conv = 0.f;
#pragma unroll
          for (int i = 0; i < kConvL; ++i) {
            st[i] = Elem<T>::from_f(sv[i]);
            conv = __fadd_rn(conv, round_to<T>(__fmul_rn(sv[i], wc[i])));
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

// ------------------------------------------------- QKV GEMV + RoPE + KV write
// One CTA per head of the packed QKV projection ([Q heads | K heads | V heads],
// D = 64 rows each): the 8 warps compute the head's 64 outputs for every
// stream (rows in the accumulation order of gemv_kernel), round them as
// F.linear stores them, and warp 0 finishes the head for each stream with the
// code of the RoPE + KV-write kernels: q/k RMSNorm, the rotary angles of the
// stream's position, rotate-half, the frame-table term, the store to q_out or
// to the cache slot (V heads: the copy).  Replaces the QKV F.linear and
// kani_rope_kv_write of the decode step (optimized_decode.py:215-240).
struct RopeKvParams {
  int hq, hk;
  const float* inv_freq;
  const int64_t* positions;  // [batch]
  const void* qw;
  const void* kw;
  float eps;
  const void* table;
  int64_t table_rows;
  const int64_t* frame_pos;  // [batch] or NULL (= positions)
  int tpf, tpf_shift;
  void* q_out;
  int64_t qobs, qohs;
  void* k_cache;
  void* v_cache;
  int64_t cbs, chs, css, clen;
  const int64_t* slots;  // [batch]
  int32_t* err;
};

constexpr int kRopeD = 64;  // head_dim the fused epilogue serves
constexpr int kRopeRowsPerWarp = kRopeD / kGemvWarps;

// NORM: the input RMSNorm prologue; QKN: the per-head q / k RMSNorm; TABLE: the frame term
//
// Everything that no earlier launch writes is fetched before the
// programmatic-launch wait: all 8 weight rows of each warp, and for warp 0
// the lane's rotary frequencies and the head-norm weight chunks.  Right after
// the wait warp 0 reads each stream's position, slot and frame-table row, so
// their latency overlaps the input norm and the dot products.
template <typename T, int B, int CH, bool NORM, bool QKN, bool TABLE>
__global__ void __launch_bounds__(kGemvThreads) gemv_rope_kv_kernel(GemvParams p, RopeKvParams r) {
  constexpr int E = 8;
  constexpr int K = CH * 256;
  constexpr int RW = kRopeRowsPerWarp;
  constexpr int LOG2L = 2;  // (D/2)/E = 4 lanes per head
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ float s_part[kGemvWarps][B];
  __shared__ __align__(16) T s_head[B][kRopeD];
  T* as = reinterpret_cast<T*>(smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int head = blockIdx.x;
  const T* W = static_cast<const T*>(p.w);
  const int row0 = head * kRopeD + warp * RW;

  uint4 wv[RW][CH];
#pragma unroll
  for (int q = 0; q < RW; ++q)
#pragma unroll
    for (int c = 0; c < CH; ++c) wv[q][c] = ld16_stream(W + (int64_t)(row0 + q) * p.w_stride + c * 256 + lane * E);
  const NormIn in{p.x, p.x_stride, p.res, p.res_stride, p.res_out, p.res_out_stride, p.norm_w, p.eps, p.batch};
  const uint4 nw0 = first_norm_chunk<T, B, K, NORM>(in, tid);
  // warp 0: lanes 0..3 carry the head's chunk pairs (lo, hi), the other lanes
  // help with the sin/cos
  const int jj = lane & 3;
  const bool mine = lane < 4;
  const int lo = jj * E, hi = kRopeD / 2 + jj * E;
  const bool is_q = head < r.hq, is_k = !is_q && head < r.hq + r.hk;
  const int kv = is_q ? 0 : (is_k ? head - r.hq : head - r.hq - r.hk);
  LaneFreqs<T, LOG2L> lf{};
  uint4 hwlo = make_uint4(0u, 0u, 0u, 0u), hwhi = hwlo;
  if (warp == 0 && (is_q || is_k)) {
    lf = lane_freqs<T, LOG2L>(r.inv_freq, LOG2L, lane);
    if constexpr (QKN) {
      const T* nw = static_cast<const T*>(is_q ? r.qw : r.kw);
      hwlo = ld16_ro(nw + lo);
      hwhi = ld16_ro(nw + hi);
    }
  }
  l2_prefetch_share(p.pf);
  griddep_launch_dependents();
  griddep_wait();

  int64_t pos[B], slot[B];
  uint4 plo[B], phi[B];
  bool frame_ok[B];
  if (warp == 0) {
#pragma unroll
    for (int b = 0; b < B; ++b) {
      pos[b] = 0;
      slot[b] = -1;
      frame_ok[b] = true;
      plo[b] = phi[b] = make_uint4(0u, 0u, 0u, 0u);
      if (b < p.batch) {
        pos[b] = r.positions[b];
        slot[b] = r.slots[b];
        if constexpr (TABLE) {
          const int64_t fp = r.frame_pos ? r.frame_pos[b] : pos[b];
          const int64_t frame = fp < 0 ? -1 : (r.tpf_shift >= 0 ? (fp >> r.tpf_shift) : fp / r.tpf);
          frame_ok[b] = frame >= 0 && frame < r.table_rows;
          if (frame_ok[b] && mine && (is_q || is_k)) {
            const T* pr = static_cast<const T*>(r.table) + frame * kRopeD;
            plo[b] = ld16_ro(pr + lo);
            phi[b] = ld16_ro(pr + hi);
          }
        }
      }
    }
  }
  stage_input<T, B, K, NORM, kGemvThreads>(in, as, s_part, tid, lane, warp, nw0);

  float acc[RW][B];
#pragma unroll
  for (int q = 0; q < RW; ++q)
#pragma unroll
    for (int b = 0; b < B; ++b) acc[q][b] = 0.f;
#pragma unroll
  for (int c = 0; c < CH; ++c) {
#pragma unroll
    for (int b = 0; b < B; ++b) {
      float af[E];
      unpack16<T>(reinterpret_cast<const uint4*>(as + b * K + c * 256)[lane], af);
#pragma unroll
      for (int q = 0; q < RW; ++q) {
        float wf[E];
        unpack16<T>(wv[q][c], wf);
#pragma unroll
        for (int e = 0; e < E; ++e) acc[q][b] = fmaf(wf[e], af[e], acc[q][b]);
      }
    }
  }
#pragma unroll
  for (int q = 0; q < RW; ++q)
#pragma unroll
    for (int b = 0; b < B; ++b) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[q][b] += __shfl_xor_sync(0xffffffffu, acc[q][b], o);
      if (lane == 0) s_head[b][warp * RW + q] = Elem<T>::from_f(acc[q][b]);
    }
  __syncthreads();
  if (warp != 0) return;

  // warp 0 finishes the head, one stream after another
#pragma unroll
  for (int b = 0; b < B; ++b) {
    if (b >= p.batch) break;
    const bool slot_ok = slot[b] >= 0 && slot[b] < r.clen;
    if (lane == 0 && r.err && (head == r.hq || (head == 0 && TABLE))) {
      int bits = 0;
      if (head == r.hq && !slot_ok) bits |= KANI_FLAG_SLOT_OOB;
      if (TABLE && head == 0 && !frame_ok[b]) bits |= KANI_FLAG_FRAME_OOB;
      if (bits) atomicOr(r.err, bits);
    }
    const uint4 xlo = *reinterpret_cast<const uint4*>(&s_head[b][lo]);
    const uint4 xhi = *reinterpret_cast<const uint4*>(&s_head[b][hi]);
    if (!is_q && !is_k) {  // V head: copy into the cache slot
      if (mine && slot_ok) {
        T* dst = static_cast<T*>(r.v_cache) + b * r.cbs + kv * r.chs + slot[b] * r.css;
        st16(dst + lo, xlo);
        st16(dst + hi, xhi);
      }
      continue;
    }
    float cs[E], sn[E], nsn[E], pl[E], ph[E];
    warp_cos_sin<T, LOG2L>(lf, (float)pos[b], LOG2L, lane, cs, sn);
#pragma unroll
    for (int e = 0; e < E; ++e) nsn[e] = -sn[e];
    if constexpr (TABLE) {
      unpack16<T>(plo[b], pl);
      unpack16<T>(phi[b], ph);
    }
    T* dst = is_q ? static_cast<T*>(r.q_out) + b * r.qobs + head * r.qohs
                  : static_cast<T*>(r.k_cache) + b * r.cbs + kv * r.chs + slot[b] * r.css;
    const bool live = mine && (is_q || slot_ok);
    rope_chunk_store_w<T, QKN, TABLE>(xlo, xhi, live, cs, nsn, sn, pl, ph, frame_ok[b], hwlo, hwhi, lo, hi, LOG2L,
                                      kRopeD, r.eps, dst);
  }
}

#ifndef KANI_GATE_UP_THREADS
#define KANI_GATE_UP_THREADS 512
#endif
// Block size of the gate/up (SiLU·mul) GEMV at one stream.  Every CTA reads
// and normalises the same input row, so 576 CTAs of 256 threads hammer the
// same few L2 lines; 288 CTAs of 512 threads (the same warps, one row pair
// each, every weight still requested before the launch wait) measured
// 233.3-233.7 against 235.7-235.8 us per bs = 1 step, 144 of 1024 threads
// 242.9-244.1.
constexpr int kGateUpThreads = KANI_GATE_UP_THREADS;

template <typename T, int B, int CH>
int launch_gemv_bk(const GemvParams& prm, bool norm, int epi, cudaStream_t s) {
  const size_t smem = (size_t)B * CH * 256 * sizeof(T);
  auto go = [&](auto kern, int nt = kGemvThreads) -> int {
    const int nw = nt / 32;
    const int want = (prm.n + nw - 1) / nw;
    const int grid = want < 4096 ? want : 4096;
    if (smem > 48 * 1024) {
      const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return (int)e;
    }
    const cudaError_t e = launch_pdl(kern, dim3(grid), dim3(nt), smem, s, prm);
    note_launch();
    return e == cudaSuccess ? KANI_OK : (int)e;
  };
  if constexpr (B == 1 && kGateUpThreads != kGemvThreads) {
    if (epi == 1 && norm) return go(gemv_kernel<T, B, CH, true, 1, kGateUpThreads>, kGateUpThreads);
  }
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
  const kani::L2Prefetch pf = kani::take_l2_prefetch();
  if (batch < 0 || n_out < 0 || k < 0) return KANI_ERR_INVALID_ARG;
  if (batch == 0 || n_out == 0) return KANI_OK;
  const int rc = kani::check_gemv(dtype, x, x_row_stride, residual, residual_row_stride, residual_out,
                                  residual_out_row_stride, norm_weight, weight, weight_row_stride, n_out, k, batch, y,
                                  y_row_stride);
  if (rc != KANI_OK) return rc;
  kani::GemvParams prm{x, x_row_stride, residual, residual_row_stride, residual_out, residual_out_row_stride,
                       norm_weight, eps, weight, weight_row_stride, n_out, k, (int)batch, y, y_row_stride,
                       nullptr, 0, nullptr, pf};
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
  const kani::L2Prefetch pf = kani::take_l2_prefetch();
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
                       conv_state, conv_state_batch_stride, conv_weight, pf};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool norm = norm_weight != nullptr;
  if (dtype == KANI_DTYPE_BF16) return kani::launch_gemv<__nv_bfloat16>(prm, norm, 2, s);
  return kani::launch_gemv<__half>(prm, norm, 2, s);
}

namespace kani {
namespace {

template <typename T, int B, bool NORM, bool QKN, bool TABLE>
int launch_rope_kv_b(const GemvParams& prm, const RopeKvParams& r, cudaStream_t s) {
  constexpr int CH = 4;  // K = 1024
  const size_t smem = (size_t)B * CH * 256 * sizeof(T);
  auto kern = gemv_rope_kv_kernel<T, B, CH, NORM, QKN, TABLE>;
  const int grid = r.hq + 2 * r.hk;
  const cudaError_t e = launch_pdl(kern, dim3(grid), dim3(kGemvThreads), smem, s, prm, r);
  note_launch();
  return e == cudaSuccess ? KANI_OK : (int)e;
}

template <typename T, bool NORM, bool QKN, bool TABLE>
int launch_rope_kv_t(const GemvParams& prm, const RopeKvParams& r, cudaStream_t s) {
  if (prm.batch <= 1) return launch_rope_kv_b<T, 1, NORM, QKN, TABLE>(prm, r, s);
  if (prm.batch <= 2) return launch_rope_kv_b<T, 2, NORM, QKN, TABLE>(prm, r, s);
  return launch_rope_kv_b<T, 4, NORM, QKN, TABLE>(prm, r, s);
}

template <typename T>
int launch_rope_kv(const GemvParams& prm, const RopeKvParams& r, bool norm, bool qkn, bool table, cudaStream_t s) {
  // the decode step always normalises the input; the head norm and the table vary
  if (!norm) return KANI_ERR_UNSUPPORTED;
  if (qkn) return table ? launch_rope_kv_t<T, true, true, true>(prm, r, s) : launch_rope_kv_t<T, true, true, false>(prm, r, s);
  return table ? launch_rope_kv_t<T, true, false, true>(prm, r, s) : launch_rope_kv_t<T, true, false, false>(prm, r, s);
}

}  // namespace
}  // namespace kani

extern "C" int kani_gemv_rope_kv(int32_t dtype, const void* x, int64_t x_row_stride, const void* residual,
                                 int64_t residual_row_stride, void* residual_out, int64_t residual_out_row_stride,
                                 const void* norm_weight, float eps, const void* qkv_weight,
                                 int64_t weight_row_stride, int32_t k, int64_t batch, int32_t num_q_heads,
                                 int32_t num_kv_heads, int32_t head_dim, const float* inv_freq,
                                 const int64_t* positions, const void* q_norm_w, const void* k_norm_w,
                                 float head_eps, const void* frame_table, int64_t frame_rows,
                                 const int64_t* frame_pos, int32_t tokens_per_frame, void* q_out,
                                 int64_t q_out_batch_stride, int64_t q_out_head_stride, void* k_cache,
                                 void* v_cache, int64_t cache_batch_stride, int64_t cache_head_stride,
                                 int64_t cache_slot_stride, int64_t cache_len, const int64_t* slots,
                                 int32_t* err_flag, void* stream) {
  const kani::L2Prefetch pf = kani::take_l2_prefetch();
  if (batch < 0 || k < 0 || num_q_heads < 0 || num_kv_heads < 0) return KANI_ERR_INVALID_ARG;
  if (batch == 0) return KANI_OK;
  if (batch > 4 || k != 1024 || head_dim != kani::kRopeD || num_q_heads < 1 || num_kv_heads < 1)
    return KANI_ERR_UNSUPPORTED;
  if (!inv_freq || !positions || !q_out || !k_cache || !v_cache || !slots) return KANI_ERR_INVALID_ARG;
  if ((q_norm_w == nullptr) != (k_norm_w == nullptr)) return KANI_ERR_INVALID_ARG;
  if (frame_table && (frame_rows < 0 || tokens_per_frame < 1)) return KANI_ERR_INVALID_ARG;
  const int32_t n_rows = (num_q_heads + 2 * num_kv_heads) * head_dim;
  const int rc = kani::check_gemv(dtype, x, x_row_stride, residual, residual_row_stride, residual_out,
                                  residual_out_row_stride, norm_weight, qkv_weight, weight_row_stride, n_rows, k,
                                  batch, q_out, n_rows);
  if (rc != KANI_OK) return rc;
  if (!kani::aligned16(q_out) || !kani::aligned16(k_cache) || !kani::aligned16(v_cache) || q_out_head_stride % 8 ||
      q_out_batch_stride % 8 || cache_batch_stride % 8 || cache_head_stride % 8 || cache_slot_stride % 8 ||
      (q_norm_w && (!kani::aligned16(q_norm_w) || !kani::aligned16(k_norm_w))) ||
      (frame_table && !kani::aligned16(frame_table)))
    return KANI_ERR_UNSUPPORTED;
  kani::GemvParams prm{x, x_row_stride, residual, residual_row_stride, residual_out, residual_out_row_stride,
                       norm_weight, eps, qkv_weight, weight_row_stride, n_rows, k, (int)batch, q_out, 0,
                       nullptr, 0, nullptr, pf};
  int shift = -1;
  if (tokens_per_frame > 0 && (tokens_per_frame & (tokens_per_frame - 1)) == 0)
    for (shift = 0; (1 << shift) < tokens_per_frame; ++shift) {
    }
  kani::RopeKvParams r{num_q_heads, num_kv_heads, inv_freq, positions, q_norm_w, k_norm_w, head_eps, frame_table,
                       frame_rows, frame_pos, tokens_per_frame, shift, q_out, q_out_batch_stride, q_out_head_stride,
                       k_cache, v_cache, cache_batch_stride, cache_head_stride, cache_slot_stride, cache_len, slots,
                       err_flag};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool norm = norm_weight != nullptr, qkn = q_norm_w != nullptr, table = frame_table != nullptr;
  if (dtype == KANI_DTYPE_BF16) return kani::launch_rope_kv<__nv_bfloat16>(prm, r, norm, qkn, table, s);
  return kani::launch_rope_kv<__half>(prm, r, norm, qkn, table, s);
}
