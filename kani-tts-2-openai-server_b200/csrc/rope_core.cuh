// RoPE building blocks shared by the RoPE + KV-write kernels (rope_kv.cu) and
// the QKV GEMV whose epilogue applies them (gemv.cu): the launch parameters,
// per-token metadata, the sin/cos of the rotary angles and the per-chunk
// norm + rotate-half + frame term + store.  The arithmetic is described in
// rope_kv.cu.
#pragma once

#include "common.cuh"

namespace kani {
namespace {

struct RopeParams {
  int64_t n_tokens;
  int64_t seq_tokens;
  int hq, hk, d;
  const void* q;
  int64_t qts;
  const void* k;
  int64_t kts;
  const void* v;
  int64_t vts;
  const float* inv_freq;
  const int64_t* positions;
  const void* cos;
  const void* sin;
  const void* qw;
  const void* kw;
  float eps;
  const void* table;
  int64_t table_rows;
  const int64_t* frame_pos;
  int tpf;
  int tpf_shift;  // log2(tpf) when tpf is a power of two, else -1
  void* q_out;
  int64_t qots, qohs;
  void* k_cache;
  void* v_cache;
  int64_t cbs, chs, css, clen;
  const int64_t* slots;
  int32_t* err;
  long long wait_cycles;  // bound of the bulk kernel's first mbarrier wait (WaitBound)
  unsigned wait_suspend_ns;
};

struct TokenMeta {
  int64_t b;
  int64_t slot;
  int64_t frame;
  bool slot_ok;
  bool frame_ok;
};

// Stream index and frame row of token t.  The divisions are avoided in the
// usual cases (one stream, one token per stream, power-of-two tokens per
// frame): a 64-bit division is a long software sequence on the GPU.
template <bool TABLE>
__device__ __forceinline__ TokenMeta token_meta(const RopeParams& p, int64_t t) {
  TokenMeta m;
  if (p.seq_tokens == 1) m.b = t;
  else if (p.n_tokens == p.seq_tokens) m.b = 0;
  else m.b = t / p.seq_tokens;
  m.slot = p.slots ? p.slots[t] : (t - m.b * p.seq_tokens);
  m.slot_ok = m.slot >= 0 && m.slot < p.clen;
  m.frame = 0;
  m.frame_ok = true;
  if constexpr (TABLE) {
    const int64_t fp = p.frame_pos ? p.frame_pos[t] : p.positions[t];
    m.frame = fp < 0 ? -1 : (p.tpf_shift >= 0 ? (fp >> p.tpf_shift) : fp / p.tpf);
    m.frame_ok = m.frame >= 0 && m.frame < p.table_rows;
  }
  return m;
}

// Same as token_meta, from already-loaded position / slot / frame values.
template <bool TABLE>
__device__ __forceinline__ TokenMeta token_meta_vals(const RopeParams& p, int64_t t, int64_t slot,
                                                     int64_t fp) {
  TokenMeta m;
  if (p.seq_tokens == 1) m.b = t;
  else if (p.n_tokens == p.seq_tokens) m.b = 0;
  else m.b = t / p.seq_tokens;
  m.slot = slot;
  m.slot_ok = m.slot >= 0 && m.slot < p.clen;
  m.frame = 0;
  m.frame_ok = true;
  if constexpr (TABLE) {
    m.frame = fp < 0 ? -1 : (p.tpf_shift >= 0 ? (fp >> p.tpf_shift) : fp / p.tpf);
    m.frame_ok = m.frame >= 0 && m.frame < p.table_rows;
  }
  return m;
}

template <bool TABLE>
__device__ __forceinline__ void flag_token(const RopeParams& p, const TokenMeta& m) {
  if (p.err == nullptr) return;
  int bits = 0;
  if (!m.slot_ok) bits |= KANI_FLAG_SLOT_OOB;
  if (TABLE && !m.frame_ok) bits |= KANI_FLAG_FRAME_OOB;
  if (bits) atomicOr(p.err, bits);
}

__device__ __forceinline__ float rrms_of(float ss, int n, float eps) {
  return 1.0f / sqrtf(ss / (float)n + eps);
}

// sin and cos of one fp32 angle with a shared argument reduction.
// Method: Cody-Waite reduction by pi/2 (W. J. Cody and W. Waite, "Software
// Manual for the Elementary Functions", 1980) in its fused-multiply-add form:
// pi/2 = C1 + C2 + C3 with C1 = fp32(pi/2), C2 = fp32(pi/2 - C1),
// C3 = fp32(pi/2 - C1 - C2); then the Taylor series of sin and cos on
// [-pi/4, pi/4] (through x^11 and x^12; truncation below 2^-30), then the
// quadrant swap and signs.  Measured against float64 sin/cos over
// |x| <= 65536: <= 1.5 fp32 ulp.  Larger angles (not produced by the decode
// positions of this model family) use sinf / cosf.
__device__ __forceinline__ void sincos_reduced(float x, float* s_out, float* c_out) {
  if (!(fabsf(x) <= 65536.0f)) {  // also catches NaN / inf
    *s_out = sinf(x);
    *c_out = cosf(x);
    return;
  }
  const float n = rintf(x * 0.636619746685028076f);  // x * fp32(2/pi)
  float r = fmaf(-n, 1.57079637050628662f, x);
  r = fmaf(-n, -4.37113882867379300e-08f, r);
  r = fmaf(-n, -1.71512451000588189e-15f, r);
  const float r2 = r * r;
  // sin r = r (1 - r2/3! + r2^2/5! - r2^3/7! + r2^4/9! - r2^5/11!)
  float ps = fmaf(r2, -2.5052108385441720e-8f, 2.7557319223985891e-6f);
  ps = fmaf(r2, ps, -1.9841269841269841e-4f);
  ps = fmaf(r2, ps, 8.3333333333333333e-3f);
  ps = fmaf(r2, ps, -1.6666666666666667e-1f);
  const float sr = fmaf(r * r2, ps, r);
  // cos r = 1 - r2/2! + r2^2/4! - r2^3/6! + r2^4/8! - r2^5/10! + r2^6/12!
  float pc = fmaf(r2, 2.0876756987868099e-9f, -2.7557319223985891e-7f);
  pc = fmaf(r2, pc, 2.4801587301587302e-5f);
  pc = fmaf(r2, pc, -1.3888888888888889e-3f);
  pc = fmaf(r2, pc, 4.1666666666666667e-2f);
  pc = fmaf(r2, pc, -0.5f);
  const float cr = fmaf(r2, pc, 1.0f);
  const int q = static_cast<int>(n) & 3;
  const float sv = (q & 1) ? cr : sr;
  const float cv = (q & 1) ? sr : cr;
  *s_out = (q & 2) ? -sv : sv;
  *c_out = ((q + 1) & 2) ? -cv : cv;
}

// cos/sin (rounded to T) of frequencies jj*E .. jj*E+E-1 at angle position
// posf.  Lane = hh * L + jj: the 32/L lanes that share chunk jj compute the E
// values between them (one sincos each when 32/L >= E) and exchange them
// with shuffles.  Every lane of the warp must call this.  LOG2L_CT >= 0 fixes
// the lane geometry at compile time (constant shuffle sources); -1 reads it
// from log2l.  `own_freq` holds the lane's frequencies for each round
// (lane_freqs below), loaded ahead of time so no global load sits on the
// critical path.
template <typename T, int LOG2L_CT>
struct LaneFreqs {
  static constexpr int E = VecN<T>::value;
  static constexpr int R = LOG2L_CT >= 0 ? (E + (32 >> LOG2L_CT) - 1) / (32 >> LOG2L_CT) : E;
  float f[R];
};

template <typename T, int LOG2L_CT>
__device__ __forceinline__ LaneFreqs<T, LOG2L_CT> lane_freqs(const float* __restrict__ inv_freq, int log2l_rt,
                                                             int lane) {
  constexpr int E = VecN<T>::value;
  LaneFreqs<T, LOG2L_CT> lf;
  const int log2l = LOG2L_CT >= 0 ? LOG2L_CT : log2l_rt;
  const int log2g = 5 - log2l;
  const int G = 1 << log2g;
  const int hh = lane >> log2l;
  const int jj = lane & ((1 << log2l) - 1);
#pragma unroll
  for (int r = 0; r < LaneFreqs<T, LOG2L_CT>::R; ++r) {
    const int e_own = r * G + hh;
    lf.f[r] = e_own < E ? __ldg(inv_freq + jj * E + e_own) : 0.f;
  }
  return lf;
}

template <typename T, int LOG2L_CT>
__device__ __forceinline__ void warp_cos_sin(const LaneFreqs<T, LOG2L_CT>& lf, float posf, int log2l_rt,
                                             int lane, float* cs, float* sn) {
  constexpr int E = VecN<T>::value;
  const int log2l = LOG2L_CT >= 0 ? LOG2L_CT : log2l_rt;
  const int log2g = 5 - log2l;
  const int G = 1 << log2g;
  const int hh = lane >> log2l;
  const int jj = lane & ((1 << log2l) - 1);
  const int rounds = (E + G - 1) >> log2g;
#pragma unroll
  for (int r = 0; r < LaneFreqs<T, LOG2L_CT>::R; ++r) {
    if (LOG2L_CT < 0 && r >= rounds) break;
    float cv = 0.f, sv = 0.f;
    if (r * G + hh < E) {
      float sr, cr;
      sincos_reduced(__fmul_rn(lf.f[r], posf), &sr, &cr);
      cv = round_to<T>(cr);
      sv = round_to<T>(sr);
    }
#pragma unroll
    for (int e = 0; e < E; ++e) {
      if ((e >> log2g) == r) {  // uniform across the warp (constant with LOG2L_CT)
        const int src = ((e & (G - 1)) << log2l) | jj;
        cs[e] = __shfl_sync(0xffffffffu, cv, src);
        sn[e] = __shfl_sync(0xffffffffu, sv, src);
      }
    }
  }
}

// One lane's two chunks (elements [lo, lo+E) and [hi, hi+E)) of one head:
// optional RMSNorm (an L-lane shuffle tree over the head, so every lane of
// the warp must call this, live or not), rotate-half, optional frame term,
// one rounding, store at dst + lo / dst + hi.  The arithmetic runs on
// sm_100's paired fp32 units (__fmul2_rn / __fadd2_rn: two independent
// round-to-nearest operations per instruction, bit-identical to the scalar
// form).  nsn holds -sin.
// rope_chunk_store_w takes the two norm-weight chunks (elements [lo, lo+E)
// and [hi, hi+E) of the head-norm weight) already loaded, so a caller can
// fetch them ahead of time; rope_chunk_store loads them from nw.
template <typename T, bool NORM, bool TABLE>
__device__ __forceinline__ void rope_chunk_store_w(uint4 xlo, uint4 xhi, bool live, const float* cs,
                                                   const float* nsn, const float* sn, const float* pl,
                                                   const float* ph, bool frame_ok, uint4 nwlo, uint4 nwhi,
                                                   int lo, int hi, int log2l, int d, float eps, T* dst) {
  constexpr int E = VecN<T>::value;
  float a[E], b[E];
  unpack16<T>(xlo, a);
  unpack16<T>(xhi, b);
  if constexpr (NORM) {
    float ss = 0.f;
    if (live) {
#pragma unroll
      for (int e = 0; e < E; ++e) {
        ss = fmaf(a[e], a[e], ss);
        ss = fmaf(b[e], b[e], ss);
      }
    }
    for (int off = (1 << log2l) >> 1; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (live) {
      float wl[E], wh[E];
      unpack16<T>(nwlo, wl);
      unpack16<T>(nwhi, wh);
      const float r = rrms_of(ss, d, eps);
      const float2 r2 = make_float2(r, r);
#pragma unroll
      for (int e = 0; e < E; e += 2) {
        const float2 na = __fmul2_rn(__fmul2_rn(make_float2(a[e], a[e + 1]), r2), make_float2(wl[e], wl[e + 1]));
        const float2 nb = __fmul2_rn(__fmul2_rn(make_float2(b[e], b[e + 1]), r2), make_float2(wh[e], wh[e + 1]));
        a[e] = round_to<T>(na.x);
        a[e + 1] = round_to<T>(na.y);
        b[e] = round_to<T>(nb.x);
        b[e + 1] = round_to<T>(nb.y);
      }
    }
  }
  if (!live) return;
  float ylo[E], yhi[E];
#pragma unroll
  for (int e = 0; e < E; e += 2) {
    const float2 a2 = make_float2(a[e], a[e + 1]);
    const float2 b2 = make_float2(b[e], b[e + 1]);
    const float2 c2 = make_float2(cs[e], cs[e + 1]);
    const float2 s2 = make_float2(sn[e], sn[e + 1]);
    const float2 n2 = make_float2(nsn[e], nsn[e + 1]);
    float2 l2 = __fadd2_rn(__fmul2_rn(a2, c2), __fmul2_rn(b2, n2));  // a cos - b sin
    float2 h2 = __fadd2_rn(__fmul2_rn(b2, c2), __fmul2_rn(a2, s2));  // b cos + a sin
    if constexpr (TABLE) {
      if (frame_ok) {
        l2 = __fadd2_rn(l2, make_float2(pl[e], pl[e + 1]));
        h2 = __fadd2_rn(h2, make_float2(ph[e], ph[e + 1]));
      }
    }
    ylo[e] = l2.x;
    ylo[e + 1] = l2.y;
    yhi[e] = h2.x;
    yhi[e + 1] = h2.y;
  }
  st16(dst + lo, pack16<T>(ylo));
  st16(dst + hi, pack16<T>(yhi));
}

template <typename T, bool NORM, bool TABLE>
__device__ __forceinline__ void rope_chunk_store(uint4 xlo, uint4 xhi, bool live, const float* cs,
                                                 const float* nsn, const float* sn, const float* pl,
                                                 const float* ph, bool frame_ok, const T* nw, int lo,
                                                 int hi, int log2l, int d, float eps, T* dst) {
  uint4 wlo = make_uint4(0u, 0u, 0u, 0u), whi = wlo;
  if constexpr (NORM) {
    if (live) {
      wlo = ld16_ro(nw + lo);
      whi = ld16_ro(nw + hi);
    }
  }
  rope_chunk_store_w<T, NORM, TABLE>(xlo, xhi, live, cs, nsn, sn, pl, ph, frame_ok, wlo, whi, lo, hi, log2l, d, eps,
                                     dst);
}

}  // namespace
}  // namespace kani
