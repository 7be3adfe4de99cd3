// Rotary embedding of Q/K fused with the static KV-cache write (sm_100a).
//
// Reference algorithm, per token and head (all fp32, one rounding per store):
//   optional q/k RMSNorm of the head, rounded to the storage type
//       (kani_tts/optimized_decode.py:220-221 via triton_kernels.py:17-35)
//   angle_i = inv_freq[i] * float(pos)   for i < D/2, shared by both halves
//       (optimized_decode.py:229-232; inv_freq = bf16(theta^(-2i/D)) * alpha,
//        kani_tts/model.py:180-196, optimized_decode.py:104-111)
//   cos_i, sin_i rounded to the storage type (optimized_decode.py:233-234)
//   y_i = x_i*cos_i + sign_i * x_{(i+D/2)%D} * sin_i,  sign = -1 for i < D/2
//       (triton_kernels.py:121-130; the products and the sum are separately
//        rounded fp32 operations, no fused multiply-add)
//   optional frame term: y_i += table[frame, i] (fp32, before the one rounding)
//   K_rot and raw V are stored at cache[b, h, slot, :]
//       (static_cache.py:131-140).
//
// Vector kernel: a rope item is one lane holding the 16-byte vector of
// elements [jE, jE+E) of the first half of a head AND the matching vector of
// the second half, so the rotate-half partner is already in registers and no
// shuffle is needed.  A head is L = (D/2)/E lanes (bf16, D=64: 4 lanes); its
// sum of squares for the fused norm is an L-wide xor-shuffle tree.  Per token
// the items are [Q heads | K heads | V heads], padded to whole warps, so a
// head never straddles a warp and a token's K and V land in one CTA; a CTA
// of up to 256 threads carries `tpb` tokens.  With cos/sin built in-kernel,
// the lanes of a warp split the frequencies among themselves and exchange
// them by shuffles (see the kernel).
//
// Generic kernel: any even D and any alignment — one warp per
// (token, head) with scalar accesses.
#include "common.cuh"
#include "rope_core.cuh"

namespace kani {
namespace {

// ------------------------------------------------------------ vector kernel
// Lane layout inside a warp: lane = hh * L + jj, hh in [0, 32/L) the head slot,
// jj in [0, L) the chunk.  A rope lane needs cos/sin of frequencies
// jj*E .. jj*E+E-1; the 32/L lanes sharing a chunk jj compute those E
// frequencies between them (one sinf/cosf pair each when 32/L >= E) and
// exchange them with shuffles, so there is no shared memory and no block
// barrier: every warp runs on its own, its global loads are issued first and
// their latency overlaps the trig.
template <typename T, bool NORM, bool TABLE, bool CS_GIVEN>
__global__ void __launch_bounds__(256, NORM ? 3 : 4)
rope_vec_kernel(RopeParams p, int log2l, int ipt, int iptr, int tpb) {
  constexpr int E = VecN<T>::value;
  const int L = 1 << log2l;
  const int half = p.d >> 1;
  const int tl = threadIdx.x / iptr;
  const int item = threadIdx.x - tl * iptr;
  const int64_t t = (int64_t)blockIdx.x * tpb + tl;
  const bool tok_ok = t < p.n_tokens;
  const int lane = threadIdx.x & 31;
  const int head_item = item >> log2l;
  const int j = item & (L - 1);
  // kind: 0 = Q rope, 1 = K rope, 2 = V copy, 3 = idle lane
  int kind = 3, h = 0;
  if (tok_ok && item < ipt) {
    if (head_item < p.hq) {
      kind = 0;
      h = head_item;
    } else if (head_item < p.hq + p.hk) {
      kind = 1;
      h = head_item - p.hq;
    } else {
      kind = 2;
      h = head_item - p.hq - p.hk;
    }
  }
  const int lo = j * E, hi = half + j * E;

  // 1. the head's data: independent of everything else, issued first
  uint4 xlo = make_uint4(0, 0, 0, 0), xhi = xlo, plo = xlo, phi = xlo;
  if (kind < 3) {
    const T* base = kind == 0 ? static_cast<const T*>(p.q) + t * p.qts
                  : kind == 1 ? static_cast<const T*>(p.k) + t * p.kts
                              : static_cast<const T*>(p.v) + t * p.vts;
    const T* src = base + (int64_t)h * p.d;
    xlo = ld16_stream(src + lo);
    xhi = ld16_stream(src + hi);
  }
  // 2. token metadata (slot, frame) and the frame-table row
  TokenMeta m{};
  if (tok_ok) {
    m = token_meta<TABLE>(p, t);
    if (item == 0) flag_token<TABLE>(p, m);
  }
  if constexpr (TABLE) {
    if (kind < 2 && m.frame_ok) {
      const T* pr = static_cast<const T*>(p.table) + m.frame * p.d;
      plo = ld16_ro(pr + lo);
      phi = ld16_ro(pr + hi);
    }
  }
  // 3. cos/sin of this lane's E frequencies (both halves share them unless
  //    explicit cos/sin rows are given)
  float clo[E], slo[E];
  float chi_[CS_GIVEN ? E : 1], shi_[CS_GIVEN ? E : 1];
  float* chi = CS_GIVEN ? chi_ : clo;
  float* shi = CS_GIVEN ? shi_ : slo;
  if constexpr (CS_GIVEN) {
    if (kind < 2) {
      unpack16<T>(ld16_ro(static_cast<const T*>(p.cos) + lo), clo);
      unpack16<T>(ld16_ro(static_cast<const T*>(p.cos) + hi), chi);
      unpack16<T>(ld16_ro(static_cast<const T*>(p.sin) + lo), slo);
      unpack16<T>(ld16_ro(static_cast<const T*>(p.sin) + hi), shi);
    }
  } else {
    // warp-uniform: skip when no lane of the warp rotates (a V-only warp)
    if (__any_sync(0xffffffffu, kind < 2)) {
      const int log2g = 5 - log2l;            // 32/L lanes share one chunk
      const int G = 1 << log2g;
      const int hh = lane >> log2l;
      const int jj = lane & (L - 1);
      const float posf = tok_ok ? (float)p.positions[t] : 0.f;
      const int rounds = (E + G - 1) >> log2g;
      for (int r = 0; r < rounds; ++r) {
        const int e_own = r * G + hh;
        float cv = 0.f, sv = 0.f;
        if (e_own < E) {
          const float ang = __fmul_rn(__ldg(p.inv_freq + jj * E + e_own), posf);
          cv = round_to<T>(cosf(ang));
          sv = round_to<T>(sinf(ang));
        }
#pragma unroll
        for (int e = 0; e < E; ++e) {
          if ((e >> log2g) == r) {  // uniform across the warp
            const int src = ((e & (G - 1)) << log2l) | jj;
            clo[e] = __shfl_sync(0xffffffffu, cv, src);
            slo[e] = __shfl_sync(0xffffffffu, sv, src);
          }
        }
      }
    }
  }

  // 4. optional per-head RMSNorm (an L-lane shuffle tree per head)
  float a[E], b[E];
  unpack16<T>(xlo, a);
  unpack16<T>(xhi, b);
  if constexpr (NORM) {
    float ss = 0.f;
    if (kind < 2) {
#pragma unroll
      for (int e = 0; e < E; ++e) {
        ss = fmaf(a[e], a[e], ss);
        ss = fmaf(b[e], b[e], ss);
      }
    }
    for (int off = L >> 1; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (kind < 2) {
      const T* w = static_cast<const T*>(kind == 0 ? p.qw : p.kw);
      float wl[E], wh[E];
      unpack16<T>(ld16_ro(w + lo), wl);
      unpack16<T>(ld16_ro(w + hi), wh);
      const float r = rrms_of(ss, p.d, p.eps);
#pragma unroll
      for (int e = 0; e < E; ++e) {
        a[e] = round_to<T>(__fmul_rn(__fmul_rn(a[e], r), wl[e]));
        b[e] = round_to<T>(__fmul_rn(__fmul_rn(b[e], r), wh[e]));
      }
    }
  }

  // 5. rotate, add the frame term, store
  if (kind < 2) {
    float ylo[E], yhi[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
      ylo[e] = __fadd_rn(__fmul_rn(a[e], clo[e]), __fmul_rn(-b[e], slo[e]));
      yhi[e] = __fadd_rn(__fmul_rn(b[e], chi[e]), __fmul_rn(a[e], shi[e]));
    }
    if constexpr (TABLE) {
      if (m.frame_ok) {
        float pl[E], ph[E];
        unpack16<T>(plo, pl);
        unpack16<T>(phi, ph);
#pragma unroll
        for (int e = 0; e < E; ++e) {
          ylo[e] = __fadd_rn(ylo[e], pl[e]);
          yhi[e] = __fadd_rn(yhi[e], ph[e]);
        }
      }
    }
    if (kind == 0) {
      T* dst = static_cast<T*>(p.q_out) + t * p.qots + (int64_t)h * p.qohs;
      st16(dst + lo, pack16<T>(ylo));
      st16(dst + hi, pack16<T>(yhi));
    } else if (m.slot_ok) {
      T* dst = static_cast<T*>(p.k_cache) + m.b * p.cbs + (int64_t)h * p.chs + m.slot * p.css;
      st16(dst + lo, pack16<T>(ylo));
      st16(dst + hi, pack16<T>(yhi));
    }
  } else if (kind == 2 && m.slot_ok) {
    T* dst = static_cast<T*>(p.v_cache) + m.b * p.cbs + (int64_t)h * p.chs + m.slot * p.css;
    st16(dst + lo, xlo);
    st16(dst + hi, xhi);
  }
}

// ------------------------------------------------------ shared warp helpers

// ------------------------------------------------------------- token kernel
// Two warps per token: warp 0 rotates all Q heads, warp 1 rotates the K heads
// and copies the V heads.  A lane carries QI Q heads (hh, hh + G, ...) or KI
// K and V heads that all use the SAME E frequencies, so per warp the
// sin/cos, their shuffles and the token metadata are computed once for QI
// (or 2*KI) head vectors.  All of the warp's global loads are issued before
// the trig.  Used for short calls (decode steps) when num_q_heads <= QI*G
// and num_kv_heads <= KI*G (bf16, D=64: G=8, 16 Q / 8 KV heads -> QI=2, KI=1).
template <typename T, bool NORM, bool TABLE, int QI, int KI>
__global__ void __launch_bounds__(256)
rope_token_kernel(RopeParams p, int log2l) {
  // a decode step's attention (kani_decode_attention_step) may start streaming
  // the older cache rows now; it reads q and the rows written here after this
  // grid completes
  griddep_launch_dependents();
  griddep_wait();  // launched as a programmatic dependent: the inputs come from the launch before
  constexpr int E = VecN<T>::value;
  constexpr int NI = QI > KI ? QI : KI;
  const int L = 1 << log2l;
  const int G = 32 >> log2l;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 6) + (warp >> 1);
  if (t >= p.n_tokens) return;  // warp-uniform exit
  const bool qrole = (warp & 1) == 0;
  const int hh = lane >> log2l;
  const int jj = lane & (L - 1);
  const int lo = jj * E, hi = (p.d >> 1) + jj * E;

  // 1. head data
  uint4 xlo[NI], xhi[NI], vlo[KI], vhi[KI];
  if (qrole) {
    const T* base = static_cast<const T*>(p.q) + t * p.qts;
#pragma unroll
    for (int i = 0; i < QI; ++i) {
      const int h = hh + i * G;
      if (h < p.hq) {
        xlo[i] = ld16_stream(base + (int64_t)h * p.d + lo);
        xhi[i] = ld16_stream(base + (int64_t)h * p.d + hi);
      }
    }
  } else {
    const T* kb = static_cast<const T*>(p.k) + t * p.kts;
    const T* vb = static_cast<const T*>(p.v) + t * p.vts;
#pragma unroll
    for (int i = 0; i < KI; ++i) {
      const int h = hh + i * G;
      if (h < p.hk) {
        xlo[i] = ld16_stream(kb + (int64_t)h * p.d + lo);
        xhi[i] = ld16_stream(kb + (int64_t)h * p.d + hi);
        vlo[i] = ld16_stream(vb + (int64_t)h * p.d + lo);
        vhi[i] = ld16_stream(vb + (int64_t)h * p.d + hi);
      }
    }
  }
  // 2. token metadata and the frame-table row
  const TokenMeta m = token_meta<TABLE>(p, t);
  if (qrole && lane == 0) flag_token<TABLE>(p, m);
  uint4 plo = make_uint4(0, 0, 0, 0), phi = plo;
  if constexpr (TABLE) {
    if (m.frame_ok) {
      const T* pr = static_cast<const T*>(p.table) + m.frame * p.d;
      plo = ld16_ro(pr + lo);
      phi = ld16_ro(pr + hi);
    }
  }
  // 3. cos/sin
  float cs[E], sn[E];
  warp_cos_sin<T, -1>(lane_freqs<T, -1>(p.inv_freq, log2l, lane), (float)p.positions[t], log2l, lane, cs,
                      sn);
  float nsn[E];
#pragma unroll
  for (int e = 0; e < E; ++e) nsn[e] = -sn[e];
  float pl[E], ph[E];
  if constexpr (TABLE) {
    unpack16<T>(plo, pl);
    unpack16<T>(phi, ph);
  }
  // 4. per head: norm, rotate, frame term, store
  const int nh = qrole ? p.hq : p.hk;
  const T* nw = static_cast<const T*>(qrole ? p.qw : p.kw);
  T* qdst = static_cast<T*>(p.q_out) + t * p.qots;
  T* kdst = static_cast<T*>(p.k_cache) + m.b * p.cbs + m.slot * p.css;
#pragma unroll
  for (int i = 0; i < NI; ++i) {
    if (i >= (qrole ? QI : KI)) break;  // warp-uniform
    const int h = hh + i * G;
    const bool live = h < nh && (qrole || m.slot_ok);
    T* dst = qrole ? qdst + (int64_t)h * p.qohs : kdst + (int64_t)h * p.chs;
    rope_chunk_store<T, NORM, TABLE>(xlo[i], xhi[i], live, cs, nsn, sn, pl, ph, m.frame_ok, nw, lo, hi,
                                     log2l, p.d, p.eps, dst);
  }
  if (!qrole && m.slot_ok) {
    T* vdst = static_cast<T*>(p.v_cache) + m.b * p.cbs + m.slot * p.css;
#pragma unroll
    for (int i = 0; i < KI; ++i) {
      const int h = hh + i * G;
      if (h < p.hk) {
        st16(vdst + (int64_t)h * p.chs + lo, vlo[i]);
        st16(vdst + (int64_t)h * p.chs + hi, vhi[i]);
      }
    }
  }
}

// -------------------------------------------------------------- bulk kernel
// Long calls (prefill-sized token counts).  One CTA of kBulkTPS warps per
// group of kBulkTPS tokens; the hardware block scheduler balances the groups
// over the SMs.  Thread 0 brings the group's Q, K and V rows into shared
// memory with plain TMA bulk copies (cp.async.bulk completing on one
// mbarrier; every copy targets this CTA only) and pulls the CTA's share of
// the frame table into L2; shared memory, not registers, holds the bytes in
// flight, and each warp fetches its token's position, slot and frame row and
// computes the token's sin/cos while the rows stream in.  Each warp
// then owns one whole token: its lanes carry QI Q heads, KI K heads and KI V
// heads that all use the same E frequencies, so the sin/cos, their shuffles
// and the token metadata are computed once per token.  The mbarrier wait is
// bounded: on a timeout the warp raises KANI_FLAG_TIMEOUT, waits once more
// (with the default bound) for the copies and returns.  The kernel releases
// its programmatic dependents after its stores, not at entry.
constexpr int kBulkTPS = 4;
constexpr long long kWaitCycles = 2000000000LL;  // ~1 s at the B200 clock

__device__ __forceinline__ uint32_t smem_u32(const void* ptr) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(ptr));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

// One wait attempt.  With a suspend hint the thread may sleep (up to the hint,
// in ns) until the phase completes, so a waiting warp leaves the issue slots
// free; with none (a test's short limit) it only tests the phase, since a
// try_wait without a hint may still block for a system-defined time.
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity, uint32_t suspend_ns) {
  uint32_t ok;
  if (suspend_ns == 0) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(suspend_ns)
        : "memory");
  }
  return ok != 0;
}

__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity,
                                                  long long limit = kWaitCycles,
                                                  uint32_t suspend_ns = kWaitSuspendNs) {
  if (mbar_try_wait(bar, parity, suspend_ns)) return true;
  const long long start = clock64();
  while (!mbar_try_wait(bar, parity, suspend_ns)) {
    if (clock64() - start > limit) return false;
  }
  return true;
}

// global -> shared bulk copy; addresses 16-byte aligned, bytes a multiple of 16
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// Hint: pull [src, src + bytes) into L2 (bytes a multiple of 16).
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Copy `cnt` token rows of `row` bytes (source rows `stride` bytes apart) to
// consecutive shared memory: one copy when the rows are contiguous.
__device__ __forceinline__ void bulk_rows(uint32_t dst, const char* src, uint32_t row, int64_t stride,
                                          int cnt, uint32_t bar) {
  if (stride == (int64_t)row) {
    bulk_g2s(dst, src, row * cnt, bar);
  } else {
    for (int i = 0; i < cnt; ++i) bulk_g2s(dst + i * row, src + i * stride, row, bar);
  }
}

template <typename T, bool NORM, bool TABLE, int QI, int KI, int LOG2L_CT>
__global__ void __launch_bounds__(kBulkTPS * 32)
rope_bulk_kernel(RopeParams p, int log2l_rt) {
  const int log2l = LOG2L_CT >= 0 ? LOG2L_CT : log2l_rt;
  constexpr int E = VecN<T>::value;
  constexpr int ES = (int)sizeof(T);
  extern __shared__ __align__(128) unsigned char stage[];
  __shared__ __align__(8) uint64_t bar_storage;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const uint32_t qrow = (uint32_t)(p.hq * p.d * ES);
  const uint32_t krow = (uint32_t)(p.hk * p.d * ES);
  // stage layout: [Q rows][K rows][V rows]
  const int64_t t0 = (int64_t)blockIdx.x * kBulkTPS;
  const int cnt = (int)(p.n_tokens - t0 < kBulkTPS ? p.n_tokens - t0 : kBulkTPS);
  const uint32_t bar = smem_u32(&bar_storage);

  // launched as a programmatic dependent: read nothing global before the
  // previous grid has completed (the next launch is released at the end)
  griddep_wait();
  if (tid == 0) {
    mbar_init(bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    const uint32_t base = smem_u32(stage);
    mbar_expect_tx(bar, (uint32_t)cnt * (qrow + 2 * krow));
    bulk_rows(base, reinterpret_cast<const char*>(static_cast<const T*>(p.q) + t0 * p.qts), qrow,
              p.qts * ES, cnt, bar);
    bulk_rows(base + kBulkTPS * qrow, reinterpret_cast<const char*>(static_cast<const T*>(p.k) + t0 * p.kts),
              krow, p.kts * ES, cnt, bar);
    bulk_rows(base + kBulkTPS * (qrow + krow),
              reinterpret_cast<const char*>(static_cast<const T*>(p.v) + t0 * p.vts), krow, p.vts * ES, cnt,
              bar);
    if constexpr (TABLE) {
      // this CTA's share of the frame table goes to L2 while the rows stream in
      const int64_t per = (p.table_rows + gridDim.x - 1) / gridDim.x;
      const int64_t r0 = (int64_t)blockIdx.x * per;
      const int64_t r1 = r0 + per < p.table_rows ? r0 + per : p.table_rows;
      if (r1 > r0)
        bulk_prefetch_l2(static_cast<const T*>(p.table) + r0 * p.d, (uint32_t)((r1 - r0) * p.d * ES));
    }
  }
  __syncthreads();  // the barrier is initialised before anyone waits on it
  if (warp >= cnt) return;  // warp 0 always stays, so the CTA outlives its copies

  const int64_t t = t0 + warp;
  const int L = 1 << log2l;
  const int G = 32 >> log2l;
  const int hh = lane >> log2l;
  const int jj = lane & (L - 1);
  const int lo = jj * E, hi = (p.d >> 1) + jj * E;

  // Everything that does not need the staged rows is fetched while they
  // stream in: the lane's frequencies, the token's position / slot / frame
  // and the frame-table row.
  const LaneFreqs<T, LOG2L_CT> lf = lane_freqs<T, LOG2L_CT>(p.inv_freq, log2l, lane);
  const int64_t pos = p.positions[t];
  const int64_t slot = p.slots ? p.slots[t]
                               : (p.seq_tokens == 1 ? 0 : t - (t / p.seq_tokens) * p.seq_tokens);
  const int64_t fp = p.frame_pos ? p.frame_pos[t] : pos;
  const TokenMeta m = token_meta_vals<TABLE>(p, t, slot, fp);
  uint4 plo = make_uint4(0, 0, 0, 0), phi = plo;
  if constexpr (TABLE) {
    if (m.frame_ok) {
      const T* pr = static_cast<const T*>(p.table) + m.frame * p.d;
      plo = ld16_ro(pr + lo);
      phi = ld16_ro(pr + hi);
    }
  }

  // cos/sin and the frame row do not depend on the staged rows: computed while they stream in
  float cs[E], sn[E], pl[E], ph[E];
  warp_cos_sin<T, LOG2L_CT>(lf, (float)pos, log2l, lane, cs, sn);
  float nsn[E];
#pragma unroll
  for (int e = 0; e < E; ++e) nsn[e] = -sn[e];
  if constexpr (TABLE) {
    unpack16<T>(plo, pl);
    unpack16<T>(phi, ph);
  }
  if (!mbar_wait_bounded(bar, 0, p.wait_cycles, p.wait_suspend_ns)) {
    if (lane == 0 && p.err != nullptr) atomicOr(p.err, KANI_FLAG_TIMEOUT);
    mbar_wait_bounded(bar, 0);  // the copies target this CTA's shared memory: default bound
    return;
  }
  if (lane == 0) flag_token<TABLE>(p, m);
  // per-lane bases (head hh); head hh + i*G is a constant stride further
  const int hstride = G * p.d;  // elements between a lane's heads in shared memory
  // Q heads
  {
    const T* src = reinterpret_cast<const T*>(stage + warp * qrow) + hh * p.d;
    T* qdst = static_cast<T*>(p.q_out) + t * p.qots + (int64_t)hh * p.qohs;
    const int64_t qstep = (int64_t)G * p.qohs;
    const T* nw = static_cast<const T*>(p.qw);
#pragma unroll
    for (int i = 0; i < QI; ++i) {
      const bool live = hh + i * G < p.hq;
      uint4 xlo = make_uint4(0, 0, 0, 0), xhi = xlo;
      if (live) {
        xlo = *reinterpret_cast<const uint4*>(src + i * hstride + lo);
        xhi = *reinterpret_cast<const uint4*>(src + i * hstride + hi);
      }
      rope_chunk_store<T, NORM, TABLE>(xlo, xhi, live, cs, nsn, sn, pl, ph, m.frame_ok, nw, lo, hi, log2l, p.d,
                                       p.eps, qdst + i * qstep);
    }
  }
  // K heads (rotated) and V heads (copied) into the cache slot
  {
    const T* ksrc = reinterpret_cast<const T*>(stage + kBulkTPS * qrow + warp * krow) + hh * p.d;
    const T* vsrc = reinterpret_cast<const T*>(stage + kBulkTPS * (qrow + krow) + warp * krow) + hh * p.d;
    const int64_t off = m.b * p.cbs + m.slot * p.css + (int64_t)hh * p.chs;
    T* kdst = static_cast<T*>(p.k_cache) + off;
    T* vdst = static_cast<T*>(p.v_cache) + off;
    const int64_t cstep = (int64_t)G * p.chs;
    const T* nw = static_cast<const T*>(p.kw);
#pragma unroll
    for (int i = 0; i < KI; ++i) {
      const bool has = hh + i * G < p.hk;
      uint4 xlo = make_uint4(0, 0, 0, 0), xhi = xlo;
      if (has) {
        xlo = *reinterpret_cast<const uint4*>(ksrc + i * hstride + lo);
        xhi = *reinterpret_cast<const uint4*>(ksrc + i * hstride + hi);
      }
      rope_chunk_store<T, NORM, TABLE>(xlo, xhi, has && m.slot_ok, cs, nsn, sn, pl, ph, m.frame_ok, nw, lo, hi,
                                       log2l, p.d, p.eps, kdst + i * cstep);
      if (has && m.slot_ok) {
        st16(vdst + i * cstep + lo, *reinterpret_cast<const uint4*>(vsrc + i * hstride + lo));
        st16(vdst + i * cstep + hi, *reinterpret_cast<const uint4*>(vsrc + i * hstride + hi));
      }
    }
  }
  // this warp's stores are issued: the next launch may be scheduled.  Released
  // here rather than at entry: at entry the next grid's CTAs take SM slots
  // while this grid still streams (measured at T = 1024: 4.8 -> 3.7 us; a
  // plain 17 MB copy: 7.15 us with the early release, 6.21 us with the late)
  griddep_launch_dependents();
}

template <typename T, bool NORM, bool TABLE, int QI, int KI, int LOG2L_CT>
int launch_bulk(const RopeParams& p, int log2l, cudaStream_t s) {
  constexpr int ES = (int)sizeof(T);
  const size_t row_bytes = (size_t)(p.hq + 2 * p.hk) * p.d * ES;
  const size_t smem = kBulkTPS * row_bytes;
  auto kern = rope_bulk_kernel<T, NORM, TABLE, QI, KI, LOG2L_CT>;
  static int smem_set[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return KANI_ERR_UNSUPPORTED;
  if (smem + 1024 > 48 * 1024 && smem_set[dev] < (int)smem) {  // static shared memory counts too
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return launch_status();
    smem_set[dev] = (int)smem;
  }
  const int64_t grid = (p.n_tokens + kBulkTPS - 1) / kBulkTPS;
  if (grid > 0x7fffffff) return KANI_ERR_UNSUPPORTED;
  RopeParams pw = p;
  const WaitBound wb = wait_bound(kWaitCycles);
  pw.wait_cycles = wb.cycles;
  pw.wait_suspend_ns = wb.suspend_ns;
  launch_pdl(kern, dim3((unsigned)grid), dim3(kBulkTPS * 32), smem, s, pw, log2l);
  return launch_status();
}

// ----------------------------------------------------------- generic kernel
template <typename T, bool NORM, bool TABLE, bool CS_GIVEN>
__global__ void __launch_bounds__(256)
rope_generic_kernel(RopeParams p, int heads_per_tok) {
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= p.n_tokens * heads_per_tok) return;  // warp-uniform exit
  const int64_t t = gw / heads_per_tok;
  const int hitem = (int)(gw - t * heads_per_tok);
  const int half = p.d >> 1;
  const TokenMeta m = token_meta<TABLE>(p, t);
  if (hitem == 0 && lane == 0) flag_token<TABLE>(p, m);

  if (hitem >= p.hq + p.hk) {  // V copy
    if (!m.slot_ok) return;
    const int h = hitem - p.hq - p.hk;
    const T* src = static_cast<const T*>(p.v) + t * p.vts + (int64_t)h * p.d;
    T* dst = static_cast<T*>(p.v_cache) + m.b * p.cbs + (int64_t)h * p.chs + m.slot * p.css;
    for (int i = lane; i < p.d; i += 32) dst[i] = src[i];
    return;
  }
  const bool is_q = hitem < p.hq;
  const int h = is_q ? hitem : hitem - p.hq;
  const T* src = is_q ? static_cast<const T*>(p.q) + t * p.qts + (int64_t)h * p.d
                      : static_cast<const T*>(p.k) + t * p.kts + (int64_t)h * p.d;
  float r = 1.f;
  if constexpr (NORM) {
    float ss = 0.f;
    for (int i = lane; i < p.d; i += 32) {
      const float x = Elem<T>::to_f(src[i]);
      ss = fmaf(x, x, ss);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    r = rrms_of(ss, p.d, p.eps);
  }
  const T* w = static_cast<const T*>(is_q ? p.qw : p.kw);
  const float pos = CS_GIVEN ? 0.f : (float)p.positions[t];
  const T* prow = (TABLE && m.frame_ok) ? static_cast<const T*>(p.table) + m.frame * p.d : nullptr;
  T* dst = nullptr;
  if (is_q) {
    dst = static_cast<T*>(p.q_out) + t * p.qots + (int64_t)h * p.qohs;
  } else if (m.slot_ok) {
    dst = static_cast<T*>(p.k_cache) + m.b * p.cbs + (int64_t)h * p.chs + m.slot * p.css;
  }
  if (dst == nullptr) return;
  for (int i = lane; i < half; i += 32) {
    float a = Elem<T>::to_f(src[i]);
    float b = Elem<T>::to_f(src[i + half]);
    if constexpr (NORM) {
      a = round_to<T>(__fmul_rn(__fmul_rn(a, r), Elem<T>::to_f(w[i])));
      b = round_to<T>(__fmul_rn(__fmul_rn(b, r), Elem<T>::to_f(w[i + half])));
    }
    float clo, slo, chi, shi;
    if constexpr (CS_GIVEN) {
      const T* cp = static_cast<const T*>(p.cos);
      const T* sp = static_cast<const T*>(p.sin);
      clo = Elem<T>::to_f(cp[i]);
      chi = Elem<T>::to_f(cp[i + half]);
      slo = Elem<T>::to_f(sp[i]);
      shi = Elem<T>::to_f(sp[i + half]);
    } else {
      const float ang = __fmul_rn(p.inv_freq[i], pos);
      clo = chi = round_to<T>(cosf(ang));
      slo = shi = round_to<T>(sinf(ang));
    }
    float ylo = __fadd_rn(__fmul_rn(a, clo), __fmul_rn(-b, slo));
    float yhi = __fadd_rn(__fmul_rn(b, chi), __fmul_rn(a, shi));
    if (prow != nullptr) {
      ylo = __fadd_rn(ylo, Elem<T>::to_f(prow[i]));
      yhi = __fadd_rn(yhi, Elem<T>::to_f(prow[i + half]));
    }
    dst[i] = Elem<T>::from_f(ylo);
    dst[i + half] = Elem<T>::from_f(yhi);
  }
}

// -------------------------------------------------------------- KV write
template <typename T, bool VEC>
__global__ void __launch_bounds__(256)
kv_write_kernel(const T* __restrict__ k, const T* __restrict__ v, int64_t batch, int hk, int d,
                T* kc, T* vc, int64_t clen, const int64_t* __restrict__ wp, int per_stream,
                int32_t* err) {
  constexpr int E = VEC ? VecN<T>::value : 1;
  const int vpr = d / E;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= batch * hk * vpr) return;
  const int64_t bh = idx / vpr;
  const int c = (int)(idx - bh * vpr);
  const int64_t b = bh / hk;
  const int64_t slot = per_stream ? wp[b] : wp[0];
  const bool ok = slot >= 0 && slot < clen;
  if (!ok) {
    if (c == 0 && (bh - b * hk) == 0 && err != nullptr) atomicOr(err, KANI_FLAG_SLOT_OOB);
    return;
  }
  const int64_t src = bh * d + (int64_t)c * E;
  const int64_t dst = (bh * clen + slot) * d + (int64_t)c * E;
  if constexpr (VEC) {
    st16(kc + dst, ld16(k + src));
    st16(vc + dst, ld16(v + src));
  } else {
    kc[dst] = k[src];
    vc[dst] = v[src];
  }
}

// ------------------------------------------------------------------ launch
constexpr int64_t kBulkMinTokens = 256;  // shorter calls use the token kernel

template <typename T, bool NORM, bool TABLE, bool CS_GIVEN>
int launch_rope_t(const RopeParams& p, cudaStream_t s) {
  constexpr int E = VecN<T>::value;
  const int half = p.d / 2;
  const bool has_v = p.v != nullptr;
  int log2l = -1;
  if (half % E == 0) {
    const int L = half / E;
    if (L >= 1 && L <= 32 && (L & (L - 1)) == 0) {
      log2l = 0;
      while ((1 << log2l) < L) ++log2l;
    }
  }
  bool vec = log2l >= 0 && aligned16(p.q) && aligned16(p.k) && aligned16(p.q_out) &&
             aligned16(p.k_cache) && p.qts % E == 0 && p.kts % E == 0 && p.qots % E == 0 &&
             p.qohs % E == 0 && p.cbs % E == 0 && p.chs % E == 0 && p.css % E == 0;
  if (has_v) vec = vec && aligned16(p.v) && aligned16(p.v_cache) && p.vts % E == 0;
  if (NORM) vec = vec && aligned16(p.qw) && aligned16(p.kw);
  if (TABLE) vec = vec && aligned16(p.table);
  if (CS_GIVEN) vec = vec && aligned16(p.cos) && aligned16(p.sin);

  if constexpr (!CS_GIVEN) {
    // long calls: bulk-copy ring; needs 16-byte token rows and strides
    if (vec && has_v && p.hq > 0 && p.hk > 0 && p.n_tokens >= kBulkMinTokens) {
      const int G = 32 >> log2l;
      const bool rows16 = ((int64_t)p.hq * p.d * (int64_t)sizeof(T)) % 16 == 0 &&
                          ((int64_t)p.hk * p.d * (int64_t)sizeof(T)) % 16 == 0;
      const int64_t stage = (int64_t)kBulkTPS * (p.hq + 2 * p.hk) * p.d * (int64_t)sizeof(T);
      if (rows16 && stage <= 200 * 1024) {
        // the common geometry (16-bit types, D = 64 -> 4 lanes per head) is
        // compiled with constant shuffle sources
        if (p.hq <= 2 * G && p.hk <= G) {
          if (sizeof(T) == 2 && log2l == 2) return launch_bulk<T, NORM, TABLE, 2, 1, 2>(p, log2l, s);
          return launch_bulk<T, NORM, TABLE, 2, 1, -1>(p, log2l, s);
        }
        if (p.hq <= 4 * G && p.hk <= 2 * G) return launch_bulk<T, NORM, TABLE, 4, 2, -1>(p, log2l, s);
      }
    }
    // two-warps-per-token kernel: needs V, Q/K/V present and the heads to fit
    if (vec && has_v && p.hq > 0 && p.hk > 0) {
      const int G = 32 >> log2l;
      const int64_t tpb = p.n_tokens < 4 ? p.n_tokens : 4;
      const int64_t grid = (p.n_tokens + tpb - 1) / tpb;
      if (grid <= 0x7fffffff) {
        const dim3 blk((unsigned)(64 * tpb));
        if (p.hq <= 2 * G && p.hk <= G) {
          launch_maybe_pdl(p.n_tokens <= kPdlMaxRows, rope_token_kernel<T, NORM, TABLE, 2, 1>, dim3((unsigned)grid), dim3(blk), 0, s, p, log2l);
          return launch_status();
        }
        if (p.hq <= 4 * G && p.hk <= 2 * G) {
          launch_maybe_pdl(p.n_tokens <= kPdlMaxRows, rope_token_kernel<T, NORM, TABLE, 4, 2>, dim3((unsigned)grid), dim3(blk), 0, s, p, log2l);
          return launch_status();
        }
      }
    }
  }
  if (vec) {
    const int heads = p.hq + p.hk + (has_v ? p.hk : 0);
    const int ipt = heads << log2l;
    const int iptr = ((ipt + 31) / 32) * 32;
    if (iptr <= 256) {
      int tpb = 256 / iptr;
      if (tpb > p.n_tokens) tpb = (int)p.n_tokens;
      const int64_t grid = (p.n_tokens + tpb - 1) / tpb;
      if (grid <= 0x7fffffff) {
        rope_vec_kernel<T, NORM, TABLE, CS_GIVEN>
            <<<(unsigned)grid, tpb * iptr, 0, s>>>(p, log2l, ipt, iptr, tpb);
        return launch_status();
      }
    }
  }
  const int heads = p.hq + p.hk + (has_v ? p.hk : 0);
  const int64_t warps = p.n_tokens * heads;
  const int64_t grid = (warps + 7) / 8;
  if (grid > 0x7fffffff) return KANI_ERR_UNSUPPORTED;
  rope_generic_kernel<T, NORM, TABLE, CS_GIVEN><<<(unsigned)grid, 256, 0, s>>>(p, heads);
  return launch_status();
}

template <typename T>
int launch_rope(const RopeParams& p, cudaStream_t s) {
  const bool norm = p.qw != nullptr;
  const bool table = p.table != nullptr;
  const bool given = p.cos != nullptr;
  if (given) {
    // the reference-signature path: no norm, no table
    if (norm || table) return KANI_ERR_UNSUPPORTED;
    return launch_rope_t<T, false, false, true>(p, s);
  }
  if (norm && table) return launch_rope_t<T, true, true, false>(p, s);
  if (norm) return launch_rope_t<T, true, false, false>(p, s);
  if (table) return launch_rope_t<T, false, true, false>(p, s);
  return launch_rope_t<T, false, false, false>(p, s);
}

}  // namespace
}  // namespace kani

using kani::RopeParams;

extern "C" int kani_rope_qk(int32_t dtype, const void* q, const void* k, const void* cos,
                            const void* sin, void* q_out, void* k_out, int32_t num_q_heads,
                            int32_t num_k_heads, int32_t head_dim, void* stream) {
  if (num_q_heads < 0 || num_k_heads < 0 || head_dim < 0) return KANI_ERR_INVALID_ARG;
  if (head_dim % 2 != 0) return KANI_ERR_UNSUPPORTED;
  if (num_q_heads == 0 && num_k_heads == 0) return KANI_OK;
  if (head_dim == 0) return KANI_OK;
  if (cos == nullptr || sin == nullptr) return KANI_ERR_INVALID_ARG;
  if (num_q_heads > 0 && (q == nullptr || q_out == nullptr)) return KANI_ERR_INVALID_ARG;
  if (num_k_heads > 0 && (k == nullptr || k_out == nullptr)) return KANI_ERR_INVALID_ARG;
  // An empty head group still needs 16-byte aligned dummies for the vector test.
  if (num_q_heads == 0) { q = k; q_out = k_out; }
  if (num_k_heads == 0) { k = q; k_out = q_out; }
  RopeParams p{};
  p.n_tokens = 1;
  p.seq_tokens = 1;
  p.hq = num_q_heads;
  p.hk = num_k_heads;
  p.d = head_dim;
  p.q = q;
  p.qts = (int64_t)num_q_heads * head_dim;
  p.k = k;
  p.kts = (int64_t)num_k_heads * head_dim;
  p.cos = cos;
  p.sin = sin;
  p.q_out = q_out;
  p.qots = (int64_t)num_q_heads * head_dim;
  p.qohs = head_dim;
  // K output viewed as a one-slot cache [1, Hk, 1, D]
  p.k_cache = k_out;
  p.cbs = 0;
  p.chs = head_dim;
  p.css = 0;
  p.clen = 1;
  p.tpf = 1;
  p.tpf_shift = 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return kani::dispatch_dtype(dtype, [&]<typename T>() { return kani::launch_rope<T>(p, s); });
}

extern "C" int kani_kv_cache_write(int32_t dtype, const void* k, const void* v, int64_t batch,
                                   int32_t num_kv_heads, int32_t head_dim, void* k_cache,
                                   void* v_cache, int64_t cache_len, const int64_t* write_pos,
                                   int32_t per_stream_pos, int32_t* err_flag, void* stream) {
  if (batch < 0 || num_kv_heads < 0 || head_dim < 0 || cache_len < 0) return KANI_ERR_INVALID_ARG;
  if (batch == 0 || num_kv_heads == 0 || head_dim == 0) return KANI_OK;
  if (!k || !v || !k_cache || !v_cache || !write_pos) return KANI_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return kani::dispatch_dtype(dtype, [&]<typename T>() {
    constexpr int E = kani::VecN<T>::value;
    const bool vec = head_dim % E == 0 && kani::aligned16(k) && kani::aligned16(v) &&
                     kani::aligned16(k_cache) && kani::aligned16(v_cache);
    const int per = vec ? head_dim / E : head_dim;
    const int64_t total = batch * num_kv_heads * per;
    const int64_t grid = (total + 255) / 256;
    if (grid > 0x7fffffff) return (int)KANI_ERR_UNSUPPORTED;
    if (vec)
      kani::kv_write_kernel<T, true><<<(unsigned)grid, 256, 0, s>>>(
          static_cast<const T*>(k), static_cast<const T*>(v), batch, num_kv_heads, head_dim,
          static_cast<T*>(k_cache), static_cast<T*>(v_cache), cache_len, write_pos,
          per_stream_pos, err_flag);
    else
      kani::kv_write_kernel<T, false><<<(unsigned)grid, 256, 0, s>>>(
          static_cast<const T*>(k), static_cast<const T*>(v), batch, num_kv_heads, head_dim,
          static_cast<T*>(k_cache), static_cast<T*>(v_cache), cache_len, write_pos,
          per_stream_pos, err_flag);
    return kani::launch_status();
  });
}

extern "C" int kani_rope_kv_write(
    int32_t dtype, int64_t batch, int64_t seq_tokens, int32_t num_q_heads, int32_t num_kv_heads,
    int32_t head_dim, const void* q, int64_t q_tok_stride, const void* k, int64_t k_tok_stride,
    const void* v, int64_t v_tok_stride, const float* inv_freq, const int64_t* positions,
    const void* q_norm_w, const void* k_norm_w, float eps, const void* frame_table,
    int64_t frame_rows, const int64_t* frame_pos, int32_t tokens_per_frame, void* q_out,
    int64_t q_out_tok_stride, int64_t q_out_head_stride, void* k_cache, void* v_cache,
    int64_t cache_batch_stride, int64_t cache_head_stride, int64_t cache_slot_stride,
    int64_t cache_len, const int64_t* write_slots, int32_t* err_flag, void* stream) {
  if (batch < 0 || seq_tokens < 0 || num_q_heads < 0 || num_kv_heads < 0 || head_dim < 0 ||
      cache_len < 0)
    return KANI_ERR_INVALID_ARG;
  if (head_dim % 2 != 0) return KANI_ERR_UNSUPPORTED;
  const int64_t n_tokens = batch * seq_tokens;
  if (n_tokens == 0 || head_dim == 0 || (num_q_heads == 0 && num_kv_heads == 0)) return KANI_OK;
  if (!inv_freq || !positions) return KANI_ERR_INVALID_ARG;
  if (num_q_heads > 0 && (!q || !q_out)) return KANI_ERR_INVALID_ARG;
  if (num_kv_heads > 0 && (!k || !v || !k_cache || !v_cache)) return KANI_ERR_INVALID_ARG;
  if ((q_norm_w == nullptr) != (k_norm_w == nullptr)) return KANI_ERR_INVALID_ARG;
  if (frame_table != nullptr && (frame_rows < 0 || tokens_per_frame <= 0))
    return KANI_ERR_INVALID_ARG;
  // Empty head groups: point the unused side at the used one so the
  // alignment test sees real pointers; no item of that kind is generated.
  if (num_q_heads == 0) { q = k; q_out = k_cache; q_tok_stride = k_tok_stride; }
  if (num_kv_heads == 0) {
    k = q; v = nullptr; k_cache = q_out; v_cache = nullptr; k_tok_stride = q_tok_stride;
  }
  RopeParams p{};
  p.n_tokens = n_tokens;
  p.seq_tokens = seq_tokens;
  p.hq = num_q_heads;
  p.hk = num_kv_heads;
  p.d = head_dim;
  p.q = q;
  p.qts = q_tok_stride;
  p.k = k;
  p.kts = k_tok_stride;
  p.v = v;
  p.vts = v_tok_stride;
  p.inv_freq = inv_freq;
  p.positions = positions;
  p.qw = q_norm_w;
  p.kw = k_norm_w;
  p.eps = eps;
  p.table = frame_table;
  p.table_rows = frame_rows;
  p.frame_pos = frame_pos;
  p.tpf = tokens_per_frame > 0 ? tokens_per_frame : 1;
  p.tpf_shift = -1;
  for (int sh = 0; sh < 31; ++sh)
    if ((1 << sh) == p.tpf) p.tpf_shift = sh;
  p.q_out = q_out;
  p.qots = q_out_tok_stride;
  p.qohs = q_out_head_stride;
  p.k_cache = k_cache;
  p.v_cache = v_cache;
  p.cbs = cache_batch_stride;
  p.chs = cache_head_stride;
  p.css = cache_slot_stride;
  // without KV heads there is no cache write, so no slot can be out of range
  p.clen = num_kv_heads == 0 ? INT64_MAX : cache_len;
  p.slots = num_kv_heads == 0 ? nullptr : write_slots;
  p.err = err_flag;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return kani::dispatch_dtype(dtype, [&]<typename T>() { return kani::launch_rope<T>(p, s); });
}
