// Next-token sampling on the device (sm_100a): repetition penalty, optional
// additive logit bias, top-k, temperature, top-p and a categorical draw, for
// a batch of independent streams, in one launch.
//
// Reference: KaniInferenceEngine._sample_next_token,
// kani_tts/inference_engine.py:349-430, which runs on the host once per token
// (a dozen small launches plus `unique()` and an `.item()` sync):
//   * penalty (375-395): every distinct token of the history gets
//       l = l > 0 ? l / rp : l * rp                 (one rounding to the dtype)
//   * audio mask (398-399, full-vocab mode): l = l + mask
//   * top-k (402-403): torch.topk(l, min(256, V)), sorted descending
//   * temperature (406-407): l = l / T                (one rounding)
//   * top-p (410-415): p = softmax(l); c = cumsum(p);
//       candidate j >= 1 is dropped when c[j-1] >= top_p
//   * draw (418-419): p' = softmax(l with dropped = -inf); torch.multinomial(p', 1)
//   * map back (422-428): topk index -> reduced index -> full token id.
// The arithmetic follows torch's CPU kernels for a bf16/f16/f32 tensor:
//   * scalar multiply/divide in fp32 with the original scalar, then one rounding;
//   * softmax in fp32: exp(x - max) scaled by 1/sum, rounded once;
//   * cumsum accumulated in order in fp32 (double for f32 tensors), each prefix rounded;
//   * the top_p comparison in the tensor's dtype (the scalar is rounded to it).
// torch.multinomial with one sample is the exponential race of
// aten/src/ATen/native/Distributions.cpp (torch 2.x): q ~ Exp(1) stored in
// the dtype, s = p' / q rounded to the dtype, token = argmax(s), first index
// on ties.  The Exp(1) draws come either from the caller (`exp_draws`) or from
// Philox4x32-10 (Salmon, Moraes, Dror & Shaw, SC 2011) keyed by the seed and
// counted by (candidate group, stream, step): u = (2m + 1) 2^-24 with m the
// top 23 bits of a Philox word, E = -log(u).
//
// Ties: torch.topk does not specify the order of equal logits; this kernel
// orders candidates by value, then by lower index (a stable descending sort).
//
// Layout: one 1024-thread CTA per stream.  The penalised row is staged in
// shared memory (coalesced loads) and each thread takes a contiguous block of
// it as order-preserving keys (in registers for rows up to 16384).  The k-th
// largest key is found by bisection on the key value inside a bracket below
// the row's largest key: each step counts the keys above a threshold with a
// warp reduction and one barrier (about 11 steps for 16-bit types).  One
// block scan gives every key above the threshold a slot and places the equal
// keys taken at the boundary (lowest indices first) directly at their sorted
// positions; the keys above are sorted by counting ranks.  One warp then runs
// temperature, both softmaxes, the cumulative sum (one lane's in-order add
// chain) and the race.  No global scratch; no waits.
#include "common.cuh"

#include <math.h>

namespace kani {
namespace {

constexpr int kSampleThreads = 1024;
constexpr int kMaxTopK = 256;
constexpr int kSampleMaxDynSmem = 200 * 1024;
constexpr int kRegItems = 16;  // items per thread held in registers (rows up to 16384)
constexpr int kStageChunks = 4;  // 16-byte row chunks in flight per thread while staging
constexpr int kLiveMax = 2048;   // keys inside the threshold bracket that one warp searches
constexpr int kLiveReg = 16;     // of those, per lane in registers (lists up to 512)

struct SampleParams {
  const void* logits;
  int64_t row_stride;
  const void* bias;
  uint32_t* seen;
  int64_t seen_words;
  int update_seen;
  float penalty, temperature, top_p;
  int vocab, top_k, ipt;
  const int64_t* index_map;
  uint64_t seed;
  const int64_t* step;
  const float* draws;
  float* draws_out;
  void* probs_out;
  int32_t* cand_out;
  int64_t* tokens;
  int64_t tokens_stride;
};

// Order-preserving unsigned key of a stored value (larger value -> larger
// key; -0 and +0 share a key).  NaN inputs are not ordered like torch.topk.
template <typename T> struct KeyOf;
template <> struct KeyOf<__nv_bfloat16> {
  using Raw = uint16_t;
  static constexpr int kBits = 16;
  static __device__ __forceinline__ uint32_t key(uint16_t b) {
    if ((b & 0x7fffu) == 0) b = 0;
    return (uint32_t)(b ^ ((b & 0x8000u) ? 0xffffu : 0x8000u));
  }
};
template <> struct KeyOf<__half> : KeyOf<__nv_bfloat16> {};

// The stored value of a key (the inverse map; -0 comes back as +0).
template <typename T>
__device__ __forceinline__ float value_of_key(uint32_t k) {
  using Raw = typename KeyOf<T>::Raw;
  const uint32_t top = 1u << (KeyOf<T>::kBits - 1);
  const uint32_t all = KeyOf<T>::kBits == 32 ? 0xffffffffu : (1u << KeyOf<T>::kBits) - 1u;
  const Raw r = (Raw)(k ^ ((k & top) ? top : all));
  T t;
  memcpy(&t, &r, sizeof(Raw));
  return Elem<T>::to_f(t);
}
template <> struct KeyOf<float> {
  using Raw = uint32_t;
  static constexpr int kBits = 32;
  static __device__ __forceinline__ uint32_t key(uint32_t b) {
    if ((b & 0x7fffffffu) == 0) b = 0;
    return b ^ ((b & 0x80000000u) ? 0xffffffffu : 0x80000000u);
  }
};

// Smallest value of a 16-bit type that is a multiple of 2^-24 together with
// every larger value: bf16 from 2^-17 (8 significant bits); every fp16 value is.
template <typename T> constexpr float kExactMin = 0.f;
template <> constexpr float kExactMin<__nv_bfloat16> = 7.62939453125e-06f;  // 2^-17

// Cumulative-sum accumulator type of torch's CPU kernel for the dtype.
template <typename T> struct CumAcc { using type = float; };
template <> struct CumAcc<float> { using type = double; };

// Philox4x32-10 block (counter c, key k); constants from the Random123 paper.
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint2 k) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t lo0 = 0xD2511F53u * c.x, hi0 = __umulhi(0xD2511F53u, c.x);
    const uint32_t lo1 = 0xCD9E8D57u * c.z, hi1 = __umulhi(0xCD9E8D57u, c.z);
    c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
    k.x += 0x9E3779B9u;
    k.y += 0xBB67AE85u;
  }
  return c;
}

// Exp(1) draw from one 32-bit word: u = (2m + 1) * 2^-24 in (0, 1), exact in fp32.
__device__ __forceinline__ float exp_draw(uint32_t w) {
  const float u = (float)(((w >> 9) << 1) | 1u) * 5.9604644775390625e-08f;
  return -logf(u);
}

template <typename T, bool REG>
__global__ void __launch_bounds__(kSampleThreads, 1) sample_kernel(SampleParams p) {
  using K = KeyOf<T>;
  using Raw = typename K::Raw;
  constexpr int E = VecN<T>::value;
  constexpr int P = kMaxTopK / 32;  // sorted positions per lane of the final warp
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ int warp_sum[2][3][32];
  __shared__ uint32_t warp_max[32];
  __shared__ int warp_tot[32];
  __shared__ __align__(16) unsigned long long cand_key[kMaxTopK];
  __shared__ int rank_part[kSampleThreads / kMaxTopK][kMaxTopK];
  __shared__ float cand_val[kMaxTopK];
  __shared__ int cand_idx[kMaxTopK];
  __shared__ float s_val[kMaxTopK];
  __shared__ int s_idx[kMaxTopK];
  __shared__ __align__(16) float s_prob[kMaxTopK];
  __shared__ uint32_t live_key[kLiveMax];
  __shared__ int live_idx[kLiveMax];
  __shared__ int sh_count;
  __shared__ long long s_tok[kMaxTopK];
  __shared__ float s_draw[kMaxTopK];
  griddep_launch_dependents();  // the bookkeeping launch after this one may be scheduled
  griddep_wait();               // up to kPdlMaxRows streams a programmatic dependent: the logits come from the launch before

  const int b = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int V = p.vocab, KK = p.top_k, ipt = p.ipt;
  const Raw* src = reinterpret_cast<const Raw*>(static_cast<const T*>(p.logits) + (int64_t)b * p.row_stride);
  const Raw* bias = static_cast<const Raw*>(p.bias);
  const uint32_t* seen = p.seen ? p.seen + (int64_t)b * p.seen_words : nullptr;
  const bool pen = seen != nullptr && p.penalty != 1.0f;
  auto as_f = [](Raw r) {
    T t;
    memcpy(&t, &r, sizeof(Raw));
    return Elem<T>::to_f(t);
  };

  // 1. stage the row in shared memory.  The row starts o elements into a
  //    16-byte chunk; it is stored shifted by o (row = row_s + o) so that whole
  //    chunks move with 16-byte loads and stores and every thread's block below
  //    stays 16-byte aligned.  Then the penalty (a sparse pass over the set bits
  //    of the history bitmap) and the bias, in the reference's order.
  T* row_s = reinterpret_cast<T*>(smem_raw);
  const int o = (int)((reinterpret_cast<uintptr_t>(src) & 15u) / sizeof(T));
  T* row = row_s + o;
  {
    const int C = (V + o + E - 1) / E;  // chunks touched by the row
    const uint4* A = reinterpret_cast<const uint4*>(reinterpret_cast<uintptr_t>(src) - (uintptr_t)o * sizeof(T));
    for (int c0 = 0; c0 < C; c0 += kStageChunks * kSampleThreads) {
      uint4 v[kStageChunks];
#pragma unroll
      for (int r = 0; r < kStageChunks; ++r) {
        const int c = c0 + r * kSampleThreads + tid;
        const int i0 = c * E - o;
        if (c < C && i0 >= 0 && i0 + E <= V) v[r] = __ldg(A + c);
      }
#pragma unroll
      for (int r = 0; r < kStageChunks; ++r) {
        const int c = c0 + r * kSampleThreads + tid;
        const int i0 = c * E - o;
        if (c >= C) continue;
        if (i0 >= 0 && i0 + E <= V) {
          reinterpret_cast<uint4*>(row_s)[c] = v[r];
        } else {  // the partial first / last chunk: element loads inside the row only
          for (int e = 0; e < E; ++e) {
            const int i = i0 + e;
            if (i >= 0 && i < V) {
              const Raw x = __ldg(src + i);
              memcpy(row + i, &x, sizeof(Raw));
            }
          }
        }
      }
    }
  }
  __syncthreads();
  if (pen) {
    for (int w = tid; w < (V + 31) / 32; w += kSampleThreads) {
      uint32_t m = __ldg(seen + w);
      while (m) {
        const int i = 32 * w + __ffs(m) - 1;
        m &= m - 1u;
        if (i < V) {
          const float v = Elem<T>::to_f(row[i]);
          row[i] = Elem<T>::from_f(v > 0.f ? __fdiv_rn(v, p.penalty) : __fmul_rn(v, p.penalty));
        }
      }
    }
    __syncthreads();
  }
  if (bias) {
    for (int i = tid; i < V; i += kSampleThreads)
      row[i] = Elem<T>::from_f(__fadd_rn(Elem<T>::to_f(row[i]), as_f(__ldg(bias + i))));
    __syncthreads();
  }

  // this thread's block of the row: [base, base + ipt), ipt a multiple of E,
  // read from shared memory as 16-byte vectors; with REG the keys stay in
  // registers (ipt <= kRegItems), otherwise every pass re-reads shared memory
  const int base = tid * ipt;  // in row_s positions; row index = position - o
  auto keys_at = [&](int sp, uint32_t* key) {
    const uint4 raw = *reinterpret_cast<const uint4*>(row_s + sp);
    Raw v[E];
    memcpy(v, &raw, 16);
#pragma unroll
    for (int e = 0; e < E; ++e) key[e] = K::key(v[e]);
  };
  uint32_t rk[REG ? kRegItems : 1];
  if constexpr (REG) {
#pragma unroll
    for (int r = 0; r < kRegItems; r += E) {
      if (r < ipt) keys_at(base + r, rk + r);
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const int i = base + r + e - o;
        if (r >= ipt || i < 0 || i >= V) rk[r + e] = 0;  // never counted: thresholds are >= 1
      }
    }
  }
  // f(i, key) over this thread's items in index order
  auto for_items = [&](auto&& f) {
    if constexpr (REG) {
#pragma unroll
      for (int r = 0; r < kRegItems; ++r) {
        const int i = base + r - o;
        if (r < ipt && i >= 0 && i < V) f(i, rk[r]);
      }
    } else {
      for (int r = 0; r < ipt && base + r - o < V; r += E) {
        uint32_t key[E];
        keys_at(base + r, key);
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const int i = base + r + e - o;
          if (i >= 0 && i < V) f(i, key[e]);
        }
      }
    }
  };
  // block-wide counts of keys >= t[0..N) (each t >= 1); every thread gets the
  // totals.  Partial sums alternate between two buffers: one barrier per call.
  int parity = 0;
  auto count_ge = [&]<int N>(const uint32_t* t, int* tot) {
    int c[N];
#pragma unroll
    for (int n = 0; n < N; ++n) c[n] = 0;
    if constexpr (REG) {
#pragma unroll
      for (int r = 0; r < kRegItems; ++r)
#pragma unroll
        for (int n = 0; n < N; ++n) c[n] += rk[r] >= t[n] ? 1 : 0;
    } else {
      for_items([&](int, uint32_t k) {
#pragma unroll
        for (int n = 0; n < N; ++n) c[n] += k >= t[n] ? 1 : 0;
      });
    }
#pragma unroll
    for (int n = 0; n < N; ++n) {
      c[n] = __reduce_add_sync(0xffffffffu, c[n]);
      if (lane == 0) warp_sum[parity][n][warp] = c[n];
    }
    __syncthreads();
#pragma unroll
    for (int n = 0; n < N; ++n) tot[n] = __reduce_add_sync(0xffffffffu, warp_sum[parity][n][lane]);
    parity ^= 1;
  };

  // 2. the k-th largest key vk: the largest t with count(key >= t) >= k.
  //    Bracket it below the row's largest key (spans 2^(B-9), 2^(B-7), 2^(B-5)
  //    for B-bit keys, one barrier): count(>= lo) = c_lo >= k > count(>= hi) = c_hi.
  uint32_t mk = 0;
  for_items([&](int, uint32_t k) { mk = k > mk ? k : mk; });
  mk = __reduce_max_sync(0xffffffffu, mk);
  if (lane == 0) warp_max[warp] = mk;
  __syncthreads();
  const uint32_t maxk = __reduce_max_sync(0xffffffffu, warp_max[lane]);
  uint64_t hi = (uint64_t)maxk + 1, lo = 0;
  int c_hi = 0, c_lo = V;
  {
    uint32_t t[3];
    int c[3];
#pragma unroll
    for (int n = 0; n < 3; ++n) {
      const uint64_t w = 1ull << (K::kBits - 9 + 2 * n);
      t[n] = hi > w ? (uint32_t)(hi - w) : 1u;
    }
    count_ge.template operator()<3>(t, c);
    if (c[0] >= KK) {
      lo = t[0];
      c_lo = c[0];
    } else if (c[1] >= KK) {
      lo = t[1];
      c_lo = c[1];
      hi = t[0];
      c_hi = c[0];
    } else if (c[2] >= KK) {
      lo = t[2];
      c_lo = c[2];
      hi = t[1];
      c_hi = c[1];
    } else {
      hi = t[2];
      c_hi = c[2];
    }
  }

  // exclusive block scan of one int per thread (two barriers)
  auto block_excl_scan = [&](int v) -> int {
    int inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += u;
    }
    if (lane == 31) warp_tot[warp] = inc;
    __syncthreads();
    if (warp == 0) {
      const int t = warp_tot[lane];
      int ti = t;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, ti, o);
        if (lane >= o) ti += u;
      }
      warp_tot[lane] = ti - t;
    }
    __syncthreads();
    return warp_tot[warp] + inc - v;
  };
  // sort keys: value key, then lower index first; 32 bits when a 16-bit key and
  // a row index below 2^16 fit (16-bit types, rows held in registers)
  constexpr bool K32 = sizeof(T) == 2 && REG;
  auto put_greater = [&](int slot, uint32_t k, int i) {
    if (slot < kMaxTopK) {
      if constexpr (K32)
        reinterpret_cast<uint32_t*>(cand_key)[slot] = (k << 16) | (0xffffu - (uint32_t)i);
      else
        cand_key[slot] = ((unsigned long long)k << 32) | (unsigned long long)(0xffffffffu - (uint32_t)i);
      cand_val[slot] = value_of_key<T>(k);
      cand_idx[slot] = i;
    }
  };

  // c_gt keys above vk go to candidate slots [0, c_gt) (sorted in step 5); the
  // `need` equal keys taken at the boundary (lowest indices first) go straight
  // to their sorted positions [c_gt, k)
  int c_gt, need;
  if (c_lo - c_hi <= kLiveMax) {
    // 3a. few keys inside the bracket: keys >= hi are taken; the keys in
    //     [lo, hi) are compacted in index order and one warp finishes the search
    const int n_live = c_lo - c_hi;
    const int pos = block_excl_scan(
        [&] {
          int v = 0;
          for_items([&](int, uint32_t k) { v += k >= hi ? 1 : (k >= lo ? 512 : 0); });
          return v;
        }());
    int sure = pos & 511, live = pos >> 9;
    for_items([&](int i, uint32_t k) {
      if (k >= hi) {
        put_greater(sure++, k, i);
      } else if (k >= lo) {
        live_key[live] = k;
        live_idx[live] = i;
        ++live;
      }
    });
    __syncthreads();
    if (warp == 0) {
      uint64_t l2 = lo, h2 = hi;
      int ch = c_hi;
      // up to kLiveReg keys per lane stay in registers; a longer list is re-read
      uint32_t lk[kLiveReg];
      const bool in_reg = n_live <= 32 * kLiveReg;
#pragma unroll
      for (int j = 0; j < kLiveReg; ++j) {
        const int m = lane + 32 * j;
        lk[j] = (in_reg && m < n_live) ? live_key[m] : 0u;  // key 0 is never counted (mid >= 1)
      }
      while (h2 - l2 > 1) {
        const uint32_t mid = (uint32_t)((l2 + h2) >> 1);
        int c = 0;
        if (in_reg) {
#pragma unroll
          for (int j = 0; j < kLiveReg; ++j) c += lk[j] >= mid ? 1 : 0;
        } else {
#pragma unroll 4
          for (int m = lane; m < n_live; m += 32) c += live_key[m] >= mid ? 1 : 0;
        }
        c = __reduce_add_sync(0xffffffffu, c) + c_hi;
        if (c >= KK) {
          l2 = mid;
        } else {
          h2 = mid;
          ch = c;
        }
      }
      const uint32_t vk = (uint32_t)l2;
      const int nd = KK - ch;
      int gbase = c_hi, ebase = 0;
      const uint32_t below = (1u << lane) - 1u;
      // list order is index order: equal keys are ranked by ballots round by round
      auto place = [&](int m, uint32_t k) {
        const bool gt = m < n_live && k > vk, eq = m < n_live && k == vk;
        const uint32_t bg = __ballot_sync(0xffffffffu, gt), be = __ballot_sync(0xffffffffu, eq);
        if (gt) put_greater(gbase + __popc(bg & below), k, live_idx[m]);
        if (eq) {
          const int r = ebase + __popc(be & below);
          if (r < nd) {
            s_val[ch + r] = value_of_key<T>(k);
            s_idx[ch + r] = live_idx[m];
          }
        }
        gbase += __popc(bg);
        ebase += __popc(be);
      };
      if (in_reg) {
#pragma unroll
        for (int j = 0; j < kLiveReg; ++j)
          if (32 * j < n_live) place(lane + 32 * j, lk[j]);
      } else {
        for (int m0 = 0; m0 < n_live; m0 += 32) {
          const int m = m0 + lane;
          place(m, m < n_live ? live_key[m] : 0u);
        }
      }
      if (lane == 0) sh_count = ch;
    }
    __syncthreads();
    c_gt = sh_count;
    need = KK - c_gt;
  } else {
    // 3b. bisection inside the bracket over all keys, then one block scan of
    //     packed (greater, equal) counts (the greater total is < k <= 256)
    while (hi - lo > 1) {
      const uint32_t mid = (uint32_t)((lo + hi) >> 1);
      int c;
      count_ge.template operator()<1>(&mid, &c);
      if (c >= KK) {
        lo = mid;
      } else {
        hi = mid;
        c_hi = c;
      }
    }
    const uint32_t vk = (uint32_t)lo;
    c_gt = c_hi;
    need = KK - c_gt;
    const int excl = block_excl_scan(
        [&] {
          int v = 0;
          for_items([&](int, uint32_t k) { v += k > vk ? 1 : (k == vk ? 512 : 0); });
          return v;
        }());
    int gt_slot = excl & 511, eq_rank = excl >> 9;
    for_items([&](int i, uint32_t k) {
      if (k > vk) {
        put_greater(gt_slot++, k, i);
      } else if (k == vk) {
        if (eq_rank < need) {
          s_val[c_gt + eq_rank] = value_of_key<T>(k);
          s_idx[c_gt + eq_rank] = i;
        }
        ++eq_rank;
      }
    });
    __syncthreads();
  }

  // 5. sort the greater keys descending (all distinct): rank = number larger.
  //    Thread (q, j) counts over quarter q of the keys; a warp reads one key
  //    pair per step at a single address (a broadcast).
  {
    const int j = tid & (kMaxTopK - 1), q = tid / kMaxTopK;
    constexpr int QN = kMaxTopK / (kSampleThreads / kMaxTopK);
    int part = 0;
    if (q * QN < c_gt) {
      const int n = min(QN, c_gt - q * QN);
      if constexpr (K32) {
        const uint32_t* ck = reinterpret_cast<const uint32_t*>(cand_key);
        const uint32_t kj = j < c_gt ? ck[j] : 0xffffffffu;
        const uint4* ck4 = reinterpret_cast<const uint4*>(ck + q * QN);
#pragma unroll 4
        for (int m = 0; m < QN / 4; ++m) {
          if (4 * m < n) {
            const uint4 kk = ck4[m];
            part += kk.x > kj ? 1 : 0;
            part += (4 * m + 1 < n && kk.y > kj) ? 1 : 0;
            part += (4 * m + 2 < n && kk.z > kj) ? 1 : 0;
            part += (4 * m + 3 < n && kk.w > kj) ? 1 : 0;
          }
        }
      } else {
        const unsigned long long kj = j < c_gt ? cand_key[j] : ~0ull;
        const ulonglong2* ck2 = reinterpret_cast<const ulonglong2*>(cand_key + q * QN);
#pragma unroll 8
        for (int m = 0; m < QN / 2; ++m) {
          if (2 * m < n) {
            const ulonglong2 kk = ck2[m];
            part += kk.x > kj ? 1 : 0;
            part += (2 * m + 1 < n && kk.y > kj) ? 1 : 0;
          }
        }
      }
    }
    rank_part[q][j] = part;
  }
  __syncthreads();
  if (tid < c_gt) {
    int rank = 0;
#pragma unroll
    for (int q = 0; q < kSampleThreads / kMaxTopK; ++q) rank += rank_part[q][tid];
    s_val[rank] = cand_val[tid];
    s_idx[rank] = cand_idx[tid];
  }
  __syncthreads();
  // 6. warps 1..8 fetch every candidate's token id and Exp(1) draw into shared
  //    memory and arrive on named barrier 1; warp 0 runs temperature, softmax
  //    and top-p meanwhile and meets the barrier only before the race.
  if (warp != 0) {
    const int j = tid - 32;
    if (j < kMaxTopK) {
      if (j < KK) {
        const int idx = s_idx[j];
        s_tok[j] = p.index_map ? __ldg(p.index_map + idx) : (long long)idx;
        float d;
        if (p.draws) {
          d = __ldg(p.draws + (int64_t)b * KK + j);
        } else {
          const uint64_t step = p.step ? (uint64_t)*p.step : 0ull;
          const uint4 w = philox4x32_10(make_uint4((uint32_t)(j >> 2), (uint32_t)b, (uint32_t)step,
                                                   (uint32_t)(step >> 32)),
                                        make_uint2((uint32_t)p.seed, (uint32_t)(p.seed >> 32)));
          const int q = j & 3;
          d = exp_draw(q == 0 ? w.x : q == 1 ? w.y : q == 2 ? w.z : w.w);
        }
        s_draw[j] = d;
      }
      __syncwarp();
      asm volatile("bar.arrive 1, %0;" ::"n"(32 + kMaxTopK) : "memory");
    }
    return;
  }

  // 7. warp 0: lane owns sorted positions lane*P .. lane*P+P-1
  float x[P];
#pragma unroll
  for (int e = 0; e < P; ++e) {
    const int j = lane * P + e;
    float v = j < KK ? s_val[j] : -INFINITY;
    if (j < KK && p.temperature != 1.0f) v = round_to<T>(__fdiv_rn(v, p.temperature));
    x[e] = v;
  }
  const float mx = __shfl_sync(0xffffffffu, x[0], 0);

  auto softmax = [&](int keep, float* out) {
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < P; ++e) {
      const int j = lane * P + e;
      out[e] = j < keep ? expf(__fsub_rn(x[e], mx)) : 0.f;
      s = __fadd_rn(s, out[e]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
    const float inv = __frcp_rn(s);
#pragma unroll
    for (int e = 0; e < P; ++e) out[e] = round_to<T>(__fmul_rn(out[e], inv));
  };

  float pr[P];
  int keep = KK;
  if (p.top_p < 1.0f) {
    softmax(KK, pr);
    // first dropped position: smallest j >= 1 with round(c[j-1]) >= round(top_p),
    // c the in-order running sum (fp32; double for f32).  Every value of a
    // 16-bit type at or above kExactMin<T> is a multiple of 2^-24, so while the
    // sum stays below 1 every partial sum is exact whatever the order: a warp
    // scan then gives the in-order sums bit for bit.  Otherwise one lane runs
    // the in-order add chain.
    const float thr = round_to<T>(p.top_p);
    bool done = false;
    if constexpr (sizeof(T) == 2) {
      float loc[P], run = 0.f;
#pragma unroll
      for (int e = 0; e < P; ++e) {
        run = __fadd_rn(run, pr[e]);
        loc[e] = run;
      }
      float incl = run;  // inclusive scan of lane totals
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl = __fadd_rn(incl, v);
      }
      float ex = __shfl_up_sync(0xffffffffu, incl, 1);
      if (lane == 0) ex = 0.f;
      int first = P;  // first position of this lane whose sum reaches the threshold
#pragma unroll
      for (int e = P - 1; e >= 0; --e) {
        const int j = lane * P + e;
        if (j + 1 < KK && round_to<T>(__fadd_rn(ex, loc[e])) >= thr) first = e;
      }
      const uint32_t any = __ballot_sync(0xffffffffu, first < P);
      const int hl = any ? __ffs(any) - 1 : 31;  // lane holding the decisive position
      const int he = __shfl_sync(0xffffffffu, first, hl);
      const int jd = any ? hl * P + he : KK - 2;  // last position whose sum is used
      // exact up to jd when every value there is >= kExactMin<T> and the sum at
      // jd (the largest: the values are non-negative) is below 1; a computed sum
      // below 1 implies every partial sum below 1 (rounding is monotone)
      uint32_t pmin = 0xffffffffu;  // non-negative floats order like their bits
      float sd = 0.f;
#pragma unroll
      for (int e = 0; e < P; ++e) {
        const int j = lane * P + e;
        if (j <= jd) pmin = min(pmin, __float_as_uint(pr[e]));
        if (j == jd) sd = __fadd_rn(ex, loc[e]);
      }
      pmin = __reduce_min_sync(0xffffffffu, pmin);
      sd = __shfl_sync(0xffffffffu, sd, jd < 0 ? 0 : jd / P);
      if (jd < 0 || (__uint_as_float(pmin) >= kExactMin<T> && sd < 1.0f)) {
        keep = any ? jd + 1 : KK;
        done = true;
      }
    }
    if (!done) {
      float4* sp4 = reinterpret_cast<float4*>(s_prob);
      sp4[lane * 2] = make_float4(pr[0], pr[1], pr[2], pr[3]);
      sp4[lane * 2 + 1] = make_float4(pr[4], pr[5], pr[6], pr[7]);
      __syncwarp();
      if (lane == 0) {
        using Acc = typename CumAcc<T>::type;
        Acc c = 0;
        for (int j0 = 0; j0 < KK - 1; j0 += 8) {
          const float4 a = sp4[j0 / 4], bq = sp4[j0 / 4 + 1];
          const float pv[8] = {a.x, a.y, a.z, a.w, bq.x, bq.y, bq.z, bq.w};
          Acc cs[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            c += (Acc)pv[e];
            cs[e] = c;
          }
          int hit = 8;
#pragma unroll
          for (int e = 7; e >= 0; --e)
            if (j0 + e + 1 < KK && round_to<T>((float)cs[e]) >= thr) hit = e;
          if (hit < 8) {
            keep = j0 + hit + 1;
            break;
          }
        }
      }
      keep = __shfl_sync(0xffffffffu, keep, 0);
    }
  }
  softmax(keep, pr);

  // 8. exponential race over the kept candidates: first maximum of round(p / round(E))
  asm volatile("bar.sync 1, %0;" ::"n"(32 + kMaxTopK) : "memory");
  float draw[P];
#pragma unroll
  for (int e = 0; e < P; ++e) draw[e] = lane * P + e < KK ? s_draw[lane * P + e] : 1.f;
  float best = -1.f;
  int best_j = 0x7fffffff;
#pragma unroll
  for (int e = 0; e < P; ++e) {
    const int j = lane * P + e;
    if (j < KK) {
      const float s = round_to<T>(__fdiv_rn(pr[e], round_to<T>(draw[e])));
      if (s > best) {
        best = s;
        best_j = j;
      }
      if (p.draws_out) p.draws_out[(int64_t)b * KK + j] = draw[e];
      if (p.probs_out) static_cast<T*>(p.probs_out)[(int64_t)b * KK + j] = Elem<T>::from_f(pr[e]);
      if (p.cand_out) p.cand_out[(int64_t)b * KK + j] = s_idx[j];
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oj = __shfl_xor_sync(0xffffffffu, best_j, o);
    if (ob > best || (ob == best && oj < best_j)) {
      best = ob;
      best_j = oj;
    }
  }
  if (best_j >= KK) best_j = 0;  // unreachable: position 0 always has a positive score
  if (lane == 0) {
    int idx = s_idx[best_j];
    if (idx < 0 || idx >= V) idx = 0;  // unreachable: every sorted slot holds a row index
    p.tokens[(int64_t)b * p.tokens_stride] = s_tok[best_j];
    if (p.update_seen && p.seen) atomicOr(p.seen + (int64_t)b * p.seen_words + (idx >> 5), 1u << (idx & 31));
  }
}

template <typename T>
int launch_sample(SampleParams prm, int64_t batch, cudaStream_t s) {
  constexpr int E = VecN<T>::value;
  int ipt = (prm.vocab + E - 1 + kSampleThreads - 1) / kSampleThreads;  // room for a shift of up to E-1
  ipt = (ipt + E - 1) / E * E;
  const size_t smem = (size_t)ipt * kSampleThreads * sizeof(T);
  if (smem > (size_t)kSampleMaxDynSmem) return KANI_ERR_UNSUPPORTED;
  prm.ipt = ipt;
  auto kern = ipt <= kRegItems ? sample_kernel<T, true> : sample_kernel<T, false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return (int)e;
  launch_maybe_pdl(batch <= kPdlMaxRows, kern, dim3((unsigned)batch), dim3(kSampleThreads), smem, s, prm);
  return launch_status();
}

}  // namespace
}  // namespace kani

extern "C" int kani_sample_tokens(int32_t dtype, const void* logits, int64_t logits_row_stride, int64_t batch,
                                  int32_t vocab, const void* logit_bias, uint32_t* seen_bitmap,
                                  int64_t seen_row_words, int32_t update_seen, float repetition_penalty,
                                  float temperature, float top_p, int32_t top_k, const int64_t* index_map,
                                  uint64_t seed, const int64_t* step_counter, const float* exp_draws,
                                  float* draws_out, void* probs_out, int32_t* cand_out, int64_t* tokens_out,
                                  int64_t tokens_out_stride, void* stream) {
  if (batch < 0) return KANI_ERR_INVALID_ARG;
  if (batch == 0) return KANI_OK;
  if (batch > 0x7fffffff || vocab < 1 || top_k < 1 || top_k > kani::kMaxTopK || top_k > vocab)
    return KANI_ERR_INVALID_ARG;
  if (!logits || !tokens_out) return KANI_ERR_INVALID_ARG;
  if (!(temperature > 0.f) || !isfinite(temperature) || !(repetition_penalty > 0.f) ||
      !isfinite(repetition_penalty) || isnan(top_p))
    return KANI_ERR_INVALID_ARG;
  if (batch > 1 && (logits_row_stride < vocab || tokens_out_stride < 1)) return KANI_ERR_INVALID_ARG;
  if (seen_bitmap && seen_row_words < (vocab + 31) / 32) return KANI_ERR_INVALID_ARG;
  kani::SampleParams prm{};
  prm.logits = logits;
  prm.row_stride = logits_row_stride;
  prm.bias = logit_bias;
  prm.seen = seen_bitmap;
  prm.seen_words = seen_row_words;
  prm.update_seen = update_seen;
  prm.penalty = repetition_penalty;
  prm.temperature = temperature;
  prm.top_p = top_p;
  prm.vocab = vocab;
  prm.top_k = top_k;
  prm.index_map = index_map;
  prm.seed = seed;
  prm.step = step_counter;
  prm.draws = exp_draws;
  prm.draws_out = draws_out;
  prm.probs_out = probs_out;
  prm.cand_out = cand_out;
  prm.tokens = tokens_out;
  prm.tokens_stride = tokens_out_stride;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return kani::dispatch_dtype(dtype, [&]<typename T>() { return kani::launch_sample<T>(prm, batch, s); });
}
