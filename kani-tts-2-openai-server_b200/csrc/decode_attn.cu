// GQA decode attention over the valid cache prefix (sm_100a).
//
// Computes, per stream b and query head hq (KV head h = hq / G),
//     out[b, hq, :] = softmax_j(scale * q[b, hq, :] . K[b, h, j, :]) V[b, h, j, :],
// over cache slots j in [0, kv_len[b]).  This is the attention the reference
// decode step runs as SDPA over the whole static buffer with an additive
// -inf mask (kani_tts/optimized_decode.py:243-248; mask built at
// kani_tts/inference_engine.py:259-265 and opened slot by slot at :643,
// always a prefix); here only the valid prefix is read.
//
// Structure: one thread-block cluster of CTAs per (b, h) (8 in the register
// variant; 1, 2, 4 or 8 in the TMA variant, as many as it takes to give the
// GPU about four CTAs per SM).  The valid prefix is split evenly over the
// cluster's CTAs; inside a CTA, lane
// = (key group kg in 0..7, dim slice ds in 0..3): four lanes share one key,
// each holding D/4 dims of it and of all G query heads, so a score is a
// 2-step shuffle sum and K/V rows are read with 16-byte loads.  Each lane
// keeps an online softmax (running max, sum, weighted V) per query head in
// fp32 (base-2 exponentials, the query pre-scaled by scale * log2 e).  The
// partials are merged across key groups by shuffles, across the CTA's warps
// through shared memory, and across the cluster through distributed shared
// memory in CTA rank 0, which writes the normalised output with one
// rounding.  No global scratch is used; the cluster barriers are hardware
// barriers that every CTA of the cluster reaches.  With contiguous cache rows
// the K/V range is staged by TMA (decode_attn_kernel below: each CTA pushes
// its partial into rank 0, one split barrier); otherwise the register
// variant reads it directly (rank 0 pulls the partials between two barriers).
#include <atomic>

#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace kani {
namespace {

constexpr int kClusterCTAs = 8;
constexpr int kAttnThreads = 128;

struct AttnParams {
  const void* q;
  int64_t qb, qh;  // strides of q [B, Hq, D]
  const void* k;
  const void* v;
  int64_t cb, ch, cs;  // cache strides [B, Hk, S, D]
  int64_t cache_len;
  const int64_t* kv_len;
  void* out;
  int64_t ob, oh;  // strides of out [B, Hq, D]
  float qscale;    // scale * log2(e)
  int32_t* err;
  long long wait_cycles = 0;  // bound of each tile's first mbarrier wait (WaitBound)
  unsigned wait_suspend_ns = 0;
};

// 2^x with the hardware approximation (ex2.approx: relative error ~2^-22,
// ample for softmax weights that end in a bf16 output).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float merge_weight(float m, float mnew) {
  return m == -INFINITY ? 0.f : ex2(m - mnew);
}

template <typename T, int G, int D>
__global__ void __cluster_dims__(kClusterCTAs, 1, 1) __launch_bounds__(kAttnThreads)
decode_attn_reg_kernel(AttnParams p) {
  griddep_launch_dependents();  // a dependent GEMV may start streaming its weights
  constexpr int DL = D / 4;           // dims per lane
  constexpr int VE = VecN<T>::value;  // elements per 16-byte vector
  constexpr int NV = DL / VE;         // 16-byte vectors per lane per row
  constexpr int NW = kAttnThreads / 32;
  cg::cluster_group cluster = cg::this_cluster();
  const int crank = (int)cluster.block_rank();
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kg = lane >> 2, ds = lane & 3;

  __shared__ float w_m[NW][G], w_l[NW][G];
  __shared__ float w_acc[NW][G][D];
  __shared__ float c_m[G], c_l[G];
  __shared__ float c_acc[G][D];

  int64_t len = p.kv_len[b];
  if (len > p.cache_len) {
    if (crank == 0 && threadIdx.x == 0 && h == 0 && p.err != nullptr) atomicOr(p.err, KANI_FLAG_SLOT_OOB);
    len = p.cache_len;
  }
  if (len < 0) len = 0;
  const int64_t chunk = (len + kClusterCTAs - 1) / kClusterCTAs;
  const int64_t k0 = crank * chunk;
  const int64_t k1 = k0 + chunk < len ? k0 + chunk : len;

  // the G query heads of this KV head, this lane's dims, pre-scaled
  float q[G][DL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const T* qp = static_cast<const T*>(p.q) + b * p.qb + (int64_t)(h * G + g) * p.qh + ds * DL;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      float f[VE];
      unpack16<T>(ld16(qp + v * VE), f);
#pragma unroll
      for (int e = 0; e < VE; ++e) q[g][v * VE + e] = f[e] * p.qscale;
    }
  }

  float m[G], l[G], acc[G][DL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int d = 0; d < DL; ++d) acc[g][d] = 0.f;
  }

  const T* kbase = static_cast<const T*>(p.k) + b * p.cb + (int64_t)h * p.ch + ds * DL;
  const T* vbase = static_cast<const T*>(p.v) + b * p.cb + (int64_t)h * p.ch + ds * DL;
  // warp-uniform loop: every lane reaches the shuffles
  for (int64_t base = k0 + warp * 8; base < k1; base += 8 * NW) {
    const int64_t j = base + kg;
    const bool valid = j < k1;
    uint4 kv[NV], vv[NV];
    if (valid) {
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        kv[v] = ld16_stream(kbase + j * p.cs + v * VE);
        vv[v] = ld16_stream(vbase + j * p.cs + v * VE);
      }
    }
    float kf[DL], vf[DL];
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      unpack16<T>(valid ? kv[v] : make_uint4(0, 0, 0, 0), kf + v * VE);
      unpack16<T>(valid ? vv[v] : make_uint4(0, 0, 0, 0), vf + v * VE);
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float s = 0.f;
#pragma unroll
      for (int d = 0; d < DL; ++d) s = fmaf(q[g][d], kf[d], s);
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      if (valid) {
        const float mn = fmaxf(m[g], s);
        const float corr = merge_weight(m[g], mn);
        const float pr = ex2(s - mn);
        l[g] = fmaf(l[g], corr, pr);
#pragma unroll
        for (int d = 0; d < DL; ++d) acc[g][d] = fmaf(acc[g][d], corr, pr * vf[d]);
        m[g] = mn;
      }
    }
  }

  // merge the 8 key groups of the warp (lanes with the same dim slice)
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float mo = __shfl_xor_sync(0xffffffffu, m[g], off);
      const float lo = __shfl_xor_sync(0xffffffffu, l[g], off);
      const float mn = fmaxf(m[g], mo);
      const float wa = merge_weight(m[g], mn), wb = merge_weight(mo, mn);
      l[g] = l[g] * wa + lo * wb;
#pragma unroll
      for (int d = 0; d < DL; ++d) {
        const float ao = __shfl_xor_sync(0xffffffffu, acc[g][d], off);
        acc[g][d] = acc[g][d] * wa + ao * wb;
      }
      m[g] = mn;
    }
  }
  if (kg == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      if (ds == 0) {
        w_m[warp][g] = m[g];
        w_l[warp][g] = l[g];
      }
#pragma unroll
      for (int d = 0; d < DL; ++d) w_acc[warp][g][ds * DL + d] = acc[g][d];
    }
  }
  __syncthreads();
  // merge the warps: one (head, dim) per thread
  for (int t = threadIdx.x; t < G * D; t += kAttnThreads) {
    const int g = t / D, d = t - (t / D) * D;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) mx = fmaxf(mx, w_m[w][g]);
    float ls = 0.f, as = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float wt = merge_weight(w_m[w][g], mx);
      ls += w_l[w][g] * wt;
      as += w_acc[w][g][d] * wt;
    }
    c_acc[g][d] = as;
    if (d == 0) {
      c_m[g] = mx;
      c_l[g] = ls;
    }
  }
  cluster.sync();  // every CTA's partial is in its shared memory
  if (crank == 0) {
    for (int t = threadIdx.x; t < G * D; t += kAttnThreads) {
      const int g = t / D, d = t - (t / D) * D;
      float mr[kClusterCTAs];
      float mx = -INFINITY;
#pragma unroll
      for (int r = 0; r < kClusterCTAs; ++r) {
        mr[r] = *cluster.map_shared_rank(&c_m[g], r);
        mx = fmaxf(mx, mr[r]);
      }
      float ls = 0.f, as = 0.f;
#pragma unroll
      for (int r = 0; r < kClusterCTAs; ++r) {
        const float wt = merge_weight(mr[r], mx);
        ls += *cluster.map_shared_rank(&c_l[g], r) * wt;
        as += *cluster.map_shared_rank(&c_acc[g][d], r) * wt;
      }
      T* o = static_cast<T*>(p.out) + b * p.ob + (int64_t)(h * G + g) * p.oh + d;
      *o = Elem<T>::from_f(ls > 0.f ? as / ls : 0.f);
    }
  }
  cluster.sync();  // rank 0 has read the other CTAs' shared memory
}

// ------------------------------------------------------- TMA-staged variant
// Same math and lane layout; the CTA's key range is brought into a ring of
// STAGES shared-memory stages of TILE keys (K tile + V tile) by TMA bulk
// copies completing on one mbarrier per stage (plain bulk copies, each
// targeting this CTA only), so the bytes in flight are bounded by shared
// memory instead of registers.  Needs contiguous cache rows (slot stride ==
// head_dim).  Each lane takes two keys per tile pass and rescales its running
// sums once per pair; NW warps take 16 * NW keys per pass.  Two shapes: 4
// warps over 64-key tiles (3 stages) for many streams, and 8 warps over
// 128-key tiles (2 stages) for up to 4 streams, where each CTA's share of the
// prefix (at most 256 keys of a 2048-slot cache) is one or two passes.
//
// The CTAs of a cluster merge their partials by pushing them into rank 0's
// shared memory (distributed shared-memory stores), then one split cluster
// barrier (arrive.release / wait.acquire); rank 0 finishes alone from its own
// shared memory.  A barrier phase armed at kernel entry and waited on before
// the first remote store makes sure every CTA of the cluster has started.
// Waits are bounded (KANI_FLAG_TIMEOUT); a CTA that times out contributes an
// empty partial and still reaches both barrier phases.
constexpr int kAttnTile = 64;
constexpr int kAttnStages = 3;
constexpr int kAttnWideTile = 128;
constexpr int kAttnWideStages = 2;
constexpr int kAttnWideWarps = 8;
constexpr long long kAttnWaitCycles = 2000000000LL;  // ~1 s

__device__ __forceinline__ uint32_t attn_smem_u32(const void* ptr) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(ptr));
}

// One wait attempt.  With a suspend hint the thread may sleep (up to the hint,
// in ns) until the phase completes, so a waiting warp leaves the issue slots
// free; with none (a test's short limit) it only tests the phase, since a
// try_wait without a hint may still block for a system-defined time.
__device__ __forceinline__ bool attn_try_wait(uint32_t bar, uint32_t parity, uint32_t suspend_ns) {
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

__device__ __forceinline__ bool attn_wait_bounded(uint32_t bar, uint32_t parity,
                                                  long long limit = kAttnWaitCycles,
                                                  uint32_t suspend_ns = kWaitSuspendNs) {
  if (attn_try_wait(bar, parity, suspend_ns)) return true;
  const long long start = clock64();
  while (!attn_try_wait(bar, parity, suspend_ns)) {
    if (clock64() - start > limit) return false;
  }
  return true;
}

__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

template <typename T, int G, int D, int NW, int TILE, int STAGES>
__global__ void __launch_bounds__(NW * 32)
decode_attn_kernel(AttnParams p) {
  griddep_launch_dependents();  // a dependent GEMV may start streaming its weights
  constexpr int NT = NW * 32;
  constexpr int DL = D / 4;
  constexpr int VE = VecN<T>::value;
  constexpr int NV = DL / VE;
  constexpr uint32_t ROW = D * sizeof(T);
  constexpr uint32_t TILE_BYTES = TILE * ROW;
  static_assert(TILE % (16 * NW) == 0, "a tile is whole passes of 16 keys per warp");
  extern __shared__ __align__(128) unsigned char ring[];  // [stage][K tile | V tile]
  __shared__ __align__(8) uint64_t bars[STAGES];
  __shared__ float w_m[NW][G], w_l[NW][G];
  __shared__ float w_acc[NW][G][D];
  __shared__ float g_m[kClusterCTAs][G], g_l[kClusterCTAs][G];  // rank 0: the cluster's partials
  __shared__ float g_acc[kClusterCTAs][G][D];

  cg::cluster_group cluster = cg::this_cluster();
  const int crank = (int)cluster.block_rank();
  const int ncl = (int)cluster.num_blocks();  // CTAs splitting this (b, h): 1, 2, 4 or 8
  if (ncl > 1) cluster_arrive_relaxed();      // phase 1: this CTA has started
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int kg = lane >> 2, ds = lane & 3;

  int64_t len = p.kv_len[b];
  if (len > p.cache_len) {
    if (crank == 0 && tid == 0 && h == 0 && p.err != nullptr) atomicOr(p.err, KANI_FLAG_SLOT_OOB);
    len = p.cache_len;
  }
  if (len < 0) len = 0;
  const int64_t chunk = (len + ncl - 1) / ncl;
  const int64_t k0 = crank * chunk;
  const int64_t k1 = k0 + chunk < len ? k0 + chunk : len;
  const int n = k1 > k0 ? (int)(k1 - k0) : 0;
  const int ntiles = (n + TILE - 1) / TILE;
  const char* kb = reinterpret_cast<const char*>(static_cast<const T*>(p.k) + b * p.cb + (int64_t)h * p.ch + k0 * p.cs);
  const char* vb = reinterpret_cast<const char*>(static_cast<const T*>(p.v) + b * p.cb + (int64_t)h * p.ch + k0 * p.cs);

  // thread 0: tile t into stage t % STAGES.  part 0: the whole tile; part 1:
  // the stage's expected bytes and every row but the tile's last; part 2: that
  // last row alone (the stage's phase completes once both parts have landed)
  auto issue = [&](int t, int part = 0) {
    const int st = t % STAGES;
    const int rows = n - t * TILE < TILE ? n - t * TILE : TILE;
    const uint32_t bytes = (uint32_t)rows * ROW;
    const uint32_t bar = attn_smem_u32(&bars[st]);
    const uint32_t dst = attn_smem_u32(ring + (size_t)st * 2 * TILE_BYTES);
    if (part != 2)
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(2 * bytes) : "memory");
    const uint32_t r0 = part == 2 ? (uint32_t)(rows - 1) * ROW : 0u;
    const uint32_t nb = part == 0 ? bytes : (part == 1 ? bytes - ROW : ROW);
    if (nb == 0) return;
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst + r0),
                 "l"(kb + (int64_t)t * TILE_BYTES + r0), "r"(nb), "r"(bar) : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     dst + TILE_BYTES + r0),
                 "l"(vb + (int64_t)t * TILE_BYTES + r0), "r"(nb), "r"(bar) : "memory");
  };
  // The newest row, len - 1, is the only one a decode step's previous launch
  // (its RoPE + KV write) may still be writing; it is the last row of this
  // CTA's range, so the last row of its tile.  Launched as a programmatic
  // dependent (kani_decode_attention_step), the first tiles stream in before
  // griddepcontrol.wait, all but that row, which is fetched after it; launched
  // plainly, the wait returns at once and the order does not matter.
  const int t_new = (len - 1 >= k0 && len - 1 < k1) ? (int)((len - 1 - k0) / TILE) : -1;
  if (tid == 0) {
    for (int st = 0; st < STAGES; ++st)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(attn_smem_u32(&bars[st])), "r"(1) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int t = 0; t < ntiles && t < STAGES; ++t) issue(t, t == t_new ? 1 : 0);
  }
  griddep_wait();  // q and the newest row may come from the launch before
  if (tid == 0 && t_new >= 0 && t_new < STAGES) issue(t_new, 2);

  // query heads (global) while the first tiles stream in
  float q[G][DL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const T* qp = static_cast<const T*>(p.q) + b * p.qb + (int64_t)(h * G + g) * p.qh + ds * DL;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      float f[VE];
      unpack16<T>(ld16(qp + v * VE), f);
#pragma unroll
      for (int e = 0; e < VE; ++e) q[g][v * VE + e] = f[e] * p.qscale;
    }
  }
  float m[G], l[G], acc[G][DL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int d = 0; d < DL; ++d) acc[g][d] = 0.f;
  }
  __syncthreads();  // barriers initialised

  bool failed = false;
  int t_fail = ntiles;
  for (int t = 0; t < ntiles; ++t) {
    const int st = t % STAGES;
    if (!failed && !attn_wait_bounded(attn_smem_u32(&bars[st]), (uint32_t)((t / STAGES) & 1),
                                      p.wait_cycles, p.wait_suspend_ns)) {
      failed = true;
      t_fail = t;
      if (lane == 0 && p.err != nullptr) atomicOr(p.err, KANI_FLAG_TIMEOUT);
    }
    const int rows = n - t * TILE < TILE ? n - t * TILE : TILE;
    const T* ktile = reinterpret_cast<const T*>(ring + (size_t)st * 2 * TILE_BYTES);
    const T* vtile = reinterpret_cast<const T*>(ring + (size_t)st * 2 * TILE_BYTES + TILE_BYTES);
    // two keys per lane group per pass: r0 and r0 + 8*NW
#pragma unroll 1
    for (int base = warp * 8; base < TILE; base += 16 * NW) {
      const int r0 = base + kg, r1 = base + kg + 8 * NW;
      const bool v0 = !failed && r0 < rows, v1 = !failed && r1 < rows;
      float k0f[DL], k1f[DL];
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        unpack16<T>(v0 ? ld16(ktile + r0 * D + ds * DL + v * VE) : make_uint4(0, 0, 0, 0), k0f + v * VE);
        unpack16<T>(v1 ? ld16(ktile + r1 * D + ds * DL + v * VE) : make_uint4(0, 0, 0, 0), k1f + v * VE);
      }
      float s0[G], s1[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        // paired fp32 FMAs: two dims per instruction, two chains per key
        float2 a0 = make_float2(0.f, 0.f), a1 = a0;
#pragma unroll
        for (int d = 0; d < DL; d += 2) {
          const float2 qq = make_float2(q[g][d], q[g][d + 1]);
          a0 = __ffma2_rn(qq, make_float2(k0f[d], k0f[d + 1]), a0);
          a1 = __ffma2_rn(qq, make_float2(k1f[d], k1f[d + 1]), a1);
        }
        float x0 = a0.x + a0.y, x1 = a1.x + a1.y;
        x0 += __shfl_xor_sync(0xffffffffu, x0, 1);
        x1 += __shfl_xor_sync(0xffffffffu, x1, 1);
        x0 += __shfl_xor_sync(0xffffffffu, x0, 2);
        x1 += __shfl_xor_sync(0xffffffffu, x1, 2);
        s0[g] = v0 ? x0 : -INFINITY;
        s1[g] = v1 ? x1 : -INFINITY;
      }
      if (v0 || v1) {
        float vf0[DL], vf1[DL];
#pragma unroll
        for (int v = 0; v < NV; ++v) {
          unpack16<T>(v0 ? ld16(vtile + r0 * D + ds * DL + v * VE) : make_uint4(0, 0, 0, 0), vf0 + v * VE);
          unpack16<T>(v1 ? ld16(vtile + r1 * D + ds * DL + v * VE) : make_uint4(0, 0, 0, 0), vf1 + v * VE);
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float mn = fmaxf(m[g], fmaxf(s0[g], s1[g]));
          const float corr = merge_weight(m[g], mn);
          const float p0 = v0 ? ex2(s0[g] - mn) : 0.f;
          const float p1 = v1 ? ex2(s1[g] - mn) : 0.f;
          l[g] = fmaf(l[g], corr, p0 + p1);
          const float2 c2 = make_float2(corr, corr), p02 = make_float2(p0, p0), p12 = make_float2(p1, p1);
#pragma unroll
          for (int d = 0; d < DL; d += 2) {
            const float2 w = __ffma2_rn(p02, make_float2(vf0[d], vf0[d + 1]),
                                        __fmul2_rn(p12, make_float2(vf1[d], vf1[d + 1])));
            const float2 r = __ffma2_rn(make_float2(acc[g][d], acc[g][d + 1]), c2, w);
            acc[g][d] = r.x;
            acc[g][d + 1] = r.y;
          }
          m[g] = mn;
        }
      }
    }
    if (t + STAGES < ntiles) {
      __syncthreads();  // stage st is free again
      if (tid == 0 && !failed) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        issue(t + STAGES);
      }
    }
  }
  if (failed && tid == 0) {
    // tiles t_fail .. t_fail + STAGES - 1 were issued and never consumed:
    // let those copies into this CTA's shared memory land before it exits
    for (int t = t_fail; t < ntiles && t < t_fail + STAGES; ++t)
      attn_wait_bounded(attn_smem_u32(&bars[t % STAGES]), (uint32_t)((t / STAGES) & 1));
  }

  // merge key groups (shuffles), warps (shared memory), CTAs (DSMEM)
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float mo = __shfl_xor_sync(0xffffffffu, m[g], off);
      const float lo = __shfl_xor_sync(0xffffffffu, l[g], off);
      const float mn = fmaxf(m[g], mo);
      const float wa = merge_weight(m[g], mn), wb = merge_weight(mo, mn);
      l[g] = l[g] * wa + lo * wb;
#pragma unroll
      for (int d = 0; d < DL; ++d) {
        const float ao = __shfl_xor_sync(0xffffffffu, acc[g][d], off);
        acc[g][d] = acc[g][d] * wa + ao * wb;
      }
      m[g] = mn;
    }
  }
  if (kg == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      if (ds == 0) {
        w_m[warp][g] = m[g];
        w_l[warp][g] = l[g];
      }
#pragma unroll
      for (int d = 0; d < DL; ++d) w_acc[warp][g][ds * DL + d] = acc[g][d];
    }
  }
  __syncthreads();
  // this CTA's partial for (g, d): warps merged; written out at once by a
  // lone CTA, pushed into rank 0's shared memory otherwise
  if (ncl > 1) asm volatile("barrier.cluster.wait.aligned;" ::: "memory");  // phase 1: all CTAs started
  float* rm = ncl > 1 ? cluster.map_shared_rank(&g_m[crank][0], 0) : nullptr;
  float* rl = ncl > 1 ? cluster.map_shared_rank(&g_l[crank][0], 0) : nullptr;
  float* ra = ncl > 1 ? cluster.map_shared_rank(&g_acc[crank][0][0], 0) : nullptr;
  for (int t = tid; t < G * D; t += NT) {
    const int g = t / D, d = t - (t / D) * D;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) mx = fmaxf(mx, w_m[w][g]);
    float ls = 0.f, as = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float wt = merge_weight(w_m[w][g], mx);
      ls += w_l[w][g] * wt;
      as += w_acc[w][g][d] * wt;
    }
    if (ncl == 1) {
      T* o = static_cast<T*>(p.out) + b * p.ob + (int64_t)(h * G + g) * p.oh + d;
      *o = Elem<T>::from_f(ls > 0.f ? as / ls : 0.f);
    } else {
      ra[t] = as;
      if (d == 0) {
        rm[g] = mx;
        rl[g] = ls;
      }
    }
  }
  if (ncl == 1) return;
  cluster_arrive_release();  // phase 2: this CTA's partial is in rank 0's shared memory
  if (crank != 0) return;    // nothing reads the other CTAs' shared memory
  cluster_wait_acquire();
  for (int t = tid; t < G * D; t += NT) {
    const int g = t / D, d = t - (t / D) * D;
    float mx = -INFINITY;
#pragma unroll
    for (int r = 0; r < kClusterCTAs; ++r)
      if (r < ncl) mx = fmaxf(mx, g_m[r][g]);
    float ls = 0.f, as = 0.f;
#pragma unroll
    for (int r = 0; r < kClusterCTAs; ++r) {
      if (r >= ncl) break;
      const float wt = merge_weight(g_m[r][g], mx);
      ls += g_l[r][g] * wt;
      as += g_acc[r][g][d] * wt;
    }
    T* o = static_cast<T*>(p.out) + b * p.ob + (int64_t)(h * G + g) * p.oh + d;
    *o = Elem<T>::from_f(ls > 0.f ? as / ls : 0.f);
  }
}

// CTAs of one decode_attn_kernel shape resident at once on the current device
// (occupancy API, once per device); 0 if its shared memory cannot be granted.
template <typename T, int G, int D, int NW, int TILE, int STAGES>
int attn_resident() {
  static std::atomic<int> resident[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  int r = resident[dev].load(std::memory_order_relaxed);
  if (r > 0) return r;
  constexpr size_t smem = (size_t)STAGES * 2 * TILE * D * sizeof(T);
  auto kern = decode_attn_kernel<T, G, D, NW, TILE, STAGES>;
  // dynamic + static shared memory may pass the 48 KB default
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return 0;
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, NW * 32, smem) != cudaSuccess || occ < 1) return 0;
  r = occ * sm_count();
  resident[dev].store(r, std::memory_order_relaxed);
  return r;
}

template <typename T, int G, int D, int NW, int TILE, int STAGES>
void launch_attn_tma(const AttnParams& p, int64_t batch, int hk, int cl, cudaStream_t s, bool dependent) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)cl, (unsigned)hk, (unsigned)batch);
  cfg.blockDim = dim3(NW * 32);
  cfg.dynamicSmemBytes = (size_t)STAGES * 2 * TILE * D * sizeof(T);
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)cl;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = dependent ? 2 : 1;
  cudaLaunchKernelEx(&cfg, decode_attn_kernel<T, G, D, NW, TILE, STAGES>, p);
}

template <typename T, int G, int D>
int launch_attn(const AttnParams& p, int64_t batch, int hk, cudaStream_t s, bool dependent) {
  if (p.cs == D) {  // contiguous cache rows: TMA-staged kernel, cluster size sized to fill the GPU
    // Few streams: 8-CTA clusters of the wide shape (8 warps, 128-key tiles),
    // when all of them fit in one wave.  Otherwise the 4-warp shape, each
    // (stream, KV head) split over the most CTAs (1, 2, 4 or 8) that still
    // fit in one wave: at 64 streams x 8 heads that is 1 (512 CTAs), at 16
    // streams 4.  A second, partial wave measured slower (64 streams, 880
    // valid slots: 27.4 us with 1024 CTAs, 23.5 us with 512)
    const int wide = attn_resident<T, G, D, kAttnWideWarps, kAttnWideTile, kAttnWideStages>();
    if (wide > 0 && batch * hk * kClusterCTAs <= wide) {
      launch_attn_tma<T, G, D, kAttnWideWarps, kAttnWideTile, kAttnWideStages>(p, batch, hk, kClusterCTAs, s,
                                                                               dependent);
      return launch_status();
    }
    const int resident = attn_resident<T, G, D, kAttnThreads / 32, kAttnTile, kAttnStages>();
    if (resident <= 0) return launch_status();
    int cl = kClusterCTAs;
    while (cl > 1 && batch * hk * cl > resident) cl >>= 1;
    launch_attn_tma<T, G, D, kAttnThreads / 32, kAttnTile, kAttnStages>(p, batch, hk, cl, s, dependent);
  } else {
    const dim3 grid(kClusterCTAs, (unsigned)hk, (unsigned)batch);
    decode_attn_reg_kernel<T, G, D><<<grid, kAttnThreads, 0, s>>>(p);
  }
  return launch_status();
}

}  // namespace
}  // namespace kani

namespace {
int decode_attention_impl(int32_t dtype, int64_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                          int32_t head_dim, const void* q, int64_t q_batch_stride, int64_t q_head_stride,
                          const void* k_cache, const void* v_cache, int64_t cache_batch_stride,
                          int64_t cache_head_stride, int64_t cache_slot_stride, int64_t cache_len,
                          const int64_t* kv_len, float scale, void* out, int64_t out_batch_stride,
                          int64_t out_head_stride, int32_t* err_flag, void* stream, bool dependent) {
  if (batch < 0 || num_q_heads < 0 || num_kv_heads < 0 || head_dim < 0 || cache_len < 0)
    return KANI_ERR_INVALID_ARG;
  if (batch == 0 || num_q_heads == 0) return KANI_OK;
  if (!q || !k_cache || !v_cache || !kv_len || !out || num_kv_heads == 0) return KANI_ERR_INVALID_ARG;
  if (num_q_heads % num_kv_heads != 0) return KANI_ERR_INVALID_ARG;
  if (batch > 65535 || num_kv_heads > 65535) return KANI_ERR_UNSUPPORTED;
  const int g = num_q_heads / num_kv_heads;
  kani::AttnParams p{q, q_batch_stride, q_head_stride, k_cache, v_cache, cache_batch_stride,
                     cache_head_stride, cache_slot_stride, cache_len, kv_len, out, out_batch_stride,
                     out_head_stride, scale * 1.4426950408889634f, err_flag};
  const kani::WaitBound wb = kani::wait_bound(kani::kAttnWaitCycles);
  p.wait_cycles = wb.cycles;
  p.wait_suspend_ns = wb.suspend_ns;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return kani::dispatch_dtype(dtype, [&]<typename T>() -> int {
    constexpr int E = kani::VecN<T>::value;
    const bool vec = kani::aligned16(q) && kani::aligned16(k_cache) && kani::aligned16(v_cache) &&
                     q_batch_stride % E == 0 && q_head_stride % E == 0 && cache_batch_stride % E == 0 &&
                     cache_head_stride % E == 0 && cache_slot_stride % E == 0;
    if (!vec) return KANI_ERR_UNSUPPORTED;
    if (head_dim == 64) {
      if (g == 1) return kani::launch_attn<T, 1, 64>(p, batch, num_kv_heads, s, dependent);
      if (g == 2) return kani::launch_attn<T, 2, 64>(p, batch, num_kv_heads, s, dependent);
      if (g == 4) return kani::launch_attn<T, 4, 64>(p, batch, num_kv_heads, s, dependent);
    } else if (head_dim == 128) {
      if (g == 1) return kani::launch_attn<T, 1, 128>(p, batch, num_kv_heads, s, dependent);
      if (g == 2) return kani::launch_attn<T, 2, 128>(p, batch, num_kv_heads, s, dependent);
    }
    return KANI_ERR_UNSUPPORTED;
  });
}
}  // namespace

extern "C" int kani_decode_attention(int32_t dtype, int64_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                                     int32_t head_dim, const void* q, int64_t q_batch_stride,
                                     int64_t q_head_stride, const void* k_cache, const void* v_cache,
                                     int64_t cache_batch_stride, int64_t cache_head_stride,
                                     int64_t cache_slot_stride, int64_t cache_len, const int64_t* kv_len,
                                     float scale, void* out, int64_t out_batch_stride,
                                     int64_t out_head_stride, int32_t* err_flag, void* stream) {
  return decode_attention_impl(dtype, batch, num_q_heads, num_kv_heads, head_dim, q, q_batch_stride, q_head_stride,
                               k_cache, v_cache, cache_batch_stride, cache_head_stride, cache_slot_stride, cache_len,
                               kv_len, scale, out, out_batch_stride, out_head_stride, err_flag, stream, false);
}

extern "C" int kani_decode_attention_step(int32_t dtype, int64_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                                          int32_t head_dim, const void* q, int64_t q_batch_stride,
                                          int64_t q_head_stride, const void* k_cache, const void* v_cache,
                                          int64_t cache_batch_stride, int64_t cache_head_stride,
                                          int64_t cache_slot_stride, int64_t cache_len, const int64_t* kv_len,
                                          float scale, void* out, int64_t out_batch_stride,
                                          int64_t out_head_stride, int32_t* err_flag, void* stream) {
  return decode_attention_impl(dtype, batch, num_q_heads, num_kv_heads, head_dim, q, q_batch_stride, q_head_stride,
                               k_cache, v_cache, cache_batch_stride, cache_head_stride, cache_slot_stride, cache_len,
                               kv_len, scale, out, out_batch_stride, out_head_stride, err_flag, stream, true);
}
