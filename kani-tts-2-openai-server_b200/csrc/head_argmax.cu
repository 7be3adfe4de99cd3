// Reduced LM head + greedy token choice for up to 8 streams, one launch
// (sm_100a).
//
// Reference: the reduced head of OptimizedDecoder (kani_tts/optimized_decode.py:
// 134-156 builds W = [lm_head[eos]; lm_head[audio_tokens_start:]], :287 runs
// logits = F.linear(hidden, W)) followed by the greedy choice
// reduced_to_full[argmax(logits)] (the reduced-to-full map of :144-148).
// Here the GEMV, the argmax and the map are one kernel:
//   * logits[b, r] = round(sum_k h[b, k] * W[r, k])  (fp32 accumulation, one
//     rounding to the storage type, as F.linear's bf16 output);
//   * token[b] = index_map[first r with the largest logits[b, r]].
// The weight rows stream from HBM once (16-byte loads, 4 rows per warp in
// flight; the first ones are issued before the programmatic-launch wait, so
// they overlap the kernel before); the hidden rows are staged in shared memory.  Each CTA folds its
// maxima, packed as (order key << 32 | ~row), into a per-stream 64-bit
// atomicMax in global scratch; the last CTA to finish (a counter after a
// fence) writes the tokens and returns the scratch to zero, so the next launch
// (e.g. the next replay of a CUDA graph) starts clean.
#include <atomic>

#include "common.cuh"
#include "gemv_input.cuh"

namespace kani {
namespace {

constexpr int kHeadThreads = 256;
constexpr int kHeadWarps = kHeadThreads / 32;
constexpr int kHeadRows = 4;   // rows per warp in flight
constexpr int kHeadMaxB = 8;

struct HeadParams {
  const void* h;
  int64_t h_stride;
  const void* w;
  int64_t w_stride;
  int rows, hidden, batch;
  const int64_t* index_map;
  void* logits;
  int64_t logits_stride;
  unsigned long long* scratch;  // [batch] packed maxima, then one CTA counter
  int64_t* tokens;
  int64_t tokens_stride;
  L2Prefetch pf;  // later launches' weights, prefetched into L2 at entry
  const void* res;     // NORM: h = round(h_in + res), normalised with norm_w (the final norm)
  int64_t res_stride;
  const void* norm_w;
  float eps;
};

template <typename T>
__device__ __forceinline__ uint32_t order_key16(T v) {
  uint16_t b;
  memcpy(&b, &v, 2);
  if ((b & 0x7fffu) == 0) b = 0;  // -0 == +0
  return (uint32_t)(b ^ ((b & 0x8000u) ? 0xffffu : 0x8000u));
}

// B streams (compile-time upper bound), CH = hidden / 256 chunks of 8 per lane;
// NORM: the hidden rows are the final residual add + RMSNorm of (h, res), with
// the arithmetic of the decode GEMVs' input prologue
template <typename T, int B, int CH, bool NORM>
__global__ void __launch_bounds__(kHeadThreads) head_argmax_kernel(HeadParams p) {
  constexpr int E = 8;  // elements per 16-byte vector
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ unsigned long long s_best[kHeadWarps][B];
  __shared__ float s_part[kHeadWarps][B];
  __shared__ bool s_last;
  T* hs = reinterpret_cast<T*>(smem_raw);  // [B][hidden]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int H = CH * 256;
  const T* W = static_cast<const T*>(p.w);
  const int gw = blockIdx.x * kHeadWarps + warp, nw = gridDim.x * kHeadWarps;
  griddep_launch_dependents();  // the sampler or the bookkeeping launch after this one may be scheduled

  // the weights do not depend on earlier launches: the first rows stream in
  // before the programmatic-launch wait, the hidden rows are read after it
  uint4 wv[kHeadRows][CH];
  auto load_rows = [&](int r0) {
#pragma unroll
    for (int q = 0; q < kHeadRows; ++q) {
      const int r = min(r0 + q, p.rows - 1);
#pragma unroll
      for (int c = 0; c < CH; ++c) wv[q][c] = ld16_stream(W + (int64_t)r * p.w_stride + c * 256 + lane * E);
    }
  };
  if (gw * kHeadRows < p.rows) load_rows(gw * kHeadRows);
  const NormIn in{p.h, p.h_stride, p.res, p.res_stride, nullptr, 0, p.norm_w, p.eps, p.batch};
  const uint4 nw0 = first_norm_chunk<T, B, CH * 256, NORM>(in, tid);
  l2_prefetch_share(p.pf);
  griddep_wait();

  // The hidden rows (or the update and residual of the final norm) are written
  // by the launch before, which may still be running while this grid is
  // resident, so they are read with coherent loads after the wait: the
  // read-only (.nc) path is only valid for data that stays unwritten for the
  // whole life of the kernel, and a stale line from an earlier read of the
  // same address (a graph replay reuses it) could be served.
  stage_input<T, B, CH * 256, NORM, kHeadThreads>(in, hs, s_part, tid, lane, warp, nw0);

  unsigned long long best[B];
#pragma unroll
  for (int b = 0; b < B; ++b) best[b] = 0ull;
  for (int r0 = gw * kHeadRows; r0 < p.rows; r0 += nw * kHeadRows) {
    if (r0 != gw * kHeadRows) load_rows(r0);
    float acc[kHeadRows][B];
#pragma unroll
    for (int q = 0; q < kHeadRows; ++q)
#pragma unroll
      for (int b = 0; b < B; ++b) acc[q][b] = 0.f;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      float wf[kHeadRows][E];
#pragma unroll
      for (int q = 0; q < kHeadRows; ++q) unpack16<T>(wv[q][c], wf[q]);
#pragma unroll
      for (int b = 0; b < B; ++b) {
        float hf[E];
        unpack16<T>(reinterpret_cast<const uint4*>(hs + b * H + c * 256)[lane], hf);
#pragma unroll
        for (int q = 0; q < kHeadRows; ++q)
#pragma unroll
          for (int e = 0; e < E; ++e) acc[q][b] = fmaf(wf[q][e], hf[e], acc[q][b]);
      }
    }
#pragma unroll
    for (int q = 0; q < kHeadRows; ++q)
#pragma unroll
      for (int b = 0; b < B; ++b) {
        float a = acc[q][b];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        acc[q][b] = a;
      }
    if (lane == 0) {
#pragma unroll
      for (int q = 0; q < kHeadRows; ++q) {
        const int r = r0 + q;
        if (r >= p.rows) break;
#pragma unroll
        for (int b = 0; b < B; ++b) {
          if (b >= p.batch) break;
          const T lv = Elem<T>::from_f(acc[q][b]);
          if (p.logits) static_cast<T*>(p.logits)[(int64_t)b * p.logits_stride + r] = lv;
          const unsigned long long pk =
              ((unsigned long long)order_key16(lv) << 32) | (unsigned long long)(0xffffffffu - (uint32_t)r);
          best[b] = pk > best[b] ? pk : best[b];
        }
      }
    }
  }

  // fold the CTA's maxima into the per-stream scratch; the last CTA finishes
  if (lane == 0) {
#pragma unroll
    for (int b = 0; b < B; ++b) s_best[warp][b] = best[b];
  }
  __syncthreads();
  if (tid < B && tid < p.batch) {
    unsigned long long m = 0ull;
#pragma unroll
    for (int w = 0; w < kHeadWarps; ++w) m = s_best[w][tid] > m ? s_best[w][tid] : m;
    atomicMax(p.scratch + tid, m);
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned long long done = atomicAdd(p.scratch + p.batch, 1ull);
    s_last = done == (unsigned long long)(gridDim.x - 1);
  }
  __syncthreads();
  if (s_last && tid < p.batch) {
    __threadfence();
    const unsigned long long m = atomicExch(p.scratch + tid, 0ull);
    const int r = (int)(0xffffffffu - (uint32_t)(m & 0xffffffffu));
    const int row = (r >= 0 && r < p.rows) ? r : 0;
    p.tokens[(int64_t)tid * p.tokens_stride] = p.index_map ? p.index_map[row] : (int64_t)row;
  }
  if (s_last && tid == 0) atomicExch(p.scratch + p.batch, 0ull);
}

template <typename T, int B>
int launch_head_b(const HeadParams& prm, cudaStream_t s) {
  const int ch = prm.hidden / 256;
  const size_t smem = (size_t)B * prm.hidden * sizeof(T);
  static int sms[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return KANI_ERR_INVALID_ARG;
  if (sms[dev] == 0) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  const int per_cta = kHeadWarps * kHeadRows;
  auto go = [&](auto kern) -> int {
    if (smem > 48 * 1024) {
      const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return (int)e;
    }
    // one full wave of resident CTAs; warps stride over the rows
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kHeadThreads, smem) != cudaSuccess || occ < 1)
      occ = 1;
    const int64_t want = (prm.rows + per_cta - 1) / per_cta, cap = (int64_t)sms[dev] * occ;
    const int grid = (int)(want < cap ? want : cap);
    const cudaError_t e = launch_pdl(kern, dim3(grid), dim3(kHeadThreads), smem, s, prm);
    note_launch();
    return e == cudaSuccess ? KANI_OK : (int)e;
  };
  const bool norm = prm.norm_w != nullptr;
  switch (ch) {
    case 2: return norm ? go(head_argmax_kernel<T, B, 2, true>) : go(head_argmax_kernel<T, B, 2, false>);
    case 4: return norm ? go(head_argmax_kernel<T, B, 4, true>) : go(head_argmax_kernel<T, B, 4, false>);
    case 8: return norm ? go(head_argmax_kernel<T, B, 8, true>) : go(head_argmax_kernel<T, B, 8, false>);
    default: return KANI_ERR_UNSUPPORTED;
  }
}

template <typename T>
int launch_head(const HeadParams& prm, cudaStream_t s) {
  if (prm.batch <= 1) return launch_head_b<T, 1>(prm, s);
  if (prm.batch <= 2) return launch_head_b<T, 2>(prm, s);
  if (prm.batch <= 4) return launch_head_b<T, 4>(prm, s);
  return launch_head_b<T, 8>(prm, s);
}

}  // namespace
}  // namespace kani

namespace {
int head_argmax_impl(int32_t dtype, const void* hidden, int64_t hidden_row_stride, const void* residual,
                     int64_t residual_row_stride, const void* norm_weight, float eps, int64_t batch,
                     int32_t hidden_size, const void* weight, int64_t weight_row_stride, int32_t rows,
                     const int64_t* index_map, void* logits_out, int64_t logits_row_stride,
                     unsigned long long* scratch, int64_t* tokens_out, int64_t tokens_out_stride, void* stream) {
  const kani::L2Prefetch pf = kani::take_l2_prefetch();
  if (batch < 0 || rows < 0 || hidden_size < 0) return KANI_ERR_INVALID_ARG;
  if (batch == 0) return KANI_OK;
  if (rows == 0 || !hidden || !weight || !scratch || !tokens_out) return KANI_ERR_INVALID_ARG;
  if (residual && !norm_weight) return KANI_ERR_INVALID_ARG;  // the add belongs to the norm
  if (batch > kani::kHeadMaxB) return KANI_ERR_UNSUPPORTED;
  if (dtype != KANI_DTYPE_BF16 && dtype != KANI_DTYPE_F16) return dtype == KANI_DTYPE_F32 ? KANI_ERR_UNSUPPORTED
                                                                                          : KANI_ERR_DTYPE;
  if (hidden_size % 256 != 0 || weight_row_stride < hidden_size || (batch > 1 && hidden_row_stride < hidden_size) ||
      (residual && batch > 1 && residual_row_stride < hidden_size))
    return KANI_ERR_INVALID_ARG;
  if (logits_out && batch > 1 && logits_row_stride < rows) return KANI_ERR_INVALID_ARG;
  if (!kani::aligned16(hidden) || !kani::aligned16(weight) || hidden_row_stride % 8 != 0 || weight_row_stride % 8 != 0 ||
      (residual && (!kani::aligned16(residual) || residual_row_stride % 8 != 0)) ||
      (norm_weight && !kani::aligned16(norm_weight)))
    return KANI_ERR_UNSUPPORTED;
  kani::HeadParams prm{hidden, hidden_row_stride, weight, weight_row_stride, rows, hidden_size, (int)batch,
                       index_map, logits_out, logits_row_stride, scratch, tokens_out, tokens_out_stride, pf,
                       residual, residual_row_stride, norm_weight, eps};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == KANI_DTYPE_BF16) return kani::launch_head<__nv_bfloat16>(prm, s);
  return kani::launch_head<__half>(prm, s);
}
}  // namespace

extern "C" int kani_head_argmax(int32_t dtype, const void* hidden, int64_t hidden_row_stride, int64_t batch,
                                int32_t hidden_size, const void* weight, int64_t weight_row_stride, int32_t rows,
                                const int64_t* index_map, void* logits_out, int64_t logits_row_stride,
                                unsigned long long* scratch, int64_t* tokens_out, int64_t tokens_out_stride,
                                void* stream) {
  return head_argmax_impl(dtype, hidden, hidden_row_stride, nullptr, 0, nullptr, 0.f, batch, hidden_size, weight,
                          weight_row_stride, rows, index_map, logits_out, logits_row_stride, scratch, tokens_out,
                          tokens_out_stride, stream);
}

extern "C" int kani_head_argmax_norm(int32_t dtype, const void* x, int64_t x_row_stride, const void* residual,
                                     int64_t residual_row_stride, const void* norm_weight, float eps, int64_t batch,
                                     int32_t hidden_size, const void* weight, int64_t weight_row_stride,
                                     int32_t rows, const int64_t* index_map, void* logits_out,
                                     int64_t logits_row_stride, unsigned long long* scratch, int64_t* tokens_out,
                                     int64_t tokens_out_stride, void* stream) {
  if (!norm_weight) {
    kani::take_l2_prefetch();
    return KANI_ERR_INVALID_ARG;
  }
  return head_argmax_impl(dtype, x, x_row_stride, residual, residual_row_stride, norm_weight, eps, batch,
                          hidden_size, weight, weight_row_stride, rows, index_map, logits_out, logits_row_stride,
                          scratch, tokens_out, tokens_out_stride, stream);
}

// ------------------------------------------------ entry point without a scratch
//
// The same launch with the cross-CTA scratch taken from a file-scope device
// array instead of caller memory: nothing to allocate or zero.  The array is
// zero at module load and every launch leaves it zero; one array per device is
// shared by all callers, so calls on one device must not overlap in time.
namespace kani {
namespace {
constexpr int kStaticScratchWords = 64;  // streams + 1 counter
static_assert(kStaticScratchWords >= kHeadMaxB + 1, "static scratch too small");
}  // namespace
}  // namespace kani

static __device__ __align__(256) unsigned long long g_head_scratch[kani::kStaticScratchWords];

// The array's device address, looked up once per device (with that device
// current) and cached.  The slots are atomic, so first calls from several host
// threads at once store the same address without a data race.  The cache
// outlives the device's primary context: after cudaDeviceReset the entry point
// must not be called again in this process (it would pass the old address).
static unsigned long long* head_static_scratch() {
  constexpr int kMaxDevices = 64;
  static std::atomic<unsigned long long*> addr[kMaxDevices] = {};
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  unsigned long long* a = addr[dev].load(std::memory_order_acquire);
  if (!a) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_head_scratch) != cudaSuccess) return nullptr;
    a = static_cast<unsigned long long*>(p);
    addr[dev].store(a, std::memory_order_release);
  }
  return a;
}

extern "C" int kani_head_argmax_noalloc(int32_t dtype, const void* hidden, int64_t hidden_row_stride,
                                        int64_t batch, int32_t hidden_size, const void* weight,
                                        int64_t weight_row_stride, int32_t rows, const int64_t* index_map,
                                        void* logits_out, int64_t logits_row_stride, int64_t* tokens_out,
                                        int64_t tokens_out_stride, void* stream) {
  if (batch < 0) return KANI_ERR_INVALID_ARG;
  if (batch == 0) return KANI_OK;
  if (batch + 1 > kani::kStaticScratchWords) return KANI_ERR_UNSUPPORTED;  // size check
  unsigned long long* scratch = head_static_scratch();
  if (!scratch) return KANI_ERR_INVALID_ARG;
  return kani_head_argmax(dtype, hidden, hidden_row_stride, batch, hidden_size, weight, weight_row_stride, rows,
                          index_map, logits_out, logits_row_stride, scratch, tokens_out, tokens_out_stride, stream);
}
