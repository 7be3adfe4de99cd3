// Batched decode projection on the tensor cores (tcgen05, sm_100a) with its
// neighbours fused, for 2..64 streams: the F.linear calls of the decode step
// (kani_tts/optimized_decode.py:215, 255, 276, 281-282) with the residual add +
// RMSNorm before them (:206, :252, :277, :280, :283) and the SiLU·mul between
// the MLP projections (triton_kernels.py:67-105).  Same arithmetic as the
// CUDA-core decode GEMV (gemv.cu), at batch sizes where the weight rows are
// better fed to 128 x N x 16 MMAs.
//
// One CTA per 128 weight rows (plain) or per 64 output features (SiLU·mul: 64
// gate rows + their 64 up rows):
//   * D[128 x N] (fp32, tensor memory; N = the batch rounded up to 16) sums
//     tcgen05.mma kind::f16 products over K;
//   * A (weights) streams through shared-memory stages of PZ 64-element K
//     tiles, one 3-D TMA load per stage ({64, rows, tiles}, tile stride 128 B);
//     for SiLU·mul a 5-D load {64, 8 rows, gate|up, 8-row group, tiles} lays
//     the 8-row atoms out as gate, up, gate, up, ..., so MMA row m is the gate
//     (bit 3 of m clear) or up (bit 3 set) row of feature (m >> 4) * 8 + m % 8;
//   * B (activations): with a norm prologue every CTA computes
//     a = round((round(x + residual) * rr) * w) for all streams into a
//     resident K-major 128-byte-swizzle operand (CTA 0 also writes
//     round(x + residual) out); without one, B tiles stream with the A stage;
//   * one thread issues the TMA loads and the MMAs; bounded waits
//     (KANI_FLAG_TIMEOUT);
//   * epilogue: 16 warps read the accumulators (lane quarter w % 4, column
//     group w / 4), round to the storage type and store; for SiLU·mul the
//     gate lane takes the up value from lane ^ 8 and stores
//     round(silu(gate) * up);
//   * split K (plain projections with few row tiles, e.g. the 1024-row output
//     projections): a cluster of C CTAs per row tile sums K / C each; the fp32
//     partials meet in distributed shared memory, and CTA rank r adds rows
//     [r 128 / C, (r + 1) 128 / C) over the C partials in rank order
//     (deterministic), then rounds and stores.
#include <cooperative_groups.h>

#include <algorithm>

#include "tc_common.cuh"

namespace cg = cooperative_groups;

namespace kani {
namespace {

constexpr int kGtThreads = 512;
constexpr int kGtN = 64;            // most streams
constexpr int kGtMaxStages = 16;
constexpr int kGtMaxNormK = 1024;   // the norm prologue keeps all of B resident
constexpr uint32_t kGtTmemCols = 64;
constexpr size_t kGtSmemBudget = 230400;

struct GemmTcParams {
  CUtensorMap tmap_w;  // weights (3-D plain, 5-D gate|up)
  CUtensorMap tmap_x;  // streamed activations {64, batch, tiles} (no norm prologue)
  const void* x;
  int64_t x_stride;
  const void* res;
  int64_t res_stride;
  void* res_out;
  int64_t res_out_stride;
  const void* norm_w;
  float eps;
  int n_out, k, batch, n_mma, stages, pz;
  int split;  // CTAs per cluster along K (1 = no split)
  void* out;
  int64_t out_stride;
  int32_t* err;
};

template <typename T>
__device__ __forceinline__ uint32_t round1_bits(float f) {
  if constexpr (std::is_same_v<T, __nv_bfloat16>) {
    return tc::bf16_rne_bits(__float_as_uint(f));
  } else {
    return (uint32_t)__half_as_ushort(__float2half_rn(f));
  }
}

// byte offset of 8-element chunk c8 of stream row n in the resident B operand
// (K tiles of n_mma rows x 128 B, 128-byte swizzle)
__device__ __forceinline__ uint32_t b_chunk_offset(int n, int c8, int n_mma) {
  const int t = c8 >> 3, c = c8 & 7;
  return (uint32_t)t * (uint32_t)n_mma * 128u + (uint32_t)n * 128u + ((uint32_t)(c ^ (n & 7)) << 4);
}

template <typename T, bool NORM, bool SILU, bool SPLIT>
__global__ void __launch_bounds__(kGtThreads, 1) gemm_tc_kernel(const __grid_constant__ GemmTcParams p) {
  static_assert(!SPLIT || (!NORM && !SILU), "split K is for plain projections");
  extern __shared__ unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t s_full[kGtMaxStages];
  __shared__ __align__(8) uint64_t s_empty[kGtMaxStages];
  __shared__ __align__(8) uint64_t s_done;
  __shared__ uint32_t s_tmem;
  __shared__ float s_rr[kGtN];
  __shared__ int s_failed;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int PZ = p.pz;
  const int K = p.k;
  const int nkt = K / tc::kKB;                     // K tiles
  const int crank = SPLIT ? (int)blockIdx.x : 0;   // rank in the cluster (grid.x = cluster size)
  const int tile_row = SPLIT ? (int)blockIdx.y : (int)blockIdx.x;
  const int t_per = nkt / p.split;                 // K tiles of this CTA
  const int t0 = crank * t_per;
  const int nkb = t_per / PZ;                      // pipeline items
  const int n_mma = p.n_mma;
  const int S = p.stages;
  const uint32_t b_bytes = (uint32_t)n_mma * 128u;  // one K tile of the streams
  const uint32_t raw = tc::smem_addr(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  // NORM: [B resident: nkt tiles][stages: PZ A tiles]; else [stages: PZ A tiles, PZ B tiles]
  const uint32_t b_res = base;
  const uint32_t stage_base = NORM ? base + (uint32_t)nkt * b_bytes : base;
  const uint32_t stage_bytes = NORM ? (uint32_t)PZ * tc::kATileBytes : (uint32_t)PZ * (tc::kATileBytes + b_bytes);
  auto a_tile = [&](int st) { return stage_base + (uint32_t)st * stage_bytes; };
  auto load_a = [&](int kb, int st) {
    const uint32_t bar = tc::smem_addr(&s_full[st]);
    if constexpr (SILU)
      tc::tma_load_5d(a_tile(st), &p.tmap_w, 0, 0, tile_row * 8, t0 + kb * PZ, bar);
    else
      tc::tma_load_3d(a_tile(st), &p.tmap_w, tile_row * tc::kM, t0 + kb * PZ, bar);
  };
  auto load_b = [&](int kb, int st) {
    tc::tma_load_3d(a_tile(st) + (uint32_t)PZ * tc::kATileBytes, &p.tmap_x, 0, t0 + kb * PZ,
                    tc::smem_addr(&s_full[st]));
  };

  if (warp == 0) tc::tmem_alloc(&s_tmem, kGtTmemCols);
  const int first = min(S, nkb);
  if (tid == 0) {
    s_failed = 0;
    for (int st = 0; st < S; ++st) {
      tc::mbar_init(tc::smem_addr(&s_full[st]));
      tc::mbar_init(tc::smem_addr(&s_empty[st]));
    }
    tc::mbar_init(tc::smem_addr(&s_done));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tc::prefetch_map(&p.tmap_w);
    if constexpr (!NORM) tc::prefetch_map(&p.tmap_x);
    // the weights of the first stages stream in before the programmatic-launch wait
    for (int st = 0; st < first; ++st) {
      tc::expect_tx(tc::smem_addr(&s_full[st]), stage_bytes);
      load_a(st, st);
    }
  }
  griddep_launch_dependents();
  griddep_wait();

  if constexpr (NORM) {
    // ---- prologue: a = round((round(x + residual) * rr) * w) into the resident B
    const int cpr = K / 8;  // 8-element chunks per row
    const T* X = static_cast<const T*>(p.x);
    const T* R = static_cast<const T*>(p.res);
    for (int v = tid; v < n_mma * cpr; v += kGtThreads) {
      const int n = v / cpr, c8 = v % cpr;
      uint4 hv = make_uint4(0u, 0u, 0u, 0u);
      if (n < p.batch) {
        float h[8];
        unpack16<T>(ld16(X + (int64_t)n * p.x_stride + c8 * 8), h);
        if (R) {
          float rv[8];
          unpack16<T>(ld16(R + (int64_t)n * p.res_stride + c8 * 8), rv);
#pragma unroll
          for (int e = 0; e < 8; ++e) h[e] = round_to<T>(__fadd_rn(h[e], rv[e]));
        }
        hv = pack16<T>(h);
        if (p.res_out && blockIdx.x == 0)
          st16(static_cast<T*>(p.res_out) + (int64_t)n * p.res_out_stride + c8 * 8, hv);
      }
      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(b_res + b_chunk_offset(n, c8, n_mma)),
                   "r"(hv.x), "r"(hv.y), "r"(hv.z), "r"(hv.w)
                   : "memory");
    }
    __syncthreads();
    // rr per stream: warp w sums rows w, w + 16, ... (lanes over chunks, fixed order)
    for (int n = warp; n < p.batch; n += kGtThreads / 32) {
      float s = 0.f;
      for (int c8 = lane; c8 < cpr; c8 += 32) {
        uint4 hv;
        asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(hv.x), "=r"(hv.y), "=r"(hv.z), "=r"(hv.w)
                     : "r"(b_res + b_chunk_offset(n, c8, n_mma)));
        float h[8];
        unpack16<T>(hv, h);
#pragma unroll
        for (int e = 0; e < 8; ++e) s = fmaf(h[e], h[e], s);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) s_rr[n] = 1.0f / sqrtf(s / (float)K + p.eps);
    }
    __syncthreads();
    const T* W = static_cast<const T*>(p.norm_w);
    for (int v = tid; v < p.batch * cpr; v += kGtThreads) {
      const int n = v / cpr, c8 = v % cpr;
      const uint32_t addr = b_res + b_chunk_offset(n, c8, n_mma);
      uint4 hv;
      asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                   : "=r"(hv.x), "=r"(hv.y), "=r"(hv.z), "=r"(hv.w)
                   : "r"(addr));
      float h[8], wf[8];
      unpack16<T>(hv, h);
      unpack16<T>(ld16_ro(W + c8 * 8), wf);
      const float rr = s_rr[n];
#pragma unroll
      for (int e = 0; e < 8; ++e) h[e] = __fmul_rn(__fmul_rn(h[e], rr), wf[e]);
      hv = pack16<T>(h);
      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(hv.x), "r"(hv.y), "r"(hv.z),
                   "r"(hv.w)
                   : "memory");
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor-core reads
  } else {
    if (tid == 0)
      for (int st = 0; st < first; ++st) load_b(st, st);  // the streams' rows, written by the launch before
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = s_tmem;

  bool failed = false;
  if (tid == 0) {
    const uint32_t idesc = tc::idesc_f16<T>(tc::kM, n_mma);
    int issued = first, landed = 0;
    for (int kb = 0; kb < nkb; ++kb) {
      const int st = kb % S;
      if (!tc::wait(tc::smem_addr(&s_full[st]), (uint32_t)((kb / S) & 1))) {
        failed = true;
        break;
      }
      landed = kb + 1;
      tc::fence_after_sync();
      for (int q = 0; q < PZ; ++q) {
        const uint32_t at = a_tile(st) + (uint32_t)q * tc::kATileBytes;
        const uint32_t bt = NORM ? b_res + (uint32_t)(kb * PZ + q) * b_bytes
                                 : a_tile(st) + (uint32_t)PZ * tc::kATileBytes + (uint32_t)q * b_bytes;
#pragma unroll
        for (int j = 0; j < tc::kKB / 16; ++j)
          tc::mma_f16(tmem, tc::desc_sw128(at + (uint32_t)j * 32u), tc::desc_sw128(bt + (uint32_t)j * 32u), idesc,
                      kb > 0 || q > 0 || j > 0);
      }
      tc::commit(tc::smem_addr(&s_empty[st]));
      const int prev = kb - 1;  // refill the stage of item kb - 1 once its MMAs completed
      if (prev >= 0 && prev + S < nkb) {
        const int ps = prev % S;
        if (!tc::wait(tc::smem_addr(&s_empty[ps]), (uint32_t)((prev / S) & 1))) {
          failed = true;
          break;
        }
        tc::expect_tx(tc::smem_addr(&s_full[ps]), stage_bytes);
        load_a(prev + S, ps);
        if constexpr (!NORM) load_b(prev + S, ps);
        issued = prev + S + 1;
      }
    }
    if (!failed) {
      tc::commit(tc::smem_addr(&s_done));
      for (int kb = max(0, nkb - S); kb < nkb; ++kb)
        if (!tc::wait(tc::smem_addr(&s_empty[kb % S]), (uint32_t)((kb / S) & 1))) failed = true;
    } else {
      for (int t = landed; t < issued; ++t)
        if (!tc::wait(tc::smem_addr(&s_full[t % S]), (uint32_t)((t / S) & 1))) break;
    }
    if (failed) s_failed = 1;
  }
  __syncthreads();
  const bool ok = !s_failed && tc::wait(tc::smem_addr(&s_done), 0u);
  if (!ok && lane == 0) atomicOr(&s_failed, 1);
  tc::fence_after_sync();

  // ---- epilogue: warp w reads lane quarter w % 4, column groups w / 4 + 4 i
  const int quarter = warp & 3;
  const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16);
  T* Y = static_cast<T*>(p.out);
  // the output feature of this lane's accumulator row
  int feat;
  bool lane_stores;
  if constexpr (SILU) {
    feat = tile_row * 64 + (2 * quarter + (lane >> 4)) * 8 + (lane & 7);
    lane_stores = ok && ((lane >> 3) & 1) == 0 && feat < p.n_out;  // gate lanes
  } else {
    feat = tile_row * tc::kM + quarter * 32 + lane;
    lane_stores = ok && feat < p.n_out;
  }
  if constexpr (SPLIT) {
    // fp32 partial -> this CTA's (idle) stage memory as red[n][128 rows]
    float* red = reinterpret_cast<float*>(smem_raw + (stage_base - raw));
#pragma unroll 1
    for (int cgi = warp >> 2; cgi < n_mma / 16; cgi += kGtThreads / 128) {
      uint32_t v[16];
      tc::tmem_ld16(taddr + (uint32_t)(cgi * 16), v);
#pragma unroll
      for (int e = 0; e < 16; ++e) red[(cgi * 16 + e) * tc::kM + quarter * 32 + lane] = ok ? __uint_as_float(v[e]) : 0.f;
    }
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();  // every partial of this row tile is in its CTA's shared memory
    const int ncl = p.split;
    const int rows = tc::kM / ncl;
    for (int idx = tid; idx < rows * n_mma; idx += kGtThreads) {
      const int m = crank * rows + idx % rows, n = idx / rows;
      float acc = 0.f;
      for (int c = 0; c < ncl; ++c) acc += *cluster.map_shared_rank(red + n * tc::kM + m, c);
      const int f = tile_row * tc::kM + m;
      if (n < p.batch && f < p.n_out)
        reinterpret_cast<uint16_t*>(Y)[(int64_t)n * p.out_stride + f] =
            (uint16_t)(tc::round_pair<T>(__float_as_uint(acc), 0u) & 0xffffu);
    }
    cluster.sync();  // the other CTAs have read this CTA's partial
  } else {
#pragma unroll 1
  for (int cg = warp >> 2; cg < n_mma / 16; cg += kGtThreads / 128) {
    uint32_t v[16];
    tc::tmem_ld16(taddr + (uint32_t)(cg * 16), v);
    const int n_valid = min(16, p.batch - cg * 16);  // uniform
    uint32_t bits[8];  // rounded pairs
#pragma unroll
    for (int e = 0; e < 8; ++e) bits[e] = tc::round_pair<T>(v[2 * e], v[2 * e + 1]);
    if constexpr (SILU) {
      uint32_t up[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) up[e] = __shfl_xor_sync(0xffffffffu, bits[e], 8);
      if (lane_stores) {
        T* dst = Y + (int64_t)(cg * 16) * p.out_stride + feat;
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const uint32_t gb = (e & 1) ? bits[e >> 1] >> 16 : bits[e >> 1] & 0xffffu;
          const uint32_t ub = (e & 1) ? up[e >> 1] >> 16 : up[e >> 1] & 0xffffu;
          const float y = silu_mul_f(tc::from_bits16<T>(gb), tc::from_bits16<T>(ub));
          if (e < n_valid)
            reinterpret_cast<uint16_t*>(dst)[(int64_t)e * p.out_stride] = (uint16_t)round1_bits<T>(y);
        }
      }
    } else {
      if (lane_stores) {
        uint16_t* dst = reinterpret_cast<uint16_t*>(Y + (int64_t)(cg * 16) * p.out_stride + feat);
#pragma unroll
        for (int e = 0; e < 16; ++e)
          if (e < n_valid)
            dst[(int64_t)e * p.out_stride] = (uint16_t)((e & 1) ? bits[e >> 1] >> 16 : bits[e >> 1] & 0xffffu);
      }
    }
  }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_free(tmem, kGtTmemCols);
  if (tid == 0 && s_failed && p.err) atomicOr(p.err, KANI_FLAG_TIMEOUT);
}

size_t gemm_tc_stage_bytes(bool norm, int n_mma, int pz) {
  return (size_t)pz * (tc::kATileBytes + (norm ? 0 : (size_t)n_mma * 128));
}

size_t gemm_tc_smem(bool norm, int k, int n_mma, int pz, int stages, int split) {
  size_t stage_area = (size_t)stages * gemm_tc_stage_bytes(norm, n_mma, pz);
  if (split > 1) stage_area = std::max(stage_area, (size_t)tc::kM * n_mma * 4);  // the fp32 partial reuses it
  return 1024 + (norm ? (size_t)(k / tc::kKB) * n_mma * 128 : 0) + stage_area;
}

template <typename T, bool NORM, bool SILU, bool SPLIT>
int launch_gemm_tc(const GemmTcParams& prm, cudaStream_t s) {
  const size_t smem = gemm_tc_smem(NORM, prm.k, prm.n_mma, prm.pz, prm.stages, prm.split);
  auto kern = gemm_tc_kernel<T, NORM, SILU, SPLIT>;
  const cudaError_t a = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (a != cudaSuccess) return (int)a;
  const int tiles = SILU ? (prm.n_out + 63) / 64 : (prm.n_out + tc::kM - 1) / tc::kM;
  cudaError_t e;
  if constexpr (SPLIT) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)prm.split, (unsigned)tiles);
    cfg.blockDim = dim3(kGtThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)prm.split;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    e = cudaLaunchKernelEx(&cfg, kern, prm);
    note_launch();
  } else {
    e = launch_pdl(kern, dim3(tiles), dim3(kGtThreads), smem, s, prm);
  }
  return e == cudaSuccess ? KANI_OK : (int)e;
}

template <typename T>
int dispatch_gemm_tc(const GemmTcParams& prm, bool norm, bool silu, cudaStream_t s) {
  if (norm) return silu ? launch_gemm_tc<T, true, true, false>(prm, s) : launch_gemm_tc<T, true, false, false>(prm, s);
  if (silu) return launch_gemm_tc<T, false, true, false>(prm, s);
  return prm.split > 1 ? launch_gemm_tc<T, false, false, true>(prm, s) : launch_gemm_tc<T, false, false, false>(prm, s);
}

}  // namespace
}  // namespace kani

extern "C" int kani_gemm_tc(int32_t dtype, const void* x, int64_t x_row_stride, const void* residual,
                            int64_t residual_row_stride, void* residual_out, int64_t residual_out_row_stride,
                            const void* norm_weight, float eps, const void* weight, int64_t weight_row_stride,
                            int32_t n_out, int32_t k, int64_t batch, int32_t silu_pairs, void* y,
                            int64_t y_row_stride, int32_t* err_flag, void* stream) {
  using namespace kani;
  if (batch < 0 || n_out < 0 || k <= 0) return KANI_ERR_INVALID_ARG;
  if (batch == 0 || n_out == 0) return KANI_OK;
  if (!x || !weight || !y) return KANI_ERR_INVALID_ARG;
  if (dtype != KANI_DTYPE_BF16 && dtype != KANI_DTYPE_F16)
    return dtype == KANI_DTYPE_F32 ? KANI_ERR_UNSUPPORTED : KANI_ERR_DTYPE;
  const bool norm = norm_weight != nullptr;
  const bool silu = silu_pairs != 0;
  if ((residual || residual_out) && !norm) return KANI_ERR_INVALID_ARG;
  if (residual_out && (residual_out == x || residual_out == residual)) return KANI_ERR_INVALID_ARG;
  if (batch > kGtN || k % tc::kKB != 0 || (norm && k > kGtMaxNormK) || (silu && n_out % 8 != 0))
    return KANI_ERR_UNSUPPORTED;
  if (batch == 1) {  // one row: the strides are never followed
    x_row_stride = k;
    residual_row_stride = k;
    residual_out_row_stride = k;
    y_row_stride = n_out;
  }
  if (x_row_stride < k || (residual && residual_row_stride < k) || (residual_out && residual_out_row_stride < k) ||
      y_row_stride < n_out || weight_row_stride < k)
    return KANI_ERR_INVALID_ARG;
  if (!aligned16(x) || !aligned16(weight) || (residual && !aligned16(residual)) ||
      (residual_out && !aligned16(residual_out)) || (norm && !aligned16(norm_weight)) || x_row_stride % 8 != 0 ||
      weight_row_stride % 8 != 0 || (residual && residual_row_stride % 8 != 0) ||
      (residual_out && residual_out_row_stride % 8 != 0))
    return KANI_ERR_UNSUPPORTED;
  const bool bf16 = dtype == KANI_DTYPE_BF16;
  GemmTcParams prm;
  memset(&prm, 0, sizeof(prm));
  prm.x = x;
  prm.x_stride = x_row_stride;
  prm.res = residual;
  prm.res_stride = residual_row_stride;
  prm.res_out = residual_out;
  prm.res_out_stride = residual_out_row_stride;
  prm.norm_w = norm_weight;
  prm.eps = eps;
  prm.n_out = n_out;
  prm.k = k;
  prm.batch = (int)batch;
  prm.n_mma = ((int)batch + 15) / 16 * 16;
  // split K over a cluster when a plain projection has too few row tiles to keep
  // the SMs streaming (at most 8 CTAs per cluster, dividing the K tiles)
  const int nkt = k / tc::kKB;
  const int row_tiles = (n_out + tc::kM - 1) / tc::kM;
  prm.split = 1;
  if (!norm && !silu && row_tiles < 32)
    for (int c : {8, 4, 2})
      if (nkt % c == 0) {
        prm.split = c;
        break;
      }
  const int t_per = nkt / prm.split;
  // K tiles per TMA load: 2-4 consecutive 128-byte pieces per row stream equally
  // fast; 2 leaves the most stages (an odd count takes 3, or single tiles)
  prm.pz = t_per % 2 == 0 ? 2 : t_per % 3 == 0 ? 3 : 1;
  const size_t fixed = 1024 + (norm ? (size_t)nkt * prm.n_mma * 128 : 0);
  const int fit = (int)((kGtSmemBudget - fixed) / gemm_tc_stage_bytes(norm, prm.n_mma, prm.pz));
  prm.stages = std::min(std::min(fit, kGtMaxStages), t_per / prm.pz);
  if (prm.stages < 1) return KANI_ERR_UNSUPPORTED;
  prm.out = y;
  prm.out_stride = y_row_stride;
  prm.err = err_flag;
  bool enc;
  if (silu) {
    // {64 elements, 8 rows, gate|up, 8-row group, K tile}
    const cuuint64_t dims[5] = {(cuuint64_t)tc::kKB, 8u, 2u, (cuuint64_t)(n_out / 8), (cuuint64_t)(k / tc::kKB)};
    const cuuint64_t strides[4] = {(cuuint64_t)weight_row_stride * 2u, (cuuint64_t)n_out * weight_row_stride * 2u,
                                   (cuuint64_t)weight_row_stride * 16u, (cuuint64_t)tc::kKB * 2u};
    const cuuint32_t box[5] = {(cuuint32_t)tc::kKB, 8u, 2u, 8u, (cuuint32_t)prm.pz};
    enc = tc::encode_map(&prm.tmap_w, bf16, weight, 5, dims, strides, box);
  } else {
    enc = tc::encode_rows(&prm.tmap_w, bf16, weight, k, n_out, weight_row_stride, tc::kM, prm.pz);
  }
  if (enc && !norm) enc = tc::encode_rows(&prm.tmap_x, bf16, x, k, batch, x_row_stride, prm.n_mma, prm.pz);
  if (!enc) return KANI_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (bf16) return dispatch_gemm_tc<__nv_bfloat16>(prm, norm, silu, s);
  return dispatch_gemm_tc<__half>(prm, norm, silu, s);
}
