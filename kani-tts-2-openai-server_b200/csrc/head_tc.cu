// Reduced LM head + greedy choice for up to 64 streams on the 5th-generation
// tensor cores (tcgen05, sm_100a).
//
// Reference: logits = F.linear(hidden, audio_lm_head_weight)
// (kani_tts/optimized_decode.py:287, head built at :134-156) and the greedy
// reduced_to_full[argmax(logits)] (:144-148) — for a batch of streams, where
// the head is a GEMM [streams x hidden] x [hidden x rows].
//
// One CTA per tile of 128 head rows (a 1-D grid over the rows):
//   * D[128 rows x N] (fp32, in tensor memory; N = the batch rounded up to 16)
//     accumulates tcgen05.mma kind::f16 products A[128 x 16] * B[N x 16]^T
//     over the hidden dimension;
//   * a pipeline stage holds PZ (2, or 1 for an odd tile count) tiles of 64
//     hidden elements: A (128 head rows x 64 per tile) and B (the streams'
//     hidden rows x 64 per tile, zero-filled past the batch by the TMA), each
//     brought by ONE 3-D TMA load over the view {64 elements, rows, tiles}
//     (tile stride 128 bytes), so every row request covers PZ x 128
//     contiguous bytes — 2-D boxes of 128-byte rows stream the head measurably
//     slower.  As many stages as shared memory holds (4 at 64 streams, 6 at
//     16) are in flight.  The weight loads of the first stages are issued
//     before the programmatic-launch wait (the weights do not depend on the
//     launch before); the stream rows (written by it) after;
//   * both operands use the K-major 128-byte-swizzle canonical layout: a tile
//     row is 64 elements (128 bytes), 8-row atoms 1024 bytes apart (SBO), the
//     16-byte chunks of row r XOR-permuted by r % 8 — the layout a TMA tile
//     load with CU_TENSOR_MAP_SWIZZLE_128B writes; the 16-wide K steps inside
//     a row start 32 bytes apart;
//   * one thread issues the TMA loads and the MMAs: MMA batch kb is committed
//     to the stage's "empty" barrier, and the stage of batch kb - 1 is refilled
//     once that barrier completes; all waits are bounded (KANI_FLAG_TIMEOUT);
//   * epilogue: each warp loads 32 rows x 16 columns of D from tensor memory
//     (tcgen05.ld 32x32b; 16 warps cover 128 rows x 64 columns in one pass),
//     rounds to the storage type (F.linear's output),
//     optionally stores the logits, and reduces per stream the packed
//     (order key << 16 | 0xffff - row) with a warp max; one 32-bit atomicMax
//     per stream and CTA into the scratch; the last CTA (a counter after a
//     fence) writes the mapped tokens and returns the scratch to zero.
#include <algorithm>

#include "tc_common.cuh"

namespace kani {
namespace {

// 16 warps: in the epilogue warp w reads TMEM lane quarter w % 4 (its 32 rows)
// and column group w / 4 (16 streams), so 64 streams take one pass
constexpr int kTcThreads = 512;
constexpr int kTcM = tc::kM;     // head rows per CTA (MMA M)
constexpr int kTcN = 64;         // most streams (MMA N)
constexpr int kTcKB = tc::kKB;   // hidden elements per tile: one 128-byte swizzle row
constexpr int kTcMaxStages = 16;
constexpr int kTcMaxHidden = 1024;
constexpr uint32_t kTmemCols = 64;  // fp32 accumulators: one column per stream slot
constexpr uint32_t kABytes = tc::kATileBytes;  // one K tile of the head rows
constexpr size_t kTcSmemBudget = 230400;          // dynamic shared memory (227 KB less the static part)

struct HeadTcParams {
  CUtensorMap tmap_w;  // head rows: {64, rows, tiles}, box {64, 128, PZ}, 128-byte swizzle
  CUtensorMap tmap_h;  // stream rows: {64, batch, tiles}, box {64, N, PZ}, 128-byte swizzle
  int rows, hidden, batch, n_mma, stages, pz;
  const int64_t* index_map;
  void* logits;
  int64_t logits_stride;
  uint32_t* scratch;  // [batch] packed maxima, then one CTA counter
  int64_t* tokens;
  int64_t tokens_stride;
  int32_t* err;
};

// Total-order key of a 16-bit float's bits (ascending with the value; -0 == +0).
__device__ __forceinline__ uint32_t order_key16(uint32_t b) {
  if ((b & 0x7fffu) == 0) b = 0;
  return b ^ ((b & 0x8000u) ? 0xffffu : 0x8000u);
}

template <typename T>
__global__ void __launch_bounds__(kTcThreads, 1) head_tc_kernel(const __grid_constant__ HeadTcParams p) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t s_full[kTcMaxStages];   // stage landed (TMA bytes)
  __shared__ __align__(8) uint64_t s_empty[kTcMaxStages];  // stage read (MMA commit)
  __shared__ __align__(8) uint64_t s_done;
  __shared__ uint32_t s_tmem;
  __shared__ uint32_t s_best[kTcN];
  __shared__ int s_failed;
  __shared__ bool s_last;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int PZ = p.pz;
  const int nkb = p.hidden / kTcKB / PZ;  // pipeline items of PZ tiles
  const int n_mma = p.n_mma;
  const int S = p.stages;
  const int r0 = blockIdx.x * kTcM;
  // 1024-byte aligned stages (the 128-byte swizzle repeats every 8 rows):
  // stage s = [head rows: PZ tiles of 128 x 128 B][stream rows: PZ tiles of n_mma x 128 B]
  const uint32_t raw = tc::smem_addr(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t b_bytes = (uint32_t)n_mma * 128u;
  const uint32_t stage_bytes = (uint32_t)PZ * (kABytes + b_bytes);
  auto a_tile = [&](int st) { return base + (uint32_t)st * stage_bytes; };
  auto b_tile = [&](int st) { return a_tile(st) + (uint32_t)PZ * kABytes; };
  auto load_a = [&](int kb, int st) { tc::tma_load_3d(a_tile(st), &p.tmap_w, r0, kb * PZ, tc::smem_addr(&s_full[st])); };
  auto load_b = [&](int kb, int st) { tc::tma_load_3d(b_tile(st), &p.tmap_h, 0, kb * PZ, tc::smem_addr(&s_full[st])); };

  if (warp == 0) {
    tc::tmem_alloc(&s_tmem, kTmemCols);
  }
  if (tid < kTcN) s_best[tid] = 0u;
  bool failed = false;
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
    tc::prefetch_map(&p.tmap_h);
    // the head rows of the first stages stream in before the programmatic-launch
    // wait; each stage's barrier expects both of its loads
    for (int st = 0; st < first; ++st) {
      tc::expect_tx(tc::smem_addr(&s_full[st]), stage_bytes);
      load_a(st, st);
    }
  }
  griddep_launch_dependents();
  griddep_wait();
  if (tid == 0)
    for (int st = 0; st < first; ++st) load_b(st, st);  // the streams' rows, written by the launch before
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = s_tmem;

  if (tid == 0) {
    const uint32_t idesc = tc::idesc_f16<T>(kTcM, n_mma);
    int issued = first;  // tiles whose loads were issued
    int landed = 0;      // ... and whose full barrier was seen
    for (int kb = 0; kb < nkb; ++kb) {
      const int st = kb % S;
      if (!tc::wait(tc::smem_addr(&s_full[st]), (uint32_t)((kb / S) & 1))) {
        failed = true;
        break;
      }
      landed = kb + 1;
      tc::fence_after_sync();
      for (int q = 0; q < PZ; ++q) {
        const uint32_t at = a_tile(st) + (uint32_t)q * kABytes, bt = b_tile(st) + (uint32_t)q * b_bytes;
#pragma unroll
        for (int j = 0; j < kTcKB / 16; ++j) {
          const uint64_t ad = tc::desc_sw128(at + (uint32_t)j * 32u);
          const uint64_t bd = tc::desc_sw128(bt + (uint32_t)j * 32u);
          const uint32_t acc = (kb > 0 || q > 0 || j > 0) ? 1u : 0u;
          tc::mma_f16(tmem, ad, bd, idesc, acc != 0u);
        }
      }
      tc::commit(tc::smem_addr(&s_empty[st]));
      // refill the stage of tile kb - 1 with tile kb - 1 + S once its MMAs completed
      const int prev = kb - 1;
      if (prev >= 0 && prev + S < nkb) {
        const int ps = prev % S;
        if (!tc::wait(tc::smem_addr(&s_empty[ps]), (uint32_t)((prev / S) & 1))) {
          failed = true;
          break;
        }
        tc::expect_tx(tc::smem_addr(&s_full[ps]), stage_bytes);
        load_a(prev + S, ps);
        load_b(prev + S, ps);
        issued = prev + S + 1;
      }
    }
    if (!failed) {
      tc::commit(tc::smem_addr(&s_done));
      // the stage commits no refill waited for (one per stage), so that no
      // arrive is pending on this CTA's shared memory when it exits
      for (int kb = max(0, nkb - S); kb < nkb; ++kb)
        if (!tc::wait(tc::smem_addr(&s_empty[kb % S]), (uint32_t)((kb / S) & 1))) failed = true;
    } else {
      // give copies still in flight a bounded time to land before the CTA exits
      for (int t = landed; t < issued; ++t)
        if (!tc::wait(tc::smem_addr(&s_full[t % S]), (uint32_t)((t / S) & 1))) break;
    }
    if (failed) s_failed = 1;
  }
  __syncthreads();  // thread 0's loop is over: s_failed is final, every MMA is issued
  const bool ok = !s_failed && tc::wait(tc::smem_addr(&s_done), 0u);
  if (!ok && lane == 0) atomicOr(&s_failed, 1);
  tc::fence_after_sync();

  // ---- epilogue: warp w holds rows r0 + 32 (w % 4) + lane and the stream
  // columns of groups w / 4, w / 4 + 4, ... (16 columns each, up to n_mma)
  const int quarter = warp & 3;
  const int row = r0 + quarter * 32 + lane;
  const bool row_ok = ok && row < p.rows;
  const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16);
#pragma unroll 1
  for (int q = warp >> 2; q < n_mma / 16; q += kTcThreads / 128) {  // columns past the MMA width were never written
    uint32_t v[16];
    tc::tmem_ld16(taddr + (uint32_t)(q * 16), v);
    // Round, then build the packed keys with selects only: a data-dependent
    // branch per element (e.g. around the logits store) costs a divergence
    // round trip each, several times the arithmetic.
    const int n_valid = min(16, p.batch - q * 16);  // uniform
    uint32_t bits[16], pk[16];
#pragma unroll
    for (int e = 0; e < 16; e += 2) {
      const uint32_t pair = tc::round_pair<T>(v[e], v[e + 1]);
      bits[e] = pair & 0xffffu;
      bits[e + 1] = pair >> 16;
    }
#pragma unroll
    for (int e = 0; e < 16; ++e)
      pk[e] = (row_ok && e < n_valid) ? ((order_key16(bits[e]) << 16) | (0xffffu - (uint32_t)row)) : 0u;
    if (p.logits != nullptr && row_ok) {
      uint16_t* dst = static_cast<uint16_t*>(p.logits) + (int64_t)(q * 16) * p.logits_stride + row;
#pragma unroll
      for (int e = 0; e < 16; ++e)
        if (e < n_valid) dst[(int64_t)e * p.logits_stride] = (uint16_t)bits[e];
    }
    // Transpose-reduce over the warp: at each step a lane keeps the half of its
    // columns selected by one lane bit and takes the max with the partner's copy
    // of that half; after 4 steps lane l holds column (l >> 1) & 15 reduced over
    // 16 lanes, and one more exchange covers all 32.
#pragma unroll
    for (int m = 16, n = 8; m >= 2; m >>= 1, n >>= 1) {
      const bool upper = (lane & m) != 0;
#pragma unroll
      for (int i = 0; i < n; ++i) {
        const uint32_t send = upper ? pk[i] : pk[i + n];
        const uint32_t keep = upper ? pk[i + n] : pk[i];
        pk[i] = max(keep, __shfl_xor_sync(0xffffffffu, send, m));
      }
    }
    const uint32_t col_max = max(pk[0], __shfl_xor_sync(0xffffffffu, pk[0], 1));
    const int col = q * 16 + ((lane >> 1) & 15);
    if ((lane & 1) == 0 && col < p.batch) atomicMax(&s_best[col], col_max);
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_free(tmem, kTmemCols);
  if (tid == 0 && s_failed && p.err) atomicOr(p.err, KANI_FLAG_TIMEOUT);

  // ---- fold into the per-stream scratch; the last CTA writes the tokens
  // The CTA's maxima (relaxed atomics) are ordered before thread 0's
  // acquire-release count by the barrier; the CTA that counts last acquires
  // every other CTA's release, so its exchanges read the final maxima.
  if (tid < p.batch) atomicMax(p.scratch + tid, s_best[tid]);
  __syncthreads();
  if (tid == 0) {
    uint32_t before;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(before) : "l"(p.scratch + p.batch) : "memory");
    s_last = before == gridDim.x - 1;
  }
  __syncthreads();
  if (s_last && tid < p.batch) {
    const uint32_t m = atomicExch(p.scratch + tid, 0u);
    int r = (int)(0xffffu - (m & 0xffffu));
    if (r < 0 || r >= p.rows) r = 0;
    p.tokens[(int64_t)tid * p.tokens_stride] = p.index_map ? p.index_map[r] : (int64_t)r;
  }
  if (s_last && tid == 0) atomicExch(p.scratch + p.batch, 0u);
}

size_t head_tc_stage_bytes(int n_mma, int pz) { return (size_t)pz * (kABytes + (size_t)n_mma * 128); }

// stages that fit the budget (a 1024-byte alignment pad, then the stages),
// at most one per pipeline item
int head_tc_stages(int hidden, int n_mma, int pz) {
  const int fit = (int)((kTcSmemBudget - 1024) / head_tc_stage_bytes(n_mma, pz));
  return std::min(std::min(fit, kTcMaxStages), hidden / kTcKB / pz);
}

template <typename T>
int launch_head_tc(const HeadTcParams& prm, cudaStream_t s) {
  const size_t smem = 1024 + (size_t)prm.stages * head_tc_stage_bytes(prm.n_mma, prm.pz);
  auto kern = head_tc_kernel<T>;
  const cudaError_t a = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (a != cudaSuccess) return (int)a;
  const int grid = (prm.rows + kTcM - 1) / kTcM;
  const cudaError_t e = launch_pdl(kern, dim3(grid), dim3(kTcThreads), smem, s, prm);
  return e == cudaSuccess ? KANI_OK : (int)e;
}

}  // namespace
}  // namespace kani

extern "C" int kani_head_argmax_tc(int32_t dtype, const void* hidden, int64_t hidden_row_stride, int64_t batch,
                                   int32_t hidden_size, const void* weight, int64_t weight_row_stride, int32_t rows,
                                   const int64_t* index_map, void* logits_out, int64_t logits_row_stride,
                                   uint32_t* scratch, int64_t* tokens_out, int64_t tokens_out_stride,
                                   int32_t* err_flag, void* stream) {
  if (batch < 0 || rows < 0 || hidden_size < 0) return KANI_ERR_INVALID_ARG;
  if (batch == 0) return KANI_OK;
  if (rows == 0 || !hidden || !weight || !scratch || !tokens_out) return KANI_ERR_INVALID_ARG;
  if (batch > kani::kTcN || rows > 0xffff || hidden_size % kani::kTcKB != 0 || hidden_size > kani::kTcMaxHidden)
    return KANI_ERR_UNSUPPORTED;
  if (dtype != KANI_DTYPE_BF16 && dtype != KANI_DTYPE_F16)
    return dtype == KANI_DTYPE_F32 ? KANI_ERR_UNSUPPORTED : KANI_ERR_DTYPE;
  if (weight_row_stride < hidden_size || (batch > 1 && hidden_row_stride < hidden_size) ||
      (logits_out && batch > 1 && logits_row_stride < rows))
    return KANI_ERR_INVALID_ARG;
  if (batch == 1) hidden_row_stride = hidden_size;  // one row: the stride is never followed
  if (!kani::aligned16(hidden) || !kani::aligned16(weight) || hidden_row_stride % 8 != 0 || weight_row_stride % 8 != 0)
    return KANI_ERR_UNSUPPORTED;
  const bool bf16 = dtype == KANI_DTYPE_BF16;
  kani::HeadTcParams prm;
  memset(&prm, 0, sizeof(prm));
  prm.rows = rows;
  prm.hidden = hidden_size;
  prm.batch = (int)batch;
  prm.n_mma = ((int)batch + 15) / 16 * 16;
  prm.pz = (hidden_size / kani::kTcKB) % 2 == 0 ? 2 : 1;
  prm.stages = kani::head_tc_stages(hidden_size, prm.n_mma, prm.pz);
  if (!kani::tc::encode_rows(&prm.tmap_w, bf16, weight, hidden_size, rows, weight_row_stride, kani::kTcM, prm.pz) ||
      !kani::tc::encode_rows(&prm.tmap_h, bf16, hidden, hidden_size, batch, hidden_row_stride, prm.n_mma, prm.pz))
    return KANI_ERR_UNSUPPORTED;
  prm.index_map = index_map;
  prm.logits = logits_out;
  prm.logits_stride = logits_row_stride;
  prm.scratch = scratch;
  prm.tokens = tokens_out;
  prm.tokens_stride = tokens_out_stride;
  prm.err = err_flag;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (bf16) return kani::launch_head_tc<__nv_bfloat16>(prm, s);
  return kani::launch_head_tc<__half>(prm, s);
}
