// Per-token bookkeeping of the decode loop, one launch per step (sm_100a).
//
// Reference: the host side of the decode loop, kani_tts/inference_engine.py:
// 615-619 (the position schedule prefill_len + ((i + 1) // tokens_per_frame) *
// audio_step), 638-643 (next token, position, cache slot and mask slot written
// before each replay) and 669 (the token appended to generated_ids).  Here, at
// the end of step k, for every stream b:
//   generated[b, k] = next_token[b];  input_ids[b] = next_token[b];
//   positions[b] = base_pos[b] + floor((k + 1) / tokens_per_frame) * audio_step;
//   slots[b] = base_slot[b] + k + 1;  kv_len[b] = slots[b] + 1;
// then *step = k + 1 and, when given, *rng_step += 1 (the sampler's Philox
// counter).  This replaces the half-dozen small tensor ops a step would
// otherwise launch.
#include "common.cuh"

#include <math.h>

namespace kani {
namespace {

__global__ void __launch_bounds__(256)
decode_advance_kernel(const int64_t* __restrict__ next_token, int64_t* __restrict__ input_ids,
                      int64_t* __restrict__ generated, int64_t gen_stride, int64_t gen_cols, int64_t* step,
                      int64_t* rng_step, const int64_t* __restrict__ base_pos, const int64_t* __restrict__ base_slot,
                      int tokens_per_frame, float audio_step, int64_t* __restrict__ positions,
                      int64_t* __restrict__ slots, int64_t* __restrict__ kv_len, int64_t batch) {
  griddep_wait();  // up to kPdlMaxRows streams a programmatic dependent: the token comes from the launch before
  const int64_t k = *step;
  for (int64_t b = threadIdx.x; b < batch; b += blockDim.x) {
    const int64_t t = next_token[b];
    if (k >= 0 && k < gen_cols) generated[b * gen_stride + k] = t;
    input_ids[b] = t;
    const int64_t frames = (k + 1) / tokens_per_frame;
    positions[b] = base_pos[b] + (int64_t)floorf((float)frames * audio_step);
    const int64_t sl = base_slot[b] + k + 1;
    slots[b] = sl;
    kv_len[b] = sl + 1;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    *step = k + 1;
    if (rng_step) *rng_step += 1;
  }
}

}  // namespace
}  // namespace kani

extern "C" int kani_decode_advance(const int64_t* next_token, int64_t* input_ids, int64_t* generated,
                                   int64_t gen_row_stride, int64_t gen_cols, int64_t* step, int64_t* rng_step,
                                   const int64_t* base_pos, const int64_t* base_slot, int32_t tokens_per_frame,
                                   float audio_step, int64_t* positions, int64_t* slots, int64_t* kv_len,
                                   int64_t batch, void* stream) {
  if (batch < 0 || gen_cols < 0 || tokens_per_frame < 1) return KANI_ERR_INVALID_ARG;
  if (batch == 0) return KANI_OK;
  if (!next_token || !input_ids || !generated || !step || !base_pos || !base_slot || !positions || !slots ||
      !kv_len)
    return KANI_ERR_INVALID_ARG;
  if (batch > 1 && gen_row_stride < gen_cols) return KANI_ERR_INVALID_ARG;
  const int threads = batch < 256 ? (int)((batch + 31) / 32 * 32) : 256;
  kani::launch_maybe_pdl(batch <= kani::kPdlMaxRows, kani::decode_advance_kernel, dim3(1), dim3(threads), 0,
                         static_cast<cudaStream_t>(stream), next_token, input_ids, generated, gen_row_stride, gen_cols,
                         step, rng_step, base_pos, base_slot, tokens_per_frame, audio_step, positions, slots, kv_len,
                         batch);
  return kani::launch_status();
}
