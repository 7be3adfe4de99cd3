/*
 * kani_b200.h — C ABI of the B200 (sm_100a) decode-path kernels for KaniTTS.
 *
 * These entry points replace the device work of the reference's per-token
 * decode loop: the three Triton kernels in kani_tts/triton_kernels.py, the
 * eager residual adds in kani_tts/optimized_decode.py and the scatter_ KV
 * write in kani_tts/static_cache.py.  Each entry point cites the reference
 * interface it replaces.
 *
 * Conventions (all entry points):
 *   - Every pointer is a DEVICE pointer owned by the caller; the library never
 *     allocates, frees or synchronises.  Launches go on `stream`
 *     (a cudaStream_t passed as void*; NULL = legacy default stream), so every
 *     call is capturable in a CUDA graph.
 *   - `dtype` codes: KANI_DTYPE_F32 / _BF16 / _F16.  Arithmetic is fp32 with a
 *     single round-to-nearest-even to the storage type per output element.
 *   - Strides are in ELEMENTS.  Rows / tokens / heads are described by the
 *     stride arguments; the innermost dimension is always contiguous.
 *   - Return value: KANI_OK (0), a negative KANI_ERR_* for an argument the
 *     library rejects before launching, or a positive cudaError_t from the
 *     launch.  A zero-sized problem returns KANI_OK without launching.
 *   - Data-dependent errors found on the device (a KV slot or a frame index out
 *     of range) do not trap: the offending access is skipped and a KANI_FLAG_*
 *     bit is OR-ed into the caller's device int32 `err_flag` (may be NULL).
 *   - The projection entry points (kani_gemv*, kani_gemm_tc, kani_head_argmax*)
 *     launch as programmatic dependents and start reading their weight
 *     matrices and norm weights before the launch ahead of them on the stream
 *     has finished.  Weights must therefore not be written by the immediately
 *     preceding launch; activations, residuals and every other input are read
 *     only after it completes.
 */
#ifndef KANI_B200_H
#define KANI_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define KANI_API __attribute__((visibility("default")))
#else
#define KANI_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define KANI_DTYPE_F32 0
#define KANI_DTYPE_BF16 1
#define KANI_DTYPE_F16 2

#define KANI_OK 0
#define KANI_ERR_INVALID_ARG (-1) /* null pointer, negative size, bad stride */
#define KANI_ERR_DTYPE (-2)       /* unknown or unsupported dtype code */
#define KANI_ERR_UNSUPPORTED (-3) /* shape the kernels do not implement */

#define KANI_FLAG_SLOT_OOB 1  /* a KV write slot was outside [0, cache_len) */
#define KANI_FLAG_FRAME_OOB 2 /* a frame-table row was outside [0, frame_rows) */
#define KANI_FLAG_TIMEOUT 4   /* a bounded on-chip wait gave up (the call's outputs are incomplete) */

/* Library ABI version (major*100 + minor). */
KANI_API int kani_version(void);

/* Human-readable text for a return code of this library. */
KANI_API const char* kani_status_string(int status);

/* Number of kernel launches this library has issued in this process. */
KANI_API uint64_t kani_launch_count(void);

/*
 * Bound of the on-chip waits of later launches (the TMA mbarrier waits of the
 * bulk RoPE + KV-write kernel and of decode attention), in clock64 cycles;
 * 0 restores the default (about 1 s, with a 1 ms suspend hint per try).  A
 * nonzero limit also turns the suspend hint off, so a wait can run out while
 * its copies are still in flight: the kernel then ORs KANI_FLAG_TIMEOUT into
 * its error flag, lets its own copies land (with the default bound) and
 * returns; its outputs for that launch are not valid.  A diagnostic for tests
 * of that path, process-wide.  No counterpart in the reference, whose Triton
 * kernels have no on-chip waits.  Returns KANI_ERR_INVALID_ARG for cycles < 0.
 */
KANI_API int kani_set_wait_limit(int64_t cycles);

/*
 * L2 prefetch hint for the next decode launch: the next call of kani_gemv,
 * kani_gemv_short_conv, kani_gemv_rope_kv, kani_head_argmax,
 * kani_reduce_add_rms_norm or kani_silu_mul made on the same host thread
 * takes these (up to two) device ranges and clears them; every CTA
 * of that launch issues its share as cp.async.bulk.prefetch.L2 as it starts,
 * before the programmatic-launch wait.  The ranges must hold data no launch
 * writes (the weights of later launches), so that reading them early is safe.
 * A range with 0 bytes is unused.  Returns KANI_ERR_INVALID_ARG for negative
 * sizes or a null pointer with a size, KANI_ERR_UNSUPPORTED for a size or
 * address that is not a multiple of 16 bytes.  No counterpart in the reference,
 * whose decode step launches each F.linear on its own.
 */
KANI_API int kani_set_l2_prefetch(const void* ptr0, int64_t bytes0, const void* ptr1, int64_t bytes1);

/*
 * RMSNorm over the last dimension:  y = round(x * rsqrt(mean(x^2) + eps) * w).
 * Replaces `_rms_norm_kernel` and its launch in `fused_rms_norm`
 * (kani_tts/triton_kernels.py:17-35, :38-60).  Unlike the reference, an fp32
 * input yields a true fp32 output (the reference stores bf16-rounded values).
 *   x, y:   [rows, n] with row strides x_row_stride / y_row_stride (y may alias x)
 *   weight: [n], dtype w_dtype
 */
KANI_API int kani_rms_norm(int32_t dtype, int32_t w_dtype,
                  const void* x, int64_t x_row_stride,
                  const void* weight,
                  void* y, int64_t y_row_stride,
                  int64_t rows, int64_t n, float eps, void* stream);

/*
 * Residual add fused into RMSNorm:  h = round(x + residual);
 * y = round(h * rsqrt(mean(h^2) + eps) * w); residual_out = h.
 * Replaces the eager `hidden = hidden + F.linear(...)` at
 * kani_tts/optimized_decode.py:252, :277, :283 together with the following
 * `fused_rms_norm` call (optimized_decode.py:206, :280, :286).
 * y may alias x; residual_out may alias x or residual (element-wise in place).
 */
KANI_API int kani_add_rms_norm(int32_t dtype, int32_t w_dtype,
                      const void* x, int64_t x_row_stride,
                      const void* residual, int64_t r_row_stride,
                      const void* weight,
                      void* y, int64_t y_row_stride,
                      void* residual_out, int64_t h_row_stride,
                      int64_t rows, int64_t n, float eps, void* stream);

/*
 * The residual add + RMSNorm that follows a projection computed as S fp32 partial
 * products over slices of K (a batched GEMM with an fp32 output, one product per
 * slice): d = round(p[0] + ... + p[S-1]) summed in split order (F.linear's
 * output), then h = round(d + residual), y = round(h * rsqrt(mean(h^2) + eps) * w),
 * as kani_add_rms_norm.  Replaces `hidden = hidden + F.linear(...)` and the next
 * `fused_rms_norm` (kani_tts/optimized_decode.py:252, 277, 283 with :206, :280,
 * :286) for batched decode, where the K-split GEMM with an fp32 output is faster
 * than the plain one.
 *   partials: fp32, element (s, row, k) at s * split_stride + row * partial_row_stride + k;
 *             the splits must not overlap; 16-byte aligned, strides multiples of 4
 *   residual, y, residual_out: [rows, n] of dtype; y must differ from residual_out
 *   n: a multiple of 4, at most 4096
 */
KANI_API int kani_reduce_add_rms_norm(int32_t dtype, int32_t w_dtype, const float* partials, int64_t split_stride,
                                      int64_t partial_row_stride, int32_t splits, const void* residual,
                                      int64_t r_row_stride, const void* weight, void* y, int64_t y_row_stride,
                                      void* residual_out, int64_t h_row_stride, int64_t rows, int64_t n, float eps,
                                      void* stream);

/*
 * SiLU-gated activation: y[r, i] = round(silu(g[r, i]) * u[r, i]) where each
 * input row is [g (n) | u (n)].
 * Replaces `_silu_mul_kernel` and `fused_silu_mul`
 * (kani_tts/triton_kernels.py:67-82, :85-105).
 *   gate_up: [rows, 2n] with row stride in_row_stride; y: [rows, n].
 */
KANI_API int kani_silu_mul(int32_t dtype,
                  const void* gate_up, int64_t in_row_stride,
                  void* y, int64_t out_row_stride,
                  int64_t rows, int64_t n, void* stream);

/*
 * Rotate-half RoPE of one token's Q and K heads with one shared cos/sin row,
 * in ONE launch (the reference issues two).
 * Replaces `_rope_kernel` and `fused_rope` (kani_tts/triton_kernels.py:112-165).
 *   q, q_out: [num_q_heads, head_dim]; k, k_out: [num_k_heads, head_dim]
 *   cos, sin: [head_dim] (same dtype as q)
 *   y[i] = x[i]*cos[i] + sign(i)*x[(i+D/2) % D]*sin[i], sign = -1 for i < D/2.
 */
KANI_API int kani_rope_qk(int32_t dtype,
                 const void* q, const void* k,
                 const void* cos, const void* sin,
                 void* q_out, void* k_out,
                 int32_t num_q_heads, int32_t num_k_heads, int32_t head_dim,
                 void* stream);

/*
 * Static KV-cache write of one token per stream:
 *   k_cache[b, h, slot_b, :] = k[b, h, :];  v_cache[b, h, slot_b, :] = v[b, h, :]
 * with slot_b = write_pos[b] if per_stream_pos else write_pos[0].
 * Replaces the scatter_ in `StaticLfm2HybridConvCache.update`
 * (kani_tts/static_cache.py:110-142; write position :81, :144-146).
 *   k, v: [batch, num_kv_heads, head_dim] contiguous;
 *   k_cache, v_cache: [batch, num_kv_heads, cache_len, head_dim] contiguous;
 *   write_pos: device int64.  An out-of-range slot skips the write and sets
 *   KANI_FLAG_SLOT_OOB.
 */
KANI_API int kani_kv_cache_write(int32_t dtype,
                        const void* k, const void* v,
                        int64_t batch, int32_t num_kv_heads, int32_t head_dim,
                        void* k_cache, void* v_cache, int64_t cache_len,
                        const int64_t* write_pos, int32_t per_stream_pos,
                        int32_t* err_flag, void* stream);

/*
 * Fused attention-input step of one decode (or prefill) call, per token t of
 * n_tokens = batch * seq_tokens:
 *   1. optional per-head RMSNorm of Q and K (weights q_norm_w / k_norm_w [head_dim]),
 *      rounded to dtype (kani_tts/optimized_decode.py:220-221);
 *   2. cos/sin built in-kernel: angle_i = inv_freq[i] * float(positions[t]),
 *      rounded to dtype (optimized_decode.py:229-234, learnable-alpha inv_freq
 *      from kani_tts/model.py:180-196 and optimized_decode.py:104-111);
 *   3. rotate-half RoPE of Q and K in fp32 (triton_kernels.py:121-130);
 *   4. optional BemaTTS frame-position term: + frame_table[frame_pos[t] / tokens_per_frame]
 *      broadcast over heads (frame_pos NULL -> positions), added in fp32 before the
 *      single rounding;
 *   5. Q -> q_out[t*q_out_tok_stride + h*q_out_head_stride + i];
 *      K (rotated) and V (raw) -> k_cache / v_cache at
 *      b*cache_batch_stride + h*cache_head_stride + slot*cache_slot_stride + i,
 *      slot = write_slots[t] (static_cache.py:131-140).
 * Replaces optimized_decode.py:220-240 (q/k norm, cos/sin glue, fused_rope,
 * past_key_values.update).  Inputs are read at
 * q + t*q_tok_stride + h*head_dim (likewise k, v), so the packed QKV
 * projection output can be passed without a copy.
 */
KANI_API int kani_rope_kv_write(int32_t dtype,
                       int64_t batch, int64_t seq_tokens,
                       int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                       const void* q, int64_t q_tok_stride,
                       const void* k, int64_t k_tok_stride,
                       const void* v, int64_t v_tok_stride,
                       const float* inv_freq, const int64_t* positions,
                       const void* q_norm_w, const void* k_norm_w, float eps,
                       const void* frame_table, int64_t frame_rows,
                       const int64_t* frame_pos, int32_t tokens_per_frame,
                       void* q_out, int64_t q_out_tok_stride, int64_t q_out_head_stride,
                       void* k_cache, void* v_cache,
                       int64_t cache_batch_stride, int64_t cache_head_stride,
                       int64_t cache_slot_stride, int64_t cache_len,
                       const int64_t* write_slots,
                       int32_t* err_flag, void* stream);

/*
 * GQA decode attention over the valid cache prefix, one query token per stream:
 *   out[b, hq, :] = softmax_j(scale * q[b, hq, :] . K[b, hq/G, j, :]) V[b, hq/G, j, :]
 * for slots j in [0, kv_len[b]) (kv_len: device int64 [batch]; values above
 * cache_len are clamped and flag KANI_FLAG_SLOT_OOB), G = num_q_heads / num_kv_heads.
 * Replaces the SDPA over the whole -inf-masked static buffer of
 * kani_tts/optimized_decode.py:243-248 (mask: kani_tts/inference_engine.py:259-265,
 * opened slot by slot at :643, always a prefix).  fp32 online softmax, one
 * rounding of the output.  head_dim 64 (G = 1, 2, 4) or 128 (G = 1, 2);
 * 16-byte aligned rows.
 *   q, out: [batch, num_q_heads, head_dim] with batch / head strides
 *   k_cache, v_cache: [batch, num_kv_heads, cache_len, head_dim] with strides
 */
KANI_API int kani_decode_attention(int32_t dtype, int64_t batch, int32_t num_q_heads,
                          int32_t num_kv_heads, int32_t head_dim,
                          const void* q, int64_t q_batch_stride, int64_t q_head_stride,
                          const void* k_cache, const void* v_cache,
                          int64_t cache_batch_stride, int64_t cache_head_stride,
                          int64_t cache_slot_stride, int64_t cache_len,
                          const int64_t* kv_len, float scale,
                          void* out, int64_t out_batch_stride, int64_t out_head_stride,
                          int32_t* err_flag, void* stream);

/*
 * kani_decode_attention for one decode step, launched as a programmatic
 * dependent of the launch before it on the stream: the cache rows
 * [0, kv_len[b] - 1) start streaming, and kv_len is read, before that launch has
 * completed; q and the newest row, kv_len[b] - 1, are read after it.  So the
 * launch just before may write q and the newest row (the step's RoPE + KV
 * write, kani_tts/optimized_decode.py:220-240 then :243-248), but kv_len and the
 * older rows must already be final.  Same arguments and bit-identical results as
 * kani_decode_attention.
 */
KANI_API int kani_decode_attention_step(int32_t dtype, int64_t batch, int32_t num_q_heads,
                          int32_t num_kv_heads, int32_t head_dim,
                          const void* q, int64_t q_batch_stride, int64_t q_head_stride,
                          const void* k_cache, const void* v_cache,
                          int64_t cache_batch_stride, int64_t cache_head_stride,
                          int64_t cache_slot_stride, int64_t cache_len,
                          const int64_t* kv_len, float scale,
                          void* out, int64_t out_batch_stride, int64_t out_head_stride,
                          int32_t* err_flag, void* stream);

/*
 * LFM2 gated short-convolution decode step for `batch` streams:
 *   [Bg | C | x] = bcx[b] (3*hidden, the in_proj output);  Bx = Bg * x;
 *   state[b] = roll(state[b], -1 along the kernel axis) with Bx in the last column;
 *   y[b] = C * sum_i(state[b, :, i] * conv_w[:, i])
 * with the rounding of the eager bf16 ops (bit-identical to them).
 * Replaces kani_tts/optimized_decode.py:256-277 (between in_proj and out_proj).
 *   bcx: [batch, 3*hidden] (row stride); state: [batch, hidden, kernel_len]
 *   (batch stride, contiguous per stream); conv_w: [hidden, kernel_len];
 *   y: [batch, hidden] (row stride).  kernel_len in 2..4; all four buffers and
 *   the row / batch strides 16-byte aligned (KANI_ERR_UNSUPPORTED otherwise).
 */
KANI_API int kani_short_conv_step(int32_t dtype, const void* bcx, int64_t bcx_row_stride,
                         void* state, int64_t state_batch_stride, const void* conv_w,
                         void* y, int64_t y_row_stride, int64_t batch, int32_t hidden,
                         int32_t kernel_len, void* stream);

/*
 * Next-token sampling for `batch` streams, one launch, no host sync.
 * Replaces KaniInferenceEngine._sample_next_token
 * (kani_tts/inference_engine.py:349-430) and its per-token `.item()`:
 *   1. repetition penalty on the tokens set in `seen_bitmap`
 *      (l > 0 ? l / rp : l * rp, rounded to the logits dtype; skipped when
 *      rp == 1 or the bitmap is NULL);
 *   2. optional additive `logit_bias` [vocab] (the full-vocab audio mask);
 *   3. top-k (k = top_k <= 256), ordered by value, ties by lower index;
 *   4. temperature (l / T when T != 1), softmax, in-order cumulative sum, and
 *      top-p (candidate j >= 1 dropped when cumsum[j-1] >= top_p, compared in
 *      the logits dtype; skipped when top_p >= 1);
 *   5. softmax of the kept candidates and torch.multinomial's exponential
 *      race: token = argmax_j round(p_j / round(E_j)), E_j ~ Exp(1).
 *   logits: [batch, vocab] with a row stride; seen_bitmap: [batch, seen_row_words]
 *   uint32 (bit i of the row = index i seen), updated with the sampled index
 *   when update_seen != 0; index_map: [vocab] int64 (index -> token id, e.g.
 *   the reduced-to-full map), NULL = identity.
 *   E_j: from exp_draws [batch, top_k] fp32 when non-NULL, else Philox4x32-10
 *   keyed by `seed`, counter (j / 4, stream, *step_counter) (step 0 when
 *   step_counter is NULL).  Optional outputs, each [batch, top_k]: draws_out
 *   (the E_j used), probs_out (the kept distribution, logits dtype),
 *   cand_out (the candidates' indices, sorted).  tokens_out[b * stride] gets
 *   the token id.  vocab * dtype size is limited to about 200 KB per row.
 */
KANI_API int kani_sample_tokens(int32_t dtype, const void* logits, int64_t logits_row_stride,
                       int64_t batch, int32_t vocab, const void* logit_bias,
                       uint32_t* seen_bitmap, int64_t seen_row_words, int32_t update_seen,
                       float repetition_penalty, float temperature, float top_p, int32_t top_k,
                       const int64_t* index_map, uint64_t seed, const int64_t* step_counter,
                       const float* exp_draws, float* draws_out, void* probs_out,
                       int32_t* cand_out, int64_t* tokens_out, int64_t tokens_out_stride,
                       void* stream);

/*
 * Reduced LM head + greedy choice for up to 8 streams, one launch:
 *   logits[b, r] = round(sum_k hidden[b, k] * weight[r, k])  (fp32 accumulation)
 *   tokens_out[b * stride] = index_map[first r with the largest logits[b, r]]
 * Replaces F.linear(hidden, audio_lm_head_weight) (kani_tts/optimized_decode.py:287,
 * head built at :134-156) and the greedy reduced_to_full[argmax(...)] (:144-148).
 *   hidden: [batch, hidden_size] (row stride); weight: [rows, hidden_size] (row
 *   stride); bf16 or fp16; hidden_size one of 512, 1024, 2048; rows and strides
 *   16-byte aligned.  logits_out [batch, rows] (row stride) may be NULL.
 *   scratch: batch + 1 uint64 of device memory, zero before the first call; every
 *   call leaves it zero (one call at a time per scratch buffer).
 *   index_map: [rows] int64, NULL = identity.  batch > 8: KANI_ERR_UNSUPPORTED.
 */
KANI_API int kani_head_argmax(int32_t dtype, const void* hidden, int64_t hidden_row_stride, int64_t batch,
                     int32_t hidden_size, const void* weight, int64_t weight_row_stride, int32_t rows,
                     const int64_t* index_map, void* logits_out, int64_t logits_row_stride,
                     unsigned long long* scratch, int64_t* tokens_out, int64_t tokens_out_stride,
                     void* stream);

/*
 * kani_head_argmax with the decode step's final residual add + RMSNorm
 * (optimized_decode.py:283 + :286) folded in front of the head: each CTA forms
 * h = round(x + residual) (residual may be NULL: h = x) and
 * round((h * rsqrt(mean(h^2) + eps)) * norm_weight) in shared memory, with the
 * arithmetic of the decode GEMVs' normed input (kani_gemv with norm_weight),
 * then runs the head, the argmax and the map as kani_head_argmax does.  The
 * logits are those of kani_gemv(x, residual, norm_weight, weight) bit for bit.
 * The new residual stream is not written (the step ends here).
 *   x, residual: [batch, hidden_size] rows; norm_weight: [hidden_size], non-NULL.
 */
KANI_API int kani_head_argmax_norm(int32_t dtype, const void* x, int64_t x_row_stride, const void* residual,
                          int64_t residual_row_stride, const void* norm_weight, float eps, int64_t batch,
                          int32_t hidden_size, const void* weight, int64_t weight_row_stride, int32_t rows,
                          const int64_t* index_map, void* logits_out, int64_t logits_row_stride,
                          unsigned long long* scratch, int64_t* tokens_out, int64_t tokens_out_stride,
                          void* stream);

/*
 * kani_head_argmax without the scratch argument, for callers that cannot
 * allocate device memory: a host whose allocator belongs to another framework,
 * code that may not call cudaMalloc while a stream is being captured, or a
 * real-time thread that must not block on an allocation.  There is no
 * counterpart in the reference (which allocates through PyTorch).
 * The cross-CTA scratch is a file-scope device array of 64 words, zero when the
 * library loads and left zero by every call.  Every GPU that loads the library
 * holds one copy until the process exits.  The first call on a device looks up
 * the array's device address with cudaGetSymbolAddress (with that device
 * current) and keeps it: make that first call before any stream capture.
 * batch + 1 above 64 returns KANI_ERR_UNSUPPORTED before any launch (the kernel
 * itself serves up to 8 streams).  All calls on a device share the array, so
 * calls that overlap on the GPU race; issue them on one stream.  The cached
 * address belongs to the device's primary context: after cudaDeviceReset do
 * not call this entry point again in the same process.
 */
KANI_API int kani_head_argmax_noalloc(int32_t dtype, const void* hidden, int64_t hidden_row_stride,
                     int64_t batch, int32_t hidden_size, const void* weight,
                     int64_t weight_row_stride, int32_t rows, const int64_t* index_map,
                     void* logits_out, int64_t logits_row_stride, int64_t* tokens_out,
                     int64_t tokens_out_stride, void* stream);

/*
 * Reduced LM head + greedy choice for 2..64 streams on the tensor cores
 * (tcgen05.mma, fp32 accumulators in tensor memory), one launch:
 *   logits[b, r] = round(sum_k hidden[b, k] * weight[r, k])  (fp32 accumulation)
 *   tokens_out[b * stride] = index_map[first r with the largest logits[b, r]]
 * Replaces, for a batch of streams, F.linear(hidden, audio_lm_head_weight)
 * (kani_tts/optimized_decode.py:287, head built at :134-156) and the greedy
 * reduced_to_full[argmax(...)] (:144-148).
 *   hidden: [batch, hidden_size]; weight: [rows, hidden_size]; bf16 or fp16;
 *   hidden_size a multiple of 64, at most 1024; rows <= 65535; pointers and row
 *   strides 16-byte aligned.  logits_out [batch, rows] (row stride) may be NULL.
 *   scratch: batch + 1 uint32 of device memory, zero before the first call; every
 *   call leaves it zero (one call at a time per scratch buffer).
 *   err_flag (may be NULL): KANI_FLAG_TIMEOUT when an on-chip wait gave up.
 *   batch > 64 or another shape: KANI_ERR_UNSUPPORTED.
 */
KANI_API int kani_head_argmax_tc(int32_t dtype, const void* hidden, int64_t hidden_row_stride, int64_t batch,
                     int32_t hidden_size, const void* weight, int64_t weight_row_stride, int32_t rows,
                     const int64_t* index_map, void* logits_out, int64_t logits_row_stride,
                     uint32_t* scratch, int64_t* tokens_out, int64_t tokens_out_stride,
                     int32_t* err_flag, void* stream);

/*
 * kani_gemv's operation for 2..64 streams on the tensor cores (tcgen05.mma, fp32
 * accumulators in tensor memory; 128 weight rows per CTA, or 64 gate + 64 up rows
 * with silu_pairs):
 *   y[b, r] = round(sum_k a[b, k] * weight[r, k])   (fp32 accumulation)
 * a = x, or with norm_weight round((round(x + residual) * rr) * norm_weight)
 * (residual may be NULL; residual_out, when given, receives round(x + residual));
 * silu_pairs != 0: weight holds 2 * n_out rows (gate, then up) and
 *   y[b, r] = round(silu(round(gate_r)) * round(up_r)).
 * Replaces, for a batch of streams, the F.linear calls of the decode step
 * (kani_tts/optimized_decode.py:215, 255, 276, 281-282) with the residual add +
 * RMSNorm before them (:206, :252, :277, :280, :283) and the SiLU·mul after the
 * gate/up projection (triton_kernels.py:67-105).
 *   bf16 / fp16; k a multiple of 64 (at most 1024 with norm_weight); batch <= 64;
 *   n_out a multiple of 8 with silu_pairs; x, weight, residual, residual_out and
 *   norm_weight 16-byte aligned with row strides a multiple of 8 elements.
 *   err_flag (may be NULL): KANI_FLAG_TIMEOUT when an on-chip wait gave up.
 */
KANI_API int kani_gemm_tc(int32_t dtype, const void* x, int64_t x_row_stride, const void* residual,
                     int64_t residual_row_stride, void* residual_out, int64_t residual_out_row_stride,
                     const void* norm_weight, float eps, const void* weight, int64_t weight_row_stride,
                     int32_t n_out, int32_t k, int64_t batch, int32_t silu_pairs, void* y,
                     int64_t y_row_stride, int32_t* err_flag, void* stream);

/*
 * Decode GEMV for up to 8 streams with its neighbours fused:
 *   y[b, r] = round(sum_k a[b, k] * weight[r, k])   (fp32 accumulation)
 * a = x, or with norm_weight the RMSNorm of the residual stream:
 *   h = round(x + residual) (residual may be NULL: h = x; residual_out, when given,
 *   receives h), a = round((h * rr) * norm_weight), rr = 1 / sqrt(mean(h^2) + eps).
 * silu_pairs != 0: weight holds 2 * n_out rows (gate, then up) and
 *   y[b, r] = round(silu(round(gate_r)) * round(up_r)).
 * Replaces the F.linear calls of the decode step (kani_tts/optimized_decode.py:
 * 215, 255, 276, 281-282) with the residual add + RMSNorm before them (:206, :252,
 * :277, :280, :283) and the SiLU·mul between the MLP GEMVs (triton_kernels.py:67-105).
 *   x, residual, residual_out: [batch, k] (row strides, 16-byte aligned rows);
 *   weight: [n_out or 2 n_out, k] (row stride); y: [batch, n_out] (row stride);
 *   bf16 / fp16; k = 1024 or 4608; batch <= 8; residual_out must not be x or residual.
 */
KANI_API int kani_gemv(int32_t dtype, const void* x, int64_t x_row_stride, const void* residual,
                     int64_t residual_row_stride, void* residual_out, int64_t residual_out_row_stride,
                     const void* norm_weight, float eps, const void* weight, int64_t weight_row_stride,
                     int32_t n_out, int32_t k, int64_t batch, int32_t silu_pairs, void* y,
                     int64_t y_row_stride, void* stream);

/*
 * kani_gemv with the LFM2 gated short-conv decode step as its epilogue: the
 * in_proj GEMV (weight [3 * hidden, k]: B rows, C rows, x rows; optional
 * residual add + RMSNorm prologue as in kani_gemv) followed, per channel c, by
 * the step of kani_short_conv_step on conv_state[b, c, :] (updated in place) and
 * conv_weight[c, :], writing y[b, c].  Replaces optimized_decode.py:255-277
 * (in_proj through the conv) in one launch.  kernel_len must be 3; k = 1024.
 */
KANI_API int kani_gemv_short_conv(int32_t dtype, const void* x, int64_t x_row_stride, const void* residual,
                     int64_t residual_row_stride, void* residual_out, int64_t residual_out_row_stride,
                     const void* norm_weight, float eps, const void* in_proj_weight,
                     int64_t weight_row_stride, int32_t hidden, int32_t k, int64_t batch,
                     void* conv_state, int64_t conv_state_batch_stride, const void* conv_weight,
                     int32_t kernel_len, void* y, int64_t y_row_stride, void* stream);

/*
 * Per-token decode-loop bookkeeping, one launch (replaces the host writes of
 * kani_tts/inference_engine.py:615-619, 638-643, 669).  With k = *step, for each
 * stream b: generated[b, k] = input_ids[b] = next_token[b] (generated written
 * only for k < gen_cols); positions[b] = base_pos[b] +
 * floor((k + 1) / tokens_per_frame) * audio_step; slots[b] = base_slot[b] + k + 1;
 * kv_len[b] = slots[b] + 1.  Then *step = k + 1 and, if rng_step is not NULL,
 * *rng_step += 1.  All pointers are device int64 arrays ([batch], generated
 * [batch, gen_cols] with a row stride; step and rng_step single values).
 */
KANI_API int kani_decode_advance(const int64_t* next_token, int64_t* input_ids, int64_t* generated,
                     int64_t gen_row_stride, int64_t gen_cols, int64_t* step, int64_t* rng_step,
                     const int64_t* base_pos, const int64_t* base_slot, int32_t tokens_per_frame,
                     float audio_step, int64_t* positions, int64_t* slots, int64_t* kv_len,
                     int64_t batch, void* stream);

/*
 * The QKV GEMV of a decode step (input residual add + RMSNorm prologue as in
 * kani_gemv; weight [(Hq + 2 Hk) * 64, k], Q rows then K then V) fused with
 * kani_rope_kv_write's per-head work, one CTA per head: q/k RMSNorm (q_norm_w /
 * k_norm_w, both or neither), rotary angles inv_freq * positions[b], rotate-half,
 * the frame-table term (frame_table may be NULL), Q into q_out [batch, Hq, 64]
 * (batch / head strides), K and V into cache[b, h, slots[b], :].  Replaces
 * optimized_decode.py:215-240 (QKV F.linear through the cache update) in one
 * launch.  batch <= 4, k = 1024, head_dim = 64, norm_weight required.
 */
KANI_API int kani_gemv_rope_kv(int32_t dtype, const void* x, int64_t x_row_stride, const void* residual,
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
                     int32_t* err_flag, void* stream);

/*
 * Generated tokens -> NeMo codec codes for `batch` streams (replaces
 * NemoAudioPlayer.get_nano_codes, kani_tts/core.py:86-108):
 *   a stream's audio segment is its tokens before the first `eos_token`
 *   (end-of-speech); frames = segment length / 4 (an incomplete frame is dropped);
 *   codes_out[b, c, f] = tokens[b, 4 f + c] - c * codebook_size - audio_tokens_start,
 *   -1 past the stream's frames.  tokens: [batch, n_tokens] int64 (row stride);
 *   codes_out: [batch, 4, max_frames] int64, max_frames >= n_tokens / 4;
 *   frames_out: [batch] int64; status_out: [batch] int32, bit 0 = a negative code,
 *   bit 1 = no complete frame, bit 2 = no end-of-speech token.
 */
KANI_API int kani_codec_codes(const int64_t* tokens, int64_t tokens_row_stride, int64_t batch,
                     int64_t n_tokens, int64_t eos_token, int64_t audio_tokens_start,
                     int64_t codebook_size, int64_t* codes_out, int64_t max_frames,
                     int64_t* frames_out, int32_t* status_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KANI_B200_H */
