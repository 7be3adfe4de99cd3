// Generated audio tokens -> NeMo codec codes for B streams (sm_100a).
//
// Reference: NemoAudioPlayer.get_nano_codes, kani_tts/core.py:86-108, which
// runs on the host after generation:
//   * the audio segment is the tokens between start-of-speech and the first
//     end-of-speech (here: a stream's generated tokens before its first
//     end-of-speech token, all of them if it has none);
//   * an incomplete last frame is dropped (len // 4 frames of 4 tokens);
//   * code[c, f] = token[4 f + c] - c * codebook_size - audio_tokens_start;
//   * a negative code is an error ("Invalid audio tokens!"), and so are zero
//     complete frames ("No complete audio frames generated!").
// Output [B, 4, max_frames] int64 (frames past a stream's count are -1), the
// frame count per stream and a status word per stream instead of exceptions:
// bit 0 = a negative code, bit 1 = no complete frame, bit 2 = no end-of-speech.
// One CTA per stream: the first end-of-speech position is a block minimum,
// then one thread per frame.
#include "common.cuh"

namespace kani {
namespace {

constexpr int kCodecThreads = 256;

__global__ void __launch_bounds__(kCodecThreads)
codec_codes_kernel(const int64_t* __restrict__ tokens, int64_t tokens_stride, int64_t n_tokens, int64_t eos,
                   int64_t audio_start, int64_t codebook, int64_t* __restrict__ codes, int64_t max_frames,
                   int64_t* __restrict__ frames_out, int32_t* __restrict__ status_out) {
  __shared__ unsigned long long s_first;
  __shared__ int s_bad;
  const int64_t b = blockIdx.x;
  const int64_t* tk = tokens + b * tokens_stride;
  if (threadIdx.x == 0) {
    s_first = (unsigned long long)n_tokens;
    s_bad = 0;
  }
  __syncthreads();
  for (int64_t i = threadIdx.x; i < n_tokens; i += kCodecThreads)
    if (tk[i] == eos) {
      atomicMin(&s_first, (unsigned long long)i);
      break;  // later positions of this thread are larger
    }
  __syncthreads();
  const int64_t len = (int64_t)s_first;
  int64_t nf = len / 4;
  if (nf > max_frames) nf = max_frames;
  int64_t* out = codes + b * 4 * max_frames;
  int bad = 0;
  for (int64_t f = threadIdx.x; f < max_frames; f += kCodecThreads) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      int64_t v = -1;
      if (f < nf) {
        v = tk[4 * f + c] - c * codebook - audio_start;
        bad |= v < 0;
      }
      out[c * max_frames + f] = v;
    }
  }
  if (bad) atomicOr(&s_bad, 1);
  __syncthreads();
  if (threadIdx.x == 0) {
    frames_out[b] = nf;
    status_out[b] = (s_bad ? 1 : 0) | (nf == 0 ? 2 : 0) | (len == n_tokens ? 4 : 0);
  }
}

}  // namespace
}  // namespace kani

extern "C" int kani_codec_codes(const int64_t* tokens, int64_t tokens_row_stride, int64_t batch, int64_t n_tokens,
                                int64_t eos_token, int64_t audio_tokens_start, int64_t codebook_size,
                                int64_t* codes_out, int64_t max_frames, int64_t* frames_out, int32_t* status_out,
                                void* stream) {
  if (batch < 0 || n_tokens < 0 || max_frames < 0) return KANI_ERR_INVALID_ARG;
  if (batch == 0) return KANI_OK;
  if (batch > 0x7fffffff || !tokens || !codes_out || !frames_out || !status_out) return KANI_ERR_INVALID_ARG;
  if (batch > 1 && tokens_row_stride < n_tokens) return KANI_ERR_INVALID_ARG;
  if (max_frames < n_tokens / 4) return KANI_ERR_INVALID_ARG;
  kani::codec_codes_kernel<<<(unsigned)batch, kani::kCodecThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      tokens, tokens_row_stride, n_tokens, eos_token, audio_tokens_start, codebook_size, codes_out, max_frames,
      frames_out, status_out);
  return kani::launch_status();
}
