"""Host-side position and frequency preparation for the fused RoPE kernel.

These produce the device inputs of ``fused_rope_kv_write``:

* ``frame_level_positions`` — BemaTTS prefill position ids: text tokens
  advance by 1, each frame of ``tokens_per_frame`` audio tokens advances by
  ``audio_step`` (kani_tts/model.py:78-138; the function's own code, not its
  docstring example, is the definition: with audio_step=0.5 the example
  yields [0, 1, 2, 2, 2, 2, 2.5]).
* ``decode_position_schedule`` — decode step i (0-based after the two
  host-side steps) uses ``prefill_seq_len + ((i + 1) // tokens_per_frame) *
  audio_step`` (kani_tts/inference_engine.py:615-619); its KV slot is
  ``prefill_seq_len + 1 + i`` (inference_engine.py:600, 640-642).
* ``learnable_inv_freq`` — per-layer frequencies
  ``(bf16(theta^(-2i/D)) * alpha).float()`` with
  ``alpha = alpha_min + (alpha_max - alpha_min) * sigmoid(w)`` computed in
  bf16 (kani_tts/model.py:180-196, optimized_decode.py:104-111).
"""
from __future__ import annotations

import torch


def frame_level_positions(input_ids: torch.Tensor, audio_tokens_start: int,
                          tokens_per_frame: int = 4, audio_step: float = 1.0) -> torch.Tensor:
    """[B, S] position ids (float when audio_step is a float, as in the reference)."""
    is_audio = input_ids >= audio_tokens_start
    zeros = torch.zeros(input_ids.shape[0], 1, dtype=torch.long, device=input_ids.device)
    text_before = torch.cat([zeros, (~is_audio).long()], dim=1).cumsum(dim=1)[:, :-1]
    audio_before = torch.cat([zeros, is_audio.long()], dim=1).cumsum(dim=1)[:, :-1]
    return text_before + (audio_before // tokens_per_frame) * audio_step


def decode_position_schedule(prefill_seq_len: int, max_new_tokens: int, tokens_per_frame: int = 4,
                             audio_step: float = 1.0, device=None) -> torch.Tensor:
    """int64 [max_new_tokens] angle positions of the graph-replayed decode steps."""
    steps = torch.arange(max_new_tokens, device=device)
    return (prefill_seq_len + (steps + 1) // tokens_per_frame * audio_step).long()


def decode_write_slots(prefill_seq_len: int, max_new_tokens: int, device=None) -> torch.Tensor:
    """int64 [max_new_tokens] KV slots of the graph-replayed decode steps."""
    return prefill_seq_len + 1 + torch.arange(max_new_tokens, device=device, dtype=torch.long)


def learnable_inv_freq(head_dim: int, rope_theta: float, alpha_weight: float | torch.Tensor = 0.0,
                       alpha_min: float = 0.1, alpha_max: float = 2.0) -> torch.Tensor:
    """fp32 [head_dim/2] inverse frequencies of one attention layer (computed on CPU)."""
    base = rope_theta
    exponents = torch.arange(0, head_dim, 2, dtype=torch.int64).to(torch.bfloat16) / head_dim
    inv_freq_base = 1.0 / (base ** exponents)
    w = alpha_weight if isinstance(alpha_weight, torch.Tensor) else torch.tensor(alpha_weight)
    w = w.detach().to("cpu", torch.bfloat16)
    alpha = alpha_min + (alpha_max - alpha_min) * torch.sigmoid(w)
    return (inv_freq_base * alpha).float()
