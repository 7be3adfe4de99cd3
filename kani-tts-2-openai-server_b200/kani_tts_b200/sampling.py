"""Sampling parameters and host helpers for the device sampler.

The reference samples each token on the host
(``KaniInferenceEngine._sample_next_token``, kani_tts/inference_engine.py:349-430)
with the generation settings of config.py:28-31 (temperature 0.5, top_p 0.85,
repetition penalty 1.2, overridable from the environment) and a top-k of 256.
Here one ``kani_sample_tokens`` launch samples every stream on the device;
the repetition history is a per-stream bitmap over the logits' index space
that the kernel extends with each sampled index, so the decode loop needs no
``unique()`` and no ``.item()``.
"""
from __future__ import annotations

import os
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class SamplingParams:
    """Generation settings (defaults: config.py:28-31, inference_engine.py:402)."""
    temperature: float = 0.5
    top_p: float = 0.85
    repetition_penalty: float = 1.2
    top_k: int = 256
    seed: int = 0

    def __post_init__(self):
        if not (self.temperature > 0 and self.temperature < float("inf")):
            raise ValueError(f"temperature must be positive and finite, got {self.temperature}")
        if not (self.repetition_penalty > 0 and self.repetition_penalty < float("inf")):
            raise ValueError(f"repetition_penalty must be positive and finite, got {self.repetition_penalty}")
        if self.top_p != self.top_p:
            raise ValueError("top_p is NaN")
        if not 1 <= self.top_k <= 256:
            raise ValueError(f"top_k must be in [1, 256], got {self.top_k}")

    @classmethod
    def from_env(cls, **overrides) -> "SamplingParams":
        """The reference's environment overrides (config.py:27-31)."""
        kw = dict(temperature=float(os.getenv("TEMPERATURE", "0.5")),
                  top_p=float(os.getenv("TOP_P", "0.85")),
                  repetition_penalty=float(os.getenv("REPETITION_PENALTY", "1.2")))
        kw.update(overrides)
        return cls(**kw)


def seen_bitmap(history: torch.Tensor, vocab: int, full_to_reduced: torch.Tensor | None = None,
                device: torch.device | None = None) -> torch.Tensor:
    """Per-stream bitmap [B, ceil(vocab / 32)] int32 of the indices in ``history``
    ([B, T] token ids), mapped through ``full_to_reduced`` (entries < 0 are not
    in the sampled vocabulary and are dropped, inference_engine.py:377-383).
    Bit i of word w marks index 32 w + i."""
    h = torch.as_tensor(history).long()
    if h.dim() == 1:
        h = h.view(1, -1)
    dev = device if device is not None else h.device
    h = h.to(dev)
    idx = full_to_reduced.to(dev)[h] if full_to_reduced is not None else h
    valid = (idx >= 0) & (idx < vocab)
    b = h.shape[0]
    words = (vocab + 31) // 32
    bits = torch.zeros(b, words * 32, dtype=torch.bool, device=dev)
    rows = torch.arange(b, device=dev).view(-1, 1).expand_as(idx)
    bits[rows[valid], idx[valid]] = True
    w = (bits.view(b, words, 32).long() << torch.arange(32, device=dev)).sum(-1)
    return (w - ((w >> 31) << 32)).to(torch.int32)
