"""LFM2-style model description for the decode path: config and weights.

Parameter names follow the HF LFM2 checkpoint layout that the reference
loads (kani_tts/model.py, kani_tts/optimized_decode.py:54-132), so a real
state dict and the synthetic one below are interchangeable:

    model.embed_tokens.weight                       [V, H]
    model.layers.{i}.operator_norm.weight           [H]
    model.layers.{i}.ffn_norm.weight                [H]
    model.layers.{i}.feed_forward.w1/w3.weight      [F, H]   (gate / up)
    model.layers.{i}.feed_forward.w2.weight         [H, F]   (down)
    attention layers:
    model.layers.{i}.self_attn.{q,k,v}_proj.weight  [Hq*D | Hk*D, H]
    model.layers.{i}.self_attn.{q,k}_layernorm.weight [D]
    model.layers.{i}.self_attn.out_proj.weight      [H, Hq*D]
    model.learnable_rope_layers.{i}.alpha_weight    []       (bf16 scalar)
    short-conv layers:
    model.layers.{i}.conv.in_proj.weight            [3H, H]
    model.layers.{i}.conv.conv.weight               [H, 1, L]
    model.layers.{i}.conv.out_proj.weight           [H, H]
    model.embedding_norm.weight                     [H]      (final norm)
    model.speaker_emb_projection.weight             [H, speaker_dim]
    lm_head.weight                                  [V, H]   (tied to the embedding)
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

# LFM2 interleave of 10 short-conv and 6 attention blocks (attention at 2, 5,
# 8, 10, 12, 14), the 16-layer layout of the 350M-class models.
LFM2_16_LAYER_TYPES = ["conv", "conv", "full_attention", "conv", "conv", "full_attention", "conv", "conv",
                       "full_attention", "conv", "full_attention", "conv", "full_attention", "conv",
                       "full_attention", "conv"]


@dataclass
class LFM2Config:
    hidden_size: int = 1024
    num_attention_heads: int = 16
    num_key_value_heads: int = 8
    head_dim: int = 64
    intermediate_size: int = 4608
    vocab_size: int = 80000
    num_hidden_layers: int = 16
    layer_types: list = field(default_factory=lambda: list(LFM2_16_LAYER_TYPES))
    conv_L_cache: int = 3
    norm_eps: float = 1e-5
    rope_theta: float = 1e6
    audio_tokens_start: int = 64410
    eos_token_id: int = 64402          # end-of-speech: the engine's EOS (core.py:599, config.py:12)
    tokens_per_frame: int = 4
    audio_step: float = 1.0
    speaker_emb_dim: int = 128
    alpha_min: float = 0.1
    alpha_max: float = 2.0

    @property
    def attn_layers(self) -> list[int]:
        return [i for i, t in enumerate(self.layer_types) if t == "full_attention"]

    @property
    def num_reduced(self) -> int:
        """Rows of the reduced head: [EOS] + audio tokens (optimized_decode.py:134-141)."""
        return 1 + self.vocab_size - self.audio_tokens_start


def tiny_config() -> LFM2Config:
    """A 4-layer model with the real head size (64) and GQA ratio (2), for tests."""
    return LFM2Config(hidden_size=128, num_attention_heads=2, num_key_value_heads=1, head_dim=64,
                      intermediate_size=256, vocab_size=700, num_hidden_layers=4,
                      layer_types=["conv", "full_attention", "conv", "full_attention"],
                      audio_tokens_start=600, eos_token_id=7, speaker_emb_dim=32)


def synthetic_state_dict(cfg: LFM2Config, seed: int = 0, device="cpu", std: float = 0.02,
                         dtype=torch.bfloat16) -> dict[str, torch.Tensor]:
    """Random-init weights ~ N(0, std) (norm weights ~ N(1, std), learnable alpha
    weight 0 -> alpha = 1.05), drawn from one seeded generator in a fixed order."""
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(seed)
    h, d = cfg.hidden_size, cfg.head_dim
    hq, hk, f = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.intermediate_size

    def w(*shape, mean=0.0):
        return (mean + std * torch.randn(*shape, generator=g, device=dev)).to(dtype)

    sd = {"model.embed_tokens.weight": w(cfg.vocab_size, h)}
    for i, kind in enumerate(cfg.layer_types):
        p = f"model.layers.{i}."
        sd[p + "operator_norm.weight"] = w(h, mean=1.0)
        sd[p + "ffn_norm.weight"] = w(h, mean=1.0)
        if kind == "full_attention":
            sd[p + "self_attn.q_proj.weight"] = w(hq * d, h)
            sd[p + "self_attn.k_proj.weight"] = w(hk * d, h)
            sd[p + "self_attn.v_proj.weight"] = w(hk * d, h)
            sd[p + "self_attn.q_layernorm.weight"] = w(d, mean=1.0)
            sd[p + "self_attn.k_layernorm.weight"] = w(d, mean=1.0)
            sd[p + "self_attn.out_proj.weight"] = w(h, hq * d)
            sd[f"model.learnable_rope_layers.{i}.alpha_weight"] = torch.zeros((), dtype=dtype, device=dev)
        else:
            sd[p + "conv.in_proj.weight"] = w(3 * h, h)
            sd[p + "conv.conv.weight"] = w(h, 1, cfg.conv_L_cache)
            sd[p + "conv.out_proj.weight"] = w(h, h)
        sd[p + "feed_forward.w1.weight"] = w(f, h)
        sd[p + "feed_forward.w3.weight"] = w(f, h)
        sd[p + "feed_forward.w2.weight"] = w(h, f)
    sd["model.embedding_norm.weight"] = w(h, mean=1.0)
    sd["model.speaker_emb_projection.weight"] = w(h, cfg.speaker_emb_dim)
    sd["lm_head.weight"] = sd["model.embed_tokens.weight"]
    return sd
