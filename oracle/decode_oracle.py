"""CPU restatement of the reference decode step — TEST INFRASTRUCTURE ONLY.

``OracleDecoder.step`` follows ``OptimizedDecoder.__call__``
(kani_tts/optimized_decode.py:175-289) line by line for B streams, with the
three Triton kernels replaced by their oracle restatements
(``oracle.kani_oracle.*_ref``) and the static-cache ``scatter_`` by direct
slot writes (static_cache.py:131-140).  The eager glue (embedding, F.linear,
the residual adds, the conv composition, SDPA with an additive mask) is the
reference's own PyTorch code path run on the CPU.  ``rounding="trunc"``
reproduces the Triton interpreter's bf16 stores (used to check against the
golden decode steps produced by running the reference decoder itself).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import kani_oracle as O


class OracleDecoder:
    def __init__(self, cfg, state_dict, batch: int, max_len: int, rounding: str = "rne"):
        self.cfg = cfg
        self.b = batch
        self.rounding = rounding
        self.dtype = torch.bfloat16
        sd = {k: v.detach().to("cpu") for k, v in state_dict.items()}
        self.sd = sd
        h, d = cfg.hidden_size, cfg.head_dim
        self.hq, self.hk, self.d = cfg.num_attention_heads, cfg.num_key_value_heads, d
        self.eps = cfg.norm_eps
        self.inv_freq = {}
        for i in cfg.attn_layers:
            aw = sd.get(f"model.learnable_rope_layers.{i}.alpha_weight", torch.tensor(0.0))
            self.inv_freq[i] = O.learnable_inv_freq_ref(d, cfg.rope_theta, float(aw), cfg.alpha_min,
                                                        cfg.alpha_max)
        head = sd["lm_head.weight"]
        self.head = torch.cat([head[cfg.eos_token_id:cfg.eos_token_id + 1], head[cfg.audio_tokens_start:]], 0)
        self.k_cache = {i: torch.zeros(batch, self.hk, max_len, d, dtype=self.dtype) for i in cfg.attn_layers}
        self.v_cache = {i: torch.zeros_like(self.k_cache[i]) for i in cfg.attn_layers}
        self.conv_state = {i: torch.zeros(batch, h, cfg.conv_L_cache, dtype=self.dtype)
                           for i, t in enumerate(cfg.layer_types) if t != "full_attention"}

    def _w(self, name):
        return self.sd[name]

    def step(self, input_ids, positions, slots, mask):
        cfg, b, hq, hk, d = self.cfg, self.b, self.hq, self.hk, self.d
        rnd = self.rounding
        hidden = F.embedding(input_ids.cpu(), self._w("model.embed_tokens.weight"))      # :197
        for i, kind in enumerate(cfg.layer_types):
            p = f"model.layers.{i}."
            normed = O.rms_norm_ref(hidden, self._w(p + "operator_norm.weight"), self.eps, rnd)   # :206
            if kind == "full_attention":
                qkv_w = torch.cat([self._w(p + "self_attn.q_proj.weight"), self._w(p + "self_attn.k_proj.weight"),
                                   self._w(p + "self_attn.v_proj.weight")], 0)
                qkv = F.linear(normed, qkv_w)                                             # :210
                q, k, v = qkv.split([hq * d, hk * d, hk * d], dim=-1)
                q = O.rms_norm_ref(q.reshape(b, 1, hq, d), self._w(p + "self_attn.q_layernorm.weight"),
                                   self.eps, rnd)                                         # :220
                k = O.rms_norm_ref(k.reshape(b, 1, hk, d), self._w(p + "self_attn.k_layernorm.weight"),
                                   self.eps, rnd)                                         # :221
                v = v.reshape(b, hk, d)
                qr = torch.empty(b, hq, 1, d, dtype=self.dtype)
                for s in range(b):                                                        # :229-237
                    cos, sin = O.rope_cos_sin_ref(self.inv_freq[i], int(positions[s]), self.dtype)
                    qr[s] = O.rope_ref(q[s, 0], cos, sin, rnd).unsqueeze(1)
                    kr = O.rope_ref(k[s, 0], cos, sin, rnd)
                    slot = int(slots[s])                                                  # :240
                    self.k_cache[i][s, :, slot] = kr
                    self.v_cache[i][s, :, slot] = v[s]
                attn = F.scaled_dot_product_attention(qr, self.k_cache[i], self.v_cache[i],
                                                      attn_mask=mask.cpu(), scale=d ** -0.5,
                                                      enable_gqa=True)                    # :243-248
                hidden = hidden + F.linear(attn.reshape(b, 1, hq * d), self._w(p + "self_attn.out_proj.weight"))
            else:                                                                         # :256-277
                bcx = F.linear(normed, self._w(p + "conv.in_proj.weight")).transpose(-1, -2)
                bg, c, xc = bcx.chunk(3, dim=-2)
                bx = bg * xc
                state = self.conv_state[i].roll(shifts=-1, dims=-1)
                state[:, :, cfg.conv_L_cache - 1] = bx[..., 0]
                self.conv_state[i].copy_(state)
                conv_out = torch.sum(state * self._w(p + "conv.conv.weight")[:, 0, :], dim=-1).unsqueeze(-1)
                y = (c * conv_out).transpose(-1, -2)
                hidden = hidden + F.linear(y, self._w(p + "conv.out_proj.weight"))
            normed = O.rms_norm_ref(hidden, self._w(p + "ffn_norm.weight"), self.eps, rnd)    # :280
            gate_up = F.linear(normed, torch.cat([self._w(p + "feed_forward.w1.weight"),
                                                  self._w(p + "feed_forward.w3.weight")], 0))
            mlp = O.silu_mul_ref(gate_up, rnd)                                            # :282
            hidden = hidden + F.linear(mlp, self._w(p + "feed_forward.w2.weight"))        # :283
        hidden = O.rms_norm_ref(hidden, self._w("model.embedding_norm.weight"), self.eps, rnd)  # :286
        return F.linear(hidden, self.head)                                                # :287
