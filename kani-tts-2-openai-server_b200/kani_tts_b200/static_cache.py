"""Static KV cache with a kernel-backed write (mirror of ``kani_tts/static_cache.py``).

``StaticKVCache`` keeps the attribute and method names that the reference
engine reads (inference_engine.py:218-228, 297-302, 342-346):
``key_cache``, ``value_cache``, ``conv_cache``, ``_write_position``,
``set_write_position``, ``advance_position``, ``max_total_len``,
``copy_from_dynamic``, ``get_seq_length``, ``reset``.  ``update`` replaces the
two ``scatter_`` launches per attention layer (static_cache.py:131-140) with
one ``kani_kv_cache_write`` launch, and ``update_fused`` performs the whole
q/k-norm + RoPE + KV write of optimized_decode.py:220-240 in one launch.

Buffers are laid out [batch, kv_heads, max_total_len, head_dim] like the
reference so SDPA can read them directly.  ``_write_position`` may hold one
slot (shared by the batch, as in the reference) or one slot per stream.
"""
from __future__ import annotations

import torch

from . import _lib
from .fused_kernels import fused_rope_kv_write, kv_cache_write


class StaticKVCache:
    """Pre-allocated K/V buffers per attention layer and conv state per layer."""

    def __init__(self, config, max_total_len: int, batch_size: int = 1,
                 dtype: torch.dtype = torch.bfloat16, device: torch.device | str | None = None,
                 per_stream_positions: bool = False):
        self.max_total_len = max_total_len
        self.batch_size = batch_size
        self._dtype = dtype
        self.device = torch.device(device) if device is not None else torch.device("cuda")
        num_kv_heads = config.num_key_value_heads
        head_dim = getattr(config, "head_dim", None) or config.hidden_size // config.num_attention_heads
        num_layers = config.num_hidden_layers
        hidden_size = config.hidden_size
        self.layer_types = (list(config.layer_types) if getattr(config, "layer_types", None)
                            else ["full_attention"] * num_layers)
        self.first_attention_layer = next(
            (i for i, t in enumerate(self.layer_types) if t == "full_attention"), 0)
        self.key_cache: list[torch.Tensor] = []
        self.value_cache: list[torch.Tensor] = []
        for i in range(num_layers):
            if self.layer_types[i] == "full_attention":
                shape = (batch_size, num_kv_heads, max_total_len, head_dim)
                self.key_cache.append(torch.zeros(shape, dtype=dtype, device=self.device))
                self.value_cache.append(torch.zeros(shape, dtype=dtype, device=self.device))
            else:
                self.key_cache.append(torch.empty(0, dtype=dtype, device=self.device))
                self.value_cache.append(torch.empty(0, dtype=dtype, device=self.device))
        conv_l = getattr(config, "conv_L_cache", 4)
        self.conv_cache = [torch.zeros(batch_size, hidden_size, conv_l, dtype=dtype, device=self.device)
                           for _ in range(num_layers)]
        n_pos = batch_size if per_stream_positions else 1
        self._write_position = torch.zeros(n_pos, dtype=torch.long, device=self.device)
        self._logical_length = 0
        # device error flag allocated now, so a later graph capture reuses it
        self.err_flag = _lib.error_flag(self.device)

    def copy_from_dynamic(self, dynamic_cache, logical_length: int) -> None:
        """One-time copy from a dynamic cache (reference static_cache.py:86-108)."""
        self._logical_length = logical_length
        for i in range(len(self.key_cache)):
            if self.layer_types[i] != "full_attention":
                continue
            if i < len(dynamic_cache.key_cache) and dynamic_cache.key_cache[i].numel() > 0:
                n = dynamic_cache.key_cache[i].shape[-2]
                self.key_cache[i][:, :, :n, :].copy_(dynamic_cache.key_cache[i])
                self.value_cache[i][:, :, :n, :].copy_(dynamic_cache.value_cache[i])
        for i in range(len(self.conv_cache)):
            if i < len(dynamic_cache.conv_cache):
                self.conv_cache[i].copy_(dynamic_cache.conv_cache[i])

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int,
               cache_kwargs=None):
        """Write [B, Hk, 1, D] K/V at the write position; return the full buffers."""
        if key_states is not None and self.layer_types[layer_idx] == "full_attention":
            kv_cache_write(key_states, value_states, self.key_cache[layer_idx],
                           self.value_cache[layer_idx], self._write_position, self.err_flag)
        return self.key_cache[layer_idx], self.value_cache[layer_idx]

    def update_fused(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, layer_idx: int,
                     inv_freq: torch.Tensor, position_ids: torch.Tensor,
                     q_norm_w: torch.Tensor | None = None, k_norm_w: torch.Tensor | None = None,
                     eps: float = 1e-5, frame_table: torch.Tensor | None = None,
                     tokens_per_frame: int = 4, frame_pos: torch.Tensor | None = None,
                     q_out: torch.Tensor | None = None):
        """q/k norm + RoPE + KV write of one decode step in one launch.

        q: [B, 1, Hq, D], k / v: [B, 1, Hk, D] (views into the QKV output);
        position_ids: [B, 1] angle positions.  Writes at ``_write_position``
        (one shared slot or one per stream).  Returns (q_rot, K buffer, V buffer).
        """
        b = self.batch_size
        slots = self._write_position
        if slots.numel() == 1 and b > 1:
            slots = slots.expand(b)
        q_rot = fused_rope_kv_write(
            q, k, v, inv_freq, position_ids.reshape(-1), self.key_cache[layer_idx],
            self.value_cache[layer_idx], slots.reshape(-1), frame_table=frame_table,
            tokens_per_frame=tokens_per_frame, q_norm_w=q_norm_w, k_norm_w=k_norm_w, eps=eps,
            frame_pos=frame_pos, q_out=q_out, err_flag=self.err_flag)
        return q_rot, self.key_cache[layer_idx], self.value_cache[layer_idx]

    def set_write_position(self, pos) -> None:
        """Set the write slot(s) before a graph replay (reference static_cache.py:144-146)."""
        if isinstance(pos, torch.Tensor):
            self._write_position.copy_(pos.reshape(self._write_position.shape))
        else:
            self._write_position.fill_(int(pos))

    def advance_position(self) -> None:
        self._logical_length += 1

    def get_seq_length(self, layer_idx: int = 0) -> int:
        return self._logical_length

    def get_mask_sizes(self, cache_position, layer_idx):
        return self._logical_length, 0

    def __len__(self) -> int:
        return len(self.key_cache)

    def __getitem__(self, layer_idx: int):
        return self.key_cache[layer_idx], self.value_cache[layer_idx]

    def reset(self) -> None:
        for i in range(len(self.key_cache)):
            if self.key_cache[i].numel() > 0:
                self.key_cache[i].zero_()
                self.value_cache[i].zero_()
        for c in self.conv_cache:
            c.zero_()
        self._logical_length = 0
        self._write_position.fill_(0)

    def read_errors(self) -> int:
        """Synchronising read-and-clear of the kernels' KANI_FLAG_* bits."""
        v = int(self.err_flag.item())
        self.err_flag.zero_()
        return v
