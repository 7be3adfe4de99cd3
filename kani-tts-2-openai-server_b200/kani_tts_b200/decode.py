"""Fused LFM2 decode step and generation engine on the B200 kernels.

``FusedDecoder`` is ``OptimizedDecoder.__call__`` (kani_tts/optimized_decode.py:
175-289) rebuilt on this library, for one or many independent speech streams:

* every residual add is folded into the RMSNorm that follows it
  (``fused_add_rms_norm``: optimized_decode.py:252/277/283 + :206/:280/:286);
* q/k per-head norm, cos/sin, RoPE (with the optional BemaTTS frame term) and
  the static KV write are one ``fused_rope_kv_write`` launch per attention
  layer (optimized_decode.py:220-240), reading the packed QKV output in place
  and writing Q straight into the attention layout;
* ``fused_silu_mul`` between the fused gate/up and down projections;
* QKV and gate/up weights are concatenated and the LM head is reduced to
  [EOS] + audio rows, as the reference does (optimized_decode.py:85-99, 134-156);
* GQA decode attention reads only each stream's valid cache prefix
  (``decode_attention``: split over an 8-CTA cluster, partials merged in
  distributed shared memory) instead of SDPA over the whole -inf-masked
  buffer (optimized_decode.py:243-248);
* the gated short-conv step between in_proj and out_proj is one
  ``short_conv_step`` launch (optimized_decode.py:256-277);
* greedy steps end in one fused head launch (the reduced head, the argmax
  and the reduced-to-full map): ``head_argmax`` (CUDA-core GEMV) up to 8
  streams, ``head_argmax_tc`` (tcgen05 tensor-core GEMM) from 9 to 64; sampled
  steps take their logits from the same launch;
* up to 4 streams, every projection is a ``gemv`` launch that folds in the
  residual add + RMSNorm before it and the SiLU·mul after the gate/up GEMV;
* otherwise up to 32 streams, every projection is a ``gemm_tc`` launch
  (tcgen05 tensor cores): the gate/up one with the SiLU·mul as its epilogue,
  the 1024-row output projections with K split over a thread-block cluster,
  and up to 8 streams the residual add + RMSNorm as the input projections'
  prologue.

Beyond 32 streams every GEMM is a cuBLAS call, the projections before a residual
add as K-split fp32 partials that the add + RMSNorm launch sums
(``reduce_add_rms_norm``); prefill attention is PyTorch SDPA.

``DecodeEngine`` adds batched prefill (the same kernels at T tokens per
stream, causal SDPA, causal depthwise conv) and a CUDA-graph decode loop
whose per-step bookkeeping (position schedule of inference_engine.py:615-619,
KV slot, mask slot, next token) also runs inside the graph, so generation
needs no host synchronisation per token.  The next token is the greedy
argmax, or, given ``SamplingParams``, the reference's penalty / top-k /
temperature / top-p / multinomial sampler (inference_engine.py:349-430) as one
``sample_tokens`` launch per step, with the repetition history kept as a
device bitmap and the Philox step counter advanced inside the graph.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import _lib
from .fused_kernels import (decode_advance, decode_attention, fused_add_rms_norm, fused_rms_norm,
                            fused_rope_kv_write, fused_silu_mul, gemm_tc, gemv, gemv_rope_kv_write, gemv_short_conv,
                            head_argmax, head_argmax_tc, linear_split_k, reduce_add_rms_norm, sample_tokens,
                            short_conv_step)
from .model import LFM2Config
from .positions import learnable_inv_freq
from .sampling import SamplingParams, seen_bitmap


class FusedDecoder:
    """Flat, fused decode forward over a static cache for `batch` streams."""

    def __init__(self, cfg: LFM2Config, state_dict: dict[str, torch.Tensor], device, batch: int,
                 max_len: int, frame_table: torch.Tensor | None = None):
        self.cfg = cfg
        self.device = dev = torch.device(device)
        self.batch = batch
        self.max_len = max_len
        self.dtype = torch.bfloat16
        h, d = cfg.hidden_size, cfg.head_dim
        self.hq, self.hk, self.d = cfg.num_attention_heads, cfg.num_key_value_heads, d
        self.q_dim, self.kv_dim = self.hq * d, self.hk * d
        self.eps = cfg.norm_eps
        self.scale = d ** -0.5
        self.frame_table = frame_table

        def t(name):
            return state_dict[name].to(dev, self.dtype).contiguous()

        self.embed = t("model.embed_tokens.weight")
        self.layers = []
        for i, kind in enumerate(cfg.layer_types):
            p = f"model.layers.{i}."
            L = {"attn": kind == "full_attention",
                 "op_norm": t(p + "operator_norm.weight"), "ffn_norm": t(p + "ffn_norm.weight"),
                 "gate_up": torch.cat([t(p + "feed_forward.w1.weight"), t(p + "feed_forward.w3.weight")], 0),
                 "down": t(p + "feed_forward.w2.weight")}
            if L["attn"]:
                L["qkv"] = torch.cat([t(p + "self_attn.q_proj.weight"), t(p + "self_attn.k_proj.weight"),
                                      t(p + "self_attn.v_proj.weight")], 0)
                L["q_norm"] = t(p + "self_attn.q_layernorm.weight")
                L["k_norm"] = t(p + "self_attn.k_layernorm.weight")
                L["o"] = t(p + "self_attn.out_proj.weight")
                aw = state_dict.get(f"model.learnable_rope_layers.{i}.alpha_weight", torch.tensor(0.0))
                L["inv_freq"] = learnable_inv_freq(d, cfg.rope_theta, aw, cfg.alpha_min, cfg.alpha_max).to(dev)
            else:
                L["in_proj"] = t(p + "conv.in_proj.weight")
                L["conv_w"] = t(p + "conv.conv.weight")[:, 0, :].contiguous()
                L["out_proj"] = t(p + "conv.out_proj.weight")
            self.layers.append(L)
        self.final_norm = t("model.embedding_norm.weight")
        head = t("lm_head.weight")
        red = torch.cat([head[cfg.eos_token_id:cfg.eos_token_id + 1], head[cfg.audio_tokens_start:]], 0)
        # F.linear's output row is padded to a multiple of 8 (16 bytes): an odd row of
        # 15591 logits sends cuBLAS to an unaligned GEMM several times slower at
        # 64 streams.  The extra zero rows are sliced off the logits; `head` is the
        # view of the real rows (the fused head kernels and the samplers see only those).
        pad = (-red.shape[0]) % 8
        self.head_padded = torch.cat([red, red.new_zeros(pad, red.shape[1])], 0) if pad else red
        self.head = self.head_padded[:red.shape[0]]
        self.num_reduced = red.shape[0]
        self.reduced_to_full = torch.cat([
            torch.tensor([cfg.eos_token_id], device=dev, dtype=torch.long),
            torch.arange(cfg.audio_tokens_start, cfg.vocab_size, device=dev, dtype=torch.long)])
        self.full_to_reduced = torch.full((cfg.vocab_size,), -1, device=dev, dtype=torch.long)
        self.full_to_reduced[self.reduced_to_full] = torch.arange(self.reduced_to_full.numel(), device=dev)
        sp = state_dict.get("model.speaker_emb_projection.weight")
        self.speaker_proj = sp.to(dev, self.dtype) if sp is not None else None
        self._pack_weights()

        # static state: caches, conv states, error flag
        self.k_cache = {i: torch.zeros(batch, self.hk, max_len, d, dtype=self.dtype, device=dev)
                        for i, L in enumerate(self.layers) if L["attn"]}
        self.v_cache = {i: torch.zeros_like(self.k_cache[i]) for i in self.k_cache}
        self.conv_state = {i: torch.zeros(batch, h, cfg.conv_L_cache, dtype=self.dtype, device=dev)
                           for i, L in enumerate(self.layers) if not L["attn"]}
        self.err_flag = _lib.error_flag(dev)
        # fused head + argmax: the CUDA-core GEMV kernel up to 8 streams (hidden 512 /
        # 1024 / 2048), the tensor-core kernel up to 64 (hidden a multiple of 64, at
        # most 1024); each keeps a cross-CTA argmax scratch that is zero between launches
        if batch <= 8 and h in (512, 1024, 2048):
            self.fused_head = "gemv"
            self.head_scratch = torch.zeros(batch + 1, dtype=torch.long, device=dev)
        elif batch <= 64 and h % 64 == 0 and h <= 1024 and red.shape[0] <= 0xffff:
            self.fused_head = "tc"
            self.head_scratch = torch.zeros(batch + 1, dtype=torch.int32, device=dev)
        else:
            self.fused_head = None
            self.head_scratch = None
        # small batches take the fused-GEMV layer path (K of every GEMV: H or the FFN size).
        # Its CUDA-core dot products scale with the batch: measured per step on B200,
        # 1 / 2 / 4 / 8 streams take 285 / 351 / 560 / 892 us against ~750-790 us for
        # cuBLAS, so it serves up to 4 streams.
        self.small_batch = (batch <= 4 and h == 1024 and cfg.intermediate_size in (1024, 4608)
                            and self.q_dim == h and cfg.conv_L_cache == 3)
        # up to 32 streams not on the fused-GEMV path: every projection runs on the
        # tensor-core GEMM (the gate/up one with the SiLU·mul as its epilogue, the
        # 1024-row ones with K split over a cluster).  Measured per step on B200
        # against cuBLAS + separate launches: 696 vs 767 us at 8 streams, 726 vs 781
        # at 16, 743 vs 741 at 32, 816 vs 731 at 64 (there every CTA also streams
        # the 128 KB activation operand from L2, half again its weight bytes).
        self.tc_batch = (not self.small_batch and batch <= 32 and h % 64 == 0 and h <= 1024
                         and cfg.intermediate_size % 8 == 0)
        self.res_buf = [torch.empty(batch, 1, h, dtype=self.dtype, device=dev) for _ in range(2)]
        self.logits_buf = torch.empty(batch, 1, self.head.shape[0], dtype=self.dtype, device=dev)
        self.argmax_buf = torch.empty(batch, dtype=torch.long, device=dev)

    # ------------------------------------------------------------ weights in HBM
    def _pack_weights(self) -> None:
        """Moves the projection weights and the padded head into one buffer in the
        order a decode step reads them (per layer: QKV or in_proj, o_proj or
        out_proj, gate/up, down; then the head), so the weights of the launches
        ahead of any launch are one contiguous range (two where the step wraps
        around).  ``weight_spans`` holds each projection's [start, end) byte range."""
        keys = []
        for L in self.layers:
            keys += [(L, k) for k in (("qkv", "o") if L["attn"] else ("in_proj", "out_proj")) + ("gate_up", "down")]
        total = sum(L[k].numel() for L, k in keys) + self.head_padded.numel()
        self.weight_arena = arena = torch.empty(total, dtype=self.dtype, device=self.device)
        es = arena.element_size()
        self.weight_spans = []
        off = 0
        for L, k in keys:
            n = L[k].numel()
            L[k] = arena[off:off + n].view_as(L[k]).copy_(L[k])
            self.weight_spans.append((off * es, (off + n) * es))
            off += n
        n = self.head_padded.numel()
        self.head_padded = arena[off:off + n].view_as(self.head_padded).copy_(self.head_padded)
        self.head = self.head_padded[:self.num_reduced]
        self.weight_spans.append((off * es, (off + n) * es))
        self._l2_plan = None

    # Each decode GEMV (and the fused head) can prefetch into L2, as it starts,
    # the weights of the launches after it, up to this many bytes past the end
    # of its own; 0 turns the prefetch off.  Off by default: it took the bs = 1
    # step from 274-276 to 266 us when the GEMVs still fetched part of their
    # weights after the launch wait, and measures within noise at one stream
    # (236.8-237.7 us off, 236.0-237.9 at 16-64 MB ahead) and slower at two and
    # four streams (301.4-301.9 against 306.1-308.2 us, 525.7-526.4 against
    # 527.6-534.7) now that every weight a GEMV needs is requested before its wait.
    l2_prefetch_ahead = 0
    # The same prefetch ahead of the cuBLAS GEMMs above 32 streams, from the add +
    # RMSNorm and SiLU·mul launches before them.  Off: at 64 streams (600 greedy
    # tokens) it measured 613-624 us per step at 0-24 MB ahead against 613-615
    # without, and 633-659 at 32-64 MB, where the K/V stream of attention
    # (about 115 MB per layer) evicts the lines before their GEMM reads them.
    l2_prefetch_large = False

    def _l2_prefetch_plan(self) -> list:
        """Per weight-reading launch of the fused-GEMV step (in step order, the head
        last): the (address, bytes) ranges it prefetches, [F(i-1), F(i)) with
        F(i) = end of its weights + ``l2_prefetch_ahead``, taken modulo the
        arena (the head's frontier wraps into the next step's first layers)."""
        ahead = int(self.l2_prefetch_ahead) // 16 * 16
        if ahead <= 0:
            return [None] * len(self.weight_spans)
        if self._l2_plan is not None and self._l2_plan[0] == ahead:
            return self._l2_plan[1]
        total = self.weight_arena.numel() * self.weight_arena.element_size()
        ahead = min(ahead, total)
        base = self.weight_arena.data_ptr()
        plan = []
        prev = ahead  # the frontier the previous step's head launch left, modulo the arena
        for _, end in self.weight_spans:
            front = end + ahead
            lo, hi = prev, front
            ranges = []
            if hi > lo:
                a, b = lo % total, (hi - 1) % total + 1
                if lo // total == (hi - 1) // total:
                    ranges.append((base + a, b - a))
                else:
                    ranges += [(base + a, total - a), (base, b)]
            plan.append(ranges or None)
            prev = max(prev, front)
        self._l2_plan = (ahead, plan)
        return plan

    # ------------------------------------------------------------ decode
    fused_greedy_head = True   # greedy / sampled steps may use the fused head kernels
    tc_output_projections = True  # tensor-core path: o / out / down projections on gemm_tc (split K) too
    # Decode attention launches as a programmatic dependent of the RoPE + KV
    # write and streams the older cache rows while that launch runs
    # (kani_decode_attention_step).  Measured per step on B200 (1500 tokens):
    # 1 stream 270 vs 272-275 us, 8 streams 710-713 vs 716-720, 16 neutral,
    # 64 streams about 1 % (bench: 795 vs 799-801 us); on the fused-GEMV path at
    # 2-4 streams its early-resident CTAs cost more than they save (4 streams:
    # 589 vs 562 us).
    @property
    def dependent_attention(self) -> bool:
        return self.batch == 1 or not self.small_batch

    # The norm prologue re-reads every stream's row in every CTA (from L2); beyond
    # this many streams a separate add + RMSNorm launch is cheaper (measured: equal
    # at 8 streams, 58 us per step slower at 16).
    tc_norm_prologue_max_batch = 8

    def step(self, input_ids: torch.Tensor, positions: torch.Tensor, slots: torch.Tensor,
             kv_len: torch.Tensor, mask: torch.Tensor | None = None) -> torch.Tensor:
        """One decode token per stream.

        input_ids [B, 1] int64; positions / slots / kv_len [B] int64 (angle
        position, KV slot, number of valid cache slots including this one).
        ``mask`` is accepted for interface parity with the reference step and
        ignored: the valid region is the prefix [0, kv_len).  Returns
        reduced-head logits [B, 1, num_reduced].

        Every stream must write its newest valid row: ``slots[b] == kv_len[b] - 1``
        (as ``DecodeEngine`` keeps them).  Where ``dependent_attention`` holds
        (one stream, or more than 4), the attention launch streams the rows
        below ``kv_len - 1`` while the RoPE + KV write before it still runs, so
        a step that wrote any other row would be read before the write lands.
        """
        return self._linear_head(self._final_hidden(input_ids, positions, slots, kv_len))

    def _linear_head(self, normed: torch.Tensor) -> torch.Tensor:
        """Reduced-head logits by F.linear on the padded head: [..., num_reduced] view."""
        return F.linear(normed, self.head_padded)[..., :self.num_reduced]

    # Up to 4 streams the final residual add + RMSNorm runs inside the head
    # launch (kani_head_argmax_norm) instead of a launch of its own: measured
    # 6.5 us of the bs = 1 step for that launch.
    fuse_final_norm = True

    def _head_input(self, input_ids, positions, slots, kv_len):
        """The decode layers, ending either in the final-normed hidden state or, where
        the fused head takes the final norm, in (update, residual stream)."""
        if self.small_batch and self.fused_head == "gemv" and self.fuse_final_norm:
            return self._final_hidden_small(input_ids, positions, slots, kv_len, fuse_final=True)
        return self._final_hidden(input_ids, positions, slots, kv_len)

    def _fused_head(self, normed, index_map=None, logits_out=None, out=None) -> torch.Tensor:
        fn = head_argmax if self.fused_head == "gemv" else head_argmax_tc
        if self.fused_head == "tc":
            kw = {"err_flag": self.err_flag}
        else:
            kw = {"l2_prefetch": self._l2_prefetch_plan()[-1]} if self.small_batch else {}
            if isinstance(normed, tuple):        # (update, residual stream): the final norm in the head
                normed, residual = normed
                kw.update(norm_weight=self.final_norm, residual=residual, eps=self.eps)
        return fn(normed, self.head, index_map, scratch=self.head_scratch, logits_out=logits_out, out=out, **kw)

    def step_logits(self, input_ids: torch.Tensor, positions: torch.Tensor, slots: torch.Tensor,
                    kv_len: torch.Tensor) -> torch.Tensor:
        """``step`` with the reduced head on the fused head kernel, which writes the
        logits while it computes them (its greedy token is not used).  Returns
        reduced-head logits [B, 1, num_reduced] in a static buffer."""
        if self.fused_head is None:
            return self.step(input_ids, positions, slots, kv_len)
        normed = self._head_input(input_ids, positions, slots, kv_len)
        self._fused_head(normed, logits_out=self.logits_buf.view(self.batch, -1), out=self.argmax_buf)
        return self.logits_buf

    def step_greedy(self, input_ids: torch.Tensor, positions: torch.Tensor, slots: torch.Tensor,
                    kv_len: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """One decode token per stream, greedy: the reduced head, the argmax and the
        reduced-to-full map in one launch (``head_argmax`` up to 8 streams of hidden
        size 512 / 1024 / 2048, ``head_argmax_tc`` up to 64 streams of hidden size a
        multiple of 64 up to 1024).  Returns the full token ids [B]."""
        if self.fused_head is None:
            raise ValueError("the fused greedy head serves at most 64 streams (hidden size at most 1024, "
                             "or 2048 up to 8 streams)")
        normed = self._head_input(input_ids, positions, slots, kv_len)
        return self._fused_head(normed, self.reduced_to_full, out=out)

    def _final_hidden(self, input_ids, positions, slots, kv_len) -> torch.Tensor:
        """The decode layers and the final norm: [B, 1, H]."""
        if self.small_batch:
            return self._final_hidden_small(input_ids, positions, slots, kv_len)
        if self.tc_batch:
            return self._final_hidden_tc(input_ids, positions, slots, kv_len)
        return self._final_hidden_large(input_ids, positions, slots, kv_len)

    def _final_hidden_small(self, input_ids, positions, slots, kv_len, fuse_final: bool = False):
        """Up to 8 streams: every F.linear is a ``gemv`` launch that also applies the
        residual add + RMSNorm before it and, for gate/up, the SiLU·mul after it,
        the in_proj GEMV also runs the short-conv step and the QKV GEMV the
        q/k norm + RoPE + KV write, so a layer is 4 launches (conv) or 5
        (attention) instead of 8-9.  The
        residual stream alternates between two static buffers (a launch reads one
        and writes the other).  With ``fuse_final`` the last update and residual
        stream are returned as they are, for the head launch that applies the
        final add + RMSNorm itself."""
        b, hq, hk, d = self.batch, self.hq, self.hk, self.d
        hidden = F.embedding(input_ids, self.embed)              # [B, 1, H] residual stream
        delta = None
        flip = 0
        pf = iter(self._l2_prefetch_plan())

        def normed(fn, *args, **kw):
            # fn (a GEMV launch) on RMSNorm(hidden + delta); the sum becomes the new residual stream
            nonlocal hidden, flip
            if delta is None:
                return fn(hidden, *args, eps=self.eps, **kw)
            out_res = self.res_buf[flip]
            flip ^= 1
            y = fn(delta, *args, residual=hidden, residual_out=out_res, eps=self.eps, **kw)
            hidden = out_res
            return y

        for i, L in enumerate(self.layers):
            if L["attn"]:
                # QKV GEMV + q/k norm + RoPE + frame term + KV write, one launch
                q_rot = normed(gemv_rope_kv_write, L["qkv"], L["op_norm"], L["inv_freq"], positions,
                               self.k_cache[i], self.v_cache[i], slots, num_q_heads=hq, num_kv_heads=hk,
                               q_norm_w=L["q_norm"], k_norm_w=L["k_norm"], head_eps=self.eps,
                               frame_table=self.frame_table, tokens_per_frame=self.cfg.tokens_per_frame,
                               err_flag=self.err_flag, l2_prefetch=next(pf))
                attn = decode_attention(q_rot, self.k_cache[i], self.v_cache[i], kv_len, self.scale,
                                        err_flag=self.err_flag, prefix_final=self.dependent_attention)
                delta = gemv(attn.view(b, 1, self.q_dim), L["o"], l2_prefetch=next(pf))
            else:
                y = normed(gemv_short_conv, L["in_proj"], self.conv_state[i], L["conv_w"], norm_weight=L["op_norm"],
                           l2_prefetch=next(pf))
                delta = gemv(y, L["out_proj"], l2_prefetch=next(pf))
            act = normed(gemv, L["gate_up"], norm_weight=L["ffn_norm"], silu_pairs=True, l2_prefetch=next(pf))
            delta = gemv(act, L["down"], l2_prefetch=next(pf))
        if fuse_final:
            return delta, hidden   # the fused head applies the final add + RMSNorm
        normed, _ = fused_add_rms_norm(delta, hidden, self.final_norm, self.eps)
        return normed

    # Above 32 streams the projections that feed a residual add (o_proj / out_proj,
    # K = 1024, and down, K = 4608) run as cuBLAS batched GEMMs with fp32 outputs
    # over K slices, and one launch sums the slices, adds the residual and applies
    # the next RMSNorm.  Measured at 64 streams (µs per launch, graph replay):
    # down 4.6 (4 slices) against 7.9 for the bf16 GEMM, o_proj 3.2 (2 slices)
    # against 3.7, and the sum rides in the add + RMSNorm launch that follows
    # anyway.  In the whole step (64 streams, 600 tokens) the split counts gave
    # 608 µs (down 6, out 2), 612-618 (down 2-4, out 2-4), 642 (out unsplit) and
    # 697 without any split.  0 turns a projection back into F.linear.
    split_k_down = 6
    split_k_out = 2

    def _final_hidden_large(self, input_ids, positions, slots, kv_len) -> torch.Tensor:
        """Many streams: cuBLAS GEMMs with the fused norm / activation launches between
        them; the projections before a residual add come as K-split fp32 partials
        that the add + RMSNorm launch sums (``reduce_add_rms_norm``)."""
        b, hq, hk, d = self.batch, self.hq, self.hk, self.d
        hidden = F.embedding(input_ids, self.embed)              # [B, 1, H] residual stream
        # the launch before each GEMM prefetches the weights ahead of it into L2
        # (the plan's entry of that GEMM); launches without the hint skip theirs
        plan = self._l2_prefetch_plan() if self.l2_prefetch_large else [None] * len(self.weight_spans)
        gi = 0

        def proj(x, w, splits):
            return linear_split_k(x, w, splits) if splits > 1 else F.linear(x, w)

        def add_norm(delta, hidden, w, pf=None):
            if delta.dtype == torch.float32 and delta.dim() == 3 and self.dtype != torch.float32:
                return reduce_add_rms_norm(delta, hidden, w, self.eps, l2_prefetch=pf)   # K-split partials
            return fused_add_rms_norm(delta, hidden, w, self.eps)

        delta = None
        for i, L in enumerate(self.layers):
            if delta is None:
                normed = fused_rms_norm(hidden, L["op_norm"], self.eps)
            else:
                normed, hidden = add_norm(delta, hidden, L["op_norm"], plan[gi])
            gi += 1
            if L["attn"]:
                qkv = F.linear(normed, L["qkv"])                  # [B, 1, (Hq+2Hk)D]
                q, k, v = qkv.split([self.q_dim, self.kv_dim, self.kv_dim], dim=-1)
                q_rot = fused_rope_kv_write(
                    q.view(b, 1, hq, d), k.view(b, 1, hk, d), v.view(b, 1, hk, d), L["inv_freq"], positions,
                    self.k_cache[i], self.v_cache[i], slots, frame_table=self.frame_table,
                    tokens_per_frame=self.cfg.tokens_per_frame, q_norm_w=L["q_norm"], k_norm_w=L["k_norm"],
                    eps=self.eps, err_flag=self.err_flag)
                attn = decode_attention(q_rot, self.k_cache[i], self.v_cache[i], kv_len, self.scale,
                                        err_flag=self.err_flag, prefix_final=self.dependent_attention)   # [B, Hq, D]
                delta = proj(attn.view(b, 1, self.q_dim), L["o"], self.split_k_out)
            else:
                y = short_conv_step(F.linear(normed, L["in_proj"]), self.conv_state[i], L["conv_w"])
                delta = proj(y, L["out_proj"], self.split_k_out)
            gi += 1
            normed, hidden = add_norm(delta, hidden, L["ffn_norm"], plan[gi])
            act = fused_silu_mul(F.linear(normed, L["gate_up"]), l2_prefetch=plan[gi + 1])
            delta = proj(act, L["down"], self.split_k_down)
            gi += 2
        normed, _ = add_norm(delta, hidden, self.final_norm, plan[gi])
        return normed

    def _final_hidden_tc(self, input_ids, positions, slots, kv_len) -> torch.Tensor:
        """Up to 64 streams: tensor-core input and gate/up projections with the residual
        add + RMSNorm (and the SiLU·mul) fused in; output projections on the
        tensor-core GEMM with K split over a cluster (or cuBLAS).  The residual
        stream alternates between the two static buffers."""
        b, hq, hk, d = self.batch, self.hq, self.hk, self.d
        hidden = F.embedding(input_ids, self.embed)              # [B, 1, H] residual stream
        delta, ri = None, 0
        common = dict(eps=self.eps, err_flag=self.err_flag)
        if self.tc_output_projections:
            def proj(a, w):
                return gemm_tc(a, w, err_flag=self.err_flag)
        else:
            proj = F.linear
        fused_norm = b <= self.tc_norm_prologue_max_batch

        def normed_input(delta, hidden, w, ri):
            """(GEMM input, norm keyword arguments, residual stream after the step, ri)."""
            if fused_norm:
                if delta is None:
                    return hidden, dict(norm_weight=w), hidden, ri
                return delta, dict(norm_weight=w, residual=hidden, residual_out=self.res_buf[ri]), \
                    self.res_buf[ri], ri ^ 1
            if delta is None:
                return fused_rms_norm(hidden, w, self.eps), {}, hidden, ri
            normed, new_hidden = fused_add_rms_norm(delta, hidden, w, self.eps, residual_out=self.res_buf[ri])
            return normed, {}, new_hidden, ri ^ 1

        for i, L in enumerate(self.layers):
            x_in, norm_kw, hidden_next, ri = normed_input(delta, hidden, L["op_norm"], ri)
            if L["attn"]:
                qkv = gemm_tc(x_in, L["qkv"], **norm_kw, **common)
                hidden = hidden_next
                q, k, v = qkv.split([self.q_dim, self.kv_dim, self.kv_dim], dim=-1)
                q_rot = fused_rope_kv_write(
                    q.view(b, 1, hq, d), k.view(b, 1, hk, d), v.view(b, 1, hk, d), L["inv_freq"], positions,
                    self.k_cache[i], self.v_cache[i], slots, frame_table=self.frame_table,
                    tokens_per_frame=self.cfg.tokens_per_frame, q_norm_w=L["q_norm"], k_norm_w=L["k_norm"],
                    eps=self.eps, err_flag=self.err_flag)
                attn = decode_attention(q_rot, self.k_cache[i], self.v_cache[i], kv_len, self.scale,
                                        err_flag=self.err_flag, prefix_final=self.dependent_attention)
                delta = proj(attn.view(b, 1, self.q_dim), L["o"])
            else:
                bcx = gemm_tc(x_in, L["in_proj"], **norm_kw, **common)
                hidden = hidden_next
                delta = proj(short_conv_step(bcx, self.conv_state[i], L["conv_w"]), L["out_proj"])
            x_in, norm_kw, hidden_next, ri = normed_input(delta, hidden, L["ffn_norm"], ri)
            act = gemm_tc(x_in, L["gate_up"], silu_pairs=True, **norm_kw, **common)
            hidden = hidden_next
            delta = proj(act, L["down"])
        normed, _ = fused_add_rms_norm(delta, hidden, self.final_norm, self.eps)
        return normed

    def _conv_step(self, i, L, normed):
        """Gated short-conv decode step: in_proj, one fused kernel, out_proj."""
        y = short_conv_step(F.linear(normed, L["in_proj"]), self.conv_state[i], L["conv_w"])
        return F.linear(y, L["out_proj"])

    def _conv_step_eager(self, i, L, normed):
        """The reference's eager composition of the same step (optimized_decode.py:256-277)."""
        bcx = F.linear(normed, L["in_proj"]).transpose(-1, -2)   # [B, 3H, 1]
        bg, c, xc = bcx.chunk(3, dim=-2)
        bx = bg * xc
        state = self.conv_state[i].roll(shifts=-1, dims=-1)
        state[:, :, -1:] = bx                                     # cache_position >= L-1 in decode
        self.conv_state[i].copy_(state)
        conv_out = torch.sum(state * L["conv_w"], dim=-1).unsqueeze(-1)
        y = (c * conv_out).transpose(-1, -2)
        return F.linear(y, L["out_proj"])

    # ----------------------------------------------------------- prefill
    def prefill(self, input_ids: torch.Tensor, positions: torch.Tensor,
                speaker_emb: torch.Tensor | None = None) -> torch.Tensor:
        """Prompt pass for all streams (equal lengths).  input_ids [B, T];
        positions [B, T'] (T' = T + 1 with a speaker embedding, inserted at
        position 1 as inference_engine.py:475-491 does).  Fills KV slots
        0..T'-1 and the conv states; returns reduced-head logits of the last
        token [B, 1, num_reduced]."""
        b = self.batch
        x = F.embedding(input_ids, self.embed)
        if speaker_emb is not None:
            spk = F.linear(speaker_emb.to(self.dtype), self.speaker_proj).unsqueeze(1)
            x = torch.cat([x[:, :1], spk, x[:, 1:]], dim=1)
        t = x.shape[1]
        hq, hk, d = self.hq, self.hk, self.d
        slots = torch.arange(t, device=self.device, dtype=torch.long).repeat(b)
        pos = positions.reshape(-1).to(torch.long)
        hidden, delta = x, None
        for i, L in enumerate(self.layers):
            if delta is None:
                normed = fused_rms_norm(hidden, L["op_norm"], self.eps)
            else:
                normed, hidden = fused_add_rms_norm(delta, hidden, L["op_norm"], self.eps)
            if L["attn"]:
                qkv = F.linear(normed, L["qkv"])
                q, k, v = qkv.split([self.q_dim, self.kv_dim, self.kv_dim], dim=-1)
                q_rot = fused_rope_kv_write(
                    q.view(b, t, hq, d), k.view(b, t, hk, d), v.view(b, t, hk, d), L["inv_freq"], pos,
                    self.k_cache[i], self.v_cache[i], slots, frame_table=self.frame_table,
                    tokens_per_frame=self.cfg.tokens_per_frame, q_norm_w=L["q_norm"], k_norm_w=L["k_norm"],
                    eps=self.eps, err_flag=self.err_flag)
                rep = hq // hk                                    # prefill: expand K/V heads for GQA
                attn = F.scaled_dot_product_attention(
                    q_rot.transpose(1, 2), self.k_cache[i][:, :, :t].repeat_interleave(rep, dim=1),
                    self.v_cache[i][:, :, :t].repeat_interleave(rep, dim=1),
                    is_causal=True, scale=self.scale)                  # [B, Hq, T, D]
                delta = F.linear(attn.transpose(1, 2).reshape(b, t, self.q_dim), L["o"])
            else:
                bcx = F.linear(normed, L["in_proj"]).transpose(-1, -2)   # [B, 3H, T]
                bg, c, xc = bcx.chunk(3, dim=-2)
                bx = bg * xc
                lc = self.cfg.conv_L_cache
                self.conv_state[i].copy_(F.pad(bx, (lc - t, 0)) if t < lc else bx[..., t - lc:])
                conv_out = F.conv1d(bx, L["conv_w"].unsqueeze(1), padding=lc - 1, groups=bx.shape[1])[..., :t]
                delta = F.linear((c * conv_out).transpose(-1, -2), L["out_proj"])
            normed, hidden = fused_add_rms_norm(delta, hidden, L["ffn_norm"], self.eps)
            delta = F.linear(fused_silu_mul(F.linear(normed, L["gate_up"])), L["down"])
        normed, _ = fused_add_rms_norm(delta[:, -1:], hidden[:, -1:], self.final_norm, self.eps)
        return self._linear_head(normed)


class DecodeEngine:
    """Prefill + CUDA-graph decode (greedy, or sampled with ``sampling``) for
    `batch` independent streams."""

    def __init__(self, decoder: FusedDecoder, keep_mask: bool = False, sampling: SamplingParams | None = None):
        self.dec = decoder
        self.keep_mask = keep_mask   # maintain the additive mask (for steps that use one)
        self.sampling = sampling
        dev, b, s = decoder.device, decoder.batch, decoder.max_len
        self.rng_step = torch.zeros(1, dtype=torch.long, device=dev)
        self.next_tok = torch.zeros(b, dtype=torch.long, device=dev)
        self.seen = None
        self.input_ids = torch.zeros(b, 1, dtype=torch.long, device=dev)
        self.positions = torch.zeros(b, dtype=torch.long, device=dev)
        self.slots = torch.zeros(b, dtype=torch.long, device=dev)
        self.kv_len = torch.zeros(b, dtype=torch.long, device=dev)
        self.mask = torch.full((b, 1, 1, s), float("-inf"), dtype=torch.bfloat16, device=dev)
        self.step_idx = torch.zeros(1, dtype=torch.long, device=dev)
        self.base_pos = torch.zeros(b, dtype=torch.long, device=dev)
        self.base_slot = torch.zeros(b, dtype=torch.long, device=dev)
        self.generated = None
        self.graph = None
        self.logits = None

    def start(self, input_ids: torch.Tensor, speaker_emb: torch.Tensor | None, max_new_tokens: int) -> None:
        """Prefill all streams and arm the decode loop."""
        dec, cfg = self.dec, self.dec.cfg
        b, t = input_ids.shape
        t_eff = t + (1 if speaker_emb is not None else 0)
        if t_eff + max_new_tokens > dec.max_len:
            raise ValueError(f"cache of {dec.max_len} slots cannot hold {t_eff} + {max_new_tokens} tokens")
        if speaker_emb is not None:   # speaker-conditioned prompts are sequential (inference_engine.py:497-499)
            pos = torch.arange(t_eff, device=dec.device).repeat(b, 1)
        else:
            from .positions import frame_level_positions
            pos = frame_level_positions(input_ids, cfg.audio_tokens_start, cfg.tokens_per_frame,
                                        cfg.audio_step).long()
        logits = dec.prefill(input_ids, pos, speaker_emb)
        self.rng_step.zero_()
        if self.sampling is not None:
            # the prompt is the initial repetition history (inference_engine.py:553-556)
            self.seen = seen_bitmap(input_ids, dec.head.shape[0], dec.full_to_reduced, device=dec.device)
        first = self._next_token(logits[:, -1])
        self.rng_step.add_(1)
        self.input_ids.copy_(first.view(b, 1))
        self.mask.fill_(float("-inf"))
        self.mask[..., :t_eff] = 0.0
        self.base_pos.fill_(t_eff)        # decode step k: t_eff + (k // tpf) * audio_step
        self.base_slot.fill_(t_eff)       # decode step k writes slot t_eff + k
        self.step_idx.zero_()
        self.positions.copy_(self.base_pos)      # step 0; decode_advance computes the later ones
        self.slots.copy_(self.base_slot)
        self.kv_len.copy_(self.base_slot + 1)
        self.generated = torch.zeros(b, max_new_tokens, dtype=torch.long, device=dec.device)

    def _step_body(self):
        cfg = self.dec.cfg
        if self.keep_mask:
            self.mask.scatter_(3, self.slots.view(-1, 1, 1, 1), 0.0)
        if self.sampling is None and self.dec.fused_greedy_head and self.dec.fused_head is not None:
            self.logits = None
            nxt = self.dec.step_greedy(self.input_ids, self.positions, self.slots, self.kv_len, out=self.next_tok)
        elif self.dec.fused_greedy_head and self.dec.fused_head is not None:
            self.logits = self.dec.step_logits(self.input_ids, self.positions, self.slots, self.kv_len)
            nxt = self._next_token(self.logits[:, 0])
        else:
            self.logits = self.dec.step(self.input_ids, self.positions, self.slots, self.kv_len, self.mask)
            nxt = self._next_token(self.logits[:, 0])
        # record and feed back the token, next step's position / slot / length, counters
        decode_advance(nxt.view(-1), self.input_ids, self.generated, self.step_idx, self.base_pos, self.base_slot,
                       self.positions, self.slots, self.kv_len, cfg.tokens_per_frame, cfg.audio_step,
                       rng_step=self.rng_step if self.sampling is not None else None)

    def _next_token(self, logits: torch.Tensor) -> torch.Tensor:
        """[B] full token ids from reduced logits [B, V_red]: greedy, or one
        sampler launch that also extends the repetition bitmap and the step counter."""
        if self.sampling is None:
            return self.dec.reduced_to_full[logits.argmax(-1)]
        sp = self.sampling
        sample_tokens(logits, self.seen, temperature=sp.temperature, top_p=sp.top_p,
                      repetition_penalty=sp.repetition_penalty, top_k=sp.top_k,
                      index_map=self.dec.reduced_to_full, seed=sp.seed, step=self.rng_step, out=self.next_tok)
        return self.next_tok

    def capture(self) -> None:
        """Warm up once outside capture, then capture one decode step."""
        dec = self.dec
        saved = ({i: c.clone() for i, c in dec.conv_state.items()}, self.input_ids.clone(), self.mask.clone(),
                 self.step_idx.clone(), self.rng_step.clone(),
                 self.seen.clone() if self.seen is not None else None,
                 self.positions.clone(), self.slots.clone(), self.kv_len.clone())
        s = torch.cuda.Stream(device=dec.device)
        s.wait_stream(torch.cuda.current_stream(dec.device))
        with torch.cuda.stream(s):
            self._step_body()
        torch.cuda.current_stream(dec.device).wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._step_body()
        # undo the warm-up and capture steps (they ran the step twice)
        for i, c in saved[0].items():
            dec.conv_state[i].copy_(c)
        self.input_ids.copy_(saved[1])
        self.mask.copy_(saved[2])
        self.step_idx.copy_(saved[3])
        self.rng_step.copy_(saved[4])
        if saved[5] is not None:
            self.seen.copy_(saved[5])
        self.positions.copy_(saved[6])
        self.slots.copy_(saved[7])
        self.kv_len.copy_(saved[8])

    def run(self, n_steps: int) -> None:
        for _ in range(n_steps):
            self.graph.replay()
