"""CPU oracle for the KaniTTS decode-path kernels — TEST INFRASTRUCTURE ONLY.

This module restates, on the CPU with PyTorch eager ops, the reference
algorithms that the CUDA kernels replace.  It is the checker: only the tests,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may
import it, and never as the thing measured for the GPU or as a fallback.

Two families of functions:

* ``*_ref`` — the reference hot-path algorithm exactly as the reference GPU
  path computes it (fp32 arithmetic, one rounding to the storage type per
  output, the same operation order; each cites the reference file:line).
  The kernels are expected to be bit-identical to these except where a
  reduction order or a transcendental differs (sum of squares, exp, sin/cos),
  which can move a result by one unit in the last place of bf16.
* ``eager_*`` — the eager PyTorch/HF compositions the reference runs outside
  its Triton path (HF ``Lfm2RMSNorm``, ``F.silu(g) * u``,
  ``apply_rotary_pos_emb`` in bf16), the "PyTorch eager" side of the
  tolerance checks.

Rounding: on a GPU, Triton's ``x.to(tl.bfloat16)`` rounds to nearest even;
the Triton CPU interpreter (triton 3.6, ``runtime/interpreter.py``
``cast_impl`` -> ``_convert_float`` with no rounding mode) truncates instead.
The ``rounding`` argument selects ``"rne"`` (default: the hardware
reference, eager PyTorch and the CUDA kernels) or ``"trunc"`` (to reproduce
the interpreter's golden vectors bit for bit, which pins the fp32 arithmetic).

Pinning: ``tests/golden/make_golden.py`` runs the reference's own Triton
kernels (under the Triton CPU interpreter), its ``StaticLfm2HybridConvCache``,
``LearnableRotaryEmbedding`` and ``compute_frame_level_positions`` on seeded
inputs and stores the outputs in ``tests/golden/*.npz``;
``tests/test_oracle_golden.py`` checks every function here against them.
The BemaTTS frame-table term and the residual-add fusion have no reference
implementation; they are defined here (table term: ``+ table[pos //
tokens_per_frame]`` in fp32 before the final rounding) and their parity is
pinned only through their components.
"""
from __future__ import annotations

import numpy as np
import torch

# --------------------------------------------------------------- elementary


def _f32(t: torch.Tensor) -> torch.Tensor:
    return t.detach().to("cpu", torch.float32)


def _store(v: torch.Tensor, dtype: torch.dtype, rounding: str = "rne") -> torch.Tensor:
    """Round fp32 values to the storage dtype: nearest-even, or truncation
    toward zero for bf16 (the Triton interpreter's cast)."""
    if rounding == "trunc" and dtype == torch.bfloat16:
        bits = v.contiguous().view(torch.int32) & ~0xFFFF
        return bits.view(torch.float32).to(torch.bfloat16)
    if rounding not in ("rne", "trunc"):
        raise ValueError(rounding)
    return v.to(dtype)


def rms_norm_ref(x: torch.Tensor, w: torch.Tensor, eps: float, rounding: str = "rne") -> torch.Tensor:
    """Triton RMSNorm (kani_tts/triton_kernels.py:28-35): fp32 math, one rounding.

    var = sum(x*x)/N; rrms = 1/sqrt(var+eps); y = (x*rrms)*w.  The output keeps
    x's dtype; for fp32 x this is a true fp32 result (the reference kernel
    stores bf16-rounded values, see ``rms_norm_ref_storage``).
    """
    xf = _f32(x)
    n = xf.shape[-1]
    var = (xf * xf).sum(-1, keepdim=True) / n
    rr = 1.0 / torch.sqrt(var + eps)
    return _store((xf * rr) * _f32(w), x.dtype, rounding)


def rms_norm_ref_storage(x: torch.Tensor, w: torch.Tensor, eps: float,
                         rounding: str = "rne") -> torch.Tensor:
    """What the reference Triton kernel stores: bf16-rounded values in x's dtype
    (``tl.store(..., y.to(tl.bfloat16))`` into ``empty_like(x)``,
    triton_kernels.py:35, :53)."""
    xf = _f32(x)
    n = xf.shape[-1]
    var = (xf * xf).sum(-1, keepdim=True) / n
    rr = 1.0 / torch.sqrt(var + eps)
    return _store((xf * rr) * _f32(w), torch.bfloat16, rounding).to(x.dtype)


def add_rms_norm_ref(x: torch.Tensor, r: torch.Tensor, w: torch.Tensor, eps: float,
                     rounding: str = "rne"):
    """Eager residual add (optimized_decode.py:252/277/283: ``hidden + delta`` in
    the activation dtype, always nearest-even) followed by the Triton RMSNorm.
    Returns (y, h)."""
    h = (_f32(x) + _f32(r)).to(x.dtype)
    return rms_norm_ref(h, w, eps, rounding), h


def reduce_add_rms_norm_ref(partials: torch.Tensor, r: torch.Tensor, w: torch.Tensor, eps: float):
    """A projection given as fp32 partial products over slices of K, finished by
    the residual add and RMSNorm of the decode step: the partials summed in split
    order and rounded as F.linear rounds its output, then ``add_rms_norm_ref``
    (optimized_decode.py:252 + :280).  Returns (y, h)."""
    acc = partials[0].float()
    for s in range(1, partials.shape[0]):
        acc = acc + partials[s].float()
    return add_rms_norm_ref(acc.to(r.dtype).reshape(r.shape), r, w, eps)


def silu_mul_ref(gate_up: torch.Tensor, rounding: str = "rne") -> torch.Tensor:
    """Triton SiLU x mul (triton_kernels.py:77-82): (g * sigmoid(g)) * u in fp32."""
    n = gate_up.shape[-1] // 2
    g = _f32(gate_up[..., :n])
    u = _f32(gate_up[..., n:2 * n])
    return _store((g * torch.sigmoid(g)) * u, gate_up.dtype, rounding)


def _rope_f32(xf: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate-half in fp32 (triton_kernels.py:121-130): x*cos + sign*x_paired*sin,
    each product and the sum rounded separately.  cos/sin broadcast on the
    last dim."""
    half = xf.shape[-1] // 2
    paired = torch.cat([xf[..., half:], xf[..., :half]], dim=-1)
    sign = torch.cat([-torch.ones(half), torch.ones(half)])
    return xf * cos + (sign * paired) * sin


def rope_ref(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, rounding: str = "rne") -> torch.Tensor:
    """Triton RoPE of heads x [..., D] with one cos/sin row [D]
    (triton_kernels.py:112-131, launched per Q and K at :160-163)."""
    d = x.shape[-1]
    return _store(_rope_f32(_f32(x), _f32(cos).reshape(d), _f32(sin).reshape(d)), x.dtype, rounding)


def rope_compose_ref(xn: torch.Tensor, cos_rows: torch.Tensor, sin_rows: torch.Tensor,
                     table_rows: torch.Tensor | None = None) -> torch.Tensor:
    """The rotation half of ``rope_kv_write_ref`` on given inputs: heads xn
    [N, H, D] (already normed and rounded), one cos and one sin row [N, D] per
    token (already rounded), optional frame rows [N, D]; rotate-half in fp32
    (triton_kernels.py:121-130), the frame row added in fp32, one rounding to
    xn's dtype.  Used to check a kernel's rotation given its own cos/sin and
    norm outputs."""
    out = _rope_f32(_f32(xn), _f32(cos_rows).unsqueeze(1), _f32(sin_rows).unsqueeze(1))
    if table_rows is not None:
        out = out + _f32(table_rows).unsqueeze(1)
    return out.to(xn.dtype)


def rope_cos_sin_ref(inv_freq: torch.Tensor, pos, dtype=torch.bfloat16):
    """cos/sin rows of one decode step (optimized_decode.py:229-234):
    freqs = inv_freq * float(pos) (fp32); emb = cat(freqs, freqs); cos/sin
    rounded to the activation dtype.  ``pos`` may be a scalar or a [N] tensor
    (one row per token)."""
    inv = _f32(inv_freq)
    p = torch.as_tensor(pos).to(torch.int64).to(torch.float32)
    freqs = inv * p.reshape(-1, 1) if p.dim() else inv * p
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def learnable_inv_freq_ref(head_dim: int, rope_theta: float, alpha_weight: float = 0.0,
                           alpha_min: float = 0.1, alpha_max: float = 2.0) -> torch.Tensor:
    """Per-layer frequencies (kani_tts/model.py:180-196, optimized_decode.py:108):
    inv_freq_base = 1/(theta ** (arange(0, D, 2) -> bf16 / D)) in bf16,
    alpha = alpha_min + (alpha_max - alpha_min) * sigmoid(w) in bf16,
    result (inv_freq_base * alpha).float()."""
    exps = torch.arange(0, head_dim, 2, dtype=torch.int64).to(torch.bfloat16) / head_dim
    base = 1.0 / (rope_theta ** exps)
    alpha = alpha_min + (alpha_max - alpha_min) * torch.sigmoid(torch.tensor(alpha_weight, dtype=torch.bfloat16))
    return (base * alpha).float()


def kv_write_ref(k_cache: torch.Tensor, v_cache: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                 slot) -> None:
    """In-place static-cache write (static_cache.py:131-140): cache[b, h, slot, :] =
    states[b, h, 0, :].  ``slot`` is one int (shared by the batch) or one per
    stream; out-of-range slots are skipped (the kernel flags them)."""
    b = k_cache.shape[0]
    slots = [int(slot)] * b if np.ndim(slot) == 0 or np.size(slot) == 1 else [int(s) for s in slot]
    for i in range(b):
        s = slots[i] if len(slots) > 1 else slots[0]
        if 0 <= s < k_cache.shape[2]:
            k_cache[i, :, s, :] = k[i, :, 0, :]
            v_cache[i, :, s, :] = v[i, :, 0, :]


def rope_kv_write_ref(q, k, v, inv_freq, positions, k_cache, v_cache, slots, frame_table=None,
                      tokens_per_frame: int = 4, q_norm_w=None, k_norm_w=None, eps: float = 1e-5,
                      frame_pos=None):
    """Fused decode attention-input step for N tokens (optimized_decode.py:220-240).

    q: [N, Hq, D], k / v: [N, Hk, D] (N = B * T tokens, token t belongs to
    stream t // T of the [B, Hk, S, D] caches); positions / slots /
    frame_pos: [N] int64.  Per token: optional q/k RMSNorm rounded to the
    dtype; cos/sin from inv_freq * pos rounded to the dtype; rotate-half in
    fp32; optional ``+ frame_table[frame_pos // tokens_per_frame]`` in fp32;
    one rounding.  K_rot and raw V are written to the caches in place.
    Returns (q_rot [N, Hq, D], flags) with flags the KANI_FLAG_* bits the
    kernel would raise (1 = slot out of range, 2 = frame row out of range).
    """
    dtype = q.dtype
    n_tok, _, d = q.shape
    bsz = k_cache.shape[0]
    t_per = n_tok // bsz
    pos = torch.as_tensor(positions).reshape(-1).to(torch.int64)
    cos, sin = rope_cos_sin_ref(inv_freq, pos, dtype)          # [N, D]
    cos = _f32(cos).unsqueeze(1)
    sin = _f32(sin).unsqueeze(1)
    qx, kx = q, k
    if q_norm_w is not None:
        qx = rms_norm_ref(q, q_norm_w, eps)
        kx = rms_norm_ref(k, k_norm_w, eps)
    qr = _rope_f32(_f32(qx), cos, sin)
    kr = _rope_f32(_f32(kx), cos, sin)
    flags = 0
    if frame_table is not None:
        fp = pos if frame_pos is None else torch.as_tensor(frame_pos).reshape(-1).to(torch.int64)
        frame = torch.where(fp >= 0, torch.div(fp, tokens_per_frame, rounding_mode="floor"),
                            torch.full_like(fp, -1))
        ok = (frame >= 0) & (frame < frame_table.shape[0])
        if not bool(ok.all()):
            flags |= 2
        rows = _f32(frame_table)[frame.clamp(0, frame_table.shape[0] - 1)].unsqueeze(1)
        keep = ok.reshape(-1, 1, 1)
        # an out-of-range row contributes nothing (not even the sign of a zero)
        qr = torch.where(keep, qr + rows, qr)
        kr = torch.where(keep, kr + rows, kr)
    q_rot = qr.to(dtype)
    k_rot = kr.to(dtype)
    sl = torch.as_tensor(slots).reshape(-1).to(torch.int64)
    b_idx = torch.arange(n_tok) // t_per
    valid = (sl >= 0) & (sl < k_cache.shape[2])
    if not bool(valid.all()):
        flags |= 1
    k_cache[b_idx[valid], :, sl[valid], :] = k_rot[valid].to(k_cache.device)
    v_cache[b_idx[valid], :, sl[valid], :] = v[valid].to(v_cache.device)
    return q_rot, flags


def decode_attention_ref(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, kv_len,
                         scale: float) -> torch.Tensor:
    """Decode attention of the reference step (optimized_decode.py:243-248): SDPA of
    one query per stream over the static buffer with the -inf mask opened on the
    prefix [0, kv_len[b]) (inference_engine.py:259-265, :643), GQA by head groups.
    Computed in float64; returned in q's dtype.  q [B, Hq, D]; caches [B, Hk, S, D]."""
    b, hq, d = q.shape
    hk = k_cache.shape[1]
    g = hq // hk
    out = torch.zeros(b, hq, d, dtype=torch.float64)
    for s in range(b):
        n = int(kv_len[s])
        if n <= 0:
            continue
        k = k_cache[s, :, :n].double().repeat_interleave(g, dim=0)    # [Hq, n, D]
        v = v_cache[s, :, :n].double().repeat_interleave(g, dim=0)
        sc = torch.einsum("hd,hnd->hn", q[s].double(), k) * scale
        out[s] = torch.einsum("hn,hnd->hd", torch.softmax(sc, dim=-1), v)
    return out.to(q.dtype)


def short_conv_step_ref(bcx: torch.Tensor, state: torch.Tensor, conv_w: torch.Tensor) -> torch.Tensor:
    """Gated short-conv decode step, the eager ops of optimized_decode.py:258-276 on
    bcx [B, 3H] (in_proj output).  Updates `state` [B, H, L] in place; returns
    y [B, H] (every product rounded to the storage dtype, fp32 sum)."""
    h = state.shape[1]
    bg, c, x = bcx[:, :h], bcx[:, h:2 * h], bcx[:, 2 * h:3 * h]
    bx = bg * x                                         # :261
    st = state.roll(shifts=-1, dims=-1)                 # :265
    st[:, :, -1] = bx                                   # :267
    state.copy_(st)                                     # :268
    prod = (st * conv_w).float()                        # :270-271, products rounded
    conv = prod[..., 0]
    for i in range(1, prod.shape[-1]):
        conv = conv + prod[..., i]
    return c * conv.to(bcx.dtype)                       # :275


# ------------------------------------------------------ eager compositions


def eager_rms_norm_hf(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """HF ``Lfm2RMSNorm.forward`` (transformers/models/lfm2/modeling_lfm2.py):
    normalise in fp32, round to the input dtype, multiply by the weight."""
    xf = _f32(x)
    var = xf.pow(2).mean(-1, keepdim=True)
    normed = (xf * torch.rsqrt(var + eps)).to(x.dtype)
    return w.detach().cpu() * normed


def eager_silu_mul(gate_up: torch.Tensor) -> torch.Tensor:
    """``F.silu(w1(x)) * w3(x)`` of HF ``Lfm2MLP`` on a concatenated [g | u]."""
    n = gate_up.shape[-1] // 2
    g, u = gate_up[..., :n].cpu(), gate_up[..., n:2 * n].cpu()
    return torch.nn.functional.silu(g) * u


def eager_rope_hf(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """HF ``apply_rotary_pos_emb`` on one tensor: (x*cos) + (rotate_half(x)*sin)
    with every op in the activation dtype."""
    x = x.cpu()
    half = x.shape[-1] // 2
    rot = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
    return (x * cos.cpu()) + (rot * sin.cpu())


# ---------------------------------------------------------- positions (int)


def frame_level_positions_ref(input_ids: np.ndarray, audio_tokens_start: int,
                              tokens_per_frame: int = 4, audio_step: float = 1.0) -> np.ndarray:
    """BemaTTS prefill positions (kani_tts/model.py:114-138): text tokens count 1,
    audio frames count audio_step; a token's position counts what precedes it."""
    ids = np.asarray(input_ids)
    is_audio = ids >= audio_tokens_start
    text_before = np.cumsum(np.concatenate([np.zeros((ids.shape[0], 1), np.int64),
                                            (~is_audio).astype(np.int64)], axis=1), axis=1)[:, :-1]
    audio_before = np.cumsum(np.concatenate([np.zeros((ids.shape[0], 1), np.int64),
                                             is_audio.astype(np.int64)], axis=1), axis=1)[:, :-1]
    return text_before + (audio_before // tokens_per_frame) * audio_step


def decode_position_schedule_ref(prefill_seq_len: int, max_new_tokens: int,
                                 tokens_per_frame: int = 4, audio_step: float = 1.0) -> np.ndarray:
    """inference_engine.py:615-619: prefill_seq_len + ((i+1)//tpf)*audio_step, as int64."""
    i = np.arange(max_new_tokens, dtype=np.int64)
    return (prefill_seq_len + (i + 1) // tokens_per_frame * audio_step).astype(np.int64)


# ------------------------------------------------------------- comparisons


def ulp_distance(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Element-wise distance in units in the last place for bf16 / fp16 / fp32
    tensors of one dtype (ordered-integer difference of the bit patterns)."""
    assert a.dtype == b.dtype, (a.dtype, b.dtype)
    if a.dtype in (torch.bfloat16, torch.float16):
        ia = a.detach().cpu().view(torch.int16).to(torch.int64)
        ib = b.detach().cpu().view(torch.int16).to(torch.int64)
        mag = 0x7FFF
    else:
        ia = a.detach().cpu().view(torch.int32).to(torch.int64)
        ib = b.detach().cpu().view(torch.int32).to(torch.int64)
        mag = 0x7FFFFFFF
    oa = torch.where(ia < 0, -(ia & mag), ia)
    ob = torch.where(ib < 0, -(ib & mag), ib)
    return (oa - ob).abs()


def head_argmax_ref(hidden: torch.Tensor, weight: torch.Tensor, index_map: torch.Tensor | None = None
                    ) -> tuple[torch.Tensor, torch.Tensor]:
    """Reduced LM head + greedy choice (kani_tts/optimized_decode.py:287, the head
    built at :134-156, the reduced-to-full map of :144-148): logits rounded once to
    the storage type from a float64 dot product; token = map[first argmax].
    Returns (tokens [B], logits [B, rows])."""
    h = hidden.reshape(-1, hidden.shape[-1]).double()
    logits = (h @ weight.double().T).to(hidden.dtype)
    idx = torch.argmax(logits.float(), dim=-1)   # first index of the maximum
    tok = index_map[idx] if index_map is not None else idx
    return tok, logits


def codec_codes_ref(tokens: torch.Tensor, eos_token: int, audio_tokens_start: int, codebook_size: int = 4032
                    ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """NemoAudioPlayer.get_nano_codes (kani_tts/core.py:86-108) for each stream's
    generated tokens: the segment before the first end-of-speech token, cut to
    whole frames of 4, code = token - c * codebook_size - audio_tokens_start.
    The reference raises where this returns status bits: 1 = a negative code,
    2 = no complete frame, 4 = no end-of-speech token.
    Returns (codes [B, 4, T // 4] with -1 past the frames, frames [B], status [B])."""
    tokens = tokens.cpu().long()
    b_n, t = tokens.shape
    mf = t // 4
    codes = torch.full((b_n, 4, mf), -1, dtype=torch.long)
    frames = torch.zeros(b_n, dtype=torch.long)
    status = torch.zeros(b_n, dtype=torch.int32)
    for b in range(b_n):
        hit = (tokens[b] == eos_token).nonzero(as_tuple=True)[0]
        end = int(hit[0]) if hit.numel() else t
        seg = tokens[b, :end]
        seg = seg[: len(seg) - len(seg) % 4]
        nf = len(seg) // 4
        st = 0 if hit.numel() else 4
        if nf == 0:
            st |= 2
        else:
            c = seg.reshape(-1, 4) - torch.tensor([codebook_size * i for i in range(4)]) - audio_tokens_start
            if bool((c < 0).any()):
                st |= 1
            codes[b, :, :nf] = c.T
        frames[b] = nf
        status[b] = st
    return codes, frames, status


def gemv_ref(x: torch.Tensor, weight: torch.Tensor, norm_weight: torch.Tensor | None = None,
             residual: torch.Tensor | None = None, eps: float = 1e-5, silu_pairs: bool = False):
    """The decode step's F.linear with its neighbours (optimized_decode.py:175-289):
    optional residual add + RMSNorm before it (``add_rms_norm_ref`` /
    ``rms_norm_ref``), the product as a float64 dot rounded once (F.linear's
    output), optional SiLU·mul of the gate / up halves after it
    (``silu_mul_ref``).  Returns (y, h) with h the residual-stream sum (or None)."""
    h = None
    a = x
    if norm_weight is not None:
        if residual is not None:
            a, h = add_rms_norm_ref(x, residual, norm_weight, eps)
        else:
            a = rms_norm_ref(x, norm_weight, eps)
    y = (a.double() @ weight.double().T).to(x.dtype)
    if silu_pairs:
        y = silu_mul_ref(y)
    return y, h
