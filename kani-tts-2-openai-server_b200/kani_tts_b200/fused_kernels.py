"""Drop-in replacements for ``kani_tts/triton_kernels.py`` plus the fused entry points.

Same names, argument meaning and return values as the reference module
(``fused_rms_norm``, ``fused_silu_mul``, ``fused_rope``), so
``kani_tts/optimized_decode.py:14`` can bind them unchanged, plus:

* ``fused_add_rms_norm`` — the residual add of optimized_decode.py:252/277/283
  folded into the following RMSNorm;
* ``kv_cache_write`` — the scatter_ of static_cache.py:131-140;
* ``fused_rope_kv_write`` — q/k norm + cos/sin + RoPE (+ BemaTTS frame term)
  + KV write of optimized_decode.py:220-240 in one launch.

Each call validates its tensors on the host (device, dtype, shape) before a
single launch through the C ABI on the current CUDA stream; nothing
synchronises, so every op is capturable in a CUDA graph.  Differences from
the reference, all deliberate:

* an fp32 input to ``fused_rms_norm`` gives a true fp32 result (the Triton
  kernel stores bf16-rounded values into an fp32 tensor,
  triton_kernels.py:35/53);
* ``fused_rope`` is one launch for Q and K (the reference launches twice,
  triton_kernels.py:160-163);
* invalid input raises ``TypeError`` / ``ValueError`` before any launch (the
  reference wrappers do not validate).
"""
from __future__ import annotations

import math

import torch

from . import _lib
from ._lib import check, dtype_code, error_flag, load_library, ptr, require_cuda, stream_ptr

__all__ = [
    "fused_rms_norm",
    "fused_add_rms_norm",
    "linear_split_k",
    "reduce_add_rms_norm",
    "fused_silu_mul",
    "fused_rope",
    "kv_cache_write",
    "fused_rope_kv_write",
    "decode_attention",
    "short_conv_step",
    "sample_tokens",
    "head_argmax",
    "head_argmax_tc",
    "gemm_tc",
    "codec_codes",
    "gemv",
    "gemv_short_conv",
    "decode_advance",
    "gemv_rope_kv_write",
]


def _rows_view(t: torch.Tensor, n: int) -> tuple[torch.Tensor, int, int]:
    """View ``t`` as [rows, n] rows with a uniform row stride (copying if needed)."""
    if t.dim() == 0 or t.shape[-1] != n:
        raise ValueError(f"expected last dimension {n}, got shape {tuple(t.shape)}")
    if t.stride(-1) != 1:
        t = t.contiguous()
    rows = t.numel() // n if n else 0
    if rows <= 1:
        return t, rows, n
    # leading dims must collapse to one stride
    lead = [(s, st) for s, st in zip(t.shape[:-1], t.stride()[:-1]) if s != 1]
    stride = lead[-1][1] if lead else n
    if stride < n:  # overlapping rows (e.g. an expanded view)
        t = t.contiguous()
        return t, rows, n
    expect = stride
    for s, st in reversed(lead):
        if st != expect:
            t = t.contiguous()
            return t, rows, n
        expect = st * s
    return t, rows, stride


def fused_rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """RMSNorm over the last dim (reference ``fused_rms_norm``, triton_kernels.py:38-60).

    Args:
        x: [..., N] bf16 / fp16 / fp32 CUDA tensor.
        weight: [N] norm weight (bf16 / fp16 / fp32).
        eps: epsilon added to mean(x^2).
    Returns:
        [..., N] tensor of x's dtype.
    """
    require_cuda(x, "x")
    require_cuda(weight, "weight")
    lib = load_library()
    n = x.shape[-1] if x.dim() else 0
    if weight.dim() != 1 or weight.shape[0] != n:
        raise ValueError(f"weight must have shape [{n}], got {tuple(weight.shape)}")
    if weight.device != x.device:
        raise ValueError("x and weight must be on the same device")
    code, wcode = dtype_code(x, "x"), dtype_code(weight, "weight")
    weight = weight.contiguous()
    xv, rows, xs = _rows_view(x, n)
    y = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    check(lib.kani_rms_norm(code, wcode, ptr(xv), xs, ptr(weight), ptr(y), n, rows, n, float(eps),
                            stream_ptr(x.device)), "kani_rms_norm")
    return y


def fused_add_rms_norm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                       eps: float = 1e-6, out: torch.Tensor | None = None,
                       residual_out: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """``h = x + residual`` (rounded to the dtype, like the eager add) then RMSNorm of h.

    Replaces ``hidden = hidden + F.linear(...)`` (optimized_decode.py:252, 277, 283)
    plus the next ``fused_rms_norm``.  Returns ``(normed, h)``.  ``out`` /
    ``residual_out`` may be given for in-place use (``residual_out=residual``
    updates the residual stream in place); they must be contiguous.
    """
    for t, w in ((x, "x"), (residual, "residual"), (weight, "weight")):
        require_cuda(t, w)
    lib = load_library()
    if x.shape != residual.shape:
        raise ValueError(f"x {tuple(x.shape)} and residual {tuple(residual.shape)} differ in shape")
    if x.dtype != residual.dtype:
        raise TypeError(f"x ({x.dtype}) and residual ({residual.dtype}) differ in dtype")
    n = x.shape[-1] if x.dim() else 0
    if weight.dim() != 1 or weight.shape[0] != n:
        raise ValueError(f"weight must have shape [{n}], got {tuple(weight.shape)}")
    if not (x.device == residual.device == weight.device):
        raise ValueError("x, residual and weight must be on the same device")
    code, wcode = dtype_code(x, "x"), dtype_code(weight, "weight")
    weight = weight.contiguous()
    xv, rows, xs = _rows_view(x, n)
    rv, _, rs = _rows_view(residual, n)
    for t, w in ((out, "out"), (residual_out, "residual_out")):
        if t is not None:
            require_cuda(t, w)
            if t.shape != x.shape or t.dtype != x.dtype or not t.is_contiguous() or t.device != x.device:
                raise ValueError(f"{w} must be a contiguous tensor like x")
    y = out if out is not None else torch.empty(x.shape, dtype=x.dtype, device=x.device)
    h = residual_out if residual_out is not None else torch.empty(x.shape, dtype=x.dtype, device=x.device)
    if y.data_ptr() == h.data_ptr() and y.numel() > 0:
        raise ValueError("out and residual_out must be different tensors")
    check(lib.kani_add_rms_norm(code, wcode, ptr(xv), xs, ptr(rv), rs, ptr(weight), ptr(y), n, ptr(h), n,
                                rows, n, float(eps), stream_ptr(x.device)), "kani_add_rms_norm")
    return y, h


def linear_split_k(x: torch.Tensor, weight: torch.Tensor, splits: int) -> torch.Tensor:
    """``F.linear(x, weight)`` as `splits` fp32 partial products over equal slices of
    K, one cuBLAS batched GEMM with an fp32 output: returns [splits, rows, N] fp32
    with ``partials.sum(0)`` the product.  For 64 decode streams this is faster
    than the plain bf16 GEMM (down projection, K = 4608: 4.6 against 7.9 µs with 4
    splits), and ``reduce_add_rms_norm`` finishes it together with the residual
    add and RMSNorm that follow.  (A library GEMM: cuBLAS, as F.linear is.)"""
    k = x.shape[-1]
    if k % splits:
        raise ValueError(f"K = {k} does not split into {splits} equal slices")
    if weight.dim() != 2 or weight.shape[1] != k:
        raise ValueError(f"weight must be [N, {k}]")
    x2 = x.reshape(-1, k)
    if x2.stride(-1) != 1 or weight.stride(-1) != 1:
        raise ValueError("x and weight need a contiguous last dimension")
    ks = k // splits
    n = weight.shape[0]
    xk = x2.as_strided((splits, x2.shape[0], ks), (ks, x2.stride(0), 1))
    wk = weight.as_strided((splits, ks, n), (ks, 1, weight.stride(0)))
    return torch.bmm(xk, wk, out_dtype=torch.float32)


def reduce_add_rms_norm(partials: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6,
                        out: torch.Tensor | None = None, residual_out: torch.Tensor | None = None,
                        l2_prefetch=None) -> tuple[torch.Tensor, torch.Tensor]:
    """``fused_add_rms_norm(round(partials.sum(0)), residual, weight)`` in one launch
    (``kani_reduce_add_rms_norm``): the fp32 partials of ``linear_split_k`` are summed
    in split order and rounded as F.linear rounds its output, then the residual add
    (optimized_decode.py:252, 277, 283) and the next RMSNorm (:206, :280, :286).

    Args:
        partials: fp32 [S, rows, N] (the splits and rows may carry strides).
        residual: [..., N] with rows rows (bf16 / fp16 / fp32).
    Returns ``(normed, h)`` shaped like ``residual``; ``out`` / ``residual_out`` as
    in ``fused_add_rms_norm``; ``l2_prefetch`` as in ``gemv`` (the weights of the
    GEMMs after this launch).
    """
    for t, w in ((partials, "partials"), (residual, "residual"), (weight, "weight")):
        require_cuda(t, w)
    lib = load_library()
    if partials.dtype != torch.float32 or partials.dim() != 3 or partials.stride(-1) != 1:
        raise ValueError("partials must be fp32 [splits, rows, N] with a contiguous last dimension")
    s_, rows, n = partials.shape
    if residual.shape[-1] != n or residual.numel() != rows * n:
        raise ValueError(f"residual must hold {rows} rows of {n}")
    if weight.dim() != 1 or weight.shape[0] != n:
        raise ValueError(f"weight must have shape [{n}], got {tuple(weight.shape)}")
    if not (partials.device == residual.device == weight.device):
        raise ValueError("partials, residual and weight must be on the same device")
    code, wcode = dtype_code(residual, "residual"), dtype_code(weight, "weight")
    weight = weight.contiguous()
    rv, _, rs = _rows_view(residual, n)
    for t, w in ((out, "out"), (residual_out, "residual_out")):
        if t is not None:
            require_cuda(t, w)
            if t.shape != residual.shape or t.dtype != residual.dtype or not t.is_contiguous() or \
                    t.device != residual.device:
                raise ValueError(f"{w} must be a contiguous tensor like residual")
    y = out if out is not None else torch.empty(residual.shape, dtype=residual.dtype, device=residual.device)
    h = residual_out if residual_out is not None else torch.empty(residual.shape, dtype=residual.dtype,
                                                                  device=residual.device)
    if y.data_ptr() == h.data_ptr() and y.numel() > 0:
        raise ValueError("out and residual_out must be different tensors")
    if l2_prefetch:
        _lib.set_l2_prefetch(l2_prefetch)
    check(lib.kani_reduce_add_rms_norm(code, wcode, ptr(partials), partials.stride(0), partials.stride(1), s_,
                                       ptr(rv), rs, ptr(weight), ptr(y), n, ptr(h), n, rows, n, float(eps),
                                       stream_ptr(residual.device)), "kani_reduce_add_rms_norm")
    return y, h


def fused_silu_mul(gate_up: torch.Tensor, out: torch.Tensor | None = None, l2_prefetch=None) -> torch.Tensor:
    """SiLU(gate) * up from a concatenated [gate | up] tensor (triton_kernels.py:85-105).

    Args:
        gate_up: [..., 2 * intermediate_size].
        l2_prefetch: as in ``gemv`` (the weights of the GEMMs after this launch).
    Returns:
        [..., intermediate_size] of gate_up's dtype.
    """
    require_cuda(gate_up, "gate_up")
    lib = load_library()
    code = dtype_code(gate_up, "gate_up")
    if gate_up.dim() == 0 or gate_up.shape[-1] % 2 != 0:
        raise ValueError(f"gate_up last dimension must be even, got shape {tuple(gate_up.shape)}")
    two_n = gate_up.shape[-1]
    n = two_n // 2
    gv, rows, gs = _rows_view(gate_up, two_n)
    shape = (*gate_up.shape[:-1], n)
    if out is None:
        out = torch.empty(shape, dtype=gate_up.dtype, device=gate_up.device)
    else:
        require_cuda(out, "out")
        if tuple(out.shape) != shape or out.dtype != gate_up.dtype or not out.is_contiguous():
            raise ValueError(f"out must be a contiguous {gate_up.dtype} tensor of shape {shape}")
    if l2_prefetch:
        _lib.set_l2_prefetch(l2_prefetch)
    check(lib.kani_silu_mul(code, ptr(gv), gs, ptr(out), n, rows, n, stream_ptr(gate_up.device)),
          "kani_silu_mul")
    return out


def fused_rope(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
    """Rotate-half RoPE on Q and K with one cos/sin row (triton_kernels.py:134-165).

    Args:
        q: [1, num_q_heads, 1, head_dim]; k: [1, num_k_heads, 1, head_dim].
        cos, sin: head_dim elements (any shape), same dtype as q.
    Returns:
        (q_rotated, k_rotated), same shapes as q and k.
    """
    for t, w in ((q, "q"), (k, "k"), (cos, "cos"), (sin, "sin")):
        require_cuda(t, w)
    lib = load_library()
    code = dtype_code(q, "q")
    if not (k.dtype == cos.dtype == sin.dtype == q.dtype):
        raise TypeError("q, k, cos and sin must share one dtype")
    if q.dim() < 2 or k.dim() < 2:
        raise ValueError("q and k must be [1, heads, 1, head_dim]")
    num_q, num_k, hd = q.shape[1], k.shape[1], q.shape[-1]
    if k.shape[-1] != hd or q.numel() != num_q * hd or k.numel() != num_k * hd:
        raise ValueError(f"q {tuple(q.shape)} / k {tuple(k.shape)} are not [1, heads, 1, head_dim]")
    if cos.numel() != hd or sin.numel() != hd:
        raise ValueError(f"cos and sin must hold head_dim={hd} elements")
    if hd % 2:
        raise ValueError(f"head_dim must be even, got {hd}")
    qf, kf = q.contiguous(), k.contiguous()
    cf, sf = cos.contiguous(), sin.contiguous()
    q_out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    k_out = torch.empty(k.shape, dtype=k.dtype, device=k.device)
    check(lib.kani_rope_qk(code, ptr(qf), ptr(kf), ptr(cf), ptr(sf), ptr(q_out), ptr(k_out),
                           num_q, num_k, hd, stream_ptr(q.device)), "kani_rope_qk")
    return q_out, k_out


def kv_cache_write(key_states: torch.Tensor, value_states: torch.Tensor, k_cache: torch.Tensor,
                   v_cache: torch.Tensor, write_pos: torch.Tensor,
                   err_flag: torch.Tensor | None = None) -> None:
    """``cache[b, h, slot, :] = states[b, h, 0, :]`` for K and V (static_cache.py:131-140).

    ``write_pos`` is a device int64 tensor: one element (shared by the batch,
    as in the reference) or one per stream.  A slot outside the cache is
    skipped and flagged in ``err_flag`` (default: the per-device flag).
    """
    for t, w in ((key_states, "key_states"), (value_states, "value_states"), (k_cache, "k_cache"),
                 (v_cache, "v_cache"), (write_pos, "write_pos")):
        require_cuda(t, w)
    lib = load_library()
    code = dtype_code(k_cache, "k_cache")
    if k_cache.dim() != 4 or v_cache.shape != k_cache.shape:
        raise ValueError("k_cache / v_cache must both be [batch, kv_heads, max_len, head_dim]")
    b, hk, s, d = k_cache.shape
    exp = (b, hk, 1, d)
    if tuple(key_states.shape) != exp or tuple(value_states.shape) != exp:
        raise ValueError(f"key/value states must be {exp}, got {tuple(key_states.shape)} / "
                         f"{tuple(value_states.shape)}")
    if not (key_states.dtype == value_states.dtype == v_cache.dtype == k_cache.dtype):
        raise TypeError("states and caches must share one dtype")
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("k_cache and v_cache must be contiguous")
    if write_pos.dtype != torch.int64 or write_pos.numel() not in (1, b):
        raise ValueError(f"write_pos must be int64 with 1 or {b} elements")
    wp = write_pos.contiguous()
    ks, vs = key_states.contiguous(), value_states.contiguous()
    flag = err_flag if err_flag is not None else error_flag(k_cache.device)
    per_stream = 1 if (wp.numel() == b and b > 1) else 0
    check(lib.kani_kv_cache_write(code, ptr(ks), ptr(vs), b, hk, d, ptr(k_cache), ptr(v_cache), s,
                                  ptr(wp), per_stream, ptr(flag), stream_ptr(k_cache.device)),
          "kani_kv_cache_write")


def _token_view(t: torch.Tensor, heads: int, d: int, what: str) -> tuple[int, int]:
    """Check t is [*lead, heads, d] with heads at stride d; return (tokens, token stride)."""
    if t.dim() < 2 or t.shape[-1] != d or t.shape[-2] != heads:
        raise ValueError(f"{what} must end in [{heads}, {d}], got {tuple(t.shape)}")
    if t.stride(-1) != 1 or (heads > 1 and t.stride(-2) != d):
        raise ValueError(f"{what} must have contiguous heads (strides [..., {d}, 1]), got {t.stride()}")
    lead = [(s, st) for s, st in zip(t.shape[:-2], t.stride()[:-2]) if s != 1]
    tokens = math.prod(t.shape[:-2])
    if not lead:
        return tokens, heads * d
    stride = lead[-1][1]
    expect = stride
    for s, st in reversed(lead):
        if st != expect:
            raise ValueError(f"{what}: leading dims of shape {tuple(t.shape[:-2])} / strides "
                             f"{t.stride()[:-2]} do not collapse to one token stride")
        expect = st * s
    return tokens, stride


def fused_rope_kv_write(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, inv_freq: torch.Tensor,
                        position: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                        write_pos: torch.Tensor, frame_table: torch.Tensor | None = None,
                        tokens_per_frame: int = 4, q_norm_w: torch.Tensor | None = None,
                        k_norm_w: torch.Tensor | None = None, eps: float = 1e-5,
                        frame_pos: torch.Tensor | None = None, q_out: torch.Tensor | None = None,
                        err_flag: torch.Tensor | None = None) -> torch.Tensor:
    """Fused q/k-norm + RoPE (+ frame term) + static KV write for a batch of tokens.

    Replaces optimized_decode.py:220-240.  Shapes (B streams x T tokens):
        q: [B, T, Hq, D], k / v: [B, T, Hk, D]  (views into a packed QKV output are fine:
           heads must be contiguous, leading dims must collapse to one token stride)
        inv_freq: [D/2] fp32 (learnable-alpha frequencies of the layer)
        position: [B, T] int64 angle positions (BemaTTS frame-level position ids)
        k_cache / v_cache: [B, Hk, S, D] (last dim contiguous)
        write_pos: [B, T] int64 KV slots
        frame_table: optional [F, D]; row = frame_pos // tokens_per_frame
           (frame_pos defaults to position), added to rotated Q and K
        q_norm_w / k_norm_w: optional [D] per-head RMSNorm weights (both or neither)
        q_out: optional output, indexed like q ([B, T, Hq, D] view; may be the
           transpose of a [B, Hq, T, D] tensor when B == 1 or T == 1)
    Returns q_out (rotated Q).  K and V land in the caches.  Slots or frame
    rows out of range are skipped and flagged in ``err_flag``.
    """
    for t, w in ((q, "q"), (k, "k"), (v, "v"), (inv_freq, "inv_freq"), (position, "position"),
                 (k_cache, "k_cache"), (v_cache, "v_cache"), (write_pos, "write_pos")):
        require_cuda(t, w)
    lib = load_library()
    code = dtype_code(q, "q")
    if not (k.dtype == v.dtype == k_cache.dtype == v_cache.dtype == q.dtype):
        raise TypeError("q, k, v and the caches must share one dtype")
    if q.dim() < 3:
        raise ValueError("q must be [..., heads, head_dim] with a token dimension")
    hq, d = q.shape[-2], q.shape[-1]
    if k_cache.dim() != 4 or v_cache.shape != k_cache.shape or k_cache.shape[-1] != d:
        raise ValueError("k_cache / v_cache must both be [batch, kv_heads, max_len, head_dim]")
    bsz, hk, s_len, _ = k_cache.shape
    nq, qts = _token_view(q, hq, d, "q")
    nk, kts = _token_view(k, hk, d, "k")
    nv, vts = _token_view(v, hk, d, "v")
    if not (nq == nk == nv):
        raise ValueError(f"q, k and v hold different token counts ({nq}, {nk}, {nv})")
    if nq % bsz:
        raise ValueError(f"{nq} tokens do not split over a cache batch of {bsz}")
    seq_tokens = nq // bsz
    if inv_freq.dtype != torch.float32 or inv_freq.numel() != d // 2:
        raise ValueError(f"inv_freq must be fp32 with head_dim/2 = {d // 2} elements")
    for t, w in ((position, "position"), (write_pos, "write_pos")) + (
            ((frame_pos, "frame_pos"),) if frame_pos is not None else ()):
        if t.dtype != torch.int64 or t.numel() != nq:
            raise ValueError(f"{w} must be int64 with one element per token ({nq})")
    if (q_norm_w is None) != (k_norm_w is None):
        raise ValueError("q_norm_w and k_norm_w must be given together")
    if q_norm_w is not None:
        for t, w in ((q_norm_w, "q_norm_w"), (k_norm_w, "k_norm_w")):
            require_cuda(t, w)
            if t.dtype != q.dtype or t.numel() != d:
                raise ValueError(f"{w} must be a {q.dtype} tensor of head_dim={d} elements")
    frame_rows = 0
    if frame_table is not None:
        require_cuda(frame_table, "frame_table")
        if frame_table.dtype != q.dtype or frame_table.dim() != 2 or frame_table.shape[1] != d:
            raise ValueError(f"frame_table must be a {q.dtype} [rows, {d}] tensor")
        if tokens_per_frame <= 0:
            raise ValueError("tokens_per_frame must be positive")
        frame_table = frame_table.contiguous()
        frame_rows = frame_table.shape[0]
    if k_cache.stride(-1) != 1 or k_cache.stride() != v_cache.stride():
        raise ValueError("k_cache and v_cache need the same strides with a contiguous last dim")
    if q_out is None:
        q_out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
        qots, qohs = hq * d, d
    else:
        require_cuda(q_out, "q_out")
        if q_out.shape != q.shape or q_out.dtype != q.dtype or q_out.stride(-1) != 1:
            raise ValueError("q_out must be indexed like q with a contiguous last dim")
        lead = [(s, st) for s, st in zip(q_out.shape[:-2], q_out.stride()[:-2]) if s != 1]
        qots = lead[-1][1] if lead else hq * d
        expect = qots
        for s, st in reversed(lead):
            if st != expect:
                raise ValueError("q_out leading dims do not collapse to one token stride")
            expect = st * s
        qohs = q_out.stride(-2)
    dev = q.device
    flag = err_flag if err_flag is not None else error_flag(dev)
    cs = k_cache.stride()
    pos_c, wp_c = position.contiguous(), write_pos.contiguous()
    fp_c = frame_pos.contiguous() if frame_pos is not None else None
    inv_c = inv_freq.contiguous()
    qw = q_norm_w.contiguous() if q_norm_w is not None else None
    kw = k_norm_w.contiguous() if k_norm_w is not None else None
    check(lib.kani_rope_kv_write(
        code, bsz, seq_tokens, hq, hk, d,
        ptr(q), qts, ptr(k), kts, ptr(v), vts,
        ptr(inv_c), ptr(pos_c),
        ptr(qw), ptr(kw), float(eps),
        ptr(frame_table), frame_rows, ptr(fp_c), int(tokens_per_frame),
        ptr(q_out), qots, qohs,
        ptr(k_cache), ptr(v_cache), cs[0], cs[1], cs[2], s_len,
        ptr(wp_c), ptr(flag), stream_ptr(dev)), "kani_rope_kv_write")
    return q_out


def decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, kv_len: torch.Tensor,
                     scale: float | None = None, out: torch.Tensor | None = None,
                     err_flag: torch.Tensor | None = None, prefix_final: bool = False) -> torch.Tensor:
    """GQA decode attention of one query token per stream over cache slots [0, kv_len[b]).

    Replaces SDPA over the whole -inf-masked static buffer (optimized_decode.py:243-248).
        q: [B, Hq, D] or [B, 1, Hq, D] (heads at stride D); k_cache / v_cache: [B, Hk, S, D];
        kv_len: device int64 [B].  Returns out [B, Hq, D] (or writes ``out``).
        prefix_final: a decode step whose launch just before (its RoPE + KV write)
            writes at most q and the newest row, kv_len - 1, of each stream, while
            kv_len and the older rows are already final.  Then
            ``kani_decode_attention_step`` streams those rows before that launch
            completes (same results).
    """
    for t, w in ((q, "q"), (k_cache, "k_cache"), (v_cache, "v_cache"), (kv_len, "kv_len")):
        require_cuda(t, w)
    lib = load_library()
    code = dtype_code(q, "q")
    if k_cache.dim() != 4 or v_cache.shape != k_cache.shape or k_cache.stride() != v_cache.stride():
        raise ValueError("k_cache / v_cache must both be [batch, kv_heads, max_len, head_dim] with equal strides")
    b, hk, s_len, d = k_cache.shape
    qv = q.reshape(b, -1, d) if q.is_contiguous() else q
    if qv.dim() != 3 or qv.shape[0] != b or qv.shape[2] != d or qv.stride(-1) != 1:
        raise ValueError(f"q must be [{b}, heads, {d}] with a contiguous last dim")
    hq = qv.shape[1]
    if hq % hk:
        raise ValueError(f"{hq} query heads do not group over {hk} KV heads")
    if not (k_cache.dtype == v_cache.dtype == q.dtype):
        raise TypeError("q and the caches must share one dtype")
    if kv_len.dtype != torch.int64 or kv_len.numel() != b:
        raise ValueError(f"kv_len must be int64 with {b} elements")
    if out is None:
        out = torch.empty(b, hq, d, dtype=q.dtype, device=q.device)
    elif out.numel() != b * hq * d or out.dtype != q.dtype or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous {q.dtype} tensor of {b * hq * d} elements")
    ov = out.view(b, hq, d)
    flag = err_flag if err_flag is not None else error_flag(q.device)
    cs = k_cache.stride()
    fn, name = ((lib.kani_decode_attention_step, "kani_decode_attention_step") if prefix_final
                else (lib.kani_decode_attention, "kani_decode_attention"))
    check(fn(
        code, b, hq, hk, d, ptr(qv), qv.stride(0), qv.stride(1), ptr(k_cache), ptr(v_cache),
        cs[0], cs[1], cs[2], s_len, ptr(kv_len.contiguous()),
        float(d ** -0.5 if scale is None else scale), ptr(ov), ov.stride(0), ov.stride(1), ptr(flag),
        stream_ptr(q.device)), name)
    return out


def short_conv_step(bcx: torch.Tensor, state: torch.Tensor, conv_w: torch.Tensor,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """LFM2 gated short-conv decode step (optimized_decode.py:256-277, between in_proj
    and out_proj).  bcx: [B, 1, 3H] or [B, 3H] in_proj output; state: [B, H, L]
    (updated in place); conv_w: [H, L].  Returns y [B, 1, H] (or [B, H])."""
    for t, w in ((bcx, "bcx"), (state, "state"), (conv_w, "conv_w")):
        require_cuda(t, w)
    lib = load_library()
    code = dtype_code(bcx, "bcx")
    if state.dim() != 3 or conv_w.dim() != 2:
        raise ValueError("state must be [batch, hidden, L] and conv_w [hidden, L]")
    b, h, lc = state.shape
    if tuple(conv_w.shape) != (h, lc) or bcx.shape[-1] != 3 * h or bcx.numel() != b * 3 * h:
        raise ValueError(f"bcx [..., {3 * h}] / conv_w [{h}, {lc}] do not match state {tuple(state.shape)}")
    if not (state.dtype == conv_w.dtype == bcx.dtype):
        raise TypeError("bcx, state and conv_w must share one dtype")
    if state.stride(2) != 1 or state.stride(1) != lc:
        raise ValueError("state must be contiguous per stream")
    bv, _, bs = _rows_view(bcx, 3 * h)
    shape = (*bcx.shape[:-1], h)
    if out is None:
        out = torch.empty(shape, dtype=bcx.dtype, device=bcx.device)
    check(lib.kani_short_conv_step(code, ptr(bv), bs, ptr(state), state.stride(0), ptr(conv_w.contiguous()),
                                   ptr(out), h, b, h, lc, stream_ptr(bcx.device)), "kani_short_conv_step")
    return out


def sample_tokens(logits: torch.Tensor, seen: torch.Tensor | None = None, *, temperature: float = 1.0,
                  top_p: float = 1.0, repetition_penalty: float = 1.0, top_k: int = 256,
                  index_map: torch.Tensor | None = None, logit_bias: torch.Tensor | None = None,
                  seed: int = 0, step: torch.Tensor | None = None, draws: torch.Tensor | None = None,
                  update_seen: bool = True, out: torch.Tensor | None = None,
                  return_details: bool = False):
    """Sample one token per row of ``logits`` on the device (the reference's
    ``_sample_next_token``, inference_engine.py:349-430, for B streams at once).

    Args:
        logits: [B, V] (or [B, 1, V]) bf16 / fp16 / fp32 CUDA tensor, unchanged.
        seen: [B, ceil(V / 32)] int32 bitmap of penalised indices
            (``sampling.seen_bitmap``), extended with the sampled index when
            ``update_seen``; None = no repetition penalty.
        temperature, top_p, repetition_penalty: as in the reference; k =
            min(top_k, V).
        index_map: [V] int64 index -> token id (the reduced-to-full map).
        logit_bias: [V] additive bias of the logits dtype (the audio mask of
            the full-vocab mode).
        seed, step: Philox key and a device int64 step counter (may live in a
            CUDA graph); ignored when ``draws`` [B, k] fp32 Exp(1) variates are given.
        out: [B] (or any [B, ...] view with a batch stride) int64 for the token ids.
    Returns:
        token ids [B] int64, or (tokens, details) with ``draws``, ``probs`` and
        ``cand`` [B, k] when ``return_details``.
    """
    require_cuda(logits, "logits")
    lib = load_library()
    code = dtype_code(logits, "logits")
    v = logits.shape[-1]
    lv, rows, rs = _rows_view(logits, v)
    b = rows
    if b == 0:
        raise ValueError("empty logits")
    k = min(int(top_k), v)
    if not 1 <= k <= 256:
        raise ValueError(f"top_k must be in [1, 256], got {top_k}")
    dev = logits.device
    words = (v + 31) // 32
    if seen is not None:
        require_cuda(seen, "seen")
        if seen.dtype != torch.int32 or tuple(seen.shape) != (b, words) or not seen.is_contiguous():
            raise ValueError(f"seen must be a contiguous int32 [{b}, {words}] bitmap")
    if index_map is not None:
        require_cuda(index_map, "index_map")
        if index_map.dtype != torch.int64 or index_map.numel() != v or not index_map.is_contiguous():
            raise ValueError(f"index_map must be a contiguous int64 [{v}] tensor")
    if logit_bias is not None:
        require_cuda(logit_bias, "logit_bias")
        if logit_bias.dtype != logits.dtype or logit_bias.numel() != v or not logit_bias.is_contiguous():
            raise ValueError(f"logit_bias must be a contiguous [{v}] tensor of the logits dtype")
    if step is not None:
        require_cuda(step, "step")
        if step.dtype != torch.int64 or step.numel() < 1:
            raise ValueError("step must be an int64 device tensor")
    if draws is not None:
        require_cuda(draws, "draws")
        if draws.dtype != torch.float32 or tuple(draws.shape) != (b, k) or not draws.is_contiguous():
            raise ValueError(f"draws must be a contiguous fp32 [{b}, {k}] tensor")
    if out is None:
        out = torch.empty(b, dtype=torch.int64, device=dev)
    require_cuda(out, "out")
    if out.dtype != torch.int64 or out.numel() != b:
        raise ValueError(f"out must hold {b} int64 token ids")
    out_stride = out.stride(0) if out.dim() >= 1 and b > 1 else 1
    det = None
    if return_details:
        det = {"draws": torch.empty(b, k, dtype=torch.float32, device=dev),
               "probs": torch.empty(b, k, dtype=logits.dtype, device=dev),
               "cand": torch.empty(b, k, dtype=torch.int32, device=dev)}
    check(lib.kani_sample_tokens(
        code, ptr(lv), rs, b, v, ptr(logit_bias) if logit_bias is not None else None,
        ptr(seen) if seen is not None else None, words, 1 if update_seen else 0,
        float(repetition_penalty), float(temperature), float(top_p), k,
        ptr(index_map) if index_map is not None else None, int(seed) & ((1 << 64) - 1),
        ptr(step) if step is not None else None, ptr(draws) if draws is not None else None,
        ptr(det["draws"]) if det else None, ptr(det["probs"]) if det else None,
        ptr(det["cand"]) if det else None, ptr(out), out_stride, stream_ptr(dev)), "kani_sample_tokens")
    return (out, det) if return_details else out


def gemv(x: torch.Tensor, weight: torch.Tensor, *, norm_weight: torch.Tensor | None = None,
         residual: torch.Tensor | None = None, residual_out: torch.Tensor | None = None, eps: float = 1e-5,
         silu_pairs: bool = False, out: torch.Tensor | None = None, l2_prefetch=None) -> torch.Tensor:
    """Decode GEMV for up to 8 streams with the residual add + RMSNorm before it and
    (``silu_pairs``) the SiLU·mul after it, in one launch (the F.linear calls of
    optimized_decode.py:175-289 with their neighbouring norm / activation).

    Args:
        x: [B, K] or [B, 1, K] input (the GEMV input itself, or with ``norm_weight``
            the residual-stream update that is added to ``residual`` and normalised).
        weight: [N, K] ([2N, K], gate rows then up rows, with ``silu_pairs``).
        residual_out: receives round(x + residual) (must not alias x or residual).
        l2_prefetch: up to two (address, bytes) device ranges, the weights of
            later launches, that this launch prefetches into L2 as it starts.
    Returns:
        [B, N] (or [B, 1, N] for a [B, 1, K] input).
    """
    require_cuda(x, "x")
    require_cuda(weight, "weight")
    lib = load_library()
    code = dtype_code(x, "x")
    k = x.shape[-1]
    if weight.dim() != 2 or weight.shape[1] != k or weight.dtype != x.dtype:
        raise ValueError(f"weight must be [N, {k}] of the input dtype")
    if weight.stride(1) != 1:
        weight = weight.contiguous()
    n = weight.shape[0] // 2 if silu_pairs else weight.shape[0]
    if silu_pairs and weight.shape[0] % 2:
        raise ValueError("silu_pairs needs an even number of weight rows")
    xv, b, xs = _rows_view(x, k)
    rv, rs, ov, os_ = None, 0, None, 0
    if residual is not None:
        require_cuda(residual, "residual")
        rv, rb, rs = _rows_view(residual, k)
        if rb != b:
            raise ValueError("residual must have the input's rows")
    if residual_out is not None:
        require_cuda(residual_out, "residual_out")
        if residual_out.shape[-1] != k or residual_out.stride(-1) != 1 or residual_out.numel() != b * k:
            raise ValueError(f"residual_out must be [{b}, {k}] with unit stride")
        ov, _, os_ = _rows_view(residual_out, k)
    if norm_weight is not None:
        require_cuda(norm_weight, "norm_weight")
        if norm_weight.numel() != k or norm_weight.dtype != x.dtype:
            raise ValueError(f"norm_weight must be [{k}] of the input dtype")
        norm_weight = norm_weight.contiguous()
    if out is None:
        out = torch.empty(*x.shape[:-1], n, dtype=x.dtype, device=x.device)
    ov2, ob, ys = _rows_view(out, n)
    if ob != b or ov2.data_ptr() != out.data_ptr():
        raise ValueError(f"out must be [{b}, {n}] rows with a uniform stride")
    if l2_prefetch:
        _lib.set_l2_prefetch(l2_prefetch)
    check(lib.kani_gemv(code, ptr(xv), xs, ptr(rv) if rv is not None else None, rs,
                        ptr(ov) if ov is not None else None, os_,
                        ptr(norm_weight) if norm_weight is not None else None, float(eps), ptr(weight),
                        weight.stride(0), n, k, b, 1 if silu_pairs else 0, ptr(out), ys, stream_ptr(x.device)),
          "kani_gemv")
    return out


def gemm_tc(x: torch.Tensor, weight: torch.Tensor, *, norm_weight: torch.Tensor | None = None,
            residual: torch.Tensor | None = None, residual_out: torch.Tensor | None = None, eps: float = 1e-5,
            silu_pairs: bool = False, out: torch.Tensor | None = None,
            err_flag: torch.Tensor | None = None) -> torch.Tensor:
    """``gemv``'s operation for up to 64 streams on the tensor cores
    (``kani_gemm_tc``): the decode step's F.linear (optimized_decode.py:215, 255,
    276, 281-282) with the residual add + RMSNorm before it and (``silu_pairs``)
    the SiLU·mul after it, in one launch.

    Args:
        x: [B, K] or [B, 1, K] input (with ``norm_weight``, the residual-stream
            update that is added to ``residual`` and normalised); K a multiple of
            64, at most 1024 with ``norm_weight``.
        weight: [N, K] ([2N, K], gate rows then up rows, with ``silu_pairs``).
        residual_out: receives round(x + residual) (must not alias x or residual).
        err_flag: optional int32 device word for KANI_FLAG_TIMEOUT.
    Returns:
        [B, N] (or [B, 1, N] for a [B, 1, K] input).
    """
    require_cuda(x, "x")
    require_cuda(weight, "weight")
    lib = load_library()
    code = dtype_code(x, "x")
    k = x.shape[-1]
    if weight.dim() != 2 or weight.shape[1] != k or weight.dtype != x.dtype:
        raise ValueError(f"weight must be [N, {k}] of the input dtype")
    if weight.stride(1) != 1:
        weight = weight.contiguous()
    n = weight.shape[0] // 2 if silu_pairs else weight.shape[0]
    if silu_pairs and weight.shape[0] % 2:
        raise ValueError("silu_pairs needs an even number of weight rows")
    xv, b, xs = _rows_view(x, k)
    rv, rs, ov, os_ = None, 0, None, 0
    if residual is not None:
        require_cuda(residual, "residual")
        rv, rb, rs = _rows_view(residual, k)
        if rb != b:
            raise ValueError("residual must have the input's rows")
    if residual_out is not None:
        require_cuda(residual_out, "residual_out")
        if residual_out.shape[-1] != k or residual_out.stride(-1) != 1 or residual_out.numel() != b * k:
            raise ValueError(f"residual_out must be [{b}, {k}] with unit stride")
        ov, _, os_ = _rows_view(residual_out, k)
    if norm_weight is not None:
        require_cuda(norm_weight, "norm_weight")
        if norm_weight.numel() != k or norm_weight.dtype != x.dtype:
            raise ValueError(f"norm_weight must be [{k}] of the input dtype")
        norm_weight = norm_weight.contiguous()
    if out is None:
        out = torch.empty(*x.shape[:-1], n, dtype=x.dtype, device=x.device)
    ov2, ob, ys = _rows_view(out, n)
    if ob != b or ov2.data_ptr() != out.data_ptr():
        raise ValueError(f"out must be [{b}, {n}] rows with a uniform stride")
    if err_flag is not None:
        require_cuda(err_flag, "err_flag")
        if err_flag.dtype != torch.int32:
            raise ValueError("err_flag must be an int32 device tensor")
    check(lib.kani_gemm_tc(code, ptr(xv), xs, ptr(rv) if rv is not None else None, rs,
                           ptr(ov) if ov is not None else None, os_,
                           ptr(norm_weight) if norm_weight is not None else None, float(eps), ptr(weight),
                           weight.stride(0), n, k, b, 1 if silu_pairs else 0, ptr(out), ys,
                           ptr(err_flag) if err_flag is not None else None, stream_ptr(x.device)), "kani_gemm_tc")
    return out


def gemv_short_conv(x: torch.Tensor, in_proj_weight: torch.Tensor, conv_state: torch.Tensor,
                    conv_weight: torch.Tensor, *, norm_weight: torch.Tensor | None = None,
                    residual: torch.Tensor | None = None, residual_out: torch.Tensor | None = None,
                    eps: float = 1e-5, out: torch.Tensor | None = None, l2_prefetch=None) -> torch.Tensor:
    """in_proj GEMV + the gated short-conv decode step in one launch
    (optimized_decode.py:255-277), with the optional residual add + RMSNorm
    prologue of ``gemv``.  in_proj_weight [3H, K]; conv_state [B, H, 3] (updated in
    place); conv_weight [H, 3].  ``l2_prefetch`` as in ``gemv``.  Returns y [B, H]
    (or [B, 1, H])."""
    for t, w in ((x, "x"), (in_proj_weight, "in_proj_weight"), (conv_state, "conv_state"),
                 (conv_weight, "conv_weight")):
        require_cuda(t, w)
    lib = load_library()
    code = dtype_code(x, "x")
    k = x.shape[-1]
    if conv_state.dim() != 3 or conv_weight.dim() != 2:
        raise ValueError("conv_state must be [batch, hidden, L] and conv_weight [hidden, L]")
    bsz, h, lc = conv_state.shape
    if in_proj_weight.shape != (3 * h, k) or tuple(conv_weight.shape) != (h, lc):
        raise ValueError(f"in_proj_weight [{3 * h}, {k}] and conv_weight [{h}, {lc}] expected")
    if not (in_proj_weight.dtype == conv_state.dtype == conv_weight.dtype == x.dtype):
        raise TypeError("all tensors must share the input dtype")
    if conv_state.stride(2) != 1 or conv_state.stride(1) != lc:
        raise ValueError("conv_state must be contiguous per stream")
    xv, b, xs = _rows_view(x, k)
    if b != bsz:
        raise ValueError("conv_state must have one row per stream")
    rv, rs, ov, os_ = None, 0, None, 0
    if residual is not None:
        require_cuda(residual, "residual")
        rv, _, rs = _rows_view(residual, k)
    if residual_out is not None:
        require_cuda(residual_out, "residual_out")
        ov, _, os_ = _rows_view(residual_out, k)
    if norm_weight is not None:
        require_cuda(norm_weight, "norm_weight")
        norm_weight = norm_weight.contiguous()
    if out is None:
        out = torch.empty(*x.shape[:-1], h, dtype=x.dtype, device=x.device)
    ov2, _, ys = _rows_view(out, h)
    if l2_prefetch:
        _lib.set_l2_prefetch(l2_prefetch)
    check(lib.kani_gemv_short_conv(code, ptr(xv), xs, ptr(rv) if rv is not None else None, rs,
                                   ptr(ov) if ov is not None else None, os_,
                                   ptr(norm_weight) if norm_weight is not None else None, float(eps),
                                   ptr(in_proj_weight.contiguous()), k, h, k, b, ptr(conv_state), conv_state.stride(0),
                                   ptr(conv_weight.contiguous()), lc, ptr(out), ys, stream_ptr(x.device)),
          "kani_gemv_short_conv")
    return out


def gemv_rope_kv_write(x: torch.Tensor, qkv_weight: torch.Tensor, norm_weight: torch.Tensor,
                       inv_freq: torch.Tensor, position: torch.Tensor, k_cache: torch.Tensor,
                       v_cache: torch.Tensor, write_pos: torch.Tensor, *, num_q_heads: int, num_kv_heads: int,
                       residual: torch.Tensor | None = None, residual_out: torch.Tensor | None = None,
                       eps: float = 1e-5, q_norm_w: torch.Tensor | None = None,
                       k_norm_w: torch.Tensor | None = None, head_eps: float = 1e-5,
                       frame_table: torch.Tensor | None = None, tokens_per_frame: int = 4,
                       frame_pos: torch.Tensor | None = None, q_out: torch.Tensor | None = None,
                       err_flag: torch.Tensor | None = None, l2_prefetch=None) -> torch.Tensor:
    """The attention block's QKV projection (with the input residual add +
    RMSNorm) fused with q/k norm, RoPE, the frame term and the KV write, one
    launch for up to 4 streams (optimized_decode.py:215-240).  x: [B, 1, K]
    (the residual-stream update, or the normed input's source when no
    residual); caches [B, Hk, S, 64]; position / write_pos: [B] int64.
    ``l2_prefetch`` as in ``gemv``.  Returns q_out [B, Hq, 64]."""
    require_cuda(x, "x")
    lib = load_library()
    code = dtype_code(x, "x")
    k = x.shape[-1]
    d = k_cache.shape[-1]
    xv, b, xs = _rows_view(x, k)
    rv, rs, ov, os_ = None, 0, None, 0
    if residual is not None:
        rv, _, rs = _rows_view(residual, k)
    if residual_out is not None:
        ov, _, os_ = _rows_view(residual_out, k)
    if q_out is None:
        q_out = torch.empty(b, num_q_heads, d, dtype=x.dtype, device=x.device)
    if err_flag is None:
        err_flag = error_flag(x.device)
    pos = position.reshape(-1).contiguous()
    slots = write_pos.reshape(-1).contiguous()
    fpos = frame_pos.reshape(-1).contiguous() if frame_pos is not None else None
    if l2_prefetch:
        _lib.set_l2_prefetch(l2_prefetch)
    check(lib.kani_gemv_rope_kv(
        code, ptr(xv), xs, ptr(rv) if rv is not None else None, rs, ptr(ov) if ov is not None else None, os_,
        ptr(norm_weight.contiguous()), float(eps), ptr(qkv_weight), qkv_weight.stride(0), k, b, num_q_heads,
        num_kv_heads, d, ptr(inv_freq.float().contiguous()), ptr(pos),
        ptr(q_norm_w) if q_norm_w is not None else None, ptr(k_norm_w) if k_norm_w is not None else None,
        float(head_eps), ptr(frame_table) if frame_table is not None else None,
        frame_table.shape[0] if frame_table is not None else 0, ptr(fpos) if fpos is not None else None,
        int(tokens_per_frame), ptr(q_out), q_out.stride(0), q_out.stride(1), ptr(k_cache), ptr(v_cache),
        k_cache.stride(0), k_cache.stride(1), k_cache.stride(2), k_cache.shape[2], ptr(slots), ptr(err_flag),
        stream_ptr(x.device)), "kani_gemv_rope_kv")
    return q_out


def head_argmax(hidden: torch.Tensor, weight: torch.Tensor, index_map: torch.Tensor | None = None, *,
                scratch: torch.Tensor | None = None, logits_out: torch.Tensor | None = None,
                out: torch.Tensor | None = None, l2_prefetch=None, norm_weight: torch.Tensor | None = None,
                residual: torch.Tensor | None = None, eps: float = 1e-5) -> torch.Tensor:
    """Greedy next token from the reduced LM head (optimized_decode.py:287 and the
    reduced-to-full map of :144-148) for up to 8 streams in one launch.

    Args:
        hidden: [B, H] or [B, 1, H] final-normed hidden state (bf16 / fp16).
        weight: [rows, H] reduced head (same dtype).
        index_map: [rows] int64 row -> token id (``reduced_to_full``); None = row index.
        scratch: [B + 1] int64 device tensor, zero before the first call and left
            zero by every call; allocated (zeroed) per call when None.
        logits_out: optional [B, rows] tensor that receives the logits.
        out: optional [B] int64 tensor for the token ids.
        l2_prefetch: as in ``gemv``.
        norm_weight: with it, ``hidden`` is the residual-stream update and the
            launch first forms the final residual add + RMSNorm
            (``kani_head_argmax_norm``; optimized_decode.py:283, :286) with
            ``residual`` (None: RMSNorm of ``hidden`` alone) and ``eps``, with the
            arithmetic of ``gemv``'s normed input.
    Returns:
        [B] int64 token ids.
    """
    require_cuda(hidden, "hidden")
    require_cuda(weight, "weight")
    lib = load_library()
    code = dtype_code(hidden, "hidden")
    h = weight.shape[-1]
    if weight.dim() != 2 or hidden.shape[-1] != h:
        raise ValueError(f"hidden [..., {h}] and weight [rows, {h}] expected")
    if weight.dtype != hidden.dtype:
        raise TypeError("hidden and weight must share one dtype")
    hv, b, hs = _rows_view(hidden, h)
    if weight.stride(1) != 1:
        weight = weight.contiguous()
    rows = weight.shape[0]
    dev = hidden.device
    if scratch is None:
        scratch = torch.zeros(b + 1, dtype=torch.int64, device=dev)
    require_cuda(scratch, "scratch")
    if scratch.dtype != torch.int64 or scratch.numel() < b + 1 or not scratch.is_contiguous():
        raise ValueError(f"scratch must be a contiguous int64 tensor of >= {b + 1} elements")
    if index_map is not None:
        require_cuda(index_map, "index_map")
        if index_map.dtype != torch.int64 or index_map.numel() != rows or not index_map.is_contiguous():
            raise ValueError(f"index_map must be a contiguous int64 [{rows}] tensor")
    ls = 0
    if logits_out is not None:
        require_cuda(logits_out, "logits_out")
        if logits_out.dtype != hidden.dtype or logits_out.shape[-1] != rows or logits_out.stride(-1) != 1:
            raise ValueError(f"logits_out must be [{b}, {rows}] of the hidden dtype")
        ls = logits_out.stride(0) if logits_out.dim() > 1 else rows
    if out is None:
        out = torch.empty(b, dtype=torch.int64, device=dev)
    if out.dtype != torch.int64 or out.numel() != b:
        raise ValueError(f"out must hold {b} int64 token ids")
    rv, rs = None, 0
    if norm_weight is not None:
        require_cuda(norm_weight, "norm_weight")
        if norm_weight.numel() != h or norm_weight.dtype != hidden.dtype:
            raise ValueError(f"norm_weight must be [{h}] of the hidden dtype")
        norm_weight = norm_weight.contiguous()
        if residual is not None:
            require_cuda(residual, "residual")
            rv, rb, rs = _rows_view(residual, h)
            if rb != b or residual.dtype != hidden.dtype:
                raise ValueError("residual must have the hidden rows and dtype")
    elif residual is not None:
        raise ValueError("residual needs norm_weight (the add belongs to the final norm)")
    if l2_prefetch:
        _lib.set_l2_prefetch(l2_prefetch)
    tail = (rows, ptr(index_map) if index_map is not None else None,
            ptr(logits_out) if logits_out is not None else None, ls, ptr(scratch),
            ptr(out), out.stride(0) if b > 1 else 1, stream_ptr(dev))
    if norm_weight is None:
        check(lib.kani_head_argmax(code, ptr(hv), hs, b, h, ptr(weight), weight.stride(0), *tail), "kani_head_argmax")
    else:
        check(lib.kani_head_argmax_norm(code, ptr(hv), hs, ptr(rv) if rv is not None else None, rs, ptr(norm_weight),
                                        float(eps), b, h, ptr(weight), weight.stride(0), *tail),
              "kani_head_argmax_norm")
    return out


def head_argmax_tc(hidden: torch.Tensor, weight: torch.Tensor, index_map: torch.Tensor | None = None, *,
                   scratch: torch.Tensor | None = None, logits_out: torch.Tensor | None = None,
                   out: torch.Tensor | None = None, err_flag: torch.Tensor | None = None) -> torch.Tensor:
    """Greedy next tokens from the reduced LM head for a batch of up to 64
    streams on the tensor cores (``kani_head_argmax_tc``): the batched form of
    optimized_decode.py:287 with the reduced-to-full map of :144-148.

    Args:
        hidden: [B, H] or [B, 1, H] final-normed hidden states (bf16 / fp16),
            H a multiple of 64 and at most 1024.
        weight: [rows, H] reduced head (same dtype), rows <= 65535.
        index_map: [rows] int64 row -> token id; None = row index.
        scratch: [>= B + 1] int32 device tensor, zero before the first call and
            left zero by every call; allocated (zeroed) per call when None.
        logits_out: optional [B, rows] tensor that receives the logits.
        out: optional [B] int64 tensor for the token ids.
        err_flag: optional int32 device word; bit KANI_FLAG_TIMEOUT when an
            on-chip wait gave up.
    Returns:
        [B] int64 token ids.
    """
    require_cuda(hidden, "hidden")
    require_cuda(weight, "weight")
    lib = load_library()
    code = dtype_code(hidden, "hidden")
    h = weight.shape[-1]
    if weight.dim() != 2 or hidden.shape[-1] != h:
        raise ValueError(f"hidden [..., {h}] and weight [rows, {h}] expected")
    if weight.dtype != hidden.dtype:
        raise TypeError("hidden and weight must share one dtype")
    hv, b, hs = _rows_view(hidden, h)
    if weight.stride(1) != 1:
        weight = weight.contiguous()
    rows = weight.shape[0]
    dev = hidden.device
    if scratch is None:
        scratch = torch.zeros(b + 1, dtype=torch.int32, device=dev)
    require_cuda(scratch, "scratch")
    if scratch.dtype != torch.int32 or scratch.numel() < b + 1 or not scratch.is_contiguous():
        raise ValueError(f"scratch must be a contiguous int32 tensor of >= {b + 1} elements")
    if index_map is not None:
        require_cuda(index_map, "index_map")
        if index_map.dtype != torch.int64 or index_map.numel() != rows or not index_map.is_contiguous():
            raise ValueError(f"index_map must be a contiguous int64 [{rows}] tensor")
    ls = 0
    if logits_out is not None:
        require_cuda(logits_out, "logits_out")
        if logits_out.dtype != hidden.dtype or logits_out.shape[-1] != rows or logits_out.stride(-1) != 1:
            raise ValueError(f"logits_out must be [{b}, {rows}] of the hidden dtype")
        ls = logits_out.stride(0) if logits_out.dim() > 1 else rows
    if out is None:
        out = torch.empty(b, dtype=torch.int64, device=dev)
    if out.dtype != torch.int64 or out.numel() != b:
        raise ValueError(f"out must hold {b} int64 token ids")
    if err_flag is not None:
        require_cuda(err_flag, "err_flag")
        if err_flag.dtype != torch.int32:
            raise ValueError("err_flag must be an int32 device tensor")
    check(lib.kani_head_argmax_tc(code, ptr(hv), hs, b, h, ptr(weight), weight.stride(0), rows,
                                  ptr(index_map) if index_map is not None else None,
                                  ptr(logits_out) if logits_out is not None else None, ls, ptr(scratch),
                                  ptr(out), out.stride(0) if b > 1 else 1,
                                  ptr(err_flag) if err_flag is not None else None, stream_ptr(dev)),
          "kani_head_argmax_tc")
    return out


def head_argmax_noalloc(hidden: torch.Tensor, weight: torch.Tensor, index_map: torch.Tensor | None = None, *,
                        logits_out: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """``head_argmax`` through ``kani_head_argmax_noalloc``: the cross-CTA scratch
    is the library's own device array, so nothing is allocated per call (calls on
    one device must not overlap in time)."""
    require_cuda(hidden, "hidden")
    require_cuda(weight, "weight")
    lib = load_library()
    code = dtype_code(hidden, "hidden")
    h = weight.shape[-1]
    if weight.dim() != 2 or hidden.shape[-1] != h or weight.dtype != hidden.dtype:
        raise ValueError(f"hidden [..., {h}] and weight [rows, {h}] of one dtype expected")
    hv, b, hs = _rows_view(hidden, h)
    if weight.stride(1) != 1:
        weight = weight.contiguous()
    rows = weight.shape[0]
    if index_map is not None and (index_map.dtype != torch.int64 or index_map.numel() != rows):
        raise ValueError(f"index_map must be an int64 [{rows}] tensor")
    ls = logits_out.stride(0) if logits_out is not None and logits_out.dim() > 1 else rows
    if out is None:
        out = torch.empty(b, dtype=torch.int64, device=hidden.device)
    check(lib.kani_head_argmax_noalloc(code, ptr(hv), hs, b, h, ptr(weight), weight.stride(0), rows,
                                       ptr(index_map) if index_map is not None else None,
                                       ptr(logits_out) if logits_out is not None else None, ls, ptr(out),
                                       out.stride(0) if b > 1 else 1, stream_ptr(hidden.device)),
          "kani_head_argmax_noalloc")
    return out


def decode_advance(next_token: torch.Tensor, input_ids: torch.Tensor, generated: torch.Tensor,
                   step: torch.Tensor, base_pos: torch.Tensor, base_slot: torch.Tensor, positions: torch.Tensor,
                   slots: torch.Tensor, kv_len: torch.Tensor, tokens_per_frame: int = 4, audio_step: float = 1.0,
                   rng_step: torch.Tensor | None = None) -> None:
    """End-of-step bookkeeping of the decode loop in one launch
    (inference_engine.py:615-619, 638-643, 669): record the token, feed it back,
    compute the next step's position / slot / valid length, advance the step
    counter (and the sampler's, if given).  All device int64 tensors; [B] except
    ``generated`` [B, max_new] and the single-value counters."""
    ts = [next_token, input_ids, generated, step, base_pos, base_slot, positions, slots, kv_len]
    for t in ts + ([rng_step] if rng_step is not None else []):
        require_cuda(t, "bookkeeping tensor")
        if t.dtype != torch.int64:
            raise ValueError("bookkeeping tensors must be int64")
    b = next_token.numel()
    for t in (input_ids, base_pos, base_slot, positions, slots, kv_len):
        if t.numel() != b or not t.is_contiguous():
            raise ValueError(f"per-stream tensors must be contiguous with {b} elements")
    if generated.dim() != 2 or generated.shape[0] != b or generated.stride(1) != 1:
        raise ValueError("generated must be [B, max_new] with unit column stride")
    lib = load_library()
    check(lib.kani_decode_advance(ptr(next_token.contiguous()), ptr(input_ids), ptr(generated), generated.stride(0),
                                  generated.shape[1], ptr(step), ptr(rng_step) if rng_step is not None else None,
                                  ptr(base_pos), ptr(base_slot), int(tokens_per_frame), float(audio_step),
                                  ptr(positions), ptr(slots), ptr(kv_len), b, stream_ptr(next_token.device)),
          "kani_decode_advance")


def codec_codes(tokens: torch.Tensor, eos_token: int, audio_tokens_start: int, codebook_size: int = 4032):
    """NeMo codec codes of generated audio tokens (core.py:86-108) for B streams.

    Args:
        tokens: [B, T] int64 generated token ids (device).
    Returns:
        (codes [B, 4, T // 4] int64 (-1 past a stream's frames), frames [B] int64,
        status [B] int32: bit 0 a negative code, bit 1 no complete frame, bit 2 no
        end-of-speech token).
    """
    require_cuda(tokens, "tokens")
    lib = load_library()
    if tokens.dtype != torch.int64 or tokens.dim() != 2:
        raise ValueError("tokens must be an int64 [batch, n_tokens] tensor")
    if tokens.stride(1) != 1:
        tokens = tokens.contiguous()
    b, t = tokens.shape
    mf = t // 4
    dev = tokens.device
    codes = torch.empty(b, 4, mf, dtype=torch.int64, device=dev)
    frames = torch.empty(b, dtype=torch.int64, device=dev)
    status = torch.empty(b, dtype=torch.int32, device=dev)
    check(lib.kani_codec_codes(ptr(tokens), tokens.stride(0), b, t, int(eos_token), int(audio_tokens_start),
                               int(codebook_size), ptr(codes), mf, ptr(frames), ptr(status), stream_ptr(dev)),
          "kani_codec_codes")
    return codes, frames, status


def launch_count() -> int:
    """Kernel launches issued by the library so far in this process."""
    return _lib.launch_count()
