"""Generate the golden vectors in tests/golden/*.npz from the reference itself.

Run where the reference checkout is available, naming it in
KANI_REFERENCE_DIR:

    KANI_REFERENCE_DIR=<checkout> python tests/golden/make_golden.py

What runs, all on the CPU:
  * the reference's three Triton kernels (kani_tts/triton_kernels.py) under
    the Triton interpreter (TRITON_INTERPRET=1);
  * StaticLfm2HybridConvCache.update (kani_tts/static_cache.py);
  * LearnableRotaryEmbedding and compute_frame_level_positions
    (kani_tts/model.py);
  * HF Lfm2RMSNorm (the eager norm the reference's model uses) for the
    fp32 residual-add + norm case.
The reference package __init__ imports NeMo, which is absent, so a bare
``kani_tts`` package object pointing at the checkout is registered instead;
the static cache and model modules import ``Lfm2HybridConvCache``, which the
installed transformers no longer has, so a placeholder class is added.  The
reference files are read, never modified.

Inputs are seeded (torch.Generator per tensor, seeds 0, 1, 2, ... in argument
order) and saved next to the outputs; bf16 tensors are stored as their uint16
bit patterns (key suffix ``__bf16``).
"""
from __future__ import annotations

import importlib
import os
import sys
import types
from pathlib import Path

import numpy as np

os.environ["TRITON_INTERPRET"] = "1"
import torch  # noqa: E402

REF = Path(os.environ["KANI_REFERENCE_DIR"]) if os.environ.get("KANI_REFERENCE_DIR") else None
OUT = Path(__file__).resolve().parent


def _import_reference():
    if REF is None:
        raise SystemExit("set KANI_REFERENCE_DIR to the reference checkout")
    import transformers.models.lfm2.modeling_lfm2 as hf
    if not hasattr(hf, "Lfm2HybridConvCache"):
        class Lfm2HybridConvCache:  # placeholder for the removed HF class (type use only)
            pass
        hf.Lfm2HybridConvCache = Lfm2HybridConvCache
    pkg = types.ModuleType("kani_tts")
    pkg.__path__ = [str(REF / "kani_tts")]
    sys.modules["kani_tts"] = pkg
    tk = importlib.import_module("kani_tts.triton_kernels")
    sc = importlib.import_module("kani_tts.static_cache")
    md = importlib.import_module("kani_tts.model")
    return tk, sc, md, hf


def _gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def randn(shape, seed, dtype=torch.bfloat16, mean=0.0, std=1.0):
    return (mean + std * torch.randn(shape, generator=_gen(seed))).to(dtype)


def pack(d: dict) -> dict:
    out = {}
    for k, v in d.items():
        if isinstance(v, torch.Tensor):
            if v.dtype == torch.bfloat16:
                out[k + "__bf16"] = v.contiguous().view(torch.int16).numpy().view(np.uint16)
            else:
                out[k] = v.contiguous().numpy()
        else:
            out[k] = np.asarray(v)
    return out


def save(name: str, cases: dict[str, dict]) -> None:
    flat = {}
    for case, d in cases.items():
        for k, v in pack(d).items():
            flat[f"{case}/{k}"] = v
    np.savez_compressed(OUT / f"{name}.npz", **flat)
    print(f"wrote {name}.npz: {len(cases)} cases")


def make_config(hf, hidden=1024, heads=16, kv_heads=8, layers=2, layer_types=None, theta=1e6):
    from transformers import Lfm2Config
    cfg = Lfm2Config(hidden_size=hidden, num_attention_heads=heads, num_key_value_heads=kv_heads,
                     num_hidden_layers=layers, layer_types=layer_types or ["conv", "full_attention"])
    cfg.rope_theta = theta
    return cfg


def main() -> None:
    tk, sc, md, hf = _import_reference()

    # ---------------------------------------------------- Triton RMSNorm
    cases = {}
    for name, shape, n, dtype in [("hidden_bf16", (4, 1024), 1024, torch.bfloat16),
                                  ("decode_bf16", (1, 1, 1024), 1024, torch.bfloat16),
                                  ("qnorm_bf16", (1, 1, 16, 64), 64, torch.bfloat16),
                                  ("knorm_bf16", (1, 1, 8, 64), 64, torch.bfloat16),
                                  ("odd_bf16", (3, 100), 100, torch.bfloat16),
                                  ("fp32_storage", (8, 1024), 1024, torch.float32)]:
        x = randn(shape, 0, dtype)
        w = randn((n,), 1, dtype, mean=1.0, std=0.02)
        eps = 1e-5
        y = tk.fused_rms_norm(x, w, eps)
        cases[name] = dict(x=x, w=w, eps=np.float32(eps), y=y)
    save("triton_rms_norm", cases)

    # ------------------------------------- residual add + norm (eager paths)
    cases = {}
    x = randn((8, 1024), 0, torch.float32)
    r = randn((8, 1024), 1, torch.float32)
    g = randn((1024,), 2, torch.float32, mean=1.0, std=0.02)
    norm = hf.Lfm2RMSNorm(1024, eps=1e-5)
    with torch.no_grad():
        norm.weight.copy_(g)
        h = x + r
        y = norm(h)
    cases["config1_fp32_hf"] = dict(x=x, r=r, w=g, eps=np.float32(1e-5), h=h, y=y)
    xb = randn((4, 1024), 3, torch.bfloat16)
    rb = randn((4, 1024), 4, torch.bfloat16)
    wb = randn((1024,), 5, torch.bfloat16, mean=1.0, std=0.02)
    hb = xb + rb                                   # optimized_decode.py:252 (bf16 eager add)
    yb = tk.fused_rms_norm(hb, wb, 1e-5)           # next norm (optimized_decode.py:280)
    cases["decode_bf16_triton"] = dict(x=xb, r=rb, w=wb, eps=np.float32(1e-5), h=hb, y=yb)
    save("add_rms_norm", cases)

    # ------------------------------------------------------ Triton SiLU*mul
    cases = {}
    for name, shape in [("rows4_bf16", (4, 9216)), ("decode_bf16", (1, 1, 9216)),
                        ("odd_bf16", (3, 200))]:
        gu = randn(shape, 0)
        cases[name] = dict(gate_up=gu, y=tk.fused_silu_mul(gu))
    save("triton_silu_mul", cases)

    # ------------------------------- learnable-alpha inv_freq (model.py:141-196)
    cases = {}
    cfg = make_config(hf)
    for i, wa in enumerate([0.0, 0.3, -1.2]):
        rope = md.LearnableRotaryEmbedding(cfg, layer_idx=1, total_attention_layers=1)
        with torch.no_grad():
            rope.alpha_weight.fill_(wa)
            inv = (rope.inv_freq_base * rope.alpha).float()   # optimized_decode.py:108
        cases[f"alpha{i}"] = dict(head_dim=np.int64(64), theta=np.float64(1e6),
                                  alpha_weight=np.float32(wa), inv_freq=inv)
    save("inv_freq", cases)

    # ------------------------------------- Triton RoPE with decode cos/sin rows
    cases = {}
    rope = md.LearnableRotaryEmbedding(cfg, layer_idx=1, total_attention_layers=1)
    with torch.no_grad():
        inv = (rope.inv_freq_base * rope.alpha).float()
    for i, pos in enumerate([0, 1, 777, 2047]):
        q = randn((1, 16, 1, 64), 2 * i)
        k = randn((1, 8, 1, 64), 2 * i + 1)
        # optimized_decode.py:229-234
        p = torch.tensor([[pos]], dtype=torch.long)[0, 0].float()
        freqs = inv * p
        emb = torch.cat([freqs, freqs])
        cos, sin = emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)
        qo, ko = tk.fused_rope(q, k, cos, sin)
        cases[f"pos{pos}"] = dict(q=q, k=k, cos=cos, sin=sin, inv_freq=inv, pos=np.int64(pos),
                                  q_out=qo, k_out=ko)
    save("triton_rope", cases)

    # ------------------------------------------- static cache update (scatter_)
    cases = {}
    for name, bsz, slot in [("b1_slot5", 1, 5), ("b2_slot0", 2, 0), ("b1_last", 1, 15)]:
        cache = sc.StaticLfm2HybridConvCache(cfg, max_total_len=16, batch_size=bsz,
                                             dtype=torch.bfloat16, device="cpu")
        k_prev = randn((bsz, 8, 16, 64), 10)
        v_prev = randn((bsz, 8, 16, 64), 11)
        cache.key_cache[1].copy_(k_prev)
        cache.value_cache[1].copy_(v_prev)
        k = randn((bsz, 8, 1, 64), 12)
        v = randn((bsz, 8, 1, 64), 13)
        cache.set_write_position(slot)
        kf, vf = cache.update(k, v, 1)
        cases[name] = dict(k_prev=k_prev, v_prev=v_prev, k=k, v=v, slot=np.int64(slot),
                           k_cache=kf.clone(), v_cache=vf.clone())
    save("static_cache_update", cases)

    # ------------------------------------------------ frame-level positions
    cases = {}
    ids_doc = torch.tensor([[100, 200, 64410, 68442, 72474, 76506, 300]])
    for i, step in enumerate([1.0, 0.5]):
        cases[f"docstring_step{i}"] = dict(
            input_ids=ids_doc, audio_tokens_start=np.int64(64410), tokens_per_frame=np.int64(4),
            audio_step=np.float64(step),
            positions=md.compute_frame_level_positions(ids_doc, 64410, 4, step).float())
    ids_mix = torch.randint(0, 80000, (2, 40), generator=_gen(7))
    cases["mixed_step1"] = dict(
        input_ids=ids_mix, audio_tokens_start=np.int64(64410), tokens_per_frame=np.int64(4),
        audio_step=np.float64(1.0),
        positions=md.compute_frame_level_positions(ids_mix, 64410, 4, 1.0).float())
    save("frame_positions", cases)

    save("decode_step", decode_step_cases(sc, md, hf))
    save("sampling", sampling_cases())
    save("codec_codes", codec_cases())
    print("golden vectors written to", OUT)


def codec_cases():
    """NemoAudioPlayer.get_nano_codes (kani_tts/core.py:86-108) on token sequences
    built as the engine returns them: prompt ending with start-of-speech, the
    generated audio tokens, end-of-speech.  NeMo itself is absent, so placeholder
    ``nemo.collections.tts.models`` modules let ``kani_tts.core`` import; the
    function reads only the four attributes of the stand-in object.  Where the
    reference raises, the case records the message instead of codes."""
    import types as _t
    for name in ["nemo", "nemo.collections", "nemo.collections.tts", "nemo.collections.tts.models"]:
        sys.modules.setdefault(name, _t.ModuleType(name))
    if not hasattr(sys.modules["nemo.collections.tts.models"], "AudioCodecModel"):
        class AudioCodecModel:  # placeholder (type use only)
            pass
        sys.modules["nemo.collections.tts.models"].AudioCodecModel = AudioCodecModel
    core = importlib.import_module("kani_tts.core")
    tl = 64400
    player = _t.SimpleNamespace(start_of_speech=tl + 1, end_of_speech=tl + 2, codebook_size=4032,
                                audio_tokens_start=tl + 10)
    g = _gen(77)

    def audio(n):
        c = torch.arange(n) % 4
        return tl + 10 + c * 4032 + torch.randint(0, 4032, (n,), generator=g)

    prompt = torch.cat([torch.randint(0, tl, (20,), generator=g), torch.tensor([tl + 1])])
    cases = {}
    for name, gen in {
        "whole_frames": audio(48),
        "partial_frame": audio(51),
        "one_frame": audio(5),
        "negative_code": torch.cat([audio(8), torch.tensor([tl + 10 + 4032 * 2 - 1]), audio(3)]),
        "no_frame": audio(3),
    }.items():
        gen_ids = torch.cat([gen, torch.tensor([tl + 2])])
        out_ids = torch.cat([prompt, gen_ids])
        d = dict(generated=gen_ids)
        try:
            codes, n = core.NemoAudioPlayer.get_nano_codes(player, out_ids)
            d.update(codes=codes, frames=n)
        except ValueError as e:
            d.update(error=np.array(str(e)))
        cases[name] = d
    return cases


def _tie_free_logits(v: int, n_top: int, lo: float, hi: float, seed: int) -> torch.Tensor:
    """bf16 logits [1, v] whose n_top largest values are distinct bf16 numbers
    drawn from [lo, hi) at random positions; the rest lie below lo."""
    g = _gen(seed)
    grid = torch.arange(0, 65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    grid = grid[torch.isfinite(grid) & (grid >= lo) & (grid < hi)]
    pick = grid[torch.randperm(grid.numel(), generator=g)[:n_top]]
    out = (torch.randn(1, v, generator=g) * 1.5 + (lo - 6.0)).clamp(max=lo - 0.5).to(torch.bfloat16)
    pos = torch.randperm(v, generator=g)[:n_top]
    out[0, pos] = pick
    return out


def sampling_cases():
    """KaniInferenceEngine._sample_next_token (kani_tts/inference_engine.py:349-430)
    run on the CPU with a stand-in engine object holding the attributes it reads.
    torch.topk and torch.multinomial are wrapped: the topk wrapper records the
    reference's candidates; the multinomial wrapper records the final
    distribution and draws the sample by the exponential race torch.multinomial
    performs for one sample (argmax(probs / q), q ~ Exp(1) in the probs dtype),
    with q taken from stored fp32 draws so the selected token is reproducible."""
    import types as _t
    ie = importlib.import_module("kani_tts.inference_engine")
    sample = ie.KaniInferenceEngine._sample_next_token
    vocab, audio_start, eos = 80000, 64410, 7
    n_red = 1 + vocab - audio_start
    reduced_to_full = torch.cat([torch.tensor([eos]), torch.arange(audio_start, vocab)])
    full_to_reduced = torch.full((vocab,), -1, dtype=torch.long)
    full_to_reduced[eos] = 0
    full_to_reduced[audio_start:] = torch.arange(1, n_red)
    audio_mask = torch.full((1, vocab), float("-inf"), dtype=torch.bfloat16)
    audio_mask[0, audio_start:] = 0.0
    audio_mask[0, eos] = 0.0

    specs = {
        # name: (reduced?, penalty, temperature, top_p, (n_top, lo, hi), seed)
        "config_defaults": (True, 1.2, 0.5, 0.85, (300, 1.0, 16.0), 10),
        "engine_defaults": (True, 1.0, 0.7, 0.95, (300, 1.0, 16.0), 11),
        "no_top_p": (True, 1.1, 1.0, 1.0, (300, 1.0, 16.0), 12),
        "deep_nucleus": (True, 1.2, 1.0, 0.95, (300, 0.5, 4.0), 13),
        "full_vocab_mask": (False, 1.2, 0.5, 0.85, (300, 1.0, 16.0), 14),
    }
    cases = {}
    real_topk, real_multinomial = torch.topk, torch.multinomial
    for name, (reduced, rp, temp, top_p, (n_top, lo, hi), seed) in specs.items():
        v = n_red if reduced else vocab
        g = _gen(100 + seed)
        for attempt in range(50):
            logits = _tie_free_logits(n_red, n_top, lo, hi, 1000 * seed + attempt)
            if not reduced:   # full vocab: the same values on the EOS + audio ids, text ids anywhere
                full = (torch.randn(1, vocab, generator=g) * 3.0).to(torch.bfloat16)
                full[0, reduced_to_full] = logits[0]
                logits = full
            prompt = torch.randint(0, 64400, (1, 120), generator=g)
            gen_red = torch.randint(0, n_red, (1, 80), generator=g)
            history = torch.cat([prompt, reduced_to_full[gen_red]], dim=1)
            # the penalised row must be tie-free inside the top k + 1
            pen = logits.clone()
            ids = history[0].unique()
            ridx = full_to_reduced[ids] if reduced else ids
            ridx = ridx[ridx >= 0]
            pl = pen[0, ridx]
            pen[0, ridx] = torch.where(pl > 0, pl / rp, pl * rp) if rp != 1.0 else pl
            if not reduced:
                pen = pen + audio_mask
            top = torch.sort(pen.float(), descending=True).values[0, :257]
            if bool((top[1:] < top[:-1]).all()):
                break
        else:
            raise RuntimeError(f"no tie-free draw for {name}")
        draws = -torch.log(torch.rand(1, 256, generator=g).clamp_min(2.0 ** -24))
        rec = {}

        def topk(x, k, dim=-1, **kw):
            vals, idx = real_topk(x, k, dim=dim, **kw)
            rec["topk_values"], rec["topk_indices"] = vals.clone(), idx.clone()
            return vals, idx

        def multinomial(probs, num_samples, **kw):
            rec["probs"] = probs.clone()
            q = draws[:, :probs.shape[-1]].to(probs.dtype)
            return torch.argmax(probs / q, dim=-1, keepdim=True)

        stand_in = _t.SimpleNamespace(
            optimized_decoder=_t.SimpleNamespace(full_to_reduced=full_to_reduced,
                                                 reduced_to_full=reduced_to_full),
            vocab_size=vocab, repetition_penalty=rp, temperature=temp, top_p=top_p,
            _audio_logit_mask=None if reduced else audio_mask)
        torch.topk, torch.multinomial = topk, multinomial
        try:
            tok = sample(stand_in, logits.clone(), history)
        finally:
            torch.topk, torch.multinomial = real_topk, real_multinomial
        cases[name] = dict(logits=logits, history=history, reduced=np.bool_(reduced),
                           repetition_penalty=np.float64(rp), temperature=np.float64(temp),
                           top_p=np.float64(top_p), draws=draws.float(), token=tok.view(-1),
                           topk_values=rec["topk_values"], topk_indices=rec["topk_indices"],
                           probs=rec["probs"])
    return cases


def decode_step_cases(sc, md, hf):
    """Three decode steps of the reference OptimizedDecoder (kani_tts/optimized_decode.py)
    on a tiny synthetic LFM2 held by a stand-in model object that exposes exactly the
    attributes OptimizedDecoder reads.  Weights come from the package's seeded
    generator (only the seed and a checksum are stored)."""
    import types as _t
    sys.path.insert(0, str(Path(__file__).resolve().parents[2] / "kani-tts-2-openai-server_b200"))
    from kani_tts_b200.model import synthetic_state_dict, tiny_config
    od = importlib.import_module("kani_tts.optimized_decode")
    cfg = tiny_config()
    seed = 1234
    sd = synthetic_state_dict(cfg, seed=seed)
    hcfg = make_config(hf, hidden=cfg.hidden_size, heads=cfg.num_attention_heads,
                       kv_heads=cfg.num_key_value_heads, layers=cfg.num_hidden_layers,
                       layer_types=list(cfg.layer_types), theta=cfg.rope_theta)
    hcfg.head_dim = cfg.head_dim
    hcfg.vocab_size = cfg.vocab_size
    hcfg.norm_eps = cfg.norm_eps
    hcfg.conv_L_cache = cfg.conv_L_cache
    ns = _t.SimpleNamespace
    W = lambda name: ns(weight=sd[name])  # noqa: E731
    layers, ropes = [], []
    for i, kind in enumerate(cfg.layer_types):
        p = f"model.layers.{i}."
        L = ns(operator_norm=W(p + "operator_norm.weight"), ffn_norm=W(p + "ffn_norm.weight"),
               feed_forward=ns(w1=W(p + "feed_forward.w1.weight"), w2=W(p + "feed_forward.w2.weight"),
                               w3=W(p + "feed_forward.w3.weight")))
        if kind == "full_attention":
            L.self_attn = ns(q_proj=W(p + "self_attn.q_proj.weight"), k_proj=W(p + "self_attn.k_proj.weight"),
                             v_proj=W(p + "self_attn.v_proj.weight"),
                             q_layernorm=W(p + "self_attn.q_layernorm.weight"),
                             k_layernorm=W(p + "self_attn.k_layernorm.weight"),
                             out_proj=W(p + "self_attn.out_proj.weight"))
            rope = md.LearnableRotaryEmbedding(hcfg, layer_idx=i, total_attention_layers=2)
            with torch.no_grad():
                rope.alpha_weight.copy_(sd[f"model.learnable_rope_layers.{i}.alpha_weight"])
            ropes.append(rope)
        else:
            L.conv = ns(in_proj=W(p + "conv.in_proj.weight"), conv=W(p + "conv.conv.weight"),
                        out_proj=W(p + "conv.out_proj.weight"))
            ropes.append(None)
        layers.append(L)
    emb = torch.nn.Embedding(cfg.vocab_size, cfg.hidden_size)
    with torch.no_grad():
        emb.weight.copy_(sd["model.embed_tokens.weight"].float())
    emb = emb.to(torch.bfloat16)
    stand_in = ns(config=hcfg, parameters=lambda: iter([sd["lm_head.weight"]]),
                  model=ns(embed_tokens=emb, layers=layers, learnable_rope_layers=ropes,
                           embedding_norm=W("model.embedding_norm.weight"), pos_emb=None),
                  lm_head=W("lm_head.weight"))
    dec = od.OptimizedDecoder(stand_in, cfg.audio_tokens_start, cfg.eos_token_id)

    max_len, prefix = 16, 5
    cache = sc.StaticLfm2HybridConvCache(hcfg, max_total_len=max_len, batch_size=1, dtype=torch.bfloat16,
                                         device="cpu")
    init = {}
    for i in cfg.attn_layers:
        kp = randn((1, cfg.num_key_value_heads, max_len, cfg.head_dim), 100 + i)
        vp = randn((1, cfg.num_key_value_heads, max_len, cfg.head_dim), 200 + i)
        kp[:, :, prefix:] = 0
        vp[:, :, prefix:] = 0
        cache.key_cache[i].copy_(kp)
        cache.value_cache[i].copy_(vp)
        init[f"k_init_{i}"], init[f"v_init_{i}"] = kp, vp
    for i, kind in enumerate(cfg.layer_types):
        if kind != "full_attention":
            cs = randn((1, cfg.hidden_size, cfg.conv_L_cache), 300 + i)
            cache.conv_cache[i].copy_(cs)
            init[f"conv_init_{i}"] = cs
    mask = torch.full((1, 1, 1, max_len), float("-inf"), dtype=torch.bfloat16)
    mask[..., :prefix] = 0
    tokens = [650, 7, 612]
    positions = [prefix, prefix, prefix + 1]
    out = {"seed": np.int64(seed), "max_len": np.int64(max_len), "prefix": np.int64(prefix),
           "tokens": torch.tensor(tokens), "positions": torch.tensor(positions),
           "weight_checksum": np.float64(sum(float(v.float().abs().sum()) for v in sd.values())), **init}
    with torch.no_grad():
        for step, (tok, pos) in enumerate(zip(tokens, positions)):
            slot = prefix + step
            cache.set_write_position(slot)
            mask[..., slot] = 0
            logits = dec(input_ids=torch.tensor([[tok]]), position_ids=torch.tensor([[pos]]),
                         past_key_values=cache, causal_mask=mask,
                         cache_position=torch.tensor([slot]))
            out[f"logits_{step}"] = logits.clone()
    for i in cfg.attn_layers:
        out[f"k_final_{i}"] = cache.key_cache[i].clone()
        out[f"v_final_{i}"] = cache.value_cache[i].clone()
    for i, kind in enumerate(cfg.layer_types):
        if kind != "full_attention":
            out[f"conv_final_{i}"] = cache.conv_cache[i].clone()
    return {"tiny": out}


if __name__ == "__main__":
    if len(sys.argv) > 2 and sys.argv[1] == "--only":
        _import_reference()
        makers = {"sampling": sampling_cases, "codec_codes": codec_cases}
        for name in sys.argv[2:]:
            save(name, makers[name]())
    else:
        main()
