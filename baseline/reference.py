"""Import the unmodified reference package from baseline/_ref and build its
decoder and engine around a synthetic LFM2.

The reference is imported as it stands; two things in this environment stop
a plain ``import kani_tts``, and both are bridged from the outside:

* ``kani_tts/__init__.py`` imports the product API, which imports NeMo (not
  installed).  A bare package object named ``kani_tts`` whose ``__path__`` is
  baseline/_ref/kani_tts is registered instead, so its submodules import
  without running ``__init__``.
* ``kani_tts/static_cache.py:15`` and ``kani_tts/model.py`` import
  ``Lfm2HybridConvCache`` from transformers' LFM2 module, which the installed
  transformers (5.x) no longer defines.  Both use it as a type only, so an
  empty placeholder class is added to that module.

``stand_in_model`` builds the object that ``OptimizedDecoder.__init__``
(kani_tts/optimized_decode.py:31-165) and ``KaniInferenceEngine.__init__``
(kani_tts/inference_engine.py:46-98) read — the same attribute paths the HF
``FlashCompatibleLfm2ForCausalLM`` exposes — from a state dict in the HF LFM2
layout.  The reference's own ``LearnableRotaryEmbedding`` (model.py:141-233)
supplies each attention layer's ``inv_freq``.
"""
from __future__ import annotations

import contextlib
import hashlib
import importlib
import io
import json
import sys
import types
from pathlib import Path

import torch

REF_DIR = Path(__file__).resolve().parent / "_ref"
PKG_DIR = REF_DIR / "kani_tts"


def available() -> bool:
    return (PKG_DIR / "optimized_decode.py").exists() and (REF_DIR / "MANIFEST.json").exists()


def why_unavailable() -> str:
    return ("the reference package is not installed in baseline/_ref "
            "(python baseline/install_ref.py --reference <checkout>)")


def _check_manifest() -> None:
    man = json.loads((REF_DIR / "MANIFEST.json").read_text())
    for name, h in man["files"].items():
        if hashlib.sha256((PKG_DIR / name).read_bytes()).hexdigest() != h:
            raise RuntimeError(f"baseline/_ref/kani_tts/{name} differs from the installed reference")


def import_reference() -> types.SimpleNamespace:
    """The reference modules on the hot path: triton_kernels, static_cache,
    optimized_decode, inference_engine and model."""
    if not available():
        raise ImportError(why_unavailable())
    pkg = sys.modules.get("kani_tts")
    if pkg is None or list(getattr(pkg, "__path__", [])) != [str(PKG_DIR)]:
        _check_manifest()
        import transformers.models.lfm2.modeling_lfm2 as hf
        if not hasattr(hf, "Lfm2HybridConvCache"):
            class Lfm2HybridConvCache:  # placeholder for the removed HF class (type use only)
                pass
            hf.Lfm2HybridConvCache = Lfm2HybridConvCache
        for name in [m for m in sys.modules if m == "kani_tts" or m.startswith("kani_tts.")]:
            del sys.modules[name]
        pkg = types.ModuleType("kani_tts")
        pkg.__path__ = [str(PKG_DIR)]
        sys.modules["kani_tts"] = pkg
    mods = {n: importlib.import_module(f"kani_tts.{n}")
            for n in ("triton_kernels", "static_cache", "optimized_decode", "model", "inference_engine")}
    return types.SimpleNamespace(**mods)


def hf_config(cfg):
    """transformers' Lfm2Config with the synthetic model's sizes (the attributes
    the reference reads: optimized_decode.py:37-50, static_cache.py:46-76)."""
    from transformers import Lfm2Config
    hc = Lfm2Config(hidden_size=cfg.hidden_size, num_attention_heads=cfg.num_attention_heads,
                    num_key_value_heads=cfg.num_key_value_heads, num_hidden_layers=cfg.num_hidden_layers,
                    layer_types=list(cfg.layer_types), vocab_size=cfg.vocab_size,
                    intermediate_size=cfg.intermediate_size)
    hc.head_dim = cfg.head_dim
    hc.norm_eps = cfg.norm_eps
    hc.conv_L_cache = cfg.conv_L_cache
    hc.rope_theta = cfg.rope_theta
    return hc


def stand_in_model(ref, cfg, state_dict: dict, device) -> types.SimpleNamespace:
    """An object with the attribute paths of FlashCompatibleLfm2ForCausalLM that
    OptimizedDecoder and KaniInferenceEngine read, holding `state_dict`'s bf16
    weights on `device` (no copies beyond the device move)."""
    ns = types.SimpleNamespace
    dev = torch.device(device)
    hc = hf_config(cfg)

    def W(name):
        return ns(weight=state_dict[name].to(dev, torch.bfloat16))

    n_attn = len(cfg.attn_layers)
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
            rope = ref.model.LearnableRotaryEmbedding(hc, layer_idx=i, total_attention_layers=n_attn,
                                                      alpha_min=cfg.alpha_min, alpha_max=cfg.alpha_max)
            with torch.no_grad():
                rope.alpha_weight.copy_(state_dict[f"model.learnable_rope_layers.{i}.alpha_weight"])
            ropes.append(rope.to(dev))
        else:
            L.conv = ns(in_proj=W(p + "conv.in_proj.weight"), conv=W(p + "conv.conv.weight"),
                        out_proj=W(p + "conv.out_proj.weight"))
            ropes.append(None)
        layers.append(L)
    emb = torch.nn.Embedding(cfg.vocab_size, cfg.hidden_size, device="meta")
    emb.weight = torch.nn.Parameter(state_dict["model.embed_tokens.weight"].to(dev, torch.bfloat16),
                                    requires_grad=False)
    head = W("lm_head.weight")
    return ns(config=hc, parameters=lambda: iter([head.weight]), eval=lambda: None,
              model=ns(embed_tokens=emb, layers=layers, learnable_rope_layers=ropes,
                       embedding_norm=W("model.embedding_norm.weight"), pos_emb=None,
                       speaker_emb_projection=W("model.speaker_emb_projection.weight")),
              lm_head=head)


def optimized_decoder(ref, model, cfg):
    """kani_tts.optimized_decode.OptimizedDecoder on the stand-in (its init banner
    goes to stderr, so a JSON line on stdout stays one line)."""
    with contextlib.redirect_stdout(io.StringIO()) as buf:
        dec = ref.optimized_decode.OptimizedDecoder(model, cfg.audio_tokens_start, cfg.eos_token_id)
    sys.stderr.write(buf.getvalue())
    return dec


def engine(ref, model, cfg, max_new_tokens: int, temperature: float = 0.7, top_p: float = 0.95,
           repetition_penalty: float = 1.0):
    """kani_tts.inference_engine.KaniInferenceEngine with CUDA graphs on, its
    optimized decoder already built (generate() builds it after its HF prefill,
    inference_engine.py:531-535)."""
    eng = ref.inference_engine.KaniInferenceEngine(
        model, cfg.audio_tokens_start, tokens_per_frame=cfg.tokens_per_frame, audio_step=cfg.audio_step,
        max_new_tokens=max_new_tokens, temperature=temperature, top_p=top_p,
        repetition_penalty=repetition_penalty, use_cuda_graphs=True)
    eng.optimized_decoder = optimized_decoder(ref, model, cfg)
    return eng


def capture(eng, dynamic_cache, prefill_len: int) -> None:
    """KaniInferenceEngine._initialize_cuda_graphs (inference_engine.py:230-331):
    static cache, mask and input tensors, one warm-up step, graph capture."""
    with contextlib.redirect_stdout(io.StringIO()) as buf:
        eng._initialize_cuda_graphs(dynamic_cache, prefill_len)
    sys.stderr.write(buf.getvalue())


@contextlib.contextmanager
def installed_kernels(ref):
    """Run the reference with this library's kernels dropped in
    (kani_tts_b200.install.install_into_reference); restore its own on exit."""
    from kani_tts_b200.install import install_into_reference
    od, sc, ie = ref.optimized_decode, ref.static_cache, ref.inference_engine
    saved = ([getattr(od, n) for n in ("fused_rms_norm", "fused_silu_mul", "fused_rope")],
             sc.StaticLfm2HybridConvCache, ie.StaticLfm2HybridConvCache)
    try:
        yield install_into_reference()
    finally:
        for n, f in zip(("fused_rms_norm", "fused_silu_mul", "fused_rope"), saved[0]):
            setattr(od, n, f)
        sc.StaticLfm2HybridConvCache, ie.StaticLfm2HybridConvCache = saved[1], saved[2]
