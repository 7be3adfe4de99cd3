"""The drop-in, exercised: the reference's own decoder and engine code
(``kani_tts/optimized_decode.py``, ``kani_tts/static_cache.py``,
``kani_tts/inference_engine.py``, installed unmodified in baseline/_ref) run
once with its Triton kernels and once after
``kani_tts_b200.install.install_into_reference()`` has rebound
``fused_rms_norm`` / ``fused_silu_mul`` / ``fused_rope`` in
``kani_tts.optimized_decode`` (bound there by name at optimized_decode.py:14)
and ``StaticLfm2HybridConvCache`` in the cache and engine modules.

Checks:

* ``update`` (static_cache.py:110-142 vs ``StaticKVCache.update``): the same
  K/V rows give bit-identical caches, and both return the full buffers.
* ``OptimizedDecoder.__call__`` on the tiny model of the reference-decoder
  golden (three steps, run by the reference on the CPU): logits within 2 % of
  the largest logit of both the golden and the Triton run on this GPU, same
  argmax; every cache slot outside the written ones is untouched.
* The engine's CUDA-graph capture (``_initialize_cuda_graphs``,
  inference_engine.py:230-331) of the full-size 16-layer decoder on this
  library's kernels, replayed by the loop body of ``generate``
  (inference_engine.py:641-651) for 8 teacher-forced steps: the static cache
  is this library's class, logits within 5 % of the largest logit of the Triton
  engine's, cosine > 0.999, same argmax where the top two are not near-tied.

The tolerances are those of the decode-step tests (tests/test_gpu_decode.py):
the fused norm and SiLU·mul differ from the Triton kernels by at most 1 bf16
ULP per element, and 16 layers carry such differences into the logits.
"""
from __future__ import annotations

import types

import pytest
import torch

from baseline import reference as R
from golden_io import load

from kani_tts_b200.model import LFM2Config, synthetic_state_dict, tiny_config
from kani_tts_b200.static_cache import StaticKVCache

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not R.available(), reason=R.why_unavailable())]
DEV = torch.device("cuda", 0)


@pytest.fixture(scope="module")
def ref():
    math_sdp = torch.backends.cuda.math_sdp_enabled()
    yield R.import_reference()
    torch.backends.cuda.enable_math_sdp(math_sdp)   # the reference engine turns it off


def close(got, want, frac):
    got, want = got.detach().float().cpu(), want.detach().float().cpu()
    scale = float(want.abs().max())
    err = float((got - want).abs().max())
    assert err <= frac * scale, f"max error {err} vs scale {scale}"


def same_argmax_where_clear(got, want, rel=2.0 ** -5):
    g, r = got.float().cpu().flatten(0, -2), want.float().cpu().flatten(0, -2)
    top2 = r.topk(2, dim=-1).values
    clear = (top2[:, 0] - top2[:, 1]) > rel * top2[:, 0].abs()
    assert torch.equal(g.argmax(-1)[clear], r.argmax(-1)[clear])
    return int(clear.sum())


@pytest.mark.parametrize("slot", [0, 7, 2047])
def test_update_matches_the_reference_update_bit_for_bit(ref, slot):
    cfg = LFM2Config()
    hc = R.hf_config(cfg)
    theirs = ref.static_cache.StaticLfm2HybridConvCache(hc, max_total_len=2048, batch_size=1,
                                                        dtype=torch.bfloat16, device=DEV)
    mine = StaticKVCache(hc, max_total_len=2048, batch_size=1, dtype=torch.bfloat16, device=DEV)
    g = torch.Generator().manual_seed(slot)
    layer = cfg.attn_layers[1]
    for c in (theirs, mine):
        init = torch.randn(1, cfg.num_key_value_heads, 2048, cfg.head_dim, generator=torch.Generator().manual_seed(9))
        c.key_cache[layer].copy_(init.bfloat16())
        c.value_cache[layer].copy_((-init).bfloat16())
    k = torch.randn(1, cfg.num_key_value_heads, 1, cfg.head_dim, generator=g).bfloat16().to(DEV)
    v = torch.randn(1, cfg.num_key_value_heads, 1, cfg.head_dim, generator=g).bfloat16().to(DEV)
    for c in (theirs, mine):
        c.set_write_position(slot)
    kt, vt = theirs.update(k, v, layer)
    km, vm = mine.update(k, v, layer)
    assert km.data_ptr() == mine.key_cache[layer].data_ptr() and vm.data_ptr() == mine.value_cache[layer].data_ptr()
    assert torch.equal(km, kt) and torch.equal(vm, vt)
    assert mine.read_errors() == 0


def _tiny_run(ref, model, cfg, c, use_kernels: bool):
    dec = R.optimized_decoder(ref, model, cfg)
    max_len, prefix = int(c["max_len"]), int(c["prefix"])
    cache = ref.static_cache.StaticLfm2HybridConvCache(model.config, max_total_len=max_len, batch_size=1,
                                                       dtype=torch.bfloat16, device=DEV)
    assert isinstance(cache, StaticKVCache) == use_kernels
    for i in cfg.attn_layers:
        cache.key_cache[i].copy_(c[f"k_init_{i}"])
        cache.value_cache[i].copy_(c[f"v_init_{i}"])
    for i, kind in enumerate(cfg.layer_types):
        if kind != "full_attention":
            cache.conv_cache[i].copy_(c[f"conv_init_{i}"])
    mask = torch.full((1, 1, 1, max_len), float("-inf"), dtype=torch.bfloat16, device=DEV)
    mask[..., :prefix] = 0
    logits = []
    with torch.no_grad():
        for step in range(3):
            slot = prefix + step
            cache.set_write_position(slot)
            mask[..., slot] = 0
            logits.append(dec(input_ids=c["tokens"][step].view(1, 1).to(DEV),
                              position_ids=c["positions"][step].view(1, 1).to(DEV),
                              past_key_values=cache, causal_mask=mask,
                              cache_position=torch.tensor([slot], device=DEV)).clone())
    if use_kernels:
        assert cache.read_errors() == 0
    return logits, cache


def test_reference_decoder_on_the_kernels_matches_golden_and_triton(ref):
    c = load("decode_step")["tiny"]
    cfg = tiny_config()
    sd = synthetic_state_dict(cfg, seed=int(c["seed"]))
    model = R.stand_in_model(ref, cfg, sd, DEV)
    triton_logits, triton_cache = _tiny_run(ref, model, cfg, c, use_kernels=False)
    with R.installed_kernels(ref):
        logits, cache = _tiny_run(ref, model, cfg, c, use_kernels=True)
    prefix = int(c["prefix"])
    for step in range(3):
        close(logits[step], c[f"logits_{step}"], 0.02)
        close(logits[step], triton_logits[step], 0.02)
        assert torch.equal(logits[step].float().cpu().argmax(-1), c[f"logits_{step}"].float().argmax(-1))
    for i in cfg.attn_layers:
        for got, tri, init in ((cache.key_cache[i], triton_cache.key_cache[i], c[f"k_init_{i}"]),
                               (cache.value_cache[i], triton_cache.value_cache[i], c[f"v_init_{i}"])):
            got = got.cpu()
            # slots outside the three written ones keep their contents bit for bit
            assert torch.equal(got[:, :, :prefix], init[:, :, :prefix])
            assert torch.equal(got[:, :, prefix + 3:], init[:, :, prefix + 3:])
            close(got[:, :, prefix:prefix + 3], tri[:, :, prefix:prefix + 3].cpu(), 0.02)
    for i, kind in enumerate(cfg.layer_types):
        if kind != "full_attention":
            close(cache.conv_cache[i], c[f"conv_final_{i}"], 0.02)


def _engine_run(ref, model, cfg, dyn, prefill_len, tokens, positions):
    eng = R.engine(ref, model, cfg, max_new_tokens=256)
    R.capture(eng, dyn, prefill_len)
    out = []
    for i, (tok, pos) in enumerate(zip(tokens, positions)):
        # inference_engine.py:641-651
        eng.static_input_ids.copy_(tok.view(1, 1))
        eng.static_position_ids[0, 0] = pos
        step_offset = prefill_len + i
        eng.static_cache_position[0] = step_offset
        eng.static_cache.set_write_position(step_offset)
        eng.static_mask[:, :, :, step_offset] = 0.0
        eng.cuda_graph.replay()
        eng.static_cache.advance_position()
        out.append(eng.static_logits[:, -1, :].clone())
    torch.cuda.synchronize()
    return eng, out


def test_reference_engine_captures_and_replays_the_kernels_full_size(ref):
    cfg = LFM2Config()
    sd = synthetic_state_dict(cfg, seed=11, device=DEV)
    model = R.stand_in_model(ref, cfg, sd, DEV)
    g = torch.Generator().manual_seed(5)
    prefill_len = 40
    dyn = types.SimpleNamespace(
        key_cache=[torch.randn(1, cfg.num_key_value_heads, prefill_len, cfg.head_dim, generator=g).bfloat16().to(DEV)
                   if t == "full_attention" else torch.empty(0) for t in cfg.layer_types],
        value_cache=[torch.randn(1, cfg.num_key_value_heads, prefill_len, cfg.head_dim, generator=g).bfloat16()
                     .to(DEV) if t == "full_attention" else torch.empty(0) for t in cfg.layer_types],
        conv_cache=[torch.randn(1, cfg.hidden_size, cfg.conv_L_cache, generator=g).bfloat16().to(DEV)
                    for _ in cfg.layer_types])
    tokens = torch.randint(cfg.audio_tokens_start, cfg.vocab_size, (8,), generator=g).to(DEV)
    positions = (prefill_len + torch.arange(8) // cfg.tokens_per_frame).to(DEV)
    eng_t, triton_logits = _engine_run(ref, model, cfg, dyn, prefill_len, tokens, positions)
    assert type(eng_t.static_cache) is ref.static_cache.StaticLfm2HybridConvCache
    del eng_t
    with R.installed_kernels(ref):
        eng, logits = _engine_run(ref, model, cfg, dyn, prefill_len, tokens, positions)
        assert type(eng.static_cache) is StaticKVCache
        assert eng.static_cache.read_errors() == 0
    n_clear = 0
    for got, want in zip(logits, triton_logits):
        close(got, want, 0.05)
        cos = torch.nn.functional.cosine_similarity(got.float().flatten(), want.float().flatten(), dim=0)
        assert float(cos) > 0.999
        n_clear += same_argmax_where_clear(got, want)
    assert n_clear >= 4


def test_decoder_teacher_forced_against_the_reference_triton_engine(ref):
    """This library's decode step against the reference's own Triton + CUDA-graph
    engine, full-size model, 32 steps from the same cache state, both fed the
    reference's greedy tokens: logits within 5 % of the largest logit, cosine >
    0.999, and the same argmax on every step whose top-2 margin is clear."""
    from kani_tts_b200.decode import FusedDecoder
    cfg = LFM2Config()
    sd = synthetic_state_dict(cfg, seed=23, device=DEV)
    g = torch.Generator().manual_seed(24)
    prefill_len, n = 40, 32
    dyn = types.SimpleNamespace(
        key_cache=[torch.randn(1, cfg.num_key_value_heads, prefill_len, cfg.head_dim, generator=g).bfloat16().to(DEV)
                   if t == "full_attention" else torch.empty(0) for t in cfg.layer_types],
        value_cache=[torch.randn(1, cfg.num_key_value_heads, prefill_len, cfg.head_dim, generator=g).bfloat16()
                     .to(DEV) if t == "full_attention" else torch.empty(0) for t in cfg.layer_types],
        conv_cache=[torch.randn(1, cfg.hidden_size, cfg.conv_L_cache, generator=g).bfloat16().to(DEV)
                    for _ in cfg.layer_types])
    model = R.stand_in_model(ref, cfg, sd, DEV)
    eng = R.engine(ref, model, cfg, max_new_tokens=256)
    R.capture(eng, dyn, prefill_len)
    od = eng.optimized_decoder
    positions = (prefill_len + torch.arange(n) // cfg.tokens_per_frame).to(DEV)
    tok = torch.tensor([[cfg.audio_tokens_start + 5]], device=DEV)
    inputs, ref_logits = [], []
    for i in range(n):                                   # inference_engine.py:641-651, greedy choice
        inputs.append(tok.clone())
        eng.static_input_ids.copy_(tok)
        eng.static_position_ids[0, 0] = positions[i]
        eng.static_cache_position[0] = prefill_len + i
        eng.static_cache.set_write_position(prefill_len + i)
        eng.static_mask[:, :, :, prefill_len + i] = 0.0
        eng.cuda_graph.replay()
        eng.static_cache.advance_position()
        lg = eng.static_logits[:, -1, :].clone()
        ref_logits.append(lg)
        tok = od.reduced_to_full[lg.argmax(-1)].view(1, 1)
    del eng
    dec = FusedDecoder(cfg, sd, DEV, batch=1, max_len=512)
    for i in cfg.attn_layers:
        dec.k_cache[i][:, :, :prefill_len].copy_(dyn.key_cache[i])
        dec.v_cache[i][:, :, :prefill_len].copy_(dyn.value_cache[i])
    for i in dec.conv_state:
        dec.conv_state[i].copy_(dyn.conv_cache[i])
    n_clear = 0
    for i in range(n):
        slot = torch.tensor([prefill_len + i], device=DEV)
        got = dec.step_logits(inputs[i], positions[i:i + 1], slot, slot + 1)[:, -1, :]
        close(got, ref_logits[i], 0.05)
        cos = torch.nn.functional.cosine_similarity(got.float().flatten(), ref_logits[i].float().flatten(), dim=0)
        assert float(cos) > 0.999
        n_clear += same_argmax_where_clear(got, ref_logits[i])
    assert n_clear >= n // 3
    assert int(dec.err_flag.item()) == 0
