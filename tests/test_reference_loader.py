"""The reference package installed in baseline/_ref imports through
baseline/reference.py, its decoder and engine build around the stand-in model,
and the drop-in rebinding (kani_tts_b200.install) is applied and undone.  CPU
only: no kernel runs here (tests/test_gpu_dropin.py runs them)."""
from __future__ import annotations

import pytest
import torch

from baseline import reference as R

from kani_tts_b200.model import tiny_config, synthetic_state_dict
from kani_tts_b200.static_cache import StaticKVCache

pytestmark = pytest.mark.skipif(not R.available(), reason=R.why_unavailable())


@pytest.fixture(scope="module")
def ref():
    math_sdp = torch.backends.cuda.math_sdp_enabled()
    yield R.import_reference()
    torch.backends.cuda.enable_math_sdp(math_sdp)


def test_manifest_matches_the_installed_files(ref):
    R._check_manifest()
    assert ref.optimized_decode.__file__.startswith(str(R.PKG_DIR))


def test_decoder_and_engine_build_on_the_stand_in(ref):
    cfg = tiny_config()
    sd = synthetic_state_dict(cfg, seed=1234)
    eng = R.engine(ref, R.stand_in_model(ref, cfg, sd, "cpu"), cfg, max_new_tokens=16)
    od = eng.optimized_decoder
    assert od.num_reduced == cfg.num_reduced
    assert od.attn_layer_indices == cfg.attn_layers
    # inv_freq from the reference's LearnableRotaryEmbedding equals this package's host copy
    from kani_tts_b200.positions import learnable_inv_freq
    for i in cfg.attn_layers:
        want = learnable_inv_freq(cfg.head_dim, cfg.rope_theta, sd[f"model.learnable_rope_layers.{i}.alpha_weight"])
        assert torch.equal(od.inv_freqs[i].cpu(), want)


def test_install_rebinds_and_restores(ref):
    from kani_tts_b200 import fused_kernels
    od = ref.optimized_decode
    before = od.fused_rms_norm
    with R.installed_kernels(ref) as patched:
        assert od.fused_rms_norm is fused_kernels.fused_rms_norm
        assert od.fused_silu_mul is fused_kernels.fused_silu_mul
        assert od.fused_rope is fused_kernels.fused_rope
        assert ref.static_cache.StaticLfm2HybridConvCache is StaticKVCache
        assert ref.inference_engine.StaticLfm2HybridConvCache is StaticKVCache
        assert "kani_tts.optimized_decode.fused_rope" in patched
    assert od.fused_rms_norm is before
    assert ref.inference_engine.StaticLfm2HybridConvCache is ref.static_cache.StaticLfm2HybridConvCache
