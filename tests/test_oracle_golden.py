"""Pin the CPU oracle to the reference: every oracle function against the golden
vectors that tests/golden/make_golden.py produced by running the reference's
own Triton kernels, static cache, rotary module and position code."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from golden_io import load
from oracle import kani_oracle as O

from kani_tts_b200 import positions as P


def _max_ulp(a, b) -> int:
    return int(O.ulp_distance(a, b).max()) if a.numel() else 0


@pytest.mark.parametrize("case", ["hidden_bf16", "decode_bf16", "qnorm_bf16", "knorm_bf16", "odd_bf16"])
def test_rms_norm_oracle_vs_triton(case):
    c = load("triton_rms_norm")[case]
    # the interpreter truncates on the bf16 store; with that store the oracle's
    # fp32 arithmetic reproduces it (only the sum-of-squares order differs)
    y = O.rms_norm_ref(c["x"], c["w"], float(c["eps"]), rounding="trunc")
    d = O.ulp_distance(y, c["y"])
    assert int(d.max()) <= 1
    assert float((d == 0).float().mean()) > 0.999
    # nearest-even (the hardware store) is within one ULP of the truncated value
    assert _max_ulp(O.rms_norm_ref(c["x"], c["w"], float(c["eps"])), c["y"]) <= 1


def test_rms_norm_fp32_reference_stores_bf16_values():
    """The reference kernel writes bf16-rounded values into an fp32 tensor."""
    c = load("triton_rms_norm")["fp32_storage"]
    assert c["y"].dtype == torch.float32
    assert torch.equal(c["y"], c["y"].to(torch.bfloat16).float())
    y = O.rms_norm_ref_storage(c["x"], c["w"], float(c["eps"]), rounding="trunc")
    assert _max_ulp(y.to(torch.bfloat16), c["y"].to(torch.bfloat16)) <= 1
    # the true-fp32 result is within one bf16 ULP of the (truncated) stored values
    yt = O.rms_norm_ref(c["x"], c["w"], float(c["eps"]))
    assert torch.allclose(yt, c["y"], rtol=2 ** -7, atol=0)


def test_add_rms_norm_fp32_vs_hf_eager():
    c = load("add_rms_norm")["config1_fp32_hf"]
    y, h = O.add_rms_norm_ref(c["x"], c["r"], c["w"], float(c["eps"]))
    assert torch.equal(h, c["h"])
    rel = ((y - c["y"]).abs() / c["y"].abs().clamp_min(1e-30)).max()
    assert float(rel) <= 1e-5


def test_add_rms_norm_bf16_vs_eager_add_plus_triton():
    c = load("add_rms_norm")["decode_bf16_triton"]
    y, h = O.add_rms_norm_ref(c["x"], c["r"], c["w"], float(c["eps"]), rounding="trunc")
    assert torch.equal(h, c["h"])          # the add is bit-exact
    assert _max_ulp(y, c["y"]) <= 1


@pytest.mark.parametrize("case", ["rows4_bf16", "decode_bf16", "odd_bf16"])
def test_silu_mul_oracle_vs_triton(case):
    c = load("triton_silu_mul")[case]
    y = O.silu_mul_ref(c["gate_up"], rounding="trunc")
    d = O.ulp_distance(y, c["y"])
    assert int(d.max()) <= 1
    assert float((d == 0).float().mean()) > 0.999
    assert _max_ulp(O.silu_mul_ref(c["gate_up"]), c["y"]) <= 1


@pytest.mark.parametrize("case", ["alpha0", "alpha1", "alpha2"])
def test_inv_freq_oracle_and_host_vs_reference(case):
    c = load("inv_freq")[case]
    args = (int(c["head_dim"]), float(c["theta"]), float(c["alpha_weight"]))
    assert torch.equal(O.learnable_inv_freq_ref(*args), c["inv_freq"])
    assert torch.equal(P.learnable_inv_freq(*args), c["inv_freq"])


@pytest.mark.parametrize("case", ["pos0", "pos1", "pos777", "pos2047"])
def test_rope_oracle_vs_triton(case):
    c = load("triton_rope")[case]
    cos, sin = O.rope_cos_sin_ref(c["inv_freq"], int(c["pos"]))
    assert torch.equal(cos, c["cos"]) and torch.equal(sin, c["sin"])
    # rotate-half with separately rounded fp32 products is what the interpreter computes
    assert torch.equal(O.rope_ref(c["q"], c["cos"], c["sin"], rounding="trunc"), c["q_out"])
    assert torch.equal(O.rope_ref(c["k"], c["cos"], c["sin"], rounding="trunc"), c["k_out"])
    assert _max_ulp(O.rope_ref(c["q"], c["cos"], c["sin"]), c["q_out"]) <= 1


@pytest.mark.parametrize("case", ["pos0", "pos777", "pos2047"])
def test_fused_rope_kv_oracle_composes_reference_steps(case):
    """rope_kv_write_ref (no norm, no table) == Triton RoPE + scatter_ KV write."""
    c = load("triton_rope")[case]
    q = c["q"].reshape(1, 16, 64)
    k = c["k"].reshape(1, 8, 64)
    v = torch.randn(1, 8, 64, generator=torch.Generator().manual_seed(3)).bfloat16()
    kc = torch.zeros(1, 8, 2048, 64, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    slot = int(c["pos"])
    q_rot, flags = O.rope_kv_write_ref(q, k, v, c["inv_freq"], torch.tensor([slot]), kc, vc,
                                       torch.tensor([slot]))
    assert flags == 0
    # nearest-even store: equal to the Triton RoPE on the same cos/sin rows
    assert torch.equal(q_rot.reshape(c["q_out"].shape), O.rope_ref(c["q"], c["cos"], c["sin"]))
    assert torch.equal(kc[0, :, slot], O.rope_ref(c["k"], c["cos"], c["sin"]).reshape(8, 64))
    assert _max_ulp(q_rot.reshape(c["q_out"].shape), c["q_out"]) <= 1
    assert torch.equal(vc[0, :, slot], v[0])
    others = torch.ones(kc.shape[2], dtype=torch.bool)
    others[slot] = False
    assert not bool(kc[:, :, others].any()) and not bool(vc[:, :, others].any())


@pytest.mark.parametrize("case", ["b1_slot5", "b2_slot0", "b1_last"])
def test_kv_write_oracle_vs_static_cache(case):
    c = load("static_cache_update")[case]
    kc, vc = c["k_prev"].clone(), c["v_prev"].clone()
    O.kv_write_ref(kc, vc, c["k"], c["v"], int(c["slot"]))
    assert torch.equal(kc, c["k_cache"]) and torch.equal(vc, c["v_cache"])


@pytest.mark.parametrize("case", ["docstring_step0", "docstring_step1", "mixed_step1"])
def test_frame_positions_vs_reference(case):
    c = load("frame_positions")[case]
    args = (int(c["audio_tokens_start"]), int(c["tokens_per_frame"]), float(c["audio_step"]))
    ref = c["positions"].numpy()
    assert np.array_equal(O.frame_level_positions_ref(c["input_ids"].numpy(), *args), ref)
    assert np.array_equal(P.frame_level_positions(c["input_ids"], *args).float().numpy(), ref)


def test_frame_positions_docstring_example_is_wrong_as_written():
    """model.py's docstring claims 3.0 for the last element at audio_step 0.5;
    the code gives 2.5 (the code is the definition)."""
    c = load("frame_positions")["docstring_step1"]
    assert float(c["positions"][0, -1]) == 2.5


def test_decode_schedule_known_answers():
    """model.py:1107-1117: 3 text tokens prefill at [0,1,2]; decode steps 1-4
    at position 3 and steps 5-8 at 4.  Step 1 runs on the host path with
    position = prefill length; the graph schedule covers steps 2.."""
    ids = np.array([[10, 11, 12]])
    assert np.array_equal(O.frame_level_positions_ref(ids, 64410), [[0, 1, 2]])
    sched = O.decode_position_schedule_ref(3, 7)
    steps = [3] + list(sched)              # steps 1..8
    assert steps == [3, 3, 3, 3, 4, 4, 4, 4]
    assert P.decode_position_schedule(3, 7).tolist() == list(sched)
    assert P.decode_write_slots(3, 4).tolist() == [4, 5, 6, 7]


def test_ulp_distance_helper():
    a = torch.tensor([1.0, -1.0, 0.0], dtype=torch.bfloat16)
    b = torch.tensor([1.0078125, -1.0078125, -0.0], dtype=torch.bfloat16)
    assert O.ulp_distance(a, b).tolist() == [1, 1, 0]
