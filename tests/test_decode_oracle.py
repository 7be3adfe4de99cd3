"""The oracle decode step against the reference decoder itself (CPU).

tests/golden/decode_step.npz holds three decode steps of the reference
``OptimizedDecoder`` (kani_tts/optimized_decode.py) on a tiny synthetic
LFM2, run with the reference's Triton kernels under the CPU interpreter.
With the interpreter's truncating bf16 store, the oracle restatement
reproduces those logits and cache contents."""
from __future__ import annotations

import torch

from golden_io import load
from oracle import kani_oracle as O
from oracle.decode_oracle import OracleDecoder

from kani_tts_b200.model import synthetic_state_dict, tiny_config


def _setup(rounding):
    c = load("decode_step")["tiny"]
    cfg = tiny_config()
    sd = synthetic_state_dict(cfg, seed=int(c["seed"]))
    checksum = sum(float(v.float().abs().sum()) for v in sd.values())
    assert abs(checksum - float(c["weight_checksum"])) < 1e-6 * abs(checksum), "weight generator drifted"
    dec = OracleDecoder(cfg, sd, batch=1, max_len=int(c["max_len"]), rounding=rounding)
    for i in cfg.attn_layers:
        dec.k_cache[i].copy_(c[f"k_init_{i}"])
        dec.v_cache[i].copy_(c[f"v_init_{i}"])
    for i in dec.conv_state:
        dec.conv_state[i].copy_(c[f"conv_init_{i}"])
    return c, cfg, dec


def run_steps(c, dec):
    prefix, max_len = int(c["prefix"]), int(c["max_len"])
    mask = torch.full((1, 1, 1, max_len), float("-inf"), dtype=torch.bfloat16)
    mask[..., :prefix] = 0
    out = []
    for step in range(3):
        slot = prefix + step
        mask[..., slot] = 0
        out.append(dec.step(c["tokens"][step].view(1, 1), c["positions"][step:step + 1],
                            torch.tensor([slot]), mask))
    return out


def test_oracle_decoder_reproduces_reference_decoder():
    c, cfg, dec = _setup("trunc")
    logits = run_steps(c, dec)
    for step in range(3):
        d = O.ulp_distance(logits[step], c[f"logits_{step}"])
        assert int(d.max()) <= 1, (step, int(d.max()))
        assert float((d == 0).float().mean()) > 0.95
    for i in cfg.attn_layers:
        assert int(O.ulp_distance(dec.k_cache[i], c[f"k_final_{i}"]).max()) <= 1
        assert torch.equal(dec.v_cache[i], c[f"v_final_{i}"])
    for i in dec.conv_state:
        assert torch.equal(dec.conv_state[i], c[f"conv_final_{i}"])


def test_oracle_decoder_nearest_even_is_close_to_reference():
    c, _, dec = _setup("rne")
    logits = run_steps(c, dec)
    for step in range(3):
        ref = c[f"logits_{step}"].float()
        assert float((logits[step].float() - ref).abs().max()) <= 0.02 * float(ref.abs().max())
