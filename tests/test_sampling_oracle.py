"""CPU checks of the sampling oracle: pinned to the reference's own
``_sample_next_token`` outputs (tests/golden/sampling.npz), the Philox
generator against the Random123 known-answer vectors, and the host helpers of
the device sampler (no GPU calls)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from golden_io import load
from oracle import sampling_oracle as S

from kani_tts_b200 import sampling as KS

VOCAB, AUDIO_START, EOS = 80000, 64410, 7


def maps():
    n_red = 1 + VOCAB - AUDIO_START
    r2f = torch.cat([torch.tensor([EOS]), torch.arange(AUDIO_START, VOCAB)])
    f2r = torch.full((VOCAB,), -1, dtype=torch.long)
    f2r[EOS] = 0
    f2r[AUDIO_START:] = torch.arange(1, n_red)
    return r2f, f2r


def case_inputs(c):
    r2f, f2r = maps()
    reduced = bool(c["reduced"])
    v = c["logits"].shape[-1]
    seen = S.seen_from_history(c["history"], v, f2r if reduced else None)
    bias = None
    if not reduced:
        bias = torch.full((VOCAB,), float("-inf"), dtype=torch.bfloat16)
        bias[AUDIO_START:] = 0
        bias[EOS] = 0
    return seen, (r2f if reduced else None), bias


@pytest.mark.parametrize("name", ["config_defaults", "engine_defaults", "no_top_p", "deep_nucleus",
                                  "full_vocab_mask"])
def test_sample_ref_matches_reference_sampler(name):
    c = load("sampling")[name]
    seen, imap, bias = case_inputs(c)
    out = S.sample_ref(c["logits"], seen, float(c["repetition_penalty"]), float(c["temperature"]),
                       float(c["top_p"]), c["draws"], index_map=imap, logit_bias=bias)
    assert torch.equal(out["cand"][0], c["topk_indices"][0])
    assert torch.equal(out["values"][0], c["topk_values"][0])
    assert torch.equal(out["probs"][0], c["probs"][0])
    assert int(out["tokens"][0]) == int(c["token"][0])


def test_golden_cases_cover_the_nucleus_range():
    """The cases keep between one and all 256 candidates, and one keeps >= 100."""
    kept = {n: int((c["probs"][0] > 0).sum()) for n, c in load("sampling").items()}
    assert kept["no_top_p"] == 256
    assert max(kept.values()) >= 100
    assert min(kept.values()) >= 1


def test_philox_known_answers():
    """Random123 known-answer vectors for philox4x32_10."""
    ctr = np.array([[0, 0, 0, 0], [0xFFFFFFFF] * 4, [0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344]],
                   dtype=np.uint32)
    keys = [(0, 0), (0xFFFFFFFF, 0xFFFFFFFF), (0xA4093822, 0x299F31D0)]
    want = [[0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8],
            [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD],
            [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]]
    for c, k, w in zip(ctr, keys, want):
        assert S.philox4x32_10(c.reshape(1, 4), k)[0].tolist() == w


def test_exp_draws_are_positive_and_distinct_per_stream_and_step():
    a = S.exp_draws(seed=5, batch=3, step=0)
    b = S.exp_draws(seed=5, batch=3, step=1)
    assert a.shape == (3, 256) and bool((a > 0).all()) and bool(torch.isfinite(a).all())
    assert not torch.equal(a[0], a[1]) and not torch.equal(a, b)
    assert torch.equal(a, S.exp_draws(seed=5, batch=3, step=0))
    big = S.exp_draws(seed=1, batch=64, step=7)
    assert abs(float(big.mean()) - 1.0) < 0.03           # Exp(1): mean 1, 16384 draws
    assert float(big.max()) <= -np.log(2.0 ** -24) + 1e-3


def test_seen_bitmap_matches_history_mask():
    r2f, f2r = maps()
    g = torch.Generator().manual_seed(3)
    hist = torch.cat([torch.randint(0, 64400, (2, 50), generator=g),
                      r2f[torch.randint(0, r2f.numel(), (2, 40), generator=g)]], dim=1)
    hist[0, 0] = EOS
    v = r2f.numel()
    words = KS.seen_bitmap(hist, v, f2r)
    assert words.dtype == torch.int32 and words.shape == (2, (v + 31) // 32)
    bits = ((words.view(torch.int32).unsqueeze(-1).long() >> torch.arange(32)) & 1).view(2, -1)[:, :v].bool()
    assert torch.equal(bits, S.seen_from_history(hist, v, f2r))


def test_sampling_params_validation():
    with pytest.raises(ValueError):
        KS.SamplingParams(temperature=0.0)
    with pytest.raises(ValueError):
        KS.SamplingParams(top_k=300)
    with pytest.raises(ValueError):
        KS.SamplingParams(repetition_penalty=-1.0)
    p = KS.SamplingParams()
    assert (p.temperature, p.top_p, p.repetition_penalty, p.top_k) == (0.5, 0.85, 1.2, 256)
