"""CPU checks of the output-side oracle: the codec-code mapping pinned to the
reference's own ``get_nano_codes`` (tests/golden/codec_codes.npz) and the
reduced-head greedy choice on small cases."""
from __future__ import annotations

import pytest
import torch

from golden_io import load
from oracle import kani_oracle as O

EOS, AUDIO_START = 64402, 64410


@pytest.mark.parametrize("name", ["whole_frames", "partial_frame", "one_frame", "negative_code", "no_frame"])
def test_codec_codes_ref_matches_reference(name):
    c = load("codec_codes")[name]
    codes, frames, status = O.codec_codes_ref(c["generated"].view(1, -1), EOS, AUDIO_START)
    if "error" in c:
        want = {"Invalid audio tokens!": 1, "No complete audio frames generated!": 2}[c["error"]]
        assert int(status[0]) & want
    else:
        nf = int(c["frames"][0])
        assert int(frames[0]) == nf and int(status[0]) == 0
        assert torch.equal(codes[0, :, :nf], c["codes"][0])
        assert bool((codes[0, :, nf:] == -1).all())


def test_codec_codes_ref_flags_a_missing_end_of_speech():
    toks = torch.tensor([[AUDIO_START + 1, AUDIO_START + 4032 + 2, AUDIO_START + 8064 + 3, AUDIO_START + 12096 + 4]])
    codes, frames, status = O.codec_codes_ref(toks, EOS, AUDIO_START)
    assert int(frames[0]) == 1 and int(status[0]) == 4
    assert codes[0, :, 0].tolist() == [1, 2, 3, 4]


def test_head_argmax_ref_picks_the_first_maximum():
    w = torch.zeros(6, 256, dtype=torch.bfloat16)
    w[2, 0] = 1.0
    w[4, 0] = 1.0
    h = torch.zeros(2, 256, dtype=torch.bfloat16)
    h[0, 0] = 1.0
    imap = torch.tensor([7, 100, 101, 102, 103, 104])
    tok, logits = O.head_argmax_ref(h, w, imap)
    assert tok.tolist() == [101, 7]          # ties: the lower row; all-zero row 1 -> row 0
    assert logits.dtype == torch.bfloat16 and logits.shape == (2, 6)
