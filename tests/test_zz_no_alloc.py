"""kani_head_argmax_noalloc, the entry point for callers that cannot allocate
device memory (another framework owns the allocator, a stream is being
captured, or a real-time thread must not block on cudaMalloc): its scratch is a
file-scope device array of the library.  Checked through the C ABI against
kani_head_argmax with a caller-provided scratch: identical tokens and logits on
two consecutive calls (the second call shows the array was left clean), and the
size limit refused before any launch.  Collected last, so a run that stops at
the first failure has run every other test first."""
from __future__ import annotations

import ctypes

import pytest
import torch

from kani_tts_b200 import _lib
from kani_tts_b200 import fused_kernels as K


def test_noalloc_size_check_rejects_before_any_launch():
    lib = _lib.load_library()
    before = lib.kani_launch_count()
    fake, n = ctypes.c_void_p(0x1000), ctypes.c_void_p(0)
    assert lib.kani_head_argmax_noalloc(1, fake, 1024, 64, 1024, fake, 1024, 100, n, n, 0, fake, 1, n) == -3
    assert lib.kani_head_argmax_noalloc(1, n, 0, 0, 1024, n, 1024, 100, n, n, 0, n, 1, n) == 0
    assert lib.kani_launch_count() == before


@pytest.mark.gpu
def test_noalloc_matches_scratch_entry_point_on_two_calls():
    dev = torch.device("cuda", 0)
    b, h, rows = 5, 1024, 15591
    g = torch.Generator().manual_seed(1400)
    weight = (0.05 * torch.randn(rows, h, generator=g)).to(torch.bfloat16).to(dev)
    imap = (torch.arange(rows) + 64409).to(dev)
    scratch = torch.zeros(b + 1, dtype=torch.long, device=dev)
    for _ in range(2):
        hidden = torch.randn(b, h, generator=g).to(torch.bfloat16).to(dev)
        la = torch.empty(b, rows, dtype=torch.bfloat16, device=dev)
        lb = torch.empty_like(la)
        ta = K.head_argmax(hidden, weight, imap, scratch=scratch, logits_out=la)
        tb = K.head_argmax_noalloc(hidden, weight, imap, logits_out=lb)
        torch.cuda.synchronize()
        assert torch.equal(ta, tb)
        assert torch.equal(la, lb)
    assert int(scratch.abs().sum()) == 0
