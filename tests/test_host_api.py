"""Host-side checks that need no GPU: the C-ABI library loads and exports every
symbol the header declares, argument validation rejects bad calls before any
launch, and the Python layer refuses CPU tensors (there is no CPU fallback)."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

from kani_tts_b200 import _lib
from kani_tts_b200 import fused_kernels as K

HEADER = Path(__file__).resolve().parent.parent / "include" / "kani_b200.h"


def header_symbols() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"KANI_API\s+[\w\s\*]+?\b(kani_\w+)\s*\(", text)


def test_header_declares_the_abi():
    syms = header_symbols()
    assert set(syms) == set(_lib.EXPORTED_SYMBOLS)
    assert len(syms) == len(set(syms))


def test_library_loads_and_exports_every_symbol():
    lib = _lib.load_library()
    raw = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in header_symbols():
        assert hasattr(raw, name), name
    assert lib.kani_version() == 100


def test_status_strings():
    assert _lib.status_string(0) == "ok"
    assert "invalid" in _lib.status_string(-1)
    assert "dtype" in _lib.status_string(-2)
    assert "not supported" in _lib.status_string(-3)


def _null():
    return ctypes.c_void_p(0)


def test_wait_limit_setter():
    lib = _lib.load_library()
    assert lib.kani_set_wait_limit(-1) == -1
    assert lib.kani_set_wait_limit(100) == 0
    assert lib.kani_set_wait_limit(0) == 0        # back to the default bound
    with pytest.raises(_lib.KaniError):
        _lib.set_wait_limit(-5)


def test_l2_prefetch_hint_setter():
    lib = _lib.load_library()
    a = ctypes.c_void_p(0x10000)
    assert lib.kani_set_l2_prefetch(a, -16, None, 0) == -1          # negative size
    assert lib.kani_set_l2_prefetch(None, 16, None, 0) == -1        # size without a range
    assert lib.kani_set_l2_prefetch(a, 24, None, 0) == -3           # not a multiple of 16 bytes
    assert lib.kani_set_l2_prefetch(ctypes.c_void_p(0x10008), 16, None, 0) == -3
    assert lib.kani_set_l2_prefetch(a, 4096, a, 1 << 20) == 0
    # the next GEMV entry point takes the hint even when it rejects its own
    # arguments (batch > 8 here), so a refused call leaves no stale hint behind
    fake = ctypes.c_void_p(0x1000)
    n = None
    assert lib.kani_gemv(1, fake, 1024, n, 0, n, 0, n, 1e-5, fake, 1024, 64, 1024, 9, 0, fake, 64, n) == -3
    assert lib.kani_set_l2_prefetch(None, 0, None, 0) == 0
    with pytest.raises(ValueError):
        _lib.set_l2_prefetch([(0x10000, 16)] * 3)
    with pytest.raises(_lib.KaniError):
        _lib.set_l2_prefetch([(0x10000, 17)])
    _lib.set_l2_prefetch(None)


def test_l2_prefetch_plan_covers_the_weights_once_per_step():
    """The decode step's prefetch ranges, launch by launch: each launch's ranges
    continue where the previous launch's ended, run `ahead` bytes past the end of
    its own weights, and over one step cover the weight buffer exactly once
    (the head's ranges wrap into the next step's first layers)."""
    from types import SimpleNamespace

    import torch
    from kani_tts_b200.decode import FusedDecoder

    arena = torch.empty(1 << 16, dtype=torch.bfloat16)       # 128 KB of "weights"
    total = arena.numel() * 2
    cuts = [0, 4096, 6144, 40960, 57344, 61440, 63488, 98304, 114688, total]
    for ahead in (16384, 40000 // 16 * 16, total, 3 * total):
        fake = SimpleNamespace(weight_arena=arena, weight_spans=list(zip(cuts[:-1], cuts[1:])),
                               l2_prefetch_ahead=ahead, _l2_plan=None)
        plan = FusedDecoder._l2_prefetch_plan(fake)
        assert len(plan) == len(cuts) - 1
        base = arena.data_ptr()
        covered = []
        for (_, end), ranges in zip(fake.weight_spans, plan):
            for addr, nbytes in ranges or ():
                assert nbytes > 0 and nbytes % 16 == 0 and (addr - base) % 16 == 0
                assert base <= addr and addr + nbytes <= base + total
                covered.append((addr - base, addr - base + nbytes))
        covered.sort()
        assert covered[0][0] == 0 and covered[-1][1] == total
        assert all(a[1] == b[0] for a, b in zip(covered, covered[1:]))   # no gap, no overlap
        first = plan[0][0]
        assert first[0] - base == min(ahead, total) % total or ahead >= total
    fake.l2_prefetch_ahead = 0
    fake._l2_plan = None
    assert FusedDecoder._l2_prefetch_plan(fake) == [None] * (len(cuts) - 1)


def test_weight_buffer_holds_the_projections_in_step_order():
    """The decoder's projection weights and padded head move into one buffer, in
    the order a decode step reads them; every tensor becomes a view of it with its
    values unchanged, and the spans tile the buffer with no gap."""
    from types import SimpleNamespace

    import torch
    from kani_tts_b200.decode import FusedDecoder

    g = torch.Generator().manual_seed(9)

    def w(r, c):
        return torch.randn(r, c, generator=g).to(torch.bfloat16)

    layers = [{"attn": False, "in_proj": w(12, 8), "out_proj": w(8, 8), "gate_up": w(16, 8), "down": w(8, 8)},
              {"attn": True, "qkv": w(16, 8), "o": w(8, 8), "gate_up": w(16, 8), "down": w(8, 8)}]
    want = [[v.clone() for k, v in L.items() if k != "attn"] for L in layers]
    head = w(6, 8)
    fake = SimpleNamespace(layers=layers, head_padded=head.clone(), num_reduced=5, dtype=torch.bfloat16,
                           device=torch.device("cpu"))
    FusedDecoder._pack_weights(fake)
    arena = fake.weight_arena
    order = [("in_proj", "out_proj", "gate_up", "down"), ("qkv", "o", "gate_up", "down")]
    spans = iter(fake.weight_spans)
    end = 0
    for L, keys, vals in zip(layers, order, want):
        for key in keys:
            t = L[key]
            a, b = next(spans)
            assert a == end and t.untyped_storage().data_ptr() == arena.untyped_storage().data_ptr()
            assert t.data_ptr() - arena.data_ptr() == a and b - a == t.numel() * 2
            end = b
        assert all(torch.equal(L[k], v) for k, v in zip([k for k in L if k != "attn"], vals))
    a, b = next(spans)
    assert a == end and b == arena.numel() * 2
    assert torch.equal(fake.head_padded, head) and fake.head.shape == (5, 8)
    assert fake.head.data_ptr() == fake.head_padded.data_ptr() == arena.data_ptr() + a


def test_abi_rejects_bad_arguments_without_launching():
    lib = _lib.load_library()
    before = lib.kani_launch_count()
    fake = ctypes.c_void_p(0x1000)       # never dereferenced: every call below returns early
    # negative sizes
    assert lib.kani_rms_norm(1, 1, fake, 8, fake, fake, 8, -1, 8, 1e-5, _null()) == -1
    assert lib.kani_silu_mul(1, fake, 16, fake, 8, 4, -8, _null()) == -1
    # null pointers
    assert lib.kani_rms_norm(1, 1, _null(), 8, fake, fake, 8, 4, 8, 1e-5, _null()) == -1
    assert lib.kani_add_rms_norm(1, 1, fake, 8, _null(), 8, fake, fake, 8, fake, 8, 4, 8, 1e-5,
                                 _null()) == -1
    # out and residual_out may not be the same buffer
    assert lib.kani_add_rms_norm(1, 1, fake, 8, fake, 8, fake, fake, 8, fake, 8, 4, 8, 1e-5,
                                 _null()) == -1
    # overlapping rows (stride < n)
    assert lib.kani_silu_mul(1, fake, 8, fake, 8, 4, 8, _null()) == -1
    # unknown dtype code
    assert lib.kani_rms_norm(7, 1, fake, 8, fake, fake, 8, 4, 8, 1e-5, _null()) == -2
    assert lib.kani_rms_norm(1, 9, fake, 8, fake, fake, 8, 4, 8, 1e-5, _null()) == -2
    # odd head_dim is unsupported (rotate-half needs pairs)
    assert lib.kani_rope_qk(1, fake, fake, fake, fake, fake, fake, 16, 8, 63, _null()) == -3
    # q/k norm weights must come together
    args = [1, 1, 1, 16, 8, 64, fake, 2048, fake, 2048, fake, 2048, fake, fake,
            fake, _null(), 1e-5, _null(), 0, _null(), 4, fake, 1024, 64,
            fake, fake, 8 * 2048 * 64, 2048 * 64, 64, 2048, fake, _null(), _null()]
    assert lib.kani_rope_kv_write(*args) == -1
    # missing KV write slots pointer is allowed (slot = token index); missing positions is not
    args[13] = _null()
    args[15] = fake
    assert lib.kani_rope_kv_write(*args) == -1
    assert lib.kani_kv_cache_write(1, fake, fake, 1, 8, 64, fake, fake, 16, _null(), 0, _null(),
                                   _null()) == -1
    # sampler: top_k outside [1, min(256, vocab)], non-positive temperature, NaN top_p,
    # a bitmap row shorter than the vocabulary, missing output
    n = _null()

    def sample(**kw):
        a = dict(dtype=1, logits=fake, rs=15591, b=2, v=15591, bias=n, seen=n, words=488, upd=1, rp=1.2,
                 t=0.5, top_p=0.85, k=256, imap=n, seed=0, step=n, draws=n, dout=n, pout=n, cout=n,
                 tok=fake, ts=1, stream=n)
        a.update(kw)
        return lib.kani_sample_tokens(*a.values())
    assert sample(k=257) == -1
    assert sample(k=0) == -1
    assert sample(v=100, rs=100, k=101) == -1
    assert sample(t=0.0) == -1
    assert sample(rp=0.0) == -1
    assert sample(top_p=float("nan")) == -1
    assert sample(seen=fake, words=487) == -1
    assert sample(tok=n) == -1
    assert sample(rs=100) == -1
    assert sample(dtype=5) == -2
    # the head with the final norm: no norm weight, or a residual the norm does not cover
    assert lib.kani_head_argmax_norm(1, fake, 1024, fake, 1024, n, 1e-5, 1, 1024, fake, 1024, 100, n, n, 0, fake,
                                     fake, 1, n) == -1
    # reduced head: batch above 8, fp32, hidden size not a multiple of 256, missing scratch
    assert lib.kani_head_argmax(1, fake, 1024, 9, 1024, fake, 1024, 100, n, n, 0, fake, fake, 1, n) == -3
    assert lib.kani_head_argmax(0, fake, 1024, 1, 1024, fake, 1024, 100, n, n, 0, fake, fake, 1, n) == -3
    assert lib.kani_head_argmax(1, fake, 1000, 1, 1000, fake, 1000, 100, n, n, 0, fake, fake, 1, n) == -1
    assert lib.kani_head_argmax(1, fake, 1024, 1, 1024, fake, 1024, 100, n, n, 0, n, fake, 1, n) == -1
    # tensor-core head: batch above 64, fp32, hidden size not a multiple of 64, missing scratch
    assert lib.kani_head_argmax_tc(1, fake, 1024, 65, 1024, fake, 1024, 100, n, n, 0, fake, fake, 1, n, n) == -3
    assert lib.kani_head_argmax_tc(0, fake, 1024, 9, 1024, fake, 1024, 100, n, n, 0, fake, fake, 1, n, n) == -3
    assert lib.kani_head_argmax_tc(1, fake, 1000, 9, 1000, fake, 1000, 100, n, n, 0, fake, fake, 1, n, n) == -3
    assert lib.kani_head_argmax_tc(1, fake, 1024, 9, 1024, fake, 1024, 100, n, n, 0, n, fake, 1, n, n) == -1
    # tensor-core GEMM: batch above 64, norm prologue above K = 1024, residual without a norm, silu n % 8
    assert lib.kani_gemm_tc(1, fake, 1024, n, 0, n, 0, n, 1e-5, fake, 1024, 64, 1024, 65, 0, fake, 64, n, n) == -3
    assert lib.kani_gemm_tc(1, fake, 2048, n, 0, n, 0, fake, 1e-5, fake, 2048, 64, 2048, 4, 0, fake, 64, n,
                            n) == -3
    assert lib.kani_gemm_tc(1, fake, 1024, fake, 1024, n, 0, n, 1e-5, fake, 1024, 64, 1024, 4, 0, fake, 64, n,
                            n) == -1
    assert lib.kani_gemm_tc(1, fake, 1024, n, 0, n, 0, fake, 1e-5, fake, 1024, 60, 1024, 4, 1, fake, 64, n,
                            n) == -3
    # fused GEMV: a residual without a norm, residual_out aliasing the residual, batch above 8, K unsupported
    assert lib.kani_gemv(1, fake, 1024, fake, 1024, n, 0, n, 1e-5, fake, 1024, 64, 1024, 1, 0, fake, 64, n) == -1
    assert lib.kani_gemv(1, fake, 1024, fake, 1024, fake, 1024, fake, 1e-5, fake, 1024, 64, 1024, 1, 0, fake, 64,
                         n) == -1
    assert lib.kani_gemv(1, fake, 1024, n, 0, n, 0, n, 1e-5, fake, 1024, 64, 1024, 9, 0, fake, 64, n) == -3
    assert lib.kani_gemv(1, fake, 2048, n, 0, n, 0, n, 1e-5, fake, 2048, 64, 2048, 1, 0, fake, 64, n) == -3
    # decode bookkeeping: tokens per frame below 1, missing step counter
    assert lib.kani_decode_advance(fake, fake, fake, 10, 10, fake, n, fake, fake, 0, 1.0, fake, fake, fake, 2,
                                   n) == -1
    assert lib.kani_decode_advance(fake, fake, fake, 10, 10, n, n, fake, fake, 4, 1.0, fake, fake, fake, 2, n) == -1
    # codec codes: too few frames for the tokens, missing outputs
    assert lib.kani_codec_codes(fake, 100, 2, 100, 64402, 64410, 4032, fake, 24, fake, fake, n) == -1
    assert lib.kani_codec_codes(fake, 100, 2, 100, 64402, 64410, 4032, n, 25, fake, fake, n) == -1
    # K-split reduce + add + RMSNorm: no splits, y aliasing residual_out, n not a multiple of 4,
    # overlapping splits
    assert lib.kani_reduce_add_rms_norm(1, 1, fake, 4096, 1024, 0, fake, 1024, fake, fake, 1024, fake, 1024, 4,
                                        1024, 1e-5, n) == -1
    assert lib.kani_reduce_add_rms_norm(1, 1, fake, 4096, 1024, 2, fake, 1024, fake, fake, 1024, fake, 1024, 4,
                                        1024, 1e-5, n) == -1
    assert lib.kani_reduce_add_rms_norm(1, 1, fake, 4096, 1024, 2, fake, 1022, fake, ctypes.c_void_p(0x2000), 1022,
                                        fake, 1022, 4, 1022, 1e-5, n) == -3
    assert lib.kani_reduce_add_rms_norm(1, 1, fake, 1024, 1024, 2, fake, 1024, fake, ctypes.c_void_p(0x2000), 1024,
                                        fake, 1024, 4, 1024, 1e-5, n) == -1
    assert lib.kani_launch_count() == before


def test_abi_zero_sized_calls_are_noops():
    lib = _lib.load_library()
    before = lib.kani_launch_count()
    n = _null()
    assert lib.kani_rms_norm(1, 1, n, 0, n, n, 0, 0, 1024, 1e-5, n) == 0
    assert lib.kani_add_rms_norm(1, 1, n, 0, n, 0, n, n, 0, n, 0, 0, 1024, 1e-5, n) == 0
    assert lib.kani_silu_mul(1, n, 0, n, 0, 0, 4608, n) == 0
    assert lib.kani_rope_qk(1, n, n, n, n, n, n, 0, 0, 64, n) == 0
    assert lib.kani_kv_cache_write(1, n, n, 0, 8, 64, n, n, 16, n, 0, n, n) == 0
    assert lib.kani_rope_kv_write(1, 0, 1, 16, 8, 64, n, 0, n, 0, n, 0, n, n, n, n, 1e-5, n, 0, n, 4,
                                  n, 0, 0, n, n, 0, 0, 0, 16, n, n, n) == 0
    assert lib.kani_sample_tokens(1, n, 0, 0, 15591, n, n, 0, 1, 1.2, 0.5, 0.85, 256, n, 0, n, n, n, n, n,
                                  n, 1, n) == 0
    assert lib.kani_head_argmax(1, n, 0, 0, 1024, n, 1024, 15591, n, n, 0, n, n, 1, n) == 0
    assert lib.kani_head_argmax_tc(1, n, 0, 0, 1024, n, 1024, 15591, n, n, 0, n, n, 1, n, n) == 0
    assert lib.kani_gemm_tc(1, n, 0, n, 0, n, 0, n, 1e-5, n, 1024, 64, 1024, 0, 0, n, 64, n, n) == 0
    assert lib.kani_codec_codes(n, 0, 0, 100, 64402, 64410, 4032, n, 25, n, n, n) == 0
    assert lib.kani_launch_count() == before


@pytest.mark.parametrize("call", [
    lambda: K.fused_rms_norm(torch.zeros(2, 8), torch.ones(8)),
    lambda: K.fused_add_rms_norm(torch.zeros(2, 8), torch.zeros(2, 8), torch.ones(8)),
    lambda: K.fused_silu_mul(torch.zeros(2, 16)),
    lambda: K.fused_rope(torch.zeros(1, 2, 1, 8), torch.zeros(1, 1, 1, 8), torch.zeros(8), torch.zeros(8)),
    lambda: K.sample_tokens(torch.zeros(2, 300)),
    lambda: K.head_argmax(torch.zeros(1, 256), torch.zeros(10, 256)),
    lambda: K.codec_codes(torch.zeros(1, 8, dtype=torch.long), 64402, 64410),
])
def test_cpu_tensors_are_refused(call):
    with pytest.raises(ValueError, match="CUDA"):
        call()


def test_missing_library_fails_loudly(tmp_path, monkeypatch):
    monkeypatch.setattr(_lib, "_lib", None)
    with pytest.raises(ImportError, match="no fallback"):
        _lib.load_library(tmp_path / "absent.so")
