"""The timeout path of the kernels' bounded on-chip waits, made to run for real.

The bulk RoPE + KV-write kernel and decode attention wait on TMA mbarrier
phases, bounded by default at about 1 s.  ``kani_set_wait_limit`` bounds the
first wait on each stage to a few clock cycles with the suspend hint off, so
the wait gives up while the copies are still in flight (nothing is withheld:
the copies land a microsecond later).  Each kernel must then OR
KANI_FLAG_TIMEOUT into its error flag, let its own copies land, return, and
leave the context usable: the next call with the default bound, on the same
buffers, matches the oracle exactly as a fresh call does.
"""
from __future__ import annotations

import pytest
import torch

from oracle import kani_oracle as O

from kani_tts_b200 import _lib, fused_kernels as K, positions as P

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
LIMIT_CYCLES = 4


def rnd(shape, seed, std=1.0):
    return (std * torch.randn(shape, generator=torch.Generator().manual_seed(seed))).to(torch.bfloat16)


@pytest.fixture
def short_waits():
    _lib.read_and_clear_errors(DEV)
    _lib.set_wait_limit(LIMIT_CYCLES)
    try:
        yield
    finally:
        _lib.set_wait_limit(0)


def _rope_call(s, kc, vc, flag):
    t = s["q"].shape[0]
    return K.fused_rope_kv_write(s["q"].view(1, t, 16, 64), s["k"].view(1, t, 8, 64), s["v"].view(1, t, 8, 64),
                                 s["inv"], s["pos"], kc, vc, s["pos"], frame_table=s["table"], tokens_per_frame=4,
                                 err_flag=flag)


def _rope_inputs(t):
    s = {"q": rnd((t, 16, 64), 1), "k": rnd((t, 8, 64), 2), "v": rnd((t, 8, 64), 3),
         "table": rnd((1024, 64), 4, 0.02), "inv": P.learnable_inv_freq(64, 1e6, 0.0),
         "pos": torch.arange(t, dtype=torch.long)}
    return {k: v.to(DEV) for k, v in s.items()}, s


def test_bulk_rope_wait_times_out_and_the_next_call_is_exact(short_waits):
    t = 4096                                   # the bulk kernel (>= 256 tokens), 1024 CTAs
    d, c = _rope_inputs(t)
    kc = torch.zeros(1, 8, t, 64, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    flag = torch.zeros(1, dtype=torch.int32, device=DEV)
    _rope_call(d, kc, vc, flag)
    torch.cuda.synchronize()
    assert int(flag.item()) & _lib.KANI_FLAG_TIMEOUT
    _lib.set_wait_limit(0)                     # default bound again; same buffers
    flag.zero_()
    q = _rope_call(d, kc, vc, flag)
    torch.cuda.synchronize()
    assert int(flag.item()) == 0
    kr = torch.zeros(1, 8, t, 64, dtype=torch.bfloat16)
    vr = torch.zeros_like(kr)
    qr, flags = O.rope_kv_write_ref(c["q"], c["k"], c["v"], c["inv"], c["pos"], kr, vr, c["pos"],
                                    frame_table=c["table"], tokens_per_frame=4)
    assert flags == 0
    assert torch.equal(vc.cpu(), vr)           # V rows are copies: exact
    # the rotation with in-kernel cos/sin: the RoPE tolerance of the parity tests
    for got, want in ((q.reshape(qr.shape).cpu(), qr), (kc.cpu(), kr)):
        d_ulp = O.ulp_distance(got, want)
        ok = (d_ulp <= 1) | ((got.float() - want.float()).abs()
                             <= want.float().abs().amax(-1, keepdim=True) * 2.0 ** -8)
        assert bool(ok.all())


# 8 streams run the 4-warp shape (64-key tiles, 3 stages), 2 streams the 8-warp
# shape (128-key tiles, 2 stages) in 8-CTA clusters
@pytest.mark.parametrize("lens", [[1629, 100, 2048, 1, 700, 1500, 65, 900], [1629, 2048]])
def test_decode_attention_wait_times_out_and_the_next_call_is_exact(short_waits, lens):
    b, hq, hk, dh, s_len = len(lens), 16, 8, 64, 2048
    q = rnd((b, hq, dh), 11)
    kc, vc = rnd((b, hk, s_len, dh), 12), rnd((b, hk, s_len, dh), 13)
    kv_len = torch.tensor(lens, dtype=torch.long)
    flag = torch.zeros(1, dtype=torch.int32, device=DEV)
    qd, kd, vd, ld = q.to(DEV), kc.to(DEV), vc.to(DEV), kv_len.to(DEV)
    out = torch.empty(b, hq, dh, dtype=torch.bfloat16, device=DEV)
    K.decode_attention(qd, kd, vd, ld, out=out, err_flag=flag)
    torch.cuda.synchronize()
    assert int(flag.item()) & _lib.KANI_FLAG_TIMEOUT
    _lib.set_wait_limit(0)
    flag.zero_()
    K.decode_attention(qd, kd, vd, ld, out=out, err_flag=flag)
    fresh = K.decode_attention(qd, kd, vd, ld)
    torch.cuda.synchronize()
    assert int(flag.item()) == 0
    assert torch.equal(out, fresh)
    ref = O.decode_attention_ref(q, kc, vc, kv_len, dh ** -0.5)
    err = (out.cpu().float() - ref.float()).abs()
    assert bool(((O.ulp_distance(out.cpu(), ref) <= 2) | (err <= 2e-5)).all())
