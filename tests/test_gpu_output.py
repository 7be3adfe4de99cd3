"""GPU parity of the output-side kernels: the reduced head with the greedy choice
(``kani_head_argmax``) and the codec-code mapping (``kani_codec_codes``).

Tolerances:
  * head logits: within 1 ULP of the oracle's float64 dot product rounded once
    (fp32 accumulation in another order), or within 2^-16 x sum |h w| where
    the products cancel towards zero; >= 99 % identical;
  * head token: identical to the first maximum of the kernel's own logits,
    and to the oracle's token whenever the two logit rows are identical;
  * codec codes, frame counts and status words: identical.
"""
from __future__ import annotations

import pytest
import torch

from golden_io import load
from oracle import kani_oracle as O

from kani_tts_b200 import fused_kernels as K
from kani_tts_b200._lib import KaniError

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
EOS, AUDIO_START = 64402, 64410


def rnd(shape, seed, dtype=torch.bfloat16, std=1.0):
    g = torch.Generator().manual_seed(seed)
    return (std * torch.randn(shape, generator=g)).to(dtype)


def check_head(hidden, weight, imap, tok, logits):
    ref_tok, ref_logits = O.head_argmax_ref(hidden, weight, imap)
    d = O.ulp_distance(logits.cpu(), ref_logits)
    # 1 ULP, or an fp32-accumulation bound where the products cancel towards zero
    mag = hidden.reshape(-1, hidden.shape[-1]).double().abs() @ weight.double().abs().T
    err = (logits.cpu().double() - ref_logits.double()).abs()
    ok = (d <= 1) | (err <= mag * 2.0 ** -16)
    assert bool(ok.all()), f"{int((~ok).sum())} logits outside tolerance, max ULP {int(d.max())}"
    assert float((d == 0).float().mean()) >= 0.99
    own = torch.argmax(logits.cpu().float(), dim=-1)
    want = imap[own] if imap is not None else own
    assert torch.equal(tok.cpu(), want)
    same = (d == 0).all(dim=-1)
    assert torch.equal(tok.cpu()[same], ref_tok[same])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("b,h,rows", [(1, 1024, 15591), (3, 1024, 15591), (8, 1024, 4000), (2, 512, 37),
                                      (5, 2048, 1000)])
def test_head_argmax_vs_oracle(dtype, b, h, rows):
    hidden = rnd((b, h), 1300 + b, dtype)
    weight = rnd((rows, h), 1301 + rows, dtype, std=0.05)
    imap = torch.arange(rows, dtype=torch.long) * 3 + 11
    logits = torch.empty(b, rows, dtype=dtype, device=DEV)
    tok = K.head_argmax(hidden.to(DEV), weight.to(DEV), imap.to(DEV), logits_out=logits)
    check_head(hidden, weight, imap, tok, logits)


@pytest.mark.parametrize("b,res", [(1, True), (3, True), (4, False), (8, True)])
def test_head_argmax_norm_equals_the_normed_gemv(b, res):
    """kani_head_argmax_norm (the final residual add + RMSNorm folded into the
    head): its logits are kani_gemv's with the same norm weight and residual, bit
    for bit (one input prologue, one accumulation order), its token the first
    maximum of them, mapped; and the scratch is left zero."""
    h, rows = 1024, 15591
    x = rnd((b, 1, h), 1340 + b)
    r = rnd((b, 1, h), 1341 + b) if res else None
    nw = (1.0 + 0.1 * rnd((h,), 1342, torch.float32)).to(torch.bfloat16)
    w = rnd((rows, h), 1343, std=0.05).to(DEV)
    imap = (torch.arange(rows, dtype=torch.long) * 5 + 3).to(DEV)
    logits = torch.empty(b, rows, dtype=torch.bfloat16, device=DEV)
    scratch = torch.zeros(b + 1, dtype=torch.int64, device=DEV)
    tok = K.head_argmax(x.to(DEV), w, imap, scratch=scratch, logits_out=logits, norm_weight=nw.to(DEV),
                        residual=r.to(DEV) if r is not None else None, eps=1e-5)
    want = K.gemv(x.to(DEV), w, norm_weight=nw.to(DEV), residual=r.to(DEV) if r is not None else None,
                  residual_out=torch.empty(b, 1, h, dtype=torch.bfloat16, device=DEV) if r is not None else None,
                  eps=1e-5).reshape(b, rows)
    assert torch.equal(logits, want)
    assert torch.equal(tok, imap[torch.argmax(want.float(), dim=-1)])
    assert int(scratch.abs().sum()) == 0
    with pytest.raises(ValueError):
        K.head_argmax(x.to(DEV), w, residual=x.to(DEV))            # an add without the norm


def test_head_argmax_scratch_is_left_clean_and_reused():
    """Two calls on one scratch buffer (the second sees what the first left) and a
    graph replayed with new hidden states; the scratch is all zero afterwards."""
    b, h, rows = 4, 1024, 15591
    weight = rnd((rows, h), 1310, std=0.05).to(DEV)
    scratch = torch.zeros(b + 1, dtype=torch.long, device=DEV)
    for seed in (1311, 1312):
        hidden = rnd((b, h), seed)
        logits = torch.empty(b, rows, dtype=torch.bfloat16, device=DEV)
        tok = K.head_argmax(hidden.to(DEV), weight, scratch=scratch, logits_out=logits)
        check_head(hidden, weight.cpu(), None, tok, logits)
        assert int(scratch.abs().sum()) == 0
    hid = torch.zeros(b, h, dtype=torch.bfloat16, device=DEV)
    out = torch.zeros(b, dtype=torch.long, device=DEV)
    logits = torch.empty(b, rows, dtype=torch.bfloat16, device=DEV)
    s = torch.cuda.Stream(device=DEV)
    s.wait_stream(torch.cuda.current_stream(DEV))
    with torch.cuda.stream(s):
        K.head_argmax(hid, weight, scratch=scratch, logits_out=logits, out=out)
    torch.cuda.current_stream(DEV).wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        K.head_argmax(hid, weight, scratch=scratch, logits_out=logits, out=out)
    for seed in (1313, 1314, 1315):
        hidden = rnd((b, h), seed)
        hid.copy_(hidden)
        graph.replay()
        torch.cuda.synchronize()
        check_head(hidden, weight.cpu(), None, out, logits)
    assert int(scratch.abs().sum()) == 0


def test_head_argmax_ties_and_limits():
    h, rows = 512, 300
    weight = torch.zeros(rows, h, dtype=torch.bfloat16, device=DEV)
    hidden = rnd((2, h), 1320).to(DEV)
    imap = torch.arange(rows, device=DEV) + 1000
    assert K.head_argmax(hidden, weight, imap).tolist() == [1000, 1000]      # all equal: the first row
    weight[7, 0] = 1.0
    weight[9, 0] = 1.0
    hidden[:, 0] = 2.0
    assert K.head_argmax(hidden, weight, imap).tolist() == [1007, 1007]      # equal maxima: the lower row
    with pytest.raises(KaniError):
        K.head_argmax(rnd((9, h), 1321).to(DEV), weight)                     # more than 8 streams


@pytest.mark.parametrize("name", ["whole_frames", "partial_frame", "one_frame", "negative_code", "no_frame"])
def test_codec_codes_match_reference_golden(name):
    c = load("codec_codes")[name]
    codes, frames, status = K.codec_codes(c["generated"].view(1, -1).to(DEV), EOS, AUDIO_START)
    if "error" in c:
        want = {"Invalid audio tokens!": 1, "No complete audio frames generated!": 2}[c["error"]]
        assert int(status[0]) & want
    else:
        nf = int(c["frames"][0])
        assert int(frames[0]) == nf and int(status[0]) == 0
        assert torch.equal(codes[0, :, :nf].cpu(), c["codes"][0])


def test_codec_codes_batch_vs_oracle():
    g = torch.Generator().manual_seed(1330)
    b, t = 6, 1500
    c = torch.arange(t) % 4
    toks = AUDIO_START + c * 4032 + torch.randint(0, 4032, (b, t), generator=g)
    toks[0, 1000] = EOS                       # ends mid-frame
    toks[1, 3] = EOS                          # no complete frame
    toks[2, 400] = EOS
    toks[2, 17] = AUDIO_START - 5             # a negative code
    toks[4, 0] = EOS                          # empty
    # stream 3 and 5: no end-of-speech token
    got = K.codec_codes(toks.to(DEV), EOS, AUDIO_START)
    ref = O.codec_codes_ref(toks, EOS, AUDIO_START)
    for x, y in zip(got, ref):
        assert torch.equal(x.cpu(), y)
    assert [int(s) for s in ref[2]] == [0, 2, 1, 4, 2, 4]


@pytest.mark.parametrize("b", [1, 3, 8])
@pytest.mark.parametrize("mode", ["plain_1024", "plain_4608", "norm", "add_norm", "add_norm_silu"])
def test_gemv_vs_oracle(b, mode):
    """Fused decode GEMV: the input row (or its residual add + RMSNorm) into smem,
    fp32 dot products, optional SiLU·mul.  Outputs within 1 ULP of the oracle or
    the cancellation bound; the residual sum bit-exact."""
    k = 4608 if mode == "plain_4608" else 1024
    n = {"plain_1024": 2048, "plain_4608": 1024, "norm": 3072, "add_norm": 1024, "add_norm_silu": 4608}[mode]
    silu = mode == "add_norm_silu"
    x = rnd((b, 1, k), 1500 + b)
    w = rnd((2 * n if silu else n, k), 1501, std=0.03)
    nw = (1.0 + 0.1 * rnd((k,), 1502, torch.float32)).to(torch.bfloat16) if mode != "plain_1024" and \
        mode != "plain_4608" else None
    res = rnd((b, 1, k), 1503) if mode.startswith("add") else None
    h_out = torch.empty(b, 1, k, dtype=torch.bfloat16, device=DEV) if res is not None else None
    y = K.gemv(x.to(DEV), w.to(DEV), norm_weight=nw.to(DEV) if nw is not None else None,
               residual=res.to(DEV) if res is not None else None, residual_out=h_out, silu_pairs=silu)
    ref, h_ref = O.gemv_ref(x, w, nw, res, 1e-5, silu)
    assert y.shape == (b, 1, n)
    d = O.ulp_distance(y.cpu(), ref)
    a_ref = x if nw is None else (O.add_rms_norm_ref(x, res, nw, 1e-5)[0] if res is not None
                                 else O.rms_norm_ref(x, nw, 1e-5))
    mag = (a_ref.double().abs().reshape(b, k) @ w.double().abs().T)
    if silu:   # the activation multiplies two rounded products: allow 2 ULP there
        ok = d <= 2
    else:
        err = (y.cpu().double() - ref.double()).abs().reshape(b, n)
        ok = (d.reshape(b, n) <= 1) | (err <= mag * 2.0 ** -16)
    assert bool(ok.all()), f"max ULP {int(d.max())}"
    assert float((d == 0).float().mean()) >= 0.97
    if h_out is not None:
        assert torch.equal(h_out.cpu(), h_ref)


@pytest.mark.parametrize("b", [1, 4])
def test_gemv_short_conv_equals_gemv_then_conv(b):
    """The conv epilogue computes each channel's B, C, x rows in one warp with the
    accumulation order of the plain GEMV, so it is bit-identical to
    gemv(in_proj) followed by short_conv_step, state update included."""
    h = 1024
    x = rnd((b, 1, h), 1600 + b).to(DEV)
    res = rnd((b, 1, h), 1601).to(DEV)
    nw = (1.0 + 0.1 * rnd((h,), 1602, torch.float32)).to(torch.bfloat16).to(DEV)
    w = rnd((3 * h, h), 1603, std=0.03).to(DEV)
    cw = rnd((h, 3), 1604, std=0.3).to(DEV)
    st0 = rnd((b, h, 3), 1605).to(DEV)
    ha, hb = torch.empty_like(x), torch.empty_like(x)
    st_a, st_b = st0.clone(), st0.clone()
    bcx = K.gemv(x, w, norm_weight=nw, residual=res, residual_out=ha)
    ya = K.short_conv_step(bcx, st_a, cw)
    yb = K.gemv_short_conv(x, w, st_b, cw, norm_weight=nw, residual=res, residual_out=hb)
    torch.cuda.synchronize()
    assert torch.equal(ya, yb)
    assert torch.equal(st_a, st_b)
    assert torch.equal(ha, hb)


def test_decode_advance_matches_the_reference_schedule():
    """Per-step bookkeeping against the reference loop's arithmetic
    (inference_engine.py:615-619, 638-643, 669) over 9 steps, 3 streams."""
    b, n, tpf = 3, 9, 4
    base = torch.tensor([130, 7, 40], device=DEV)
    gen = torch.zeros(b, n, dtype=torch.long, device=DEV)
    ids = torch.zeros(b, 1, dtype=torch.long, device=DEV)
    step = torch.zeros(1, dtype=torch.long, device=DEV)
    rng = torch.full((1,), 5, dtype=torch.long, device=DEV)
    pos, slots, kvl = base.clone(), base.clone(), base + 1
    for k in range(n):
        tok = torch.tensor([1000 + k, 2000 + k, 3000 + k], device=DEV)
        K.decode_advance(tok, ids, gen, step, base, base, pos, slots, kvl, tpf, 1.0, rng_step=rng)
        torch.cuda.synchronize()
        assert torch.equal(ids.view(-1).cpu(), tok.cpu())
        assert torch.equal(pos.cpu(), (base + (k + 1) // tpf).cpu())
        assert torch.equal(slots.cpu(), (base + k + 1).cpu()) and torch.equal(kvl.cpu(), (base + k + 2).cpu())
    assert int(step.item()) == n and int(rng.item()) == 5 + n
    assert torch.equal(gen.cpu(), (torch.arange(n) + torch.tensor([[1000], [2000], [3000]])))


@pytest.mark.parametrize("b,table", [(1, True), (3, True), (4, False)])
def test_gemv_rope_kv_equals_gemv_then_rope(b, table):
    """QKV GEMV with the q/k norm + RoPE + frame term + KV write in its epilogue:
    bit-identical to gemv(QKV) followed by fused_rope_kv_write (same row
    accumulation order, the same RoPE code), caches included; an out-of-range
    slot is skipped and flagged."""
    from kani_tts_b200 import _lib
    from kani_tts_b200.positions import learnable_inv_freq
    hq, hk, d, h, s_len = 16, 8, 64, 1024, 64
    x = rnd((b, 1, h), 1700 + b).to(DEV)
    res = rnd((b, 1, h), 1701).to(DEV)
    nw = (1.0 + 0.1 * rnd((h,), 1702, torch.float32)).to(torch.bfloat16).to(DEV)
    w = rnd(((hq + 2 * hk) * d, h), 1703, std=0.03).to(DEV)
    qn = (1.0 + 0.1 * rnd((d,), 1704, torch.float32)).to(torch.bfloat16).to(DEV)
    kn = (1.0 + 0.1 * rnd((d,), 1705, torch.float32)).to(torch.bfloat16).to(DEV)
    inv = learnable_inv_freq(d, 1e6, torch.tensor(0.05)).to(DEV)
    tab = rnd((32, d), 1706, std=0.02).to(DEV) if table else None
    pos = torch.tensor([5, 77, 40, 13][:b], device=DEV)
    slots = torch.tensor([3, 9, 63, 20][:b], device=DEV)
    if b == 3:
        slots[2] = 64                                    # out of range: skipped and flagged
    kc0, vc0 = rnd((b, hk, s_len, d), 1707).to(DEV), rnd((b, hk, s_len, d), 1708).to(DEV)
    kca, vca, kcb, vcb = kc0.clone(), vc0.clone(), kc0.clone(), vc0.clone()
    ha, hb = torch.empty_like(x), torch.empty_like(x)
    _lib.read_and_clear_errors(DEV)
    qkv = K.gemv(x, w, norm_weight=nw, residual=res, residual_out=ha)
    q, k, v = qkv.split([hq * d, hk * d, hk * d], dim=-1)
    qa = K.fused_rope_kv_write(q.view(b, 1, hq, d), k.view(b, 1, hk, d), v.view(b, 1, hk, d), inv, pos, kca, vca,
                               slots, frame_table=tab, tokens_per_frame=4, q_norm_w=qn, k_norm_w=kn, eps=1e-5)
    fa = _lib.read_and_clear_errors(DEV)
    qb = K.gemv_rope_kv_write(x, w, nw, inv, pos, kcb, vcb, slots, num_q_heads=hq, num_kv_heads=hk, residual=res,
                              residual_out=hb, q_norm_w=qn, k_norm_w=kn, head_eps=1e-5, frame_table=tab,
                              tokens_per_frame=4)
    fb = _lib.read_and_clear_errors(DEV)
    torch.cuda.synchronize()
    assert torch.equal(qa.reshape(b, hq, d).cpu(), qb.cpu())
    assert torch.equal(kca.cpu(), kcb.cpu()) and torch.equal(vca.cpu(), vcb.cpu())
    assert torch.equal(ha.cpu(), hb.cpu())
    assert fa == fb == (_lib.KANI_FLAG_SLOT_OOB if b == 3 else 0)
