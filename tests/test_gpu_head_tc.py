"""GPU parity of the tensor-core reduced head with the greedy choice
(``kani_head_argmax_tc``, 2..64 streams) against the oracle.

Tolerances (as for the CUDA-core head):
  * logits: within 1 ULP of the oracle's float64 dot product rounded once
    (fp32 accumulation in another order), or within 2^-16 x sum |h w| where the
    products cancel towards zero; >= 99 % identical;
  * token: identical to the first maximum of the kernel's own logits, and to the
    oracle's token whenever the two logit rows are identical.
"""
from __future__ import annotations

import pytest
import torch

from oracle import kani_oracle as O

from kani_tts_b200 import fused_kernels as K
from kani_tts_b200._lib import KaniError

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def rnd(shape, seed, dtype=torch.bfloat16, std=1.0):
    g = torch.Generator().manual_seed(seed)
    return (std * torch.randn(shape, generator=g)).to(dtype)


def check_head(hidden, weight, imap, tok, logits):
    ref_tok, ref_logits = O.head_argmax_ref(hidden, weight, imap)
    d = O.ulp_distance(logits.cpu(), ref_logits)
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
@pytest.mark.parametrize("b,h,rows", [(64, 1024, 15591), (9, 1024, 15591), (2, 1024, 4000), (33, 512, 37),
                                      (17, 128, 200), (64, 640, 129), (33, 576, 300), (1, 64, 130)])
def test_head_argmax_tc_vs_oracle(dtype, b, h, rows):
    hidden = rnd((b, h), 1400 + b, dtype)
    weight = rnd((rows, h), 1401 + rows, dtype, std=0.05)
    imap = torch.arange(rows, dtype=torch.long) * 3 + 11
    logits = torch.empty(b, rows, dtype=dtype, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    tok = K.head_argmax_tc(hidden.to(DEV), weight.to(DEV), imap.to(DEV), logits_out=logits, err_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    check_head(hidden, weight, imap, tok, logits)


def test_head_argmax_tc_without_logits_and_strided_rows():
    """No logits output; hidden rows taken from a wider buffer (row stride > H)."""
    b, h, rows = 40, 1024, 15591
    wide = rnd((b, h + 64), 1410).to(DEV)
    hidden = wide[:, :h]
    weight = rnd((rows, h), 1411, std=0.05).to(DEV)
    tok = K.head_argmax_tc(hidden, weight)
    logits = torch.empty(b, rows, dtype=torch.bfloat16, device=DEV)
    tok2 = K.head_argmax_tc(hidden, weight, logits_out=logits)
    assert torch.equal(tok, tok2)
    check_head(hidden.cpu(), weight.cpu(), None, tok2, logits)


def test_head_argmax_tc_scratch_is_left_clean_and_reused():
    """One scratch buffer across batch sizes and a replayed graph; all zero after."""
    h, rows = 1024, 15591
    weight = rnd((rows, h), 1420, std=0.05).to(DEV)
    scratch = torch.zeros(65, dtype=torch.int32, device=DEV)
    for b, seed in ((64, 1421), (9, 1422), (64, 1423), (2, 1424)):
        hidden = rnd((b, h), seed)
        logits = torch.empty(b, rows, dtype=torch.bfloat16, device=DEV)
        tok = K.head_argmax_tc(hidden.to(DEV), weight, scratch=scratch, logits_out=logits)
        check_head(hidden, weight.cpu(), None, tok, logits)
        assert int(scratch.abs().sum()) == 0
    b = 48
    hid = torch.zeros(b, h, dtype=torch.bfloat16, device=DEV)
    out = torch.zeros(b, dtype=torch.long, device=DEV)
    logits = torch.empty(b, rows, dtype=torch.bfloat16, device=DEV)
    s = torch.cuda.Stream(device=DEV)
    s.wait_stream(torch.cuda.current_stream(DEV))
    with torch.cuda.stream(s):
        K.head_argmax_tc(hid, weight, scratch=scratch, logits_out=logits, out=out)
    torch.cuda.current_stream(DEV).wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        K.head_argmax_tc(hid, weight, scratch=scratch, logits_out=logits, out=out)
    for seed in (1425, 1426, 1427):
        hidden = rnd((b, h), seed)
        hid.copy_(hidden)
        graph.replay()
        torch.cuda.synchronize()
        check_head(hidden, weight.cpu(), None, out, logits)
    assert int(scratch.abs().sum()) == 0


def test_head_argmax_tc_matches_cuda_core_head_tokens():
    """Same tokens as the CUDA-core head wherever the winning logit leads the
    runner-up by more than 2 ULP (the two kernels accumulate in different
    orders, so single logits may differ by 1 ULP)."""
    h, rows = 1024, 15591
    weight = rnd((rows, h), 1430, std=0.05).to(DEV)
    hidden = rnd((8, h), 1431).to(DEV)
    la = torch.empty(8, rows, dtype=torch.bfloat16, device=DEV)
    lb = torch.empty(8, rows, dtype=torch.bfloat16, device=DEV)
    ta = K.head_argmax(hidden, weight, logits_out=la)
    tb = K.head_argmax_tc(hidden, weight, logits_out=lb)
    top2 = la.float().topk(2, dim=-1).values
    ulp = top2[:, 0].abs() * 2.0 ** -7
    clear = (top2[:, 0] - top2[:, 1]) > 2 * ulp
    assert bool(clear.any())
    assert torch.equal(ta[clear], tb[clear])
    assert float((O.ulp_distance(la.cpu(), lb.cpu()) <= 2).float().mean()) >= 0.999


def test_head_argmax_tc_ties_and_limits():
    h, rows = 512, 300
    weight = torch.zeros(rows, h, dtype=torch.bfloat16, device=DEV)
    hidden = rnd((20, h), 1440).to(DEV)
    imap = torch.arange(rows, device=DEV) + 1000
    assert K.head_argmax_tc(hidden, weight, imap).tolist() == [1000] * 20      # all equal: the first row
    weight[7, 0] = 1.0
    weight[9, 0] = 1.0
    weight[200, 0] = 1.0
    hidden[:, 0] = 2.0
    assert K.head_argmax_tc(hidden, weight, imap).tolist() == [1007] * 20      # equal maxima: the lower row
    weight[299, 1] = 4.0
    hidden[3, 1] = 1.0
    assert K.head_argmax_tc(hidden, weight, imap).tolist()[3] == 1299          # the last row, in the last tile
    with pytest.raises(KaniError):
        K.head_argmax_tc(rnd((65, h), 1441).to(DEV), weight)                   # more than 64 streams
    with pytest.raises(KaniError):
        K.head_argmax_tc(rnd((4, 2048), 1442).to(DEV), rnd((10, 2048), 1443).to(DEV))  # hidden above 1024
