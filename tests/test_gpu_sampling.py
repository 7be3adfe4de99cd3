"""GPU parity of the device sampler (``kani_sample_tokens``) against the
reference's own sampler outputs (tests/golden/sampling.npz) and the oracle.

Tolerances:
  * sorted candidate indices: identical (ties ordered by lower index);
  * the kept distribution: within 1 ULP of the oracle's, >= 99 % identical
    (the softmax sums accumulate in a different order); within 8 ULP for
    fp32 logits (exp and the sum order differ in the last bits);
  * the sampled token: identical to the race on the kernel's own
    distribution with the same Exp(1) draws, and identical to the oracle's
    token wherever the two distributions are bit-identical;
  * Philox draws: within 4 fp32 ULP of the oracle's -log(u) (CUDA logf
    against numpy's float32 log; u itself is exact).
"""
from __future__ import annotations

import pytest
import torch

from golden_io import load
from oracle import kani_oracle as O
from oracle import sampling_oracle as S

from kani_tts_b200 import fused_kernels as K
from kani_tts_b200 import sampling as KS

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
VOCAB, AUDIO_START, EOS = 80000, 64410, 7
N_RED = 1 + VOCAB - AUDIO_START


def maps():
    r2f = torch.cat([torch.tensor([EOS]), torch.arange(AUDIO_START, VOCAB)])
    f2r = torch.full((VOCAB,), -1, dtype=torch.long)
    f2r[EOS] = 0
    f2r[AUDIO_START:] = torch.arange(1, N_RED)
    return r2f, f2r


def audio_bias():
    bias = torch.full((VOCAB,), float("-inf"), dtype=torch.bfloat16)
    bias[AUDIO_START:] = 0
    bias[EOS] = 0
    return bias


def bits_of(words: torch.Tensor, v: int) -> torch.Tensor:
    w = words.cpu().long() & 0xFFFFFFFF
    return ((w.unsqueeze(-1) >> torch.arange(32)) & 1).view(w.shape[0], -1)[:, :v].bool()


def exp1(shape, seed):
    g = torch.Generator().manual_seed(seed)
    return -torch.log(torch.rand(shape, generator=g).clamp_min(2.0 ** -24))


def check_against_oracle(tok, det, ref, draws, index_map=None):
    """Candidates exact, distribution within 1 ULP, token exact given the distribution."""
    cand = det["cand"].long().cpu()
    assert torch.equal(cand, ref["cand"])
    probs = det["probs"].cpu()
    d = O.ulp_distance(probs, ref["probs"])
    if probs.dtype == torch.float32:   # exp and the softmax sum order: a few fp32 ULP
        assert int(d.max()) <= 8, f"max ULP {int(d.max())}"
    else:
        assert int(d.max()) <= 1, f"max ULP {int(d.max())}"
        assert float((d == 0).float().mean()) >= 0.99
    j = torch.argmax(probs / draws.cpu().to(probs.dtype), dim=-1, keepdim=True)
    red = cand.gather(-1, j).view(-1)
    want = index_map.cpu()[red] if index_map is not None else red
    assert torch.equal(tok.cpu(), want)
    same = (d == 0).all(dim=-1)
    assert torch.equal(tok.cpu()[same], ref["tokens"][same])


@pytest.mark.parametrize("name", ["config_defaults", "engine_defaults", "no_top_p", "deep_nucleus",
                                  "full_vocab_mask"])
def test_sampler_matches_reference_golden(name):
    c = load("sampling")[name]
    r2f, f2r = maps()
    reduced = bool(c["reduced"])
    v = c["logits"].shape[-1]
    seen = KS.seen_bitmap(c["history"], v, f2r if reduced else None, device=DEV)
    seen0 = seen.clone()
    tok, det = K.sample_tokens(c["logits"].to(DEV), seen, temperature=float(c["temperature"]),
                               top_p=float(c["top_p"]), repetition_penalty=float(c["repetition_penalty"]),
                               index_map=r2f.to(DEV) if reduced else None,
                               logit_bias=None if reduced else audio_bias().to(DEV),
                               draws=c["draws"].to(DEV), return_details=True)
    torch.cuda.synchronize()
    assert int(tok[0]) == int(c["token"][0])
    assert torch.equal(det["cand"][0].long().cpu(), c["topk_indices"][0])
    d = O.ulp_distance(det["probs"][0].cpu(), c["probs"][0])
    assert int(d.max()) <= 1 and float((d == 0).float().mean()) >= 0.99
    assert torch.equal(det["draws"].cpu(), c["draws"])
    # the sampled index joins the penalised history (the reference appends the token)
    idx = int(f2r[tok.cpu()][0]) if reduced else int(tok[0])
    after, before = bits_of(seen, v), bits_of(seen0, v)
    assert bool(after[0, idx])
    before[0, idx] = True
    assert torch.equal(after, before)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("rp,temp,top_p", [(1.2, 0.5, 0.85), (1.0, 0.7, 0.95), (1.1, 1.0, 1.0),
                                           (1.3, 1.3, 0.5)])
def test_sampler_batch_with_ties_vs_oracle(dtype, rp, temp, top_p):
    """Six streams of N(0, 2.5) logits (many equal bf16 values at the top-k
    boundary), each with its own repetition history."""
    b, v = 6, N_RED
    g = torch.Generator().manual_seed(21)
    logits = (torch.randn(b, v, generator=g) * 2.5).to(dtype)
    hist = torch.randint(0, v, (b, 60), generator=g)
    seen_mask = S.seen_from_history(hist, v)
    draws = exp1((b, 256), 22)
    tok, det = K.sample_tokens(logits.to(DEV), KS.seen_bitmap(hist, v, device=DEV), temperature=temp,
                               top_p=top_p, repetition_penalty=rp, draws=draws.to(DEV), return_details=True)
    ref = S.sample_ref(logits, seen_mask, rp, temp, top_p, draws)
    check_against_oracle(tok, det, ref, draws)


@pytest.mark.parametrize("case", ["small_vocab", "all_equal", "masked_half", "top_k_1", "top_p_0",
                                  "vocab_1", "full_vocab_bf16", "large_vocab_f32", "top_p_near_one",
                                  "peaked_fp16"])
def test_sampler_edge_cases(case):
    g = torch.Generator().manual_seed(31)
    dtype, top_k, top_p, temp, bias = torch.bfloat16, 256, 0.85, 0.5, None
    if case == "small_vocab":
        logits = torch.randn(3, 100, generator=g).to(dtype)
    elif case == "all_equal":
        logits = torch.zeros(2, 1000, dtype=dtype)
    elif case == "masked_half":
        logits = torch.randn(2, 2000, generator=g).to(dtype)
        bias = torch.zeros(2000, dtype=dtype)
        bias[::2] = float("-inf")
    elif case == "top_k_1":
        logits = (torch.randn(4, N_RED, generator=g) * 3).to(dtype)
        top_k = 1
    elif case == "top_p_0":
        logits = torch.randn(2, N_RED, generator=g).to(dtype)
        top_p = 0.0
    elif case == "vocab_1":
        logits = torch.randn(3, 1, generator=g).to(dtype)
    elif case == "full_vocab_bf16":
        logits = (torch.randn(2, VOCAB, generator=g) * 2).to(dtype)
    elif case == "top_p_near_one":
        # one dominant candidate: the running sum reaches bf16(0.9999) = 1 only
        # through values below 2^-17 (the kernel's in-order fallback chain)
        logits = (torch.randn(3, N_RED, generator=g) * 0.5).to(dtype)
        logits[:, 5] = 14.0
        top_p, temp = 0.9999, 1.0
    elif case == "peaked_fp16":
        dtype = torch.float16
        logits = (torch.randn(3, N_RED, generator=g) * 3).to(dtype)
        top_p, temp = 0.99, 0.3
    else:
        dtype = torch.float32
        logits = torch.randn(2, 40000, generator=g) * 2
    b, v = logits.shape
    k = min(top_k, v)
    draws = exp1((b, k), 32)
    tok, det = K.sample_tokens(logits.to(DEV), None, temperature=temp, top_p=top_p, top_k=top_k,
                               logit_bias=bias.to(DEV) if bias is not None else None, draws=draws.to(DEV),
                               return_details=True)
    ref = S.sample_ref(logits, None, 1.0, temp, top_p, draws, top_k=top_k, logit_bias=bias)
    check_against_oracle(tok, det, ref, draws)
    if case == "all_equal":
        assert torch.equal(det["cand"].long().cpu(), torch.arange(256).repeat(2, 1))
    if case in ("top_k_1", "top_p_0"):
        assert torch.equal(tok.cpu(), torch.sort(logits.float(), dim=-1, descending=True, stable=True).indices[:, 0])


def test_philox_draws_match_oracle():
    b, v, seed = 4, N_RED, 0x1234_5678_9ABC
    g = torch.Generator().manual_seed(41)
    logits = (torch.randn(b, v, generator=g) * 2).to(torch.bfloat16)
    step = torch.tensor([7], dtype=torch.long, device=DEV)
    tok, det = K.sample_tokens(logits.to(DEV), None, temperature=0.5, top_p=0.85, seed=seed, step=step,
                               return_details=True)
    got = det["draws"].cpu()
    ref_draws = S.exp_draws(seed, b, 7)
    assert int(O.ulp_distance(got, ref_draws).max()) <= 4
    ref = S.sample_ref(logits, None, 1.0, 0.5, 0.85, got)
    check_against_oracle(tok, det, ref, got)
    tok2 = K.sample_tokens(logits.to(DEV), None, temperature=0.5, top_p=0.85, seed=seed, step=step)
    assert torch.equal(tok, tok2)
    step.fill_(8)
    _, det3 = K.sample_tokens(logits.to(DEV), None, temperature=0.5, top_p=0.85, seed=seed, step=step,
                              return_details=True)
    assert not torch.equal(det3["draws"].cpu(), got)


def test_sampling_frequencies_follow_the_kept_distribution():
    """4096 samples (64 streams x 64 steps) of one row against its kept distribution."""
    v, b, steps = N_RED, 64, 64
    g = torch.Generator().manual_seed(51)
    row = (torch.randn(1, v, generator=g) * 1.5).to(torch.bfloat16)
    logits = row.repeat(b, 1).to(DEV)
    ref = S.sample_ref(row, None, 1.0, 1.0, 0.9, torch.ones(1, 256))
    p, cand = ref["probs"][0].float(), ref["cand"][0]
    step = torch.zeros(1, dtype=torch.long, device=DEV)
    toks = []
    for s in range(steps):
        step.fill_(s)
        toks.append(K.sample_tokens(logits, None, temperature=1.0, top_p=0.9, seed=77, step=step).cpu())
    toks = torch.cat(toks)
    n = toks.numel()
    pos = torch.full((v,), -1, dtype=torch.long)
    pos[cand] = torch.arange(cand.numel())
    at = pos[toks]
    assert bool((at >= 0).all()) and bool((p[at] > 0).all())      # never outside the kept set
    freq = torch.bincount(at, minlength=cand.numel()).float() / n
    sigma = (p * (1 - p) / n).sqrt()
    assert bool(((freq - p).abs() <= 5 * sigma + 2e-3).all()), float((freq - p).abs().max())


def test_sampler_in_cuda_graph_matches_eager_steps():
    """Captured sample + step increment, replayed, gives the eager token sequence
    (the repetition bitmap evolves on the device in both)."""
    b, v, n = 3, N_RED, 6
    g = torch.Generator().manual_seed(61)
    logits = (torch.randn(b, v, generator=g) * 2).to(torch.bfloat16).to(DEV)
    hist = torch.randint(0, v, (b, 30), generator=g)
    kw = dict(temperature=0.7, top_p=0.9, repetition_penalty=1.3, seed=5)

    seen = KS.seen_bitmap(hist, v, device=DEV)
    step = torch.zeros(1, dtype=torch.long, device=DEV)
    eager = []
    for _ in range(n):
        eager.append(K.sample_tokens(logits, seen, step=step, **kw).clone())
        step.add_(1)
    eager_seen = seen.clone()

    seen = KS.seen_bitmap(hist, v, device=DEV)
    step = torch.zeros(1, dtype=torch.long, device=DEV)
    out = torch.zeros(b, dtype=torch.long, device=DEV)
    s = torch.cuda.Stream(device=DEV)
    s.wait_stream(torch.cuda.current_stream(DEV))
    with torch.cuda.stream(s):     # warm-up outside capture, then undo its effects
        K.sample_tokens(logits, seen.clone(), step=step.clone(), out=out.clone(), **kw)
    torch.cuda.current_stream(DEV).wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        K.sample_tokens(logits, seen, step=step, out=out, **kw)
        step.add_(1)
    replay = []
    for _ in range(n):
        graph.replay()
        replay.append(out.clone())
    torch.cuda.synchronize()
    assert torch.equal(torch.stack(replay).cpu(), torch.stack(eager).cpu())
    assert torch.equal(seen.cpu(), eager_seen.cpu())
    assert int(step.item()) == n
