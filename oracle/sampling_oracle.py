"""CPU restatement of the reference's next-token sampler — TEST INFRASTRUCTURE ONLY.

Only the tests, ``__graft_entry__.smoke()`` and the CPU legs of ``bench.py``
may import this module; it is the checker for ``kani_sample_tokens``, never
the thing measured and never a fallback.

``sample_ref`` follows ``KaniInferenceEngine._sample_next_token``
(kani_tts/inference_engine.py:349-430) step for step with the same PyTorch
CPU ops on a batch of rows:

* repetition penalty on the distinct history tokens (375-395):
  ``where(l > 0, l / rp, l * rp)`` in the logits dtype;
* the additive audio mask of the full-vocab mode (398-399);
* ``topk(min(256, V))`` (402-403) — here a stable descending sort, so equal
  logits are ordered by lower index (``torch.topk`` leaves that order
  unspecified; the golden inputs have no ties inside the top k + 1);
* temperature (406-407), softmax, cumsum and the top-p mask (410-415);
* ``torch.multinomial(probs, 1)`` (418-419).  For one sample, torch 2.x
  (aten/src/ATen/native/Distributions.cpp, ``multinomial_out``) draws
  ``q ~ Exp(1)`` in the probs dtype and returns ``argmax(probs / q)``; here
  the Exp(1) draws are an argument, so a given set of draws selects one token
  exactly;
* the reduced-index -> full-id map (422-428).

``philox4x32_10`` and ``exp_draws`` restate the counter-based generator the
kernel uses when no draws are passed: Philox4x32-10 (Salmon, Moraes, Dror &
Shaw, "Parallel random numbers: as easy as 1, 2, 3", SC 2011) keyed by the
seed, counter (candidate group, stream, step lo, step hi);
u = (2 * (w >> 9) + 1) * 2^-24 and E = -log(u).

Pinning: ``tests/golden/make_golden.py`` runs the reference's own
``_sample_next_token`` with recording wrappers around ``torch.topk`` and
``torch.multinomial`` (the latter performs the exponential race above on
stored draws) and stores inputs and outputs in ``tests/golden/sampling.npz``;
``tests/test_sampling_oracle.py`` checks ``sample_ref`` against them.
"""
from __future__ import annotations

import numpy as np
import torch


def seen_from_history(history: torch.Tensor, vocab: int, full_to_reduced: torch.Tensor | None = None
                      ) -> torch.Tensor:
    """[B, V] bool: index i was generated or prompted before (the reference's
    ``input_ids[0].unique()`` mapped through ``full_to_reduced``, 377-383)."""
    history = torch.as_tensor(history).long()
    if history.dim() == 1:
        history = history.view(1, -1)
    out = torch.zeros(history.shape[0], vocab, dtype=torch.bool)
    for b in range(history.shape[0]):
        ids = history[b].unique()
        if full_to_reduced is not None:
            ids = full_to_reduced[ids]
            ids = ids[ids >= 0]
        out[b, ids] = True
    return out


def sample_ref(logits: torch.Tensor, seen: torch.Tensor | None, repetition_penalty: float, temperature: float,
               top_p: float, draws: torch.Tensor, top_k: int = 256, index_map: torch.Tensor | None = None,
               logit_bias: torch.Tensor | None = None) -> dict:
    """One sampling step for each row of ``logits`` [B, V] (inference_engine.py:349-430).

    ``seen`` [B, V] bool marks the penalised indices; ``draws`` [B, k] fp32
    holds the Exp(1) variates of ``torch.multinomial``'s race.  Returns the
    token ids [B], the sorted candidate indices [B, k], the candidates' logits
    after the penalty [B, k] and the final distribution [B, k] (logits dtype)."""
    logits = logits.cpu()
    b_n, v = logits.shape
    k = min(top_k, v)
    toks, cands, vals, probs_all = [], [], [], []
    for b in range(b_n):
        lg = logits[b:b + 1].clone()
        if repetition_penalty != 1.0 and seen is not None:
            idx = torch.nonzero(seen[b]).flatten()
            if idx.numel():
                pl = lg[0, idx]
                lg[0, idx] = torch.where(pl > 0, pl / repetition_penalty, pl * repetition_penalty)
        if logit_bias is not None:
            lg.add_(logit_bias.view(1, -1).to(lg.dtype))
        order = torch.sort(lg.float(), dim=-1, descending=True, stable=True).indices[:, :k]
        tl = lg.gather(-1, order)
        vals.append(tl[0].clone())
        if temperature != 1.0:
            tl = tl / temperature
        if top_p < 1.0:
            p = torch.softmax(tl, dim=-1)
            c = torch.cumsum(p, dim=-1)
            mask = torch.zeros_like(c, dtype=torch.bool)
            mask[..., 1:] = c[..., :-1] >= top_p
            tl = tl.masked_fill(mask, float("-inf"))
        p = torch.softmax(tl, dim=-1)
        q = draws[b:b + 1, :k].to(p.dtype)
        j = torch.argmax(p / q, dim=-1, keepdim=True)
        red = order.gather(-1, j)
        tok = index_map[red] if index_map is not None else red
        toks.append(int(tok.view(-1)[0]))
        cands.append(order[0])
        probs_all.append(p[0])
    return {"tokens": torch.tensor(toks), "cand": torch.stack(cands), "values": torch.stack(vals),
            "probs": torch.stack(probs_all)}


# ---------------------------------------------------------------- Philox

_M0, _M1 = 0xD2511F53, 0xCD9E8D57
_W0, _W1 = 0x9E3779B9, 0xBB67AE85
_MASK = 0xFFFFFFFF


def philox4x32_10(counter: np.ndarray, key: tuple[int, int]) -> np.ndarray:
    """Philox4x32-10 on an [N, 4] uint32 array of counters; returns [N, 4] uint32."""
    c = counter.astype(np.uint64)
    k0, k1 = np.uint64(key[0] & _MASK), np.uint64(key[1] & _MASK)
    m0, m1, mask = np.uint64(_M0), np.uint64(_M1), np.uint64(_MASK)
    for _ in range(10):
        p0 = m0 * c[:, 0]
        p1 = m1 * c[:, 2]
        hi0, lo0 = p0 >> np.uint64(32), p0 & mask
        hi1, lo1 = p1 >> np.uint64(32), p1 & mask
        c = np.stack([hi1 ^ c[:, 1] ^ k0, lo1, hi0 ^ c[:, 3] ^ k1, lo0], axis=1)
        k0 = (k0 + np.uint64(_W0)) & mask
        k1 = (k1 + np.uint64(_W1)) & mask
    return c.astype(np.uint32)


def exp_draws(seed: int, batch: int, step: int, top_k: int = 256) -> torch.Tensor:
    """The kernel's Exp(1) draws [batch, top_k] fp32 for one step (no draws passed)."""
    groups = (top_k + 3) // 4
    g, b = np.meshgrid(np.arange(groups, dtype=np.uint64), np.arange(batch, dtype=np.uint64))
    ctr = np.stack([g.ravel(), b.ravel(), np.full(g.size, step & _MASK, np.uint64),
                    np.full(g.size, (step >> 32) & _MASK, np.uint64)], axis=1)
    w = philox4x32_10(ctr, (seed & _MASK, (seed >> 32) & _MASK)).reshape(batch, groups * 4)[:, :top_k]
    u = ((w >> np.uint32(9)).astype(np.uint32) * np.uint32(2) + np.uint32(1)).astype(np.float32) \
        * np.float32(2.0 ** -24)
    return torch.from_numpy(-np.log(u))
