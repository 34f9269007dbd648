"""Restatement of the reference Sampler's filters (TEST ORACLE ONLY).

mini_vllm/layers/sampler.py:13-49: x = logits.float() / T; _apply_top_k keeps ranks < k of a
descending sort (k <= 0 or >= V: no filter); _apply_top_p, on the top-k-masked x, takes
softmax over the sorted values, keeps entries whose inclusive cumulative probability is
< top_p, and always the first; the token is then argmax(softmax(x) / Exp(1)), i.e. a draw from
softmax over the kept set.

torch.sort leaves the order of equal values unspecified; this restatement uses a stable sort
(lower vocabulary id first among equals), the order hl_sample_filtered commits to.  It returns
the kept set and the exact renormalised distribution, which the GPU tests use as the checker
(membership of every draw, and empirical frequencies).

top_p >= 1 means no top-p filter for that row.  (The reference skips _apply_top_p only when every
row of the batch has top_p >= 1; in a mixed batch a top_p = 1 row is filtered too and loses the
tokens whose float32 inclusive cumulative probability reaches 1.0 — often the last token of its
top-k set, whatever its probability.  That batch-dependent effect is not reproduced.)
"""
from __future__ import annotations

import torch


def kept_set(logits_row: torch.Tensor, temperature: float, top_k: int, top_p: float) -> torch.Tensor:
    """Boolean mask [V] of the tokens the reference's filters keep for one row (bf16 or float
    logits; the comparison is done in float32 as the reference does)."""
    x = logits_row.float() / float(temperature)
    v = x.numel()
    keep = torch.ones(v, dtype=torch.bool)
    order = torch.sort(x, descending=True, stable=True).indices
    if 0 < top_k < v:
        keep[:] = False
        keep[order[:top_k]] = True
    if top_p < 1.0:
        kept_sorted = order[keep[order]]  # the top-k set, still in descending (stable) order
        xs = x[kept_sorted]
        probs = torch.softmax(xs, 0)  # float32, as the reference computes it
        cum = torch.cumsum(probs, 0)
        keep_sorted = cum < top_p
        keep_sorted[0] = True
        keep[:] = False
        keep[kept_sorted[keep_sorted]] = True
    return keep


def filtered_distribution(logits_row: torch.Tensor, temperature: float, top_k: int, top_p: float) -> torch.Tensor:
    """The reference's sampling distribution [V] (float64) for one row."""
    x = logits_row.float().double() / float(temperature)
    keep = kept_set(logits_row, temperature, top_k, top_p)
    x = x.masked_fill(~keep, float("-inf"))
    return torch.softmax(x, 0)
