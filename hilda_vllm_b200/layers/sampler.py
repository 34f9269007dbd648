"""Token sampler (mini_vllm/layers/sampler.py:7-49) plus a greedy path.

Non-greedy rows follow the reference exactly: logits / temperature, top-k, top-p, softmax,
then argmax(probs / Exp(1) noise).  Greedy rows take hl_argmax (lowest id among ties).
"""
import torch
from torch import nn

from hilda_vllm_b200 import kernels


class Sampler(nn.Module):

    def forward(self, logits: torch.Tensor, temperatures: torch.Tensor, top_ks: torch.Tensor, top_ps: torch.Tensor):
        logits = logits.float().div_(temperatures.unsqueeze(dim=1))
        logits = self._apply_top_k(logits, top_ks)
        logits = self._apply_top_p(logits, top_ps)
        probs = torch.softmax(logits, dim=-1)
        return probs.div_(torch.empty_like(probs).exponential_(1).clamp_min_(1e-10)).argmax(dim=-1)

    @staticmethod
    def greedy(logits: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        return kernels.argmax(logits, out)

    @staticmethod
    def _apply_top_k(logits: torch.Tensor, top_ks: torch.Tensor) -> torch.Tensor:
        vocab = logits.size(-1)
        ks = torch.where(top_ks > 0, torch.minimum(top_ks, torch.full_like(top_ks, vocab)), vocab)
        if torch.all(ks == vocab):
            return logits
        sorted_logits, order = torch.sort(logits, dim=-1, descending=True)
        keep = torch.arange(vocab, device=logits.device).unsqueeze(0) < ks.unsqueeze(1)
        return torch.scatter(torch.empty_like(logits), 1, order, sorted_logits.masked_fill(~keep, float("-inf")))

    @staticmethod
    def _apply_top_p(logits: torch.Tensor, top_ps: torch.Tensor) -> torch.Tensor:
        if torch.all(top_ps >= 1.0):
            return logits
        sorted_logits, order = torch.sort(logits, dim=-1, descending=True)
        cum = torch.cumsum(torch.softmax(sorted_logits, dim=-1), dim=-1)
        keep = cum < top_ps.unsqueeze(1)
        keep[:, 0] = True
        return torch.scatter(torch.empty_like(logits), 1, order, sorted_logits.masked_fill(~keep, float("-inf")))
