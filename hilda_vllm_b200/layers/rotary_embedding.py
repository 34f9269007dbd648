"""Rotary embedding cache (mini_vllm/layers/rotary_embedding.py:19-91).

The cos/sin table is built exactly as the reference builds it (fp32 inverse frequencies
base^(-2i/d), positions x frequencies, then cos and sin), so the fused QK-norm + RoPE kernel
reads the same numbers the reference multiplies by.  The model applies RoPE through
hl_qk_norm_rope; forward() is kept for callers of the reference API and does the same
arithmetic with tensor ops.
"""
from functools import lru_cache

import torch
from torch import nn


def apply_rotary_emb(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    x1, x2 = torch.chunk(x.float(), 2, dim=-1)
    return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1).to(x.dtype)


class RotaryEmbedding(nn.Module):

    def __init__(self, head_size: int, rotary_dim: int, max_position_embeddings: int, base: float) -> None:
        super().__init__()
        self.head_size = head_size
        assert rotary_dim == head_size
        inv_freq = 1.0 / (base ** (torch.arange(0, rotary_dim, 2, dtype=torch.float) / rotary_dim))
        t = torch.arange(max_position_embeddings, dtype=torch.float)
        freqs = torch.einsum("i,j -> ij", t, inv_freq)
        cache = torch.cat((freqs.cos(), freqs.sin()), dim=-1).unsqueeze_(1)
        self.register_buffer("cos_sin_cache", cache, persistent=False)

    def forward(self, positions: torch.Tensor, query: torch.Tensor, key: torch.Tensor):
        cos, sin = self.cos_sin_cache[positions].chunk(2, dim=-1)
        return apply_rotary_emb(query, cos, sin), apply_rotary_emb(key, cos, sin)


def _normalize_rope_scaling(rope_scaling):
    if rope_scaling is None:
        return None
    if isinstance(rope_scaling, dict):
        return tuple(sorted(rope_scaling.items()))
    return tuple(rope_scaling)


@lru_cache(8)
def _get_rope_cached(head_size, rotary_dim, max_position, base, rope_scaling_items=None):
    if rope_scaling_items is not None:
        scaling = dict(rope_scaling_items)
        assert scaling.get("rope_type", "default") == "default"
        base = scaling.get("rope_theta", base)
    return RotaryEmbedding(head_size, rotary_dim, max_position, base)


def get_rope(head_size: int, rotary_dim: int, max_position: int, base: float, rope_scaling=None):
    return _get_rope_cached(head_size, rotary_dim, max_position, base, _normalize_rope_scaling(rope_scaling))
