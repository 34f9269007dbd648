"""Per-step attention metadata shared by every Attention layer of the model.

Same carrier as mini_vllm/utils/context.py:5-27 (module-global, replaced by set_context and
cleared by reset_context), so callers written against the reference work unchanged.
"""
from dataclasses import dataclass

import torch


@dataclass
class Context:
    is_prefill: bool = False
    cu_seqlens_q: torch.Tensor | None = None
    cu_seqlens_k: torch.Tensor | None = None
    max_seqlen_q: int = 0
    max_seqlen_k: int = 0
    slot_mapping: torch.Tensor | None = None
    context_lens: torch.Tensor | None = None
    block_tables: torch.Tensor | None = None


_CURRENT = Context()


def get_context() -> Context:
    return _CURRENT


def set_context(is_prefill, cu_seqlens_q=None, cu_seqlens_k=None, max_seqlen_q=0, max_seqlen_k=0,
                slot_mapping=None, context_lens=None, block_tables=None) -> None:
    global _CURRENT
    _CURRENT = Context(is_prefill, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, slot_mapping,
                       context_lens, block_tables)


def reset_context() -> None:
    global _CURRENT
    _CURRENT = Context()
