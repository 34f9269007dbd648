"""Token embedding and LM head (mini_vllm/layers/embed_head.py:9-66).

Departure from the reference, on purpose: the input embedding is replicated on every
tensor-parallel rank (the reference shards it and all-reduces, embed_head.py:34-42), so the
only collectives inside the decode step are the all-reduces after o_proj and down_proj.  The
LM head stays vocabulary-sharded; with tp > 1 its logits are gathered to rank 0 as in the
reference (embed_head.py:56-66), or, for greedy decoding, every rank takes its shard's top-1
and the (value, index) pairs are all-gathered so all ranks know the token.
"""
import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch import nn

from hilda_vllm_b200.layers.linear import _tp
from hilda_vllm_b200.utils.context import get_context


class VocabParallelEmbedding(nn.Module):
    """Replicated embedding table [V, H] (every rank holds all rows)."""

    def __init__(self, num_embeddings: int, embedding_dim: int):
        super().__init__()
        self.tp_rank, self.tp_size = _tp()
        self.num_embeddings = num_embeddings
        self.weight = nn.Parameter(torch.empty(num_embeddings, embedding_dim))
        self.weight.weight_loader = self.weight_loader

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor):
        param.data.copy_(loaded_weight)

    def forward(self, x: torch.Tensor):
        return F.embedding(x, self.weight)


class ParallelLMHead(nn.Module):
    """Vocabulary-sharded LM head: rank r holds rows [r*V/tp, (r+1)*V/tp)."""

    def __init__(self, num_embeddings: int, embedding_dim: int, bias: bool = False):
        super().__init__()
        assert not bias
        self.tp_rank, self.tp_size = _tp()
        assert num_embeddings % self.tp_size == 0
        self.num_embeddings = num_embeddings
        self.num_embeddings_per_partition = num_embeddings // self.tp_size
        self.vocab_start_idx = self.num_embeddings_per_partition * self.tp_rank
        self.weight = nn.Parameter(torch.empty(self.num_embeddings_per_partition, embedding_dim))
        self.weight.weight_loader = self.weight_loader

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor):
        shard = param.data.size(0)
        param.data.copy_(loaded_weight.narrow(0, self.tp_rank * shard, shard))

    def select_rows(self, x: torch.Tensor) -> torch.Tensor:
        context = get_context()
        if context.is_prefill:
            x = x[context.cu_seqlens_q[1:] - 1].contiguous()
        return x

    def local_logits(self, x: torch.Tensor) -> torch.Tensor:
        return F.linear(self.select_rows(x), self.weight)

    def forward(self, x: torch.Tensor):
        logits = self.local_logits(x)
        if self.tp_size > 1:
            parts = [torch.empty_like(logits) for _ in range(self.tp_size)] if self.tp_rank == 0 else None
            dist.gather(logits, parts, 0)
            logits = torch.cat(parts, -1) if self.tp_rank == 0 else None
        return logits
