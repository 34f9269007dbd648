"""Attention layer: KV-cache store + paged decode / varlen prefill on the sm_100a kernels.

Drop-in for mini_vllm/layers/attention.py:93-170: same constructor, same module attributes
(k_cache/v_cache, kv_cache_dtype, prefill_*/decode_* for the FP8 mode) filled in by the model
runner, same forward(q, k, v) reading the global Context, same return shapes ([T, Hq, D] for
prefill, [B, 1, Hq, D] for decode).  The work goes through the C ABI (hilda_vllm_b200.kernels);
there is no flash-attn, Triton or CPU path.
"""
import torch
from torch import nn

from hilda_vllm_b200 import kernels
from hilda_vllm_b200.utils.context import get_context


# Module-level entry points with the reference's names and signatures.
def store_kvcache(key, value, k_cache, v_cache, slot_mapping):
    kernels.store_kvcache(key, value, k_cache, v_cache, slot_mapping)


def store_kvcache_fp8(key, value, k_cache, v_cache, slot_mapping, k_scale=None, v_scale=None):
    kernels.store_kvcache_fp8(key, value, k_cache, v_cache, slot_mapping, k_scale, v_scale)


def copy_kvcache_fp8(src_k_cache, src_v_cache, dst_k_cache, dst_v_cache, slot_mapping, k_scale=None,
                     v_scale=None):
    kernels.copy_kvcache_fp8(src_k_cache, src_v_cache, dst_k_cache, dst_v_cache, slot_mapping, k_scale, v_scale)


class Attention(nn.Module):

    def __init__(self, num_heads, head_dim, scale, num_kv_heads):
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.scale = scale
        self.num_kv_heads = num_kv_heads
        self.kv_cache_dtype = "auto"
        self.k_cache = self.v_cache = torch.tensor([])
        self.prefill_k_cache = self.prefill_v_cache = torch.tensor([])
        self.decode_k_cache = self.decode_v_cache = torch.tensor([])
        # Added by this build: per-KV-head FP8 scales and the decode split-K workspace,
        # both set by the model runner before CUDA-graph capture.
        self.k_scale: torch.Tensor | None = None
        self.v_scale: torch.Tensor | None = None
        self.decode_workspace: torch.Tensor | None = None

    def _store_target(self, context):
        """(k_cache, v_cache, k_scale, v_scale, mirror) this step's new K/V go to, or None before
        the KV pool exists (the reference's forward skips the store then, attention.py:146).
        FP8 decode steps also write the bf16 rows into the BF16 prefill cache (mirror), which the
        reference does not (attention.py:133): a block filled during decode can later be a
        prefix-cache hit whose BF16 rows the prefill reads and the prefill->decode copy re-quantises,
        and with the mirror those rows are the real ones instead of whatever the block held before."""
        if self.kv_cache_dtype == "fp8" and self.prefill_k_cache.numel() and self.decode_k_cache.numel():
            if context.is_prefill:
                return self.prefill_k_cache, self.prefill_v_cache, None, None, None
            return (self.decode_k_cache, self.decode_v_cache, self.k_scale, self.v_scale,
                    (self.prefill_k_cache, self.prefill_v_cache))
        if self.k_cache.numel() and self.v_cache.numel():
            return self.k_cache, self.v_cache, None, None, None
        return None

    def rotate_and_store(self, qkv, q_weight, k_weight, cos_sin, positions, eps) -> bool:
        """The attention prologue in one launch: QK-RMSNorm + RoPE in place on the qkv rows
        (mini_vllm/models/qwen3.py:82-85) fused with the KV-cache store that forward() would
        do.  Returns True when the store happened, so the caller passes kv_stored=True."""
        context = get_context()
        target = self._store_target(context)
        if target is None or context.slot_mapping is None:
            kernels.qk_norm_rope(qkv, self.num_heads, self.num_kv_heads, self.head_dim, q_weight, k_weight, cos_sin,
                                 positions, eps)
            return False
        k_cache, v_cache, k_scale, v_scale, mirror = target
        k_mirror, v_mirror = mirror if mirror is not None else (None, None)
        kernels.qk_norm_rope_store(qkv, self.num_heads, self.num_kv_heads, self.head_dim, q_weight, k_weight, cos_sin,
                                   positions, eps, k_cache, v_cache, context.slot_mapping, k_scale, v_scale,
                                   k_mirror=k_mirror, v_mirror=v_mirror)
        return True

    def _prefill(self, q, k, v, k_cache, v_cache, context):
        if context.block_tables is not None:
            k, v = k_cache, v_cache
        return kernels.varlen_prefill(q, k, v, context.cu_seqlens_q, context.cu_seqlens_k, context.max_seqlen_q,
                                      context.max_seqlen_k, self.scale, block_table=context.block_tables)

    def _decode(self, q, k_cache, v_cache, context, k_scale=None, v_scale=None):
        out = kernels.paged_decode(q, k_cache, v_cache, context.block_tables, context.context_lens, self.scale,
                                   workspace=self.decode_workspace, k_scale=k_scale, v_scale=v_scale)
        return out.unsqueeze(1)

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, kv_stored: bool = False):
        """kv_stored=True: rotate_and_store already wrote k/v into the cache this step."""
        context = get_context()
        if self.kv_cache_dtype == "fp8" and self.prefill_k_cache.numel() and self.decode_k_cache.numel():
            if context.is_prefill:
                if not kv_stored:
                    store_kvcache(k, v, self.prefill_k_cache, self.prefill_v_cache, context.slot_mapping)
                return self._prefill(q, k, v, self.prefill_k_cache, self.prefill_v_cache, context)
            if not kv_stored:
                store_kvcache_fp8(k, v, self.decode_k_cache, self.decode_v_cache, context.slot_mapping,
                                  self.k_scale, self.v_scale)
                store_kvcache(k, v, self.prefill_k_cache, self.prefill_v_cache, context.slot_mapping)
            return self._decode(q, self.decode_k_cache, self.decode_v_cache, context, self.k_scale, self.v_scale)

        k_cache, v_cache = self.k_cache, self.v_cache
        if k_cache.numel() and v_cache.numel() and not kv_stored:
            store_kvcache(k, v, k_cache, v_cache, context.slot_mapping)
        if context.is_prefill:
            return self._prefill(q, k, v, k_cache, v_cache, context)
        return self._decode(q, k_cache, v_cache, context)
