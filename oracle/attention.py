"""fp32 attention restatements (TEST ORACLE ONLY).

paged_decode: the reference calls flash_attn_with_kvcache(q.unsqueeze(1), k_cache, v_cache,
cache_seqlens=context_lens, block_table=block_tables, softmax_scale=scale, causal=True)
(mini_vllm/layers/attention.py:162-170) and, for FP8, hilda_paged_attention_fp8_decode
(attention.py:134-141).  For sequence b with L = context_lens[b] cached tokens, token j sits at
slot block_tables[b, j // BS] * BS + j % BS; query head h reads KV head h // (Hq/Hk);
out = softmax(scale * q K^T) V over j < L (a single query token sees every cached token).
L = 0 gives zeros.

varlen_prefill: flash_attn_varlen_func(..., causal=True, block_table) (attention.py:120-131,
149-160).  Sequence s has Lq = cu_q[s+1]-cu_q[s] queries and Lk = cu_k[s+1]-cu_k[s] keys; query
i sees keys j <= i + Lk - Lq (flash-attn aligns the causal mask to the bottom-right corner).
With a block table, key j of sequence s comes from the paged cache; without, from row
cu_k[s] + j of k / v.  Rows with no visible key are zero.
"""
from __future__ import annotations

import torch


def _gather_pages(cache, table_row, length, block_size):
    n_pages = -(-length // block_size)
    pages = torch.as_tensor(table_row[:n_pages], dtype=torch.long, device=cache.device)
    return cache[pages].reshape(-1, cache.shape[2], cache.shape[3])[:length]


def _attend(q, k, v, scale, mask=None):
    """q [Tq, Hq, D], k/v [Tk, Hk, D] fp32 -> [Tq, Hq, D]."""
    g = q.shape[1] // k.shape[1]
    k = k.repeat_interleave(g, dim=1)
    v = v.repeat_interleave(g, dim=1)
    s = torch.einsum("qhd,khd->hqk", q, k) * scale
    if mask is not None:
        s = s.masked_fill(~mask.unsqueeze(0), float("-inf"))
    row_has = torch.isfinite(s).any(-1, keepdim=True)
    p = torch.softmax(s, dim=-1)
    p = torch.where(row_has, p, torch.zeros_like(p))
    return torch.einsum("hqk,khd->qhd", p, v)


def paged_decode(q, k_cache, v_cache, block_tables, context_lens, scale, k_scale=None, v_scale=None,
                 fp8=False):
    """q [B, Hq, D]; caches [NB, BS, Hk, D] (bf16, or uint8 e4m3 bytes when fp8=True)."""
    from oracle.kv_store import dequantize_e4m3

    b, hq, d = q.shape
    bs = k_cache.shape[1]
    out = torch.zeros(b, hq, d, dtype=torch.float32, device=q.device)
    for i in range(b):
        length = int(context_lens[i])
        if length <= 0:
            continue
        row = block_tables[i].tolist()
        k = _gather_pages(k_cache, row, length, bs)
        v = _gather_pages(v_cache, row, length, bs)
        if fp8:
            k = dequantize_e4m3(k, k_scale)
            v = dequantize_e4m3(v, v_scale)
        out[i] = _attend(q[i:i + 1].float(), k.float(), v.float(), scale)[0]
    return out


def varlen_prefill(q, k, v, cu_seqlens_q, cu_seqlens_k, scale, block_table=None):
    tq, hq, d = q.shape
    out = torch.zeros(tq, hq, d, dtype=torch.float32, device=q.device)
    cq = cu_seqlens_q.tolist()
    ck = cu_seqlens_k.tolist()
    for s in range(len(cq) - 1):
        q0, q1 = cq[s], cq[s + 1]
        lq, lk = q1 - q0, ck[s + 1] - ck[s]
        if lq <= 0:
            continue
        if block_table is not None:
            bs = k.shape[1]
            kk = _gather_pages(k, block_table[s].tolist(), lk, bs)
            vv = _gather_pages(v, block_table[s].tolist(), lk, bs)
        else:
            kk, vv = k[ck[s]:ck[s + 1]], v[ck[s]:ck[s + 1]]
        i = torch.arange(lq, device=q.device).unsqueeze(1)
        j = torch.arange(lk, device=q.device).unsqueeze(0)
        mask = j <= i + (lk - lq)
        out[q0:q1] = _attend(q[q0:q1].float(), kk.float(), vv.float(), scale, mask)
    return out
