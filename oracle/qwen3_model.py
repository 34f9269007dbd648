"""Qwen3 forward with the reference engine's arithmetic, in plain torch (TEST ORACLE ONLY).

Restates mini_vllm/models/qwen3.py:15-218 and the layers it uses, eager (torch.compile off):
  RMSNorm        layers/layernorm.py:18-42 (x.float(); x * rsqrt(mean(x^2) + eps); to bf16; * w;
                 add_rms: residual = bf16(x + r) and the norm of the fp32 sum)
  RoPE           layers/rotary_embedding.py:8-50 (NeoX halves, fp32 cos/sin cache, theta 1e6)
  SiluAndMul     layers/activation.py:12-16
  attention      store_kvcache (attention.py:59-90) + the fp32 attention restatements of
                 oracle.attention in place of flash-attn
  LM head        embed_head.py:56-66 (prefill keeps each sequence's last row)
Device-agnostic: runs on CPU (the CPU baseline and the golden pin) or on CUDA tensors (the
greedy-parity reference for the GPU engine, where only the attention path differs).
Weights come as a dict of Hugging Face checkpoint names -> tensors.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from oracle import attention as oattn
from oracle import kv_store


class Qwen3Oracle:

    def __init__(self, hf_config, weights: dict[str, torch.Tensor], num_blocks: int, block_size: int,
                 device="cpu", dtype=torch.bfloat16, kv_fp8: bool = False, kv_scale: float = 1.0):
        c = hf_config
        self.c = c
        self.device = torch.device(device)
        self.dtype = dtype
        self.w = {k: v.to(self.device, dtype) for k, v in weights.items()}
        if "lm_head.weight" not in self.w:
            self.w["lm_head.weight"] = self.w["model.embed_tokens.weight"]
        self.hq = c.num_attention_heads
        self.hk = c.num_key_value_heads
        self.d = getattr(c, "head_dim", None) or c.hidden_size // c.num_attention_heads
        self.eps = c.rms_norm_eps
        self.block_size = block_size
        base = getattr(c, "rope_theta", None)
        scaling = getattr(c, "rope_scaling", None) or {}
        base = scaling.get("rope_theta", base) if isinstance(scaling, dict) else base
        inv_freq = 1.0 / (base ** (torch.arange(0, self.d, 2, dtype=torch.float, device=self.device) / self.d))
        t = torch.arange(c.max_position_embeddings, dtype=torch.float, device=self.device)
        freqs = torch.einsum("i,j -> ij", t, inv_freq)
        self.cos_sin = torch.cat((freqs.cos(), freqs.sin()), dim=-1)
        self.qkv_w, self.gate_up_w = [], []
        for i in range(c.num_hidden_layers):
            p = f"model.layers.{i}."
            self.qkv_w.append(torch.cat([self.w[p + f"self_attn.{n}_proj.weight"] for n in "qkv"], 0))
            self.gate_up_w.append(torch.cat([self.w[p + "mlp.gate_proj.weight"], self.w[p + "mlp.up_proj.weight"]], 0))
        shape = (c.num_hidden_layers, num_blocks, block_size, self.hk, self.d)
        self.k_cache = torch.zeros(shape, dtype=dtype, device=self.device)
        self.v_cache = torch.zeros(shape, dtype=dtype, device=self.device)
        # FP8 KV mode (attention.py:114-141, model_runner.py:186-194, 483-502): the bf16 caches above
        # are the prefill cache, k8/v8 the e4m3 decode cache with per-head scales.  Prefill writes
        # and reads bf16; convert() quantises prompt rows into the decode cache; a decode step
        # stores its new row quantised (and, as intended, in bf16 too, so the prefill cache holds
        # every token) and attends over the dequantised e4m3 cache.
        self.kv_fp8 = kv_fp8
        if kv_fp8:
            self.k8 = torch.zeros(shape, dtype=torch.uint8, device=self.device)
            self.v8 = torch.zeros(shape, dtype=torch.uint8, device=self.device)
            self.k_scale = torch.full((self.hk,), float(kv_scale), dtype=torch.float32, device=self.device)
            self.v_scale = torch.full((self.hk,), float(kv_scale), dtype=torch.float32, device=self.device)

    # -- layers (reference arithmetic) --
    def rms(self, x, w):
        xf = x.float()
        var = xf.pow(2).mean(dim=-1, keepdim=True)
        xf = xf * torch.rsqrt(var + self.eps)
        return xf.to(x.dtype) * w

    def add_rms(self, x, r, w):
        xf = x.float() + r.float()
        res = xf.to(x.dtype)
        var = xf.pow(2).mean(dim=-1, keepdim=True)
        xf = xf * torch.rsqrt(var + self.eps)
        return xf.to(x.dtype) * w, res

    def rope(self, x, positions):
        cs = self.cos_sin[positions].unsqueeze(1)
        cos, sin = cs.chunk(2, dim=-1)
        x1, x2 = torch.chunk(x.float(), 2, dim=-1)
        return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1).to(x.dtype)

    def store(self, layer, k, v, slot_mapping):
        kf = self.k_cache[layer].view(-1, self.hk * self.d)
        vf = self.v_cache[layer].view(-1, self.hk * self.d)
        sm = slot_mapping.to(self.device).long()
        keep = sm >= 0
        kf[sm[keep]] = k.reshape(k.shape[0], -1)[keep]
        vf[sm[keep]] = v.reshape(v.shape[0], -1)[keep]

    def convert(self, slots):
        """FP8 mode: quantise the bf16 prefill-cache rows at `slots` into the e4m3 decode cache of
        every layer (copy_kvcache_fp8, attention.py:55-56)."""
        sl = torch.as_tensor(slots, dtype=torch.long, device=self.device)
        for layer in range(self.c.num_hidden_layers):
            for src, dst, sc in ((self.k_cache, self.k8, self.k_scale), (self.v_cache, self.v8, self.v_scale)):
                rows = src[layer].view(-1, self.hk, self.d)[sl]
                dst[layer].view(-1, self.hk, self.d)[sl] = kv_store.quantize_e4m3_torch(rows, sc)

    def attention(self, layer, q, k, v, ctx):
        self.store(layer, k, v, ctx["slot_mapping"])
        scale = self.d ** -0.5
        if self.kv_fp8 and not ctx["is_prefill"]:
            sm = ctx["slot_mapping"].to(self.device).long()
            keep = sm >= 0
            for src, dst, sc in ((k, self.k8, self.k_scale), (v, self.v8, self.v_scale)):
                dst[layer].view(-1, self.hk, self.d)[sm[keep]] = kv_store.quantize_e4m3_torch(src[keep], sc)
            o = oattn.paged_decode(q, self.k8[layer], self.v8[layer], ctx["block_tables"], ctx["context_lens"], scale,
                                   self.k_scale, self.v_scale, fp8=True)
            return o.to(self.dtype)
        if ctx["is_prefill"]:
            if ctx.get("block_tables") is not None:
                o = oattn.varlen_prefill(q, self.k_cache[layer], self.v_cache[layer], ctx["cu_seqlens_q"],
                                         ctx["cu_seqlens_k"], scale, block_table=ctx["block_tables"].cpu())
            else:
                o = oattn.varlen_prefill(q, k, v, ctx["cu_seqlens_q"], ctx["cu_seqlens_k"], scale)
        else:
            o = oattn.paged_decode(q, self.k_cache[layer], self.v_cache[layer], ctx["block_tables"],
                                   ctx["context_lens"], scale)
        return o.to(self.dtype)

    def forward(self, input_ids, positions, ctx):
        w = self.w
        h = F.embedding(input_ids.to(self.device), w["model.embed_tokens.weight"])
        positions = positions.to(self.device)
        residual = None
        for i in range(self.c.num_hidden_layers):
            p = f"model.layers.{i}."
            if residual is None:
                x, residual = self.rms(h, w[p + "input_layernorm.weight"]), h
            else:
                x, residual = self.add_rms(h, residual, w[p + "input_layernorm.weight"])
            qkv = F.linear(x, self.qkv_w[i])  # the reference's fused QKVParallelLinear
            q, k, v = qkv.split([self.hq * self.d, self.hk * self.d, self.hk * self.d], dim=-1)
            q = q.reshape(-1, self.hq, self.d)
            k = k.reshape(-1, self.hk, self.d)
            v = v.reshape(-1, self.hk, self.d)
            q = self.rope(self.rms(q, w[p + "self_attn.q_norm.weight"]), positions)
            k = self.rope(self.rms(k, w[p + "self_attn.k_norm.weight"]), positions)
            o = self.attention(i, q, k, v, ctx)
            h = F.linear(o.reshape(o.shape[0], -1), w[p + "self_attn.o_proj.weight"])
            x, residual = self.add_rms(h, residual, w[p + "post_attention_layernorm.weight"])
            gate, up = F.linear(x, self.gate_up_w[i]).chunk(2, -1)  # MergedColumnParallelLinear
            h = F.linear(F.silu(gate) * up, w[p + "mlp.down_proj.weight"])
        h, _ = self.add_rms(h, residual, w["model.norm.weight"])
        return h

    def logits(self, hidden, ctx):
        if ctx["is_prefill"]:
            hidden = hidden[ctx["cu_seqlens_q"][1:].to(self.device).long() - 1]
        return F.linear(hidden, self.w["lm_head.weight"])


def prefill_context(seqs_tokens, starts, ends, block_tables, block_size):
    """Reference prepare_prefill (mini_vllm/engine/model_runner.py:614-650) for chunks
    [start, end) of each sequence; returns (input_ids, positions, ctx)."""
    ids, pos, sm = [], [], []
    cu_q, cu_k = [0], [0]
    has_prefix = False
    for toks, s, e, bt in zip(seqs_tokens, starts, ends, block_tables):
        ids += toks[s:e]
        pos += list(range(s, e))
        cu_q.append(cu_q[-1] + e - s)
        cu_k.append(cu_k[-1] + e)
        has_prefix = has_prefix or s > 0
        sm += [bt[p // block_size] * block_size + p % block_size for p in range(s, e)]
    bts = None
    if has_prefix:
        width = max(len(bt) for bt in block_tables)
        bts = torch.tensor([bt + [-1] * (width - len(bt)) for bt in block_tables], dtype=torch.int32)
    ctx = {"is_prefill": True, "cu_seqlens_q": torch.tensor(cu_q, dtype=torch.int32),
           "cu_seqlens_k": torch.tensor(cu_k, dtype=torch.int32), "slot_mapping": torch.tensor(sm, dtype=torch.int32),
           "block_tables": bts}
    return torch.tensor(ids, dtype=torch.int64), torch.tensor(pos, dtype=torch.int64), ctx


def decode_context(lengths, last_tokens, block_tables, block_size, width):
    """Reference prepare_decode for live rows (model_runner.py:684-689)."""
    sm = [bt[-1] * block_size + (n - 1) % block_size for n, bt in zip(lengths, block_tables)]
    bts = torch.tensor([bt + [-1] * (width - len(bt)) for bt in block_tables], dtype=torch.int32)
    ctx = {"is_prefill": False, "slot_mapping": torch.tensor(sm, dtype=torch.int32),
           "context_lens": torch.tensor(lengths, dtype=torch.int32), "block_tables": bts}
    return (torch.tensor(last_tokens, dtype=torch.int64), torch.tensor([n - 1 for n in lengths], dtype=torch.int64),
            ctx)
