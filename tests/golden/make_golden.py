"""Generates the golden fixtures in tests/golden/ by running the REFERENCE engine's own code
(kirsten-1/hilda-vllm, mini_vllm) on the CPU of the build container.

    python tests/golden/make_golden.py --reference /path/to/hilda-vllm

What runs from the reference, unmodified:
  - store_kvcache (mini_vllm/layers/attention.py:59-90, a Triton kernel) under TRITON_INTERPRET=1;
  - Scheduler / BlockManager / Sequence (mini_vllm/engine/*.py) driven by a seeded churn trace,
    and ModelRunner.prepare_decode / prepare_prefill (model_runner.py:551-720) bound to CPU
    tensors (pinned-memory and .cuda() calls become no-ops);
  - RMSNorm, RotaryEmbedding, SiluAndMul and the Qwen3 model modules (torch.compile disabled),
    with flash-attn replaced by the fp32 oracle (flash-attn has no CPU path).
The fixtures are small .npz / .json files; the tests never import the reference.
"""
from __future__ import annotations

import argparse
import json
import os
import random
import sys
from pathlib import Path
from types import SimpleNamespace

os.environ.setdefault("TRITON_INTERPRET", "1")
os.environ.setdefault("MINI_VLLM_DISABLE_TORCH_COMPILE", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().copy()


# --------------------------------------------------------------------------- store_kvcache
def golden_store(ref):
    """Config-1 shapes: 8 sequences, Hk=8, D=128, 64 blocks of 256."""
    from mini_vllm.layers.attention import store_kvcache

    g = torch.Generator().manual_seed(1)
    n, hq, hk, d, nb, bs = 8, 16, 8, 128, 64, 256
    qkv = torch.randn(n, (hq + 2 * hk) * d, generator=g).bfloat16()
    key = qkv[:, hq * d:(hq + hk) * d].view(n, hk, d)
    value = qkv[:, (hq + hk) * d:].view(n, hk, d)
    ctx = torch.randint(16, 1025, (n,), generator=g)
    perm = torch.randperm(nb, generator=g)
    tables, off = [], 0
    for L in ctx.tolist():
        nblk = -(-L // bs)
        tables.append(perm[off:off + nblk].tolist())
        off += nblk
    slots = [tables[i][(L - 1) // bs] * bs + (L - 1) % bs for i, L in enumerate(ctx.tolist())]
    slots[3] = -1  # a padding row must be skipped
    slot_mapping = torch.tensor(slots, dtype=torch.int32)
    k_cache = torch.zeros(nb, bs, hk, d).bfloat16()
    v_cache = torch.zeros(nb, bs, hk, d).bfloat16()
    store_kvcache(key, value, k_cache, v_cache, slot_mapping)
    touched = [s for s in slots if s >= 0]
    np.savez_compressed(
        HERE / "store_kv.npz", qkv=bits(qkv), slot_mapping=slot_mapping.numpy(), context_lens=ctx.numpy().astype(np.int32),
        block_tables=np.array([t + [-1] * (4 - len(t)) for t in tables], np.int32),
        touched_slots=np.array(touched, np.int64),
        k_rows=bits(k_cache.view(-1, hk * d)[touched]), v_rows=bits(v_cache.view(-1, hk * d)[touched]),
        k_nonzero_rows=np.array(sorted(set(torch.nonzero(k_cache.view(-1, hk * d).float().abs().sum(1)).flatten().tolist())), np.int64),
        shape=np.array([n, hq, hk, d, nb, bs]))


# --------------------------------------------------------------------------- scheduler trace
class _CpuTensorShim:
    """Makes the reference runner's pinned / .cuda() tensor calls run on the CPU."""

    def __enter__(self):
        self._tensor = torch.tensor
        self._cuda = torch.Tensor.cuda
        orig = self._tensor

        def tensor(*a, **k):
            k.pop("pin_memory", None)
            if k.get("device") == "cuda":
                k["device"] = "cpu"
            return orig(*a, **k)

        torch.tensor = tensor
        torch.Tensor.cuda = lambda self, *a, **k: self
        return self

    def __exit__(self, *exc):
        torch.tensor = self._tensor
        torch.Tensor.cuda = self._cuda


def _make_runner(max_bs, max_blocks, block_size):
    from mini_vllm.engine.model_runner import ModelRunner

    r = ModelRunner.__new__(ModelRunner)
    r.block_size = block_size
    r.max_num_decode_blocks = max_blocks
    r.enforce_eager = False
    r.graph_bs = [1, 2, 4, 8] + list(range(16, max_bs + 1, 16))
    r.debug_persistent_batching = False
    r.last_decode_batch_info = None
    r.decode_cpu_staging = dict(
        input_ids=torch.zeros(max_bs, dtype=torch.int64), positions=torch.zeros(max_bs, dtype=torch.int64),
        slot_mapping=torch.zeros(max_bs, dtype=torch.int32), context_lens=torch.zeros(max_bs, dtype=torch.int32),
        block_table_row=torch.zeros(max_blocks, dtype=torch.int32))
    r.decode_slot_seq_ids = [-1] * max_bs
    r.decode_slot_block_table_lens = [0] * max_bs
    r.decode_gpu_buffers = dict(
        input_ids=torch.zeros(max_bs, dtype=torch.int64), positions=torch.zeros(max_bs, dtype=torch.int64),
        slot_mapping=torch.full((max_bs,), -1, dtype=torch.int32), context_lens=torch.zeros(max_bs, dtype=torch.int32),
        block_tables=torch.full((max_bs, max_blocks), -1, dtype=torch.int32))
    return r


def golden_schedule_trace(ref, name, seed, num_seqs, max_bs, num_blocks, block_size, max_model_len,
                          prompt_range, out_range, eos, max_steps, chunk, shared_prefix=0):
    from mini_vllm.engine.scheduler import Scheduler
    from mini_vllm.engine.sequence import Sequence
    from mini_vllm.sampling_params import SamplingParams
    import itertools

    rng = random.Random(seed)
    Sequence.counter = itertools.count()
    cfg = SimpleNamespace(max_num_seqs=max_bs, max_num_batched_tokens=max(chunk * 2, max_model_len), eos=eos,
                          num_kvcache_blocks=num_blocks, kvcache_block_size=block_size, enable_chunked_prefill=True,
                          chunked_prefill_size=chunk, chunked_prefill_min_size=max(1, chunk // 4),
                          chunked_prefill_tile_size=max(1, chunk // 4))
    sched = Scheduler(cfg)
    max_blocks = -(-max_model_len // block_size)
    runner = _make_runner(max_bs, max_blocks, block_size)
    prefix = [rng.randrange(1, 50) for _ in range(shared_prefix)]
    prompts, params = [], []
    for i in range(num_seqs):
        plen = rng.randint(*prompt_range)
        body = [rng.randrange(1, 50) for _ in range(plen)]
        prompts.append((prefix + body)[:max(plen, 1)] if shared_prefix and i % 2 == 0 else body)
        params.append((rng.randint(*out_range), rng.random() < 0.7))
    pending = list(range(num_seqs))
    seqs = {}
    steps = []
    with _CpuTensorShim():
        for step in range(max_steps):
            # Admit new requests over time.
            while pending and rng.random() < 0.6:
                i = pending.pop(0)
                mt, ign = params[i]
                s = Sequence(prompts[i], SamplingParams(max_tokens=mt, ignore_eos=ign))
                seqs[s.seq_id] = s
                sched.add(s)
            if sched.is_finished():
                if not pending:
                    break
                continue
            try:
                scheduled, is_prefill = sched.schedule()
            except RuntimeError as exc:  # the reference's own "no runnable work" stop
                steps.append({"error": str(exc), "admitted": sorted(seqs.keys())})
                break
            rec = {"is_prefill": is_prefill,
                   "sched": [[s.slot_index, -1 if s.seq is None else s.seq.seq_id, s.token_chunk_size] for s in scheduled],
                   "admitted": sorted(seqs.keys())}
            if is_prefill:
                ids, pos = runner.prepare_prefill(scheduled)
                from mini_vllm.utils.context import get_context
                c = get_context()
                rec["prefill"] = {"input_ids": ids.tolist(), "positions": pos.tolist(),
                                  "cu_q": c.cu_seqlens_q.tolist(), "cu_k": c.cu_seqlens_k.tolist(),
                                  "max_q": c.max_seqlen_q, "max_k": c.max_seqlen_k,
                                  "slot_mapping": c.slot_mapping.tolist(),
                                  "block_tables": None if c.block_tables is None else c.block_tables.tolist()}
                toks = [rng.randrange(1, 50) if s.requires_sampling else None for s in scheduled]
            else:
                bs = len(scheduled)
                graph_bs = runner._decode_graph_batch_size(bs)
                runner.prepare_decode(scheduled)
                gb = runner.decode_gpu_buffers
                rec["graph_bs"] = graph_bs
                rec["decode"] = {k: gb[k][:graph_bs].tolist() for k in
                                 ("input_ids", "positions", "slot_mapping", "context_lens", "block_tables")}
                toks = [None if s.is_padding else (eos if rng.random() < 0.03 else rng.randrange(1, 50)) for s in scheduled]
            rec["tokens"] = toks
            sched.postprocess(scheduled, toks, is_prefill)
            rec["after"] = {"decode_slots": [-1 if s is None else s.seq_id for s in sched.decode_slots],
                            "persistent_batch_size": sched.persistent_batch_size,
                            "free_slots": sorted(sched.free_slot_indices),
                            "free_blocks": list(sched.block_manager.free_block_ids),
                            "waiting": [s.seq_id for s in sched.waiting],
                            "block_tables": {str(k): list(v.block_table) for k, v in seqs.items() if v.block_table},
                            "finished": sorted(k for k, v in seqs.items() if v.is_finished)}
            steps.append(rec)
    meta = {"seed": seed, "num_seqs": num_seqs, "max_bs": max_bs, "num_blocks": num_blocks, "block_size": block_size,
            "max_model_len": max_model_len, "eos": eos, "chunk": chunk, "prompts": prompts,
            "params": params, "cfg": vars(cfg)}
    with open(HERE / f"{name}.json", "w") as f:
        json.dump({"meta": meta, "steps": steps}, f, separators=(",", ":"))
    return len(steps)


# --------------------------------------------------------------------------- layers
def golden_layers(ref):
    from mini_vllm.layers.activation import SiluAndMul
    from mini_vllm.layers.layernorm import RMSNorm
    from mini_vllm.layers.rotary_embedding import get_rope

    g = torch.Generator().manual_seed(2)
    out = {}
    x = (torch.randn(16, 1024, generator=g) * 3).bfloat16()
    r = torch.randn(16, 1024, generator=g).bfloat16()
    norm = RMSNorm(1024, eps=1e-6)
    with torch.no_grad():
        norm.weight.copy_((1 + 0.1 * torch.randn(1024, generator=g)).bfloat16().float())
    norm = norm.bfloat16()
    y = norm(x)
    y2, r2 = norm(x, r.clone())
    out.update(rms_x=bits(x), rms_r=bits(r), rms_w=bits(norm.weight.data), rms_y=bits(y), add_y=bits(y2), add_r=bits(r2))
    # q/k norm + rope on a [T, H, 128] slice (Qwen3Attention.forward, qwen3.py:82-85)
    rope = get_rope(128, 128, 4096, 1000000.0, None)
    qn = RMSNorm(128, eps=1e-6)
    with torch.no_grad():
        qn.weight.copy_((1 + 0.1 * torch.randn(128, generator=g)).bfloat16().float())
    qn = qn.bfloat16()
    q = torch.randn(12, 4, 128, generator=g).bfloat16()
    pos = torch.randint(0, 4096, (12,), generator=g)
    qq = qn(q)
    rq, _ = rope(pos, qq, qq.clone())
    out.update(rope_q=bits(q), rope_w=bits(qn.weight.data), rope_pos=pos.numpy(), rope_out=bits(rq))
    a = torch.randn(10, 2 * 768, generator=g).bfloat16()
    out.update(silu_in=bits(a), silu_out=bits(SiluAndMul()(a)))
    np.savez_compressed(HERE / "layers.npz", **out)


# --------------------------------------------------------------------------- tiny model
def golden_tiny_model(ref):
    """A small Qwen3 (2 layers, hidden 256, 4 Q / 2 KV heads of 128, vocab 512) with weights
    from hilda_vllm_b200's seeded random init, run through the reference modules: prefill of
    three prompts, then greedy decode steps; records every step's greedy tokens and top-2 gap."""
    import torch.distributed as dist
    from transformers import Qwen3Config

    from hilda_vllm_b200.utils.loader import random_init
    from oracle import attention as oattn

    if not dist.is_initialized():
        dist.init_process_group("gloo", init_method="tcp://127.0.0.1:29533", world_size=1, rank=0)
    import mini_vllm.layers.attention as ref_attn
    from mini_vllm.models.qwen3 import Qwen3ForCausalLM
    from mini_vllm.utils.context import reset_context, set_context

    def fa_varlen(q, k, v, max_seqlen_q, cu_seqlens_q, max_seqlen_k, cu_seqlens_k, softmax_scale, causal,
                  block_table=None):
        return oattn.varlen_prefill(q, k, v, cu_seqlens_q, cu_seqlens_k, softmax_scale, block_table).to(q.dtype)

    def fa_kvcache(q, k_cache, v_cache, cache_seqlens, block_table, softmax_scale, causal):
        return oattn.paged_decode(q.squeeze(1), k_cache, v_cache, block_table, cache_seqlens, softmax_scale).to(
            q.dtype).unsqueeze(1)

    ref_attn.flash_attn_varlen_func = fa_varlen
    ref_attn.flash_attn_with_kvcache = fa_kvcache
    cfg = tiny_config()
    torch.set_default_dtype(torch.bfloat16)
    model = Qwen3ForCausalLM(cfg)
    torch.set_default_dtype(torch.float32)
    random_init(model, cfg, seed=7, std=0.02, device="cpu")
    nb, bs, hk, d = 16, 256, cfg.num_key_value_heads, 128
    kv = torch.zeros(2, cfg.num_hidden_layers, nb, bs, hk, d, dtype=torch.bfloat16)
    layer = 0
    for m in model.modules():
        if hasattr(m, "k_cache") and hasattr(m, "v_cache"):
            m.k_cache, m.v_cache = kv[0, layer], kv[1, layer]
            layer += 1
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (5, 37, 300)]
    tables = [[0], [1], [2, 3]]
    ids, pos, sm, cu = [], [], [], [0]
    for p, t in zip(prompts, tables):
        ids += p
        pos += list(range(len(p)))
        sm += [t[i // bs] * bs + i % bs for i in range(len(p))]
        cu.append(cu[-1] + len(p))
    cu_t = torch.tensor(cu, dtype=torch.int32)
    set_context(True, cu_t, cu_t, max(len(p) for p in prompts), max(len(p) for p in prompts),
                torch.tensor(sm, dtype=torch.int32), None, None)
    with torch.no_grad():
        logits = model.compute_logits(model(torch.tensor(ids), torch.tensor(pos)))
    reset_context()
    steps = []
    toks = logits.argmax(-1).tolist()
    gaps = (logits.float().topk(2, -1).values[:, 0] - logits.float().topk(2, -1).values[:, 1]).tolist()
    steps.append({"tokens": toks, "gap": gaps})
    seqs = [p + [t] for p, t in zip(prompts, toks)]
    for _ in range(8):
        lens = [len(s) for s in seqs]
        for s, t in zip(seqs, tables):
            if (len(s) - 1) // bs >= len(t):
                t.append(max(max(x) for x in tables) + 1)
        sm = [t[(n - 1) // bs] * bs + (n - 1) % bs for n, t in zip(lens, tables)]
        bt = torch.tensor([t + [-1] * (4 - len(t)) for t in tables], dtype=torch.int32)
        set_context(False, slot_mapping=torch.tensor(sm, dtype=torch.int32),
                    context_lens=torch.tensor(lens, dtype=torch.int32), block_tables=bt)
        with torch.no_grad():
            logits = model.compute_logits(model(torch.tensor([s[-1] for s in seqs]), torch.tensor([n - 1 for n in lens])))
        reset_context()
        toks = logits.argmax(-1).tolist()
        top = logits.float().topk(2, -1).values
        steps.append({"tokens": toks, "gap": (top[:, 0] - top[:, 1]).tolist()})
        seqs = [s + [t] for s, t in zip(seqs, toks)]
    with open(HERE / "tiny_model_greedy.json", "w") as f:
        json.dump({"prompts": prompts, "seed": 7, "steps": steps, "config": tiny_config_dict()}, f)


def golden_qwen3_0_6b(ref, decode_steps=32):
    """The Qwen3-0.6B configuration of this repository (28 layers, hidden 1024, 16 Q / 8 KV heads,
    vocab 151,936, tied embeddings) with the seeded random init, run through the reference
    modules: prefill of four 64-token prompts, then `decode_steps` free-running greedy decode
    steps; records each step's greedy tokens, the top-1 logit and the top-1 minus top-2 gap."""
    import torch.distributed as dist
    from transformers import AutoConfig

    from hilda_vllm_b200.utils.loader import random_init
    from oracle import attention as oattn

    if not dist.is_initialized():
        dist.init_process_group("gloo", init_method="tcp://127.0.0.1:29534", world_size=1, rank=0)
    import mini_vllm.layers.attention as ref_attn
    from mini_vllm.models.qwen3 import Qwen3ForCausalLM
    from mini_vllm.utils.context import reset_context, set_context

    def fa_varlen(q, k, v, max_seqlen_q, cu_seqlens_q, max_seqlen_k, cu_seqlens_k, softmax_scale, causal,
                  block_table=None):
        return oattn.varlen_prefill(q, k, v, cu_seqlens_q, cu_seqlens_k, softmax_scale, block_table).to(q.dtype)

    def fa_kvcache(q, k_cache, v_cache, cache_seqlens, block_table, softmax_scale, causal):
        return oattn.paged_decode(q.squeeze(1), k_cache, v_cache, block_table, cache_seqlens, softmax_scale).to(
            q.dtype).unsqueeze(1)

    ref_attn.flash_attn_varlen_func = fa_varlen
    ref_attn.flash_attn_with_kvcache = fa_kvcache
    cfg_dir = ROOT / "hilda_vllm_b200" / "model_configs" / "qwen3-0.6b"
    cfg = AutoConfig.from_pretrained(cfg_dir)
    torch.set_default_dtype(torch.bfloat16)
    model = Qwen3ForCausalLM(cfg)
    torch.set_default_dtype(torch.float32)
    seed = 11
    random_init(model, cfg, seed=seed, std=0.02, device="cpu")
    nb, bs, hk, d = 4, 256, cfg.num_key_value_heads, 128
    kv = torch.zeros(2, cfg.num_hidden_layers, nb, bs, hk, d, dtype=torch.bfloat16)
    layer = 0
    for m in model.modules():
        if hasattr(m, "k_cache") and hasattr(m, "v_cache"):
            m.k_cache, m.v_cache = kv[0, layer], kv[1, layer]
            layer += 1
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, cfg.vocab_size, (64,), generator=g).tolist() for _ in range(4)]
    tables = [[0], [1], [2], [3]]
    ids, pos, sm, cu = [], [], [], [0]
    for p, t in zip(prompts, tables):
        ids += p
        pos += list(range(len(p)))
        sm += [t[0] * bs + i for i in range(len(p))]
        cu.append(cu[-1] + len(p))
    cu_t = torch.tensor(cu, dtype=torch.int32)
    set_context(True, cu_t, cu_t, 64, 64, torch.tensor(sm, dtype=torch.int32), None, None)
    with torch.no_grad():
        logits = model.compute_logits(model(torch.tensor(ids), torch.tensor(pos)))
    reset_context()

    def record(lg):
        top = lg.float().topk(2, -1).values
        return {"tokens": lg.argmax(-1).tolist(), "top1": top[:, 0].tolist(), "gap": (top[:, 0] - top[:, 1]).tolist()}

    steps = [record(logits)]
    seqs = [p + [t] for p, t in zip(prompts, steps[0]["tokens"])]
    for _ in range(decode_steps):
        lens = [len(s) for s in seqs]
        sm = [t[0] * bs + n - 1 for n, t in zip(lens, tables)]
        bt = torch.tensor(tables, dtype=torch.int32)
        set_context(False, slot_mapping=torch.tensor(sm, dtype=torch.int32),
                    context_lens=torch.tensor(lens, dtype=torch.int32), block_tables=bt)
        with torch.no_grad():
            logits = model.compute_logits(model(torch.tensor([s[-1] for s in seqs]), torch.tensor([n - 1 for n in lens])))
        reset_context()
        steps.append(record(logits))
        seqs = [s + [t] for s, t in zip(seqs, steps[-1]["tokens"])]
    with open(HERE / "qwen3_0_6b_greedy_32.json", "w") as f:
        json.dump({"prompts": prompts, "seed": seed, "steps": steps, "config_dir": "hilda_vllm_b200/model_configs/qwen3-0.6b"}, f)


def tiny_config_dict():
    return dict(architectures=["Qwen3ForCausalLM"], model_type="qwen3", attention_bias=False, hidden_act="silu",
                hidden_size=256, intermediate_size=512, num_attention_heads=4, num_key_value_heads=2, head_dim=128,
                num_hidden_layers=2, max_position_embeddings=4096, rms_norm_eps=1e-6, rope_theta=1000000.0,
                vocab_size=512, tie_word_embeddings=True, torch_dtype="bfloat16")


def tiny_config():
    from transformers import Qwen3Config
    return Qwen3Config(**tiny_config_dict())


def golden_sampler(ref):
    """Kept-token masks of the reference Sampler's _apply_top_k / _apply_top_p
    (mini_vllm/layers/sampler.py:27-49) on seeded rows without equal logits, where the kept set
    does not depend on torch.sort's tie order."""
    from mini_vllm.layers.sampler import Sampler

    g = torch.Generator().manual_seed(31)
    rows, vocab = 48, 97
    logits = torch.randn(rows, vocab, generator=g) * 3
    temps = torch.rand(rows, generator=g) + 0.3
    top_ks = torch.randint(-1, vocab + 3, (rows,), generator=g)
    top_ks[top_ks == 0] = -1
    top_ps = (torch.rand(rows, generator=g) * 1.1).clamp(0.01, 1.0)
    top_ps[::5] = 1.0
    x = logits / temps.unsqueeze(1)
    masked = Sampler._apply_top_p(Sampler._apply_top_k(x.clone(), top_ks), top_ps)
    np.savez_compressed(HERE / "sampler_filters.npz", logits=logits.numpy(), temps=temps.numpy(),
                        top_ks=top_ks.numpy().astype(np.int32), top_ps=top_ps.numpy(),
                        keep=torch.isfinite(masked).numpy())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("HILDA_REFERENCE"),
                    help="checkout of kirsten-1/hilda-vllm (or set HILDA_REFERENCE)")
    ap.add_argument("--only", default="")
    args = ap.parse_args()
    if not args.reference:
        ap.error("pass --reference /path/to/hilda-vllm (or set HILDA_REFERENCE)")
    sys.path.insert(0, args.reference)
    only = set(filter(None, args.only.split(",")))
    if not only or "store" in only:
        golden_store(args.reference)
    if not only or "trace" in only:
        n1 = golden_schedule_trace(args.reference, "sched_trace_churn", seed=11, num_seqs=40, max_bs=16, num_blocks=40,
                                   block_size=4, max_model_len=48, prompt_range=(1, 14), out_range=(1, 24), eos=7,
                                   max_steps=400, chunk=8)
        n2 = golden_schedule_trace(args.reference, "sched_trace_prefix", seed=12, num_seqs=24, max_bs=8, num_blocks=64,
                                   block_size=4, max_model_len=64, prompt_range=(3, 30), out_range=(2, 12), eos=7,
                                   max_steps=400, chunk=8, shared_prefix=12)
        n3 = golden_schedule_trace(args.reference, "sched_trace_complete", seed=13, num_seqs=30, max_bs=16,
                                   num_blocks=400, block_size=4, max_model_len=48, prompt_range=(1, 14),
                                   out_range=(1, 30), eos=7, max_steps=600, chunk=16)
        print("trace steps", n1, n2, n3)
    if not only or "layers" in only:
        golden_layers(args.reference)
    if not only or "tiny" in only:
        golden_tiny_model(args.reference)
    if not only or "sampler" in only:
        golden_sampler(args.reference)
    if not only or "qwen3_0_6b" in only:
        golden_qwen3_0_6b(args.reference)


if __name__ == "__main__":
    main()
