"""Engine-level parity at the BASELINE configurations beyond the headline one: the whole engine
(scheduler, block manager with prefix caching, preemption, chunked prefill, GPU decode packing,
CUDA graphs, FP8 KV) against the oracle Qwen3 forward, replaying the engine's own schedule.

The engine runs a job through LLM.generate with every step synchronous (async_decode off), and a
recorder keeps what each step fed the model runner: for a prefill step the chunk [start, end) of
every scheduled sequence with its token ids and block table, for a decode step every live
sequence's tokens and block table, plus the slot lists of the FP8 prefill->decode conversions,
and the tokens the step returned.  The oracle (oracle/qwen3_model.py, same weights, same GPU)
then replays those steps in order on its own KV pool of the same size, with the same block ids
and slots, and at every step where the engine sampled a token that token must be the oracle's
argmax or tie with it within two bf16 ulps of the top logit (the rule of test_gpu_engine.py).
Because the oracle consumes the engine's tokens, the check is teacher-forced, and because it
reuses the engine's block decisions, preemption, re-prefill after preemption, prefix-cache hits
and chunk boundaries are all exercised on identical data.

Configs (BASELINE.json configs[2..4], scaled to a test):
  c3  FP8 e4m3 KV with per-head scales and a capped pool that forces preemption, re-prefill
      (with prefix-cache hits on blocks filled during decode) and decode-batch compaction;
  c4  chunked prefill over shared 2048-token prefixes (hash hits, block_tables through the
      prefill kernel) mixed with decode sequences;
  c5  the Qwen3-8B layout (hidden 4096, 32 / 8 heads: GQA 4, the tcgen05 decode kernel) with
      the layer count cut to fit a test, BF16 and FP8 KV.
"""
import json
from pathlib import Path

import pytest
import torch

from hilda_vllm_b200 import LLM, SamplingParams
from hilda_vllm_b200.utils.loader import random_weights
from oracle.qwen3_model import Qwen3Oracle, decode_context, prefill_context

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent
CFG_06B = ROOT / "hilda_vllm_b200" / "model_configs" / "qwen3-0.6b"
CFG_8B = ROOT / "hilda_vllm_b200" / "model_configs" / "qwen3-8b"


class ScheduleRecorder:
    """Wraps a single-GPU LLM's model runner and records every step it executes."""

    def __init__(self, llm):
        self.events = []
        runner = llm.model_runner
        run, convert = runner.run, runner.convert_prefill_to_decode_cache

        def rec_run(scheduled, is_prefill):
            if is_prefill:
                rows = [dict(seq_id=s.seq.seq_id, tokens=list(s.seq.token_ids), start=s.seq.num_computed_tokens,
                             end=s.seq.num_computed_tokens + s.token_chunk_size, table=list(s.seq.block_table),
                             sample=bool(s.requires_sampling)) for s in scheduled]
            else:
                # A sequence preempted after it was placed in the batch (no blocks any more) is a
                # padding row on the device; its row's token is not checked.
                rows = [None if s.is_padding or not s.seq.block_table else
                        dict(seq_id=s.seq.seq_id, tokens=list(s.seq.token_ids), table=list(s.seq.block_table))
                        for s in scheduled]
            out = run(scheduled, is_prefill)
            self.events.append(("prefill" if is_prefill else "decode", rows, list(out)))
            return out

        def rec_convert(seqs):
            bs = runner.block_size
            slots = []
            for seq in seqs:
                slots += [seq.block_table[p // bs] * bs + p % bs for p in range(seq.num_computed_tokens)]
            self.events.append(("convert", slots, None))
            return convert(seqs)

        runner.run = rec_run
        runner.convert_prefill_to_decode_cache = rec_convert


def replay_against_oracle(hf, seed, events, num_blocks, block_size=256, kv_fp8=False, kv_scale=1.0,
                          max_decode_steps=None):
    """Replays the recorded steps on the oracle; returns (checked, exact, ties, decode steps, preempt
    re-prefills) and asserts that no engine token is more than two bf16 ulps below the oracle's top."""
    weights = dict(random_weights(hf, seed, 0.02, device="cuda"))
    model = Qwen3Oracle(hf, weights, num_blocks=num_blocks, block_size=block_size, device="cuda", kv_fp8=kv_fp8,
                        kv_scale=kv_scale)
    del weights
    checked = exact = 0
    ties, bad = [], []
    decode_steps = 0
    reprefills = 0
    seen_prefill = set()

    def check(logits, toks, where):
        nonlocal checked, exact
        logits = logits.float()
        top = logits.max(-1).values
        for i, tok in enumerate(toks):
            if tok is None:
                continue
            ulp = 2.0 ** (torch.floor(torch.log2(top[i].abs())) - 7)
            gap = float(top[i] - logits[i, tok])
            checked += 1
            if int(logits[i].argmax()) == tok:
                exact += 1
            elif gap <= 2 * float(ulp):
                ties.append((where, i, gap))
            else:
                bad.append((where, i, tok, int(logits[i].argmax()), gap, float(ulp)))

    for n, (kind, rows, out) in enumerate(events):
        if kind == "convert":
            if rows:
                model.convert(rows)
            continue
        if kind == "prefill":
            for r in rows:
                if r["start"] == 0 and r["seq_id"] in seen_prefill:
                    reprefills += 1
                seen_prefill.add(r["seq_id"])
            ids, pos, ctx = prefill_context([r["tokens"] for r in rows], [r["start"] for r in rows],
                                            [r["end"] for r in rows], [r["table"] for r in rows], block_size)
            with torch.no_grad():
                logits = model.logits(model.forward(ids, pos, ctx), ctx)
            check(logits, [t if r["sample"] else None for r, t in zip(rows, out)], f"prefill {n}")
            continue
        if max_decode_steps is not None and decode_steps >= max_decode_steps:
            break
        decode_steps += 1
        live = [(r, t) for r, t in zip(rows, out) if r is not None]
        width = max(len(r["table"]) for r, _ in live)
        ids, pos, ctx = decode_context([len(r["tokens"]) for r, _ in live], [r["tokens"][-1] for r, _ in live],
                                       [r["table"] for r, _ in live], block_size, width)
        with torch.no_grad():
            logits = model.logits(model.forward(ids, pos, ctx), ctx)
        check(logits, [t for _, t in live], f"decode {n}")
    del model
    torch.cuda.empty_cache()  # the oracle's pool is as large as the engine's: give it back
    for t in ties:
        print(f"bf16 logit tie at {t[0]} row {t[1]}: engine token {t[2]:.3g} below the top logit")
    assert not bad, f"engine tokens that are not an oracle argmax (where, row, token, argmax, gap, ulp): {bad[:10]}"
    return checked, exact, ties, decode_steps, reprefills


def run_engine(model_dir, prompts, params, **kw):
    llm = LLM(str(model_dir), load_format="random", async_decode=False, **kw)
    rec = ScheduleRecorder(llm)
    outs = llm.generate(prompts, params, use_tqdm=False)
    stats = dict(llm.last_generate_stats)
    num_blocks = llm.config.num_kvcache_blocks
    llm.exit()
    del llm
    torch.cuda.empty_cache()
    return outs, rec.events, stats, num_blocks


def test_c3_fp8_kv_capped_pool_preemption_matches_oracle():
    """Config 3 scaled: Qwen3-0.6B, FP8 e4m3 KV with a non-unit per-head scale, 12 sequences whose
    prompts (U[200, 250]) cross the first 256-token page during decode, 40 greedy tokens, and a pool
    of 14 blocks: most sequences are preempted when they need their second page, re-prefilled
    (their first page, filled partly during decode, is a prefix-cache hit), converted to FP8 again
    and packed back into the persistent decode batch."""
    from transformers import AutoConfig

    hf = AutoConfig.from_pretrained(CFG_06B)
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, hf.vocab_size, (int(torch.randint(200, 251, (1,), generator=g)),),
                             generator=g).tolist() for _ in range(12)]
    sp = SamplingParams(greedy=True, max_tokens=40, ignore_eos=True)
    outs, events, stats, nb = run_engine(CFG_06B, prompts, sp, seed=0, max_num_seqs=16, max_model_len=512,
                                         max_num_batched_tokens=4096, kv_cache_dtype="fp8", kv_cache_scale=0.5,
                                         kvcache_block_cap=14, gpu_memory_utilization=0.5)
    assert all(len(o["token_ids"]) == 40 for o in outs)
    checked, exact, ties, steps, reprefills = replay_against_oracle(hf, 0, events, nb, kv_fp8=True, kv_scale=0.5)
    print(f"c3 FP8: {exact}/{checked} exact, {len(ties)} ties, {steps} decode steps, {reprefills} re-prefills, "
          f"prefill steps blocked on the pool {stats['prefill_allocation_blocked_steps']}")
    assert reprefills > 0, "the capped pool was meant to force preemption"
    # Every output token is checked except those a preempted victim took from its padding row.
    victim_tokens = sum(1 for kind, rows, out in events if kind == "decode"
                        for r, t in zip(rows, out) if r is None and t is not None)
    assert checked == 12 * 40 - victim_tokens and exact >= 0.9 * checked


def test_c4_chunked_prefill_over_shared_prefixes_matches_oracle():
    """Config 4 scaled: two groups of three prompts sharing a 2048-token prefix (hash hits on eight
    pages), suffixes of 300-900 tokens, prefill chunks of at most 1024 tokens (so chunks start
    after position 0 and read the paged cache through block_tables), mixed with four decode
    sequences of prompt 64 and 32 outputs."""
    from transformers import AutoConfig

    hf = AutoConfig.from_pretrained(CFG_06B)
    g = torch.Generator().manual_seed(4)
    prompts, params = [], []
    for _ in range(2):
        prefix = torch.randint(0, hf.vocab_size, (2048,), generator=g).tolist()
        for _ in range(3):
            n = int(torch.randint(300, 901, (1,), generator=g))
            prompts.append(prefix + torch.randint(0, hf.vocab_size, (n,), generator=g).tolist())
            params.append(SamplingParams(greedy=True, max_tokens=3, ignore_eos=True))
    for _ in range(4):
        prompts.append(torch.randint(0, hf.vocab_size, (64,), generator=g).tolist())
        params.append(SamplingParams(greedy=True, max_tokens=32, ignore_eos=True))
    order = torch.randperm(len(prompts), generator=g).tolist()
    prompts = [prompts[i] for i in order]
    params = [params[i] for i in order]
    outs, events, stats, nb = run_engine(CFG_06B, prompts, params, seed=0, max_num_seqs=16, max_model_len=4096,
                                         max_num_batched_tokens=4096, chunked_prefill_size=1024,
                                         kvcache_block_cap=96, gpu_memory_utilization=0.5)
    assert [len(o["token_ids"]) for o in outs] == [p.max_tokens for p in params]
    prefix_chunks = sum(1 for kind, rows, _ in events if kind == "prefill" for r in rows if r["start"] > 0)
    assert prefix_chunks > 0, "no chunk started after position 0"
    checked, exact, ties, steps, _ = replay_against_oracle(hf, 0, events, nb)
    print(f"c4 chunked prefill: {exact}/{checked} exact, {len(ties)} ties, {prefix_chunks} chunks over a cached "
          f"prefix")
    assert checked == sum(p.max_tokens for p in params) and exact >= 0.9 * checked


def _reduced_8b(tmp_path, layers=2):
    cfg = json.loads((CFG_8B / "config.json").read_text())
    cfg["num_hidden_layers"] = layers
    d = tmp_path / "qwen3-8b-reduced"
    d.mkdir()
    (d / "config.json").write_text(json.dumps(cfg))
    return d


@pytest.mark.parametrize("kv", ["auto", "fp8"])
def test_c5_qwen3_8b_layout_gqa4_matches_oracle(tmp_path, kv):
    """Config 5 scaled: the Qwen3-8B layer shapes (hidden 4096, 32 query / 8 KV heads: GQA 4, which
    runs the tcgen05 decode kernel; MLP 12288; untied LM head over the 151,936-token vocabulary)
    with two layers, 8 sequences of prompts U[256, 1024], 33 greedy tokens (32 decode steps)."""
    from transformers import AutoConfig

    d = _reduced_8b(tmp_path)
    hf = AutoConfig.from_pretrained(d)
    assert hf.num_attention_heads // hf.num_key_value_heads == 4
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, hf.vocab_size, (int(torch.randint(256, 1025, (1,), generator=g)),),
                             generator=g).tolist() for _ in range(8)]
    sp = SamplingParams(greedy=True, max_tokens=33, ignore_eos=True)
    outs, events, _, nb = run_engine(d, prompts, sp, seed=0, max_num_seqs=8, max_model_len=1280,
                                     max_num_batched_tokens=8192, kv_cache_dtype=kv, kvcache_block_cap=64,
                                     gpu_memory_utilization=0.5)
    checked, exact, ties, steps, _ = replay_against_oracle(hf, 0, events, nb, kv_fp8=kv == "fp8")
    print(f"c5 8B layout ({kv} KV): {exact}/{checked} exact, {len(ties)} ties, {steps} decode steps")
    assert steps == 32 and checked == 8 * 33 and exact >= 0.9 * checked
