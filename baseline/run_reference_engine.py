"""Runs the UNMODIFIED reference engine (kirsten-1/hilda-vllm's `mini_vllm`) on this GPU through
its own public API, on the bench's workloads, and prints one JSON line with its tok/s.

    python baseline/run_reference_engine.py --ref baseline/_ref [--workload c2|c4] [--temperature 0.6]

`--ref` is a directory holding the reference's `mini_vllm` package (a plain copy of the
reference tree's package directory: the reference ships no setup.py or pyproject.toml, so there
is nothing to pip-install).  Nothing of this repository is on the measured path: the reference's
own LLM, Scheduler, ModelRunner, flash-attn attention, Triton KV store and torch.compile run as
they ship.  This script only provides what the reference expects to find on disk:

* a Hugging Face model directory with the Qwen3-0.6B config of this repository, seeded
  random-init weights (Linear / Embedding N(0, 0.02), norms 1, the bench's initialisation) in a
  safetensors file, and a word-level tokenizer over the 151,936 token ids (prompts are token-id
  lists, so the tokenizer only supplies the EOS id and decodes the outputs);
* the bench's prompts (seeded random ids) and sampling settings.  The reference has no greedy
  mode (its Sampler always draws, mini_vllm/sampling_params.py:13), so the default is its own
  benchmark's temperature 0.6 (benchmarks/bench.py:186-192); ignore_eos makes every request
  produce exactly max_tokens.

Workloads: c2 = 256 sequences, prompt 64, 1024 output tokens; c4 = the
bench's mixed chunked-prefill workload (64 prompts U[4096, 8192] in groups of 8 sharing a
2048-token prefix with 1 output token, plus 128 x (64 -> 256)).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
CFG_06B = ROOT / "hilda_vllm_b200" / "model_configs" / "qwen3-0.6b"


def make_model_dir(dst: Path, seed: int) -> None:
    import torch
    from safetensors.torch import save_file
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import AutoConfig, PreTrainedTokenizerFast

    sys.path.insert(0, str(ROOT))
    from hilda_vllm_b200.utils.loader import random_weights

    cfg = json.loads((CFG_06B / "config.json").read_text())
    (dst / "config.json").write_text(json.dumps(cfg))
    hf = AutoConfig.from_pretrained(dst)
    weights = {k: v.contiguous() for k, v in random_weights(hf, seed, 0.02, device="cpu")}
    if cfg.get("tie_word_embeddings", False):
        weights.pop("lm_head.weight", None)
    save_file(weights, str(dst / "model.safetensors"))
    vocab = {f"t{i}": i for i in range(hf.vocab_size)}
    tok = Tokenizer(models.WordLevel(vocab=vocab, unk_token="t0"))
    tok.pre_tokenizer = pre_tokenizers.Whitespace()
    eos = getattr(hf, "eos_token_id", None)
    eos = eos[0] if isinstance(eos, (list, tuple)) else eos
    fast = PreTrainedTokenizerFast(tokenizer_object=tok, eos_token=f"t{eos if eos is not None else 0}",
                                   unk_token="t0")
    fast.save_pretrained(dst)


def workload(name: str, seed: int, temperature: float):
    import torch

    g = torch.Generator().manual_seed(seed)
    vocab = 151936
    if name == "c2":
        prompts = [torch.randint(0, vocab, (64,), generator=g).tolist() for _ in range(256)]
        return prompts, [dict(temperature=temperature, ignore_eos=True, max_tokens=1024)] * 256, {"max_model_len": 4096}
    prompts, params = [], []
    for _ in range(8):
        prefix = torch.randint(0, vocab, (2048,), generator=g).tolist()
        for _ in range(8):
            n = int(torch.randint(4096, 8193, (1,), generator=g))
            prompts.append(prefix + torch.randint(0, vocab, (n - 2048,), generator=g).tolist())
            params.append(dict(temperature=temperature, ignore_eos=True, max_tokens=1))
    for _ in range(128):
        prompts.append(torch.randint(0, vocab, (64,), generator=g).tolist())
        params.append(dict(temperature=temperature, ignore_eos=True, max_tokens=256))
    order = torch.randperm(len(prompts), generator=g).tolist()
    return ([prompts[i] for i in order], [params[i] for i in order],
            {"max_model_len": 8448, "max_num_batched_tokens": 8448, "chunked_prefill_size": 8192})


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="directory that contains the reference's mini_vllm package")
    ap.add_argument("--workload", default="c2", choices=["c2", "c4"])
    ap.add_argument("--temperature", type=float, default=0.6)
    ap.add_argument("--seed", type=int, default=0)
    args = ap.parse_args()
    ref = Path(args.ref).resolve()
    if not (ref / "mini_vllm" / "__init__.py").exists():
        print(json.dumps({"impl": "reference-engine", "unavailable": f"no mini_vllm package under {ref}"}))
        return
    with tempfile.TemporaryDirectory() as tmp:
        model_dir = Path(tmp)
        make_model_dir(model_dir, args.seed)
        sys.path.insert(0, str(ref))
        from mini_vllm import LLM, SamplingParams  # the reference, unmodified

        prompts, params, kw = workload(args.workload, args.seed, args.temperature)
        llm = LLM(str(model_dir), enforce_eager=False, **kw)
        llm.generate([prompts[0][:64]], SamplingParams(temperature=args.temperature, ignore_eos=True, max_tokens=8),
                     use_tqdm=False)
        sps = [SamplingParams(**p) for p in params]
        t0 = time.perf_counter()
        outs = llm.generate(prompts, sps, use_tqdm=False)
        wall = time.perf_counter() - t0
        n_out = sum(len(o["token_ids"]) for o in outs)
        stats = getattr(llm, "last_generate_stats", None) or {}
        line = {"impl": "reference-engine", "workload": args.workload, "output_tokens": n_out,
                "wall_s": round(wall, 3), "tok_s": round(n_out / wall, 1), "temperature": args.temperature,
                "source": str(ref), "stats": {k: stats[k] for k in stats if isinstance(stats[k], (int, float))}}
        print(json.dumps(line), flush=True)
        if hasattr(llm, "exit"):
            llm.exit()


if __name__ == "__main__":
    main()
