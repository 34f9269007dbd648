"""Benchmark: Qwen3-0.6B decode tok/s at 256 sequences on the B200 path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One JSON line on rank 0.  Workload: Qwen3-0.6B architecture, seeded
random init (std 0.02), BF16 weights and KV cache, 256 sequences, prompt 64 random token ids,
1024 greedy output tokens with ignore_eos, block size 256, persistent batch of 256 under CUDA
graphs.  A "step" is one decode sweep of that job: the 1023 batched decode steps that follow
the prefill (context 65 -> 1087 for all 256 sequences).

value: decode tok/s over the timed sweeps with every input already in HBM: the per-step pack
       packets are prepared before the timed region and copied device-to-device, the sampled
       tokens stay on the device (next_tokens), each step is one CUDA-graph replay (pack kernel +
       28 layers + LM head + argmax).  Timed with CUDA events, max over ranks.
e2e:   the same job through the public API (LLM.generate with host token-id prompts, outputs
       returned as host lists): host scheduler, per-step packet upload, token read-back; total
       output tokens / wall time including prefill.
roofline: the paged decode kernel timed on its own (CUDA events on its stream) over the live KV
       cache at contexts sampled across the sweep; algorithmic bytes = K+V bytes of every cached
       token + Q and O.
cpu_baseline / --impl reference: the reference algorithm on the host (the CPU oracle port of the
       reference's Qwen3 forward: eager torch with the reference's layer arithmetic and fp32
       attention), decode steps of a bounded sample of sequences at the job's mid context.
With --gpus N > 1 (torchrun), the model runs tensor-parallel over N GPUs (KV heads sharded,
all-reduce after o_proj / down_proj): "strong" scaling, same job.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CFG_DIR = ROOT / "hilda_vllm_b200" / "model_configs" / "qwen3-0.6b"
NUM_SEQS = 256
PROMPT_LEN = 64
OUTPUT_LEN = 1024
MAX_MODEL_LEN = PROMPT_LEN + OUTPUT_LEN + 256  # as benchmarks/bench_decode_heavy.py:78
METRIC = "Qwen3-0.6B decode tok/s @256 seqs"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--workload", default="c2", choices=["c1", "c2", "c3", "c4", "c5"],
                    help="c2 (default, the headline): BASELINE configs[1]; c1: the single-op KV store + paged "
                         "decode of configs[0]; c3: FP8 KV with a capped pool; c4: mixed chunked prefill + "
                         "decode with shared prefixes; c5: Qwen3-8B (TP over --gpus)")
    ap.add_argument("--kv", default="auto", choices=["auto", "bf16", "fp8"],
                    help="KV cache dtype for c5 (auto = bf16, the model dtype)")
    ap.add_argument("--tp-shard", type=int, default=1,
                    help="decode-kernel profiles: the per-GPU head counts under tensor parallelism of this degree")
    ap.add_argument("--profile", default="",
                    choices=["", "decode-kernel", "decode-kernel-tc", "decode-steps", "prefill-kernel", "small-kernels",
                             "allreduce", "reference-kernels"],
                    help="run a short profiling case instead of the benchmark: the CUDA profiler range "
                         "(cudaProfilerStart/Stop, for ncu --profile-from-start off) covers --steps "
                         "launches of the decode kernel alone (decode-kernel), of the prefill kernel "
                         "(prefill-kernel), of every other kernel (small-kernels), or --steps engine "
                         "decode steps at the job's mid context (decode-steps)")
    return ap.parse_args()


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except FileNotFoundError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        loaded = [s for s in sm if smax and s > 0.5 * smax] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------- CPU baseline
class CpuDecodeSample:
    """Decode steps of the reference algorithm on the host (the CPU oracle port), for num_seqs
    sequences whose KV cache is filled to ctx_len (random K/V stand in for the prefill)."""

    def __init__(self, num_seqs: int, ctx_len: int, max_steps: int, seed: int = 0):
        import torch
        from transformers import AutoConfig

        from hilda_vllm_b200.utils.loader import random_weights
        from oracle.qwen3_model import Qwen3Oracle

        self.threads = len(os.sched_getaffinity(0))
        torch.set_num_threads(self.threads)
        hf = AutoConfig.from_pretrained(CFG_DIR)
        weights = dict(random_weights(hf, seed, 0.02, device="cpu"))
        self.bs = 256
        self.nblk = -(-(ctx_len + max_steps + 1) // self.bs)
        self.model = Qwen3Oracle(hf, weights, num_blocks=num_seqs * self.nblk, block_size=self.bs, device="cpu")
        g = torch.Generator().manual_seed(seed)
        # The cache holds seeded random K/V rows (one random block per layer, repeated): the
        # arithmetic per decode step does not depend on the values, only on the context length.
        for cache in (self.model.k_cache, self.model.v_cache):
            one_block = torch.randn((cache.shape[0], 1, *cache.shape[2:]), generator=g).to(cache.dtype)
            cache.copy_(one_block.expand_as(cache))
        self.tables = [[i * self.nblk + j for j in range(self.nblk)] for i in range(num_seqs)]
        self.lens = [ctx_len] * num_seqs
        self.last = torch.randint(0, hf.vocab_size, (num_seqs,), generator=g).tolist()
        self.num_seqs = num_seqs

    def step(self) -> float:
        """One batched decode step; returns its wall time in seconds."""
        import torch

        from oracle.qwen3_model import decode_context

        t0 = time.perf_counter()
        self.lens = [n + 1 for n in self.lens]
        cur = [t[: -(-n // self.bs)] for n, t in zip(self.lens, self.tables)]
        ids, pos, ctx = decode_context(self.lens, self.last, cur, self.bs, self.nblk)
        with torch.no_grad():
            logits = self.model.logits(self.model.forward(ids, pos, ctx), ctx)
        self.last = logits.argmax(-1).tolist()
        return time.perf_counter() - t0


def cpu_decode_sample(num_seqs: int, ctx_len: int, steps: int, seed: int = 0):
    """(tok/s, seconds, threads) over `steps` decode steps after one warm-up step."""
    import torch

    s = CpuDecodeSample(num_seqs, ctx_len, steps + 1, seed)
    s.step()
    dt = sum(s.step() for _ in range(steps))
    return num_seqs * steps / dt, dt, torch.get_num_threads()


CPU_SAMPLE_SEQS = 32
CPU_SAMPLE_STEPS = 16  # about 10 s on 16 host threads
CPU_CTX = PROMPT_LEN + OUTPUT_LEN // 2  # mid-job context


def run_reference_arm(args):
    """The reference's hot path on the host cores (CPU oracle port), same metric and config;
    each step is one decode step of a bounded sample of the 256 sequences."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch

    sample = CpuDecodeSample(CPU_SAMPLE_SEQS, CPU_CTX, args.steps + args.warmup + 1, args.seed)
    for _ in range(args.warmup):
        sample.step()
    total = sum(sample.step() for _ in range(args.steps))
    value = CPU_SAMPLE_SEQS * args.steps / total
    desc = (f"{CPU_SAMPLE_SEQS} of the 256 sequences, one batched decode step per bench step at context "
            f"{CPU_CTX}, 28 layers, fp32 attention (reference arithmetic, CPU oracle port)")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * total / args.steps, 1),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "qwen3-0.6b decode-heavy 256x(64->1024), CPU sample", "global_batch": NUM_SEQS,
                   "seq_len": PROMPT_LEN + OUTPUT_LEN, "parallelism": "host cores"},
        "cpu_baseline": {"value": round(value, 3), "unit": "tok/s", "cores": torch.get_num_threads(), "kind": "port",
                         "sample": desc},
        "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_c1_reference(args):
    """--impl reference --workload c1: the config-1 op on the host cores (CPU oracle)."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    cpu = c1_cpu_sample(args.seed, reps=max(args.steps, 1))
    line = {"impl": "reference", "metric": "config-1 single op (KV store + paged decode, 8 seqs): ops/s",
            "value": cpu["value"], "unit": "ops/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1e3 / cpu["value"], 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) cache, q and new K/V)",
            "config": {"workload": "c1: BASELINE configs[0] on the host cores"}, "cpu_baseline": cpu,
            "e2e": {"value": cpu["value"], "unit": "ops/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- GPU arm
def run_ours(args):
    import torch
    import torch.distributed as dist

    world = args.gpus
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)

    from hilda_vllm_b200 import LLM, SamplingParams
    from hilda_vllm_b200.engine.scheduler import Scheduler

    g = torch.Generator().manual_seed(args.seed)
    vocab = 151936
    prompts = [torch.randint(0, vocab, (PROMPT_LEN,), generator=g).tolist() for _ in range(NUM_SEQS)]
    sp = SamplingParams(greedy=True, max_tokens=OUTPUT_LEN, ignore_eos=True)
    llm = LLM(str(CFG_DIR), load_format="random", seed=args.seed, max_num_seqs=NUM_SEQS,
              max_model_len=MAX_MODEL_LEN, max_num_batched_tokens=16384, tensor_parallel_size=world,
              gpu_memory_utilization=0.85, distributed_executor="external" if world > 1 else "spawn")
    if getattr(llm, "is_worker", False):
        if dist.is_initialized():
            dist.destroy_process_group()
        return  # worker ranks served rank 0's calls inside LLM(...) until it exited
    runner = llm.model_runner
    hf = llm.config.hf_config

    def fresh():
        llm.scheduler = Scheduler(llm.config)
        runner.call("reset_decode_state")

    # One full job through the engine (warms everything up) while recording its decode packets.
    runner.call("record_packets", True)
    llm.generate(prompts, sp, use_tqdm=False)
    runner.call("take_recording")
    steps_per_sweep = len(runner.recorded_packets)

    def device_sweep(probe_every=0):
        """Prefill through the engine (untimed), then the recorded decode sweep replayed with
        every input already on the device; returns (seconds, kernel probe samples)."""
        fresh()
        for p in prompts:
            llm.add_request(p, sp)
        llm.step()  # prefill of all 256 prompts (16384 tokens, one step)
        return runner.call("replay_recorded", NUM_SEQS, probe_every)

    for _ in range(args.warmup):
        device_sweep()
    sampler = ClockSampler(local)
    sampler.start()
    times = [device_sweep()[0] for _ in range(args.steps)]
    clocks = sampler.stop()
    sweep_s = max(times)
    tokens_per_sweep = NUM_SEQS * steps_per_sweep
    value = tokens_per_sweep / sweep_s

    # ---- decode-kernel roofline leg: the kernel alone on the live cache across a sweep ----
    _, samples = device_sweep(probe_every=64)
    kbytes = sum(b for b, _ in samples)
    ktime = sum(t for _, t in samples)
    peaks = {}
    peak_path = ROOT / "MEASURED_PEAKS.json"
    if peak_path.exists():
        peaks = json.loads(peak_path.read_text())
    hbm_peak = peaks.get("hbm_gbs", 6650.0)
    achieved = kbytes / ktime / 1e9
    hk = hf.num_key_value_heads // world
    g_ratio = hf.num_attention_heads // hf.num_key_value_heads
    # DRAM traffic per launch: one ncu capture of this kernel on the config-2 mid-job launch
    # (`bench.py --profile decode-kernel`: 614.70 MB read + 12.28 MB written for 609.6 MB of
    # algorithmic bytes), scaled to this run's average launch — the traffic is the cache bytes
    # read once plus the split-K partials, so it grows with the bytes processed.
    ncu_ratio = (614.70 + 12.28) / 609.6 if (g_ratio == 2 and hk == 8) else None
    bpl = kbytes / max(1, len(samples))
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                "frac": round(achieved / hbm_peak, 4),
                "traffic": int(ncu_ratio * bpl) if ncu_ratio else None,
                "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum of one config-2 mid-job launch "
                                   "(bench.py --profile decode-kernel), 1.028x algorithmic, scaled to this run's "
                                   "average launch") if ncu_ratio else None,
                # hl_paged_decode runs the tensor-core kernel from GQA 4 on, and for one KV head per
                # GPU at GQA 2 (tensor parallelism over all KV heads).
                "kernel": (f"paged_decode_tc_kernel<G={g_ratio},bf16>" if g_ratio >= 4 or (hk == 1 and g_ratio == 2)
                           else f"paged_decode_kernel<bf16,G={g_ratio},Hk={hk}>"),
                "peak_source": "of measured (MEASURED_PEAKS.json hbm_gbs)" if peaks else "of fallback (6650 GB/s)",
                "samples": len(samples), "avg_launch_us": round(1e6 * ktime / max(1, len(samples)), 2),
                "bytes_per_launch_avg": int(kbytes / max(1, len(samples)))}

    # ---- the reference's own attention kernels (flash-attn) beside ours, same inputs, this GPU ----
    ref_kernels = reference_kernel_ab(args.seed, reps=10) if world == 1 else None

    # ---- end-to-end through the public API ----
    e2e = None
    if not args.no_e2e:
        fresh()
        runner.io_bytes = {"h2d": 0, "d2h": 0}
        runner.gpu_wait_s = 0.0
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        outs = llm.generate(prompts, sp, use_tqdm=False)
        wall = time.perf_counter() - t0
        n_out = sum(len(o["token_ids"]) for o in outs)
        stats = llm.last_generate_stats
        n_steps = stats["decode_steps"] + 1
        e2e = {"value": round(n_out / wall, 1), "unit": "tok/s",
               "h2d_bytes_per_step": int(runner.io_bytes["h2d"] / n_steps),
               "d2h_bytes_per_step": int(runner.io_bytes["d2h"] / n_steps),
               "wall_s": round(wall, 3), "output_tokens": n_out,
               "prefill_s": round(stats["prefill_time_s"], 4), "decode_s": round(stats["decode_time_s"], 3),
               "decode_tok_s": round(stats["decode_throughput_toks"], 1),
               "rank0_gpu_wait_s": round(runner.gpu_wait_s, 3),
               "rank0_host_s": round(wall - runner.gpu_wait_s, 3)}
        # The same job sampled at temperature 0.6 (the reference's own benchmark setting,
        # benchmarks/bench.py:186-192): sampled on the device by the Gumbel-max kernel.
        fresh()
        t0 = time.perf_counter()
        outs_t = llm.generate(prompts, SamplingParams(temperature=0.6, max_tokens=OUTPUT_LEN, ignore_eos=True),
                              use_tqdm=False)
        wall_t = time.perf_counter() - t0
        e2e["temperature_0_6_tok_s"] = round(sum(len(o["token_ids"]) for o in outs_t) / wall_t, 1)

    cpu = None
    if not args.no_cpu and world == 1:
        rate, dt, threads = cpu_decode_sample(CPU_SAMPLE_SEQS, CPU_CTX, CPU_SAMPLE_STEPS, args.seed)
        cpu = {"value": round(rate, 2), "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": f"{CPU_SAMPLE_SEQS} sequences x {CPU_SAMPLE_STEPS} decode steps at context {CPU_CTX} "
                         f"({dt:.1f} s), reference arithmetic via the CPU oracle port"}

    # Our kernels per decode step: the pack kernel; per layer input add+RMSNorm, fused
    # QK-norm+RoPE+KV store, paged decode, post-attention add+RMSNorm, SiLU*mul; final norm;
    # argmax (cuBLAS GEMMs and torch's embedding gather are not counted).
    launches_per_step = 1 + hf.num_hidden_layers * 5 + 2

    # ---- whole-job roofline: weight bytes + KV bytes every decode step must read, per GPU ----
    d = getattr(hf, "head_dim", None) or hf.hidden_size // hf.num_attention_heads
    per_layer = hf.hidden_size * (hf.num_attention_heads + 2 * hf.num_key_value_heads) * d \
        + hf.num_attention_heads * d * hf.hidden_size + 3 * hf.hidden_size * hf.intermediate_size
    weight_bytes = 2 * (hf.num_hidden_layers * per_layer + hf.vocab_size * hf.hidden_size) / world
    kv_token_bytes = hf.num_hidden_layers * hf.num_key_value_heads * d * 2 * 2 / world
    ctx_sum = sum(NUM_SEQS * (PROMPT_LEN + 1 + s) for s in range(steps_per_sweep))
    job_bytes = steps_per_sweep * weight_bytes + ctx_sum * kv_token_bytes
    roof_tok_s = tokens_per_sweep / (job_bytes / (hbm_peak * 1e9))
    job_roofline = {"tok_s": round(roof_tok_s, 1), "bytes_per_gpu": int(job_bytes), "peak_gbs": hbm_peak,
                    "value_frac": round(value / roof_tok_s, 4),
                    "e2e_frac": round(e2e["value"] / roof_tok_s, 4) if e2e else None,
                    "what": "decode tok/s if every step only streamed its weights and KV cache from HBM at the "
                            "measured copy bandwidth (per GPU under TP)"}
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(sweep_s * 1e3, 2), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init weights std 0.02, random token ids)",
        "config": {"workload": "qwen3-0.6b decode-heavy: 256 seqs, prompt 64, 1024 greedy tokens, ignore_eos, "
                               "block 256, CUDA graphs (BASELINE configs[1])",
                   "global_batch": NUM_SEQS, "seq_len": PROMPT_LEN + OUTPUT_LEN, "parallelism": f"tp{world}",
                   "step": f"one decode sweep = {steps_per_sweep} batched decode steps",
                   "l2": "no flush: per-step KV (0.6-3.2 GB) and weights (1.2 GB) exceed the 126 MB L2"},
        "decode_ms_per_batch_step": round(sweep_s * 1e3 / steps_per_sweep, 4),
        "roofline": roofline,
        "kv_weight_roofline": job_roofline,
        "reference_kernels": ref_kernels,
        "cpu_baseline": cpu,
        "e2e": e2e,
        "clocks": clocks,
        "gpu_launches": launches_per_step * steps_per_sweep * args.steps,
    }
    completions = [o["token_ids"] for o in outs] if e2e else None
    if world == 1:
        if completions is not None:
            line["parity"] = greedy_parity(llm, prompts, completions, "this engine's prefill path (same GPU)")
        print(json.dumps(line), flush=True)
        llm.exit()
        return
    # Tensor parallel: tear the TP engine down, then check its greedy tokens on rank 0's GPU with a
    # single-GPU engine of the same seeded weights.
    import gc

    llm.exit()
    del runner, llm
    gc.collect()
    torch.cuda.empty_cache()
    if completions is not None:
        from hilda_vllm_b200 import LLM as _LLM
        ref = _LLM(str(CFG_DIR), load_format="random", seed=args.seed, max_num_seqs=64, max_model_len=MAX_MODEL_LEN,
                   max_num_batched_tokens=16384, enforce_eager=True, kvcache_block_cap=256, gpu_memory_utilization=0.5)
        line["parity"] = greedy_parity(ref, prompts, completions, "a 1-GPU engine with the same weights")
        ref.exit()
    print(json.dumps(line), flush=True)


def greedy_parity(engine, prompts, completions, against: str, seqs: int = 8, steps: int = 32) -> dict:
    """Teacher-forced check of the first `steps` decode tokens (plus the prefill token) of the first
    `seqs` sequences: engine.score_next_tokens(prompt + first s tokens) must pick token s, or hold it
    within two bf16 ulps of its top logit (a tie: bf16 logits of a random-init model often tie)."""
    import math

    lists, targets = [], []
    for p, c in zip(prompts[:seqs], completions[:seqs]):
        for k in range(min(steps + 1, len(c))):
            lists.append(list(p) + list(c[:k]))
            targets.append(int(c[k]))
    res = engine.score_next_tokens(lists, targets)
    exact = ties = bad = 0
    for r, t in zip(res, targets):
        if r["argmax"] == t:
            exact += 1
            continue
        top = r["top_logit"]
        ulp = 2.0 ** (math.floor(math.log2(abs(top))) - 7) if top != 0 else 2.0 ** -133
        if top - r["target_logit"] <= 2 * ulp:
            ties += 1
        else:
            bad += 1
    n = len(targets)
    return {"seqs": seqs, "steps": steps, "checked": n, "exact": exact, "ties": ties, "bad": bad,
            "ok": bad == 0 and exact >= 0.9 * n, "against": against + ", teacher-forced"}


def small_kernels(args, g):
    """Every kernel besides decode and prefill attention, at config-2 shapes, args.steps launches
    each inside the profiler range, timed with CUDA events: the fused QK-norm+RoPE+KV store
    (BF16 and FP8, decode batch of 256 and a 16384-token prefill), the standalone BF16 store,
    the all-layer BF16->FP8 cache copy, the decode pack kernel on a full packet, add+RMSNorm,
    SiLU*mul and the greedy argmax.  A few GB on the device at most."""
    import torch

    from hilda_vllm_b200 import kernels
    from hilda_vllm_b200.engine.decode_packer import DecodePacker
    from hilda_vllm_b200.engine.scheduler import ScheduledSequence
    from hilda_vllm_b200.engine.sequence import Sequence, SequenceStatus
    from hilda_vllm_b200.layers.rotary_embedding import RotaryEmbedding

    dev = torch.device("cuda", 0)
    hq, hk, d, bs, layers, hidden, inter, vocab = 16, 8, 128, 256, 28, 1024, 3072, 151936
    nb = 512  # 0.27 GB per BF16 cache
    cos_sin = RotaryEmbedding(d, d, 40960, 1000000.0).cos_sin_cache.to(dev).contiguous()
    qw = torch.ones(d, dtype=torch.bfloat16, device=dev)
    kc = torch.zeros(nb, bs, hk, d, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    kc8 = torch.zeros(nb, bs, hk, d, dtype=torch.float8_e4m3fn, device=dev)
    vc8 = torch.zeros_like(kc8)
    scales = torch.rand(hk, device=dev) + 0.5
    cases = {}
    # Algorithmic bytes of the fused kernel: every qkv element read, q and k written back in
    # place, the K and V rows written to the cache (2 bytes per element BF16, 1 FP8).
    for n in (NUM_SEQS, 16384):
        qkv = torch.randn(n, (hq + 2 * hk) * d, device=dev, dtype=torch.bfloat16)
        pos = torch.randint(0, 1088, (n,), device=dev)
        slots = torch.randperm(nb * bs, device=dev)[:n].to(torch.int32)
        for kv, (kcache, vcache, sc) in {"bf16": (kc, vc, None), "fp8": (kc8, vc8, scales)}.items():
            elem = 1 if kv == "fp8" else 2
            cases[f"qk_norm_rope_store_{kv}_n{n}"] = (
                lambda qkv=qkv, pos=pos, slots=slots, kcache=kcache, vcache=vcache, sc=sc: kernels.qk_norm_rope_store(
                    qkv, hq, hk, d, qw, qw, cos_sin, pos, 1e-6, kcache, vcache, slots, sc, sc),
                n * ((hq + 2 * hk) * d * 2 + (hq + hk) * d * 2 + 2 * hk * d * elem))
    n = 16384
    qkv = torch.randn(n, (hq + 2 * hk) * d, device=dev, dtype=torch.bfloat16)
    slots = torch.randperm(nb * bs, device=dev)[:n].to(torch.int32)
    key = qkv[:, hq * d:(hq + hk) * d].view(n, hk, d)
    val = qkv[:, (hq + hk) * d:].view(n, hk, d)
    cases["store_kv_bf16_n16384"] = (lambda: kernels.store_kvcache(key, val, kc, vc, slots), n * hk * d * 2 * 4)
    # all-layer BF16 -> FP8 copy (prefill-to-decode cache handoff): 8192 slots x 28 layers
    nbl = 32
    src = torch.randn(2, layers, nbl, bs, hk, d, device=dev, dtype=torch.bfloat16)
    dst = torch.zeros(2, layers, nbl, bs, hk, d, device=dev, dtype=torch.float8_e4m3fn)
    cslots = torch.randperm(nbl * bs, device=dev)[:8192].to(torch.int32)
    lsc = torch.rand(layers, hk, device=dev) + 0.5
    cases["copy_kv_bf16_to_fp8_28layers_n8192"] = (
        lambda: kernels.copy_kvcache_fp8_layers(src[0], src[1], dst[0], dst[1], cslots, lsc, lsc),
        8192 * layers * 2 * hk * d * 3)
    # decode pack kernel on a full packet (every slot a new owner with a 5-block row)
    mb = -(-MAX_MODEL_LEN // bs)
    packer = DecodePacker(NUM_SEQS, mb)
    sched = []
    for i in range(NUM_SEQS):
        seq = Sequence(list(range(577)))
        seq.status = SequenceStatus.RUNNING
        seq.num_computed_tokens = 576
        seq.block_table = [(5 * i + j) % nb for j in range(3)]
        sched.append(ScheduledSequence(seq, 1, i))
    nbytes = packer.build(sched, NUM_SEQS)
    packet = torch.from_numpy(packer.buffer[:nbytes].copy()).to(dev)
    gv = dict(slot_seq_ids=torch.full((NUM_SEQS,), -1, dtype=torch.int64, device=dev),
              slot_bt_lens=torch.zeros(NUM_SEQS, dtype=torch.int32, device=dev),
              next_tokens=torch.zeros(NUM_SEQS, dtype=torch.int64, device=dev),
              input_ids=torch.zeros(NUM_SEQS, dtype=torch.int64, device=dev),
              positions=torch.zeros(NUM_SEQS, dtype=torch.int64, device=dev),
              slot_mapping=torch.zeros(NUM_SEQS, dtype=torch.int32, device=dev),
              context_lens=torch.zeros(NUM_SEQS, dtype=torch.int32, device=dev),
              block_tables=torch.full((NUM_SEQS, mb), -1, dtype=torch.int32, device=dev))
    cases["pack_decode_full_packet_b256"] = (
        lambda: kernels.pack_decode_batch(packet, NUM_SEQS, bs, gv["slot_seq_ids"], gv["slot_bt_lens"],
                                          gv["next_tokens"], gv["input_ids"], gv["positions"], gv["slot_mapping"],
                                          gv["context_lens"], gv["block_tables"]),
        nbytes + NUM_SEQS * (8 + 4 + 8 + 8 + 8 + 4 + 4 + mb * 4))
    x = torch.randn(NUM_SEQS, hidden, device=dev, dtype=torch.bfloat16)
    res = torch.randn_like(x)
    nw = torch.ones(hidden, device=dev, dtype=torch.bfloat16)
    cases["add_rmsnorm_b256"] = (lambda: kernels.rmsnorm(x, nw, 1e-6, residual=res), NUM_SEQS * hidden * 2 * 4)
    gu = torch.randn(NUM_SEQS, 2 * inter, device=dev, dtype=torch.bfloat16)
    cases["silu_mul_b256"] = (lambda: kernels.silu_mul(gu), NUM_SEQS * inter * 2 * 3)
    logits = torch.randn(NUM_SEQS, vocab, device=dev, dtype=torch.bfloat16)
    toks = torch.zeros(NUM_SEQS, dtype=torch.int64, device=dev)
    cases["argmax_b256"] = (lambda: kernels.argmax(logits, toks), NUM_SEQS * vocab * 2)

    out = {"profile": "small-kernels"}
    stream = torch.cuda.current_stream()
    for fn, _ in cases.values():
        fn()
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    for name, (fn, nbytes_alg) in cases.items():
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / args.steps
        out[name] = {"us": round(us, 2), "alg_bytes": int(nbytes_alg), "gb_per_s": round(nbytes_alg / us / 1e3, 1)}
    torch.cuda.profiler.stop()
    print(json.dumps(out))


def allreduce_profile(args):
    """Under torchrun with --gpus N: the fused NVLink all-reduce + add + RMSNorm (one-shot and
    two-shot kernels) against NCCL all_reduce followed by the add + RMSNorm kernel, at decode
    batches of the 0.6B (hidden 1024) and 8B (hidden 4096) models.  Each variant is captured in a CUDA graph of 56 calls (one
    decode step's worth) and replayed; CUDA events, max over ranks."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from hilda_vllm_b200 import kernels
    from hilda_vllm_b200.layers.nvlink_allreduce import NvlinkAllReduce

    world = args.gpus
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    res_all = {"profile": "allreduce", "n_gpus": world}
    calls = 56
    for hidden in (1024, 4096):
        ar = NvlinkAllReduce(rank, world, 512, hidden, dev, timeout_s=20.0)
        w = torch.ones(hidden, dtype=torch.bfloat16, device=dev)
        for rows in (64, 256):
            res = torch.randn(rows, hidden, dtype=torch.bfloat16, device=dev)
            part = torch.randn(rows, hidden, dtype=torch.bfloat16, device=dev)
            out = torch.empty_like(res)

            def fused():
                ar.force_two_shot = False
                for i in range(calls):
                    ar.output(i % 2, rows).copy_(part)
                    ar.add_rmsnorm(i % 2, rows, res, w, 1e-6, out)

            def fused_2shot():
                ar.force_two_shot = True
                for i in range(calls):
                    ar.output(i % 2, rows).copy_(part)
                    ar.add_rmsnorm(i % 2, rows, res, w, 1e-6, out)

            def nccl():
                for i in range(calls):
                    y = part.clone()
                    dist.all_reduce(y)
                    kernels.rmsnorm(y, w, 1e-6, residual=res)

            def copies():
                for i in range(calls):
                    ar.output(i % 2, rows).copy_(part)
                    part.clone()

            for name, fn in (("fused_nvlink", fused), ("fused_nvlink_2shot", fused_2shot),
                             ("nccl_plus_rmsnorm", nccl), ("copies_only", copies)):
                fn()
                torch.cuda.synchronize()
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    fn()
                for _ in range(3):
                    graph.replay()
                torch.cuda.synchronize()
                dist.barrier()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(20):
                    graph.replay()
                e1.record()
                torch.cuda.synchronize()
                t = torch.tensor([e0.elapsed_time(e1) * 1e3 / (20 * calls)], device=dev)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                res_all[f"{name}_h{hidden}_rows{rows}_us_per_call"] = round(float(t.item()), 2)
                del graph
        ar.copy_error_word()
        torch.cuda.synchronize()
        ar.check_errors()
        dist.barrier()
        ar.close()
    if rank == 0:
        print(json.dumps(res_all), flush=True)
    dist.destroy_process_group()


def _paged_case(g, lens, hq, hk, dev, bs=256, fp8=False):
    """Seeded paged-decode inputs: contiguous random pages per sequence (-1 padded tables)."""
    import torch

    d = 128
    nblk = [max(1, -(-int(n) // bs)) for n in lens]
    mb = max(nblk)
    perm = torch.randperm(sum(nblk), generator=g).tolist()
    tables, off = [], 0
    for n in nblk:
        tables.append(perm[off:off + n] + [-1] * (mb - n))
        off += n
    kc = torch.randn(sum(nblk), bs, hk, d, generator=g).bfloat16().to(dev)
    vc = torch.randn(sum(nblk), bs, hk, d, generator=g).bfloat16().to(dev)
    if fp8:
        kc, vc = kc.to(torch.float8_e4m3fn), vc.to(torch.float8_e4m3fn)
    q = torch.randn(len(lens), hq, d, generator=g).bfloat16().to(dev)
    bt = torch.tensor(tables, dtype=torch.int32, device=dev)
    ln = torch.tensor([int(n) for n in lens], dtype=torch.int32, device=dev)
    return q, kc, vc, bt, ln


def _time_flushed(fn, reps, flush):
    """Mean seconds of fn() over reps launches, each timed alone with CUDA events on the current
    stream right after a read-modify-write of `flush` (larger than L2), so no launch finds the
    previous one's data in L2.  The flush keeps the GPU busy while the host enqueues the start
    event and fn's launches, so the events time GPU work, not the host's launch latency."""
    import torch

    stream = torch.cuda.current_stream()
    fn()
    torch.cuda.synchronize()
    total = 0.0
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        flush.add_(1)
        e0.record(stream)
        fn()
        e1.record(stream)
        torch.cuda.synchronize()
        total += e0.elapsed_time(e1) / 1e3
    return total / reps


def reference_kernel_ab(seed: int = 0, reps: int = 20) -> dict:
    """This repository's attention kernels against the reference's own (flash-attn 2.x, called with
    the reference's exact signatures, mini_vllm/layers/attention.py:149-170) on identical inputs on
    this GPU: decode at the config-1 shapes (8 sequences, contexts U[16, 1024]), at config-2 mid-job
    (256 sequences, contexts U[65, 1087]) and at the config-5 layout (Qwen3-8B heads, GQA 4,
    contexts U[512, 1280]); varlen chunked prefill at the config-4 shape (8 chunks of 4096-8192 new
    tokens over a 2048-token cached prefix, paged).  Each launch timed alone, L2 flushed before it."""
    import itertools

    import torch

    from hilda_vllm_b200 import kernels

    try:
        from flash_attn import flash_attn_varlen_func, flash_attn_with_kvcache
    except Exception as exc:  # pragma: no cover - depends on the installed wheel
        return {"unavailable": f"flash-attn not importable: {type(exc).__name__}"}
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator().manual_seed(seed)
    flush = torch.zeros(128 << 20, dtype=torch.float32, device=dev)  # 512 MB > 126 MB of L2
    scale = 128 ** -0.5
    res = {"timing": "CUDA events per launch, L2 flushed (512 MB read-modify-write) before each launch, mean of "
                     f"{reps}", "reference": "flash-attn 2.x with the reference's call signatures"}
    decode_cases = {
        "decode_c1": ([int(x) for x in torch.randint(16, 1025, (8,), generator=g)], 16, 8),
        "decode_c2_mid": ([int(x) for x in torch.randint(PROMPT_LEN + 1, PROMPT_LEN + OUTPUT_LEN, (NUM_SEQS,),
                                                         generator=g)], 16, 8),
        "decode_c5_layout": ([int(x) for x in torch.randint(512, 1281, (NUM_SEQS,), generator=g)], 32, 8),
    }
    for name, (lens, hq, hk) in decode_cases.items():
        q, kc, vc, bt, ln = _paged_case(g, lens, hq, hk, dev)
        out = torch.empty_like(q)
        ws = kernels.make_decode_workspace(len(lens), hq, 128, bt.shape[1], 256, dev)
        ours = _time_flushed(lambda: kernels.paged_decode(q, kc, vc, bt, ln, scale, out=out, workspace=ws), reps,
                             flush)
        q4 = q.unsqueeze(1)
        ref = _time_flushed(lambda: flash_attn_with_kvcache(q4, kc, vc, cache_seqlens=ln, block_table=bt,
                                                            softmax_scale=scale, causal=True), reps, flush)
        nbytes = sum(lens) * hk * 128 * 2 * 2 + len(lens) * hq * 128 * 2 * 2
        res[name] = {"seqs": len(lens), "hq": hq, "hk": hk, "ours_us": round(ours * 1e6, 2),
                     "reference_us": round(ref * 1e6, 2), "speedup": round(ref / ours, 3),
                     "ours_gbs": round(nbytes / ours / 1e9, 1), "reference_gbs": round(nbytes / ref / 1e9, 1)}
        del q, kc, vc, bt, ln, out, ws
    # config-4 prefill shape
    hq, hk, bs, prefix = 16, 8, 256, 2048
    chunks = [int(x) for x in torch.randint(4096, 8193, (8,), generator=g)]
    kl = [prefix + c for c in chunks]
    _, kc, vc, bt, _ = _paged_case(g, kl, hq, hk, dev)
    tq = sum(chunks)
    q = torch.randn(tq, hq, 128, generator=g).bfloat16().to(dev)
    cuq = torch.tensor([0] + list(itertools.accumulate(chunks)), dtype=torch.int32, device=dev)
    cuk = torch.tensor([0] + list(itertools.accumulate(kl)), dtype=torch.int32, device=dev)
    flops = sum(4 * hq * 128 * (c * prefix + c * (c + 1) // 2) for c in chunks)
    ours = _time_flushed(lambda: kernels.varlen_prefill(q, kc, vc, cuq, cuk, max(chunks), max(kl), scale,
                                                        block_table=bt), max(3, reps // 4), flush)
    ref = _time_flushed(lambda: flash_attn_varlen_func(q, kc, vc, max_seqlen_q=max(chunks), cu_seqlens_q=cuq,
                                                       max_seqlen_k=max(kl), cu_seqlens_k=cuk, softmax_scale=scale,
                                                       causal=True, block_table=bt), max(3, reps // 4), flush)
    res["prefill_c4"] = {"tokens": tq, "ours_us": round(ours * 1e6, 1), "reference_us": round(ref * 1e6, 1),
                         "speedup": round(ref / ours, 3), "ours_tflops": round(flops / ours / 1e12, 1),
                         "reference_tflops": round(flops / ref / 1e12, 1)}
    return res


def run_c1(args):
    """BASELINE configs[0] as a single op: the KV store of one new token per sequence plus paged
    decode attention, 8 sequences, contexts U[16, 1024], Qwen3-0.6B heads (16 Q / 8 KV, D 128),
    64 blocks of 256, BF16, N(0, 1) values, scale 1/sqrt(128), new token at position L - 1.
    value: ops/s with every input in HBM (store + decode per op, L2 flushed before each op: the
    64 MB cache would otherwise stay in the 126 MB L2).  e2e: the same op through the C ABI with
    the per-op inputs (q, new k/v, slot mapping, block tables, context lengths) in pinned host
    memory, copied in, and the output copied back, inside the timed region."""
    import torch

    from hilda_vllm_b200 import kernels

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    b, hq, hk, d, nb, bs = 8, 16, 8, 128, 64, 256
    g = torch.Generator().manual_seed(args.seed)
    lens = torch.randint(16, 1025, (b,), generator=g)
    perm = torch.randperm(nb, generator=g).tolist()
    tables, off = [], 0
    for n in lens.tolist():
        k = -(-n // bs)
        tables.append(perm[off:off + k] + [-1] * (4 - k))
        off += k
    kc = torch.randn(nb, bs, hk, d, generator=g).bfloat16().to(dev)
    vc = torch.randn(nb, bs, hk, d, generator=g).bfloat16().to(dev)
    host = {"q": torch.randn(b, hq, d, generator=g).bfloat16(), "k": torch.randn(b, hk, d, generator=g).bfloat16(),
            "v": torch.randn(b, hk, d, generator=g).bfloat16(), "bt": torch.tensor(tables, dtype=torch.int32),
            "ln": lens.to(torch.int32),
            "slots": torch.tensor([t[(n - 1) // bs] * bs + (n - 1) % bs for t, n in zip(tables, lens.tolist())],
                                  dtype=torch.int32)}
    host = {k: v.pin_memory() for k, v in host.items()}
    devt = {k: v.to(dev) for k, v in host.items()}
    out = torch.empty(b, hq, d, dtype=torch.bfloat16, device=dev)
    out_host = torch.empty_like(out, device="cpu").pin_memory()
    ws = kernels.make_decode_workspace(b, hq, d, 4, bs, dev)
    flush = torch.zeros(128 << 20, dtype=torch.float32, device=dev)  # 512 MB > 126 MB of L2

    def op():
        kernels.store_kvcache(devt["k"], devt["v"], kc, vc, devt["slots"])
        kernels.paged_decode(devt["q"], kc, vc, devt["bt"], devt["ln"], d ** -0.5, out=out, workspace=ws)

    def op_e2e():
        for k in host:
            devt[k].copy_(host[k], non_blocking=True)
        op()
        out_host.copy_(out, non_blocking=True)

    for _ in range(args.warmup):
        op()
        op_e2e()
    sampler = ClockSampler(0)
    sampler.start()
    t_dev = _time_flushed(op, args.steps, flush)
    t_e2e = _time_flushed(op_e2e, args.steps, flush)
    t_dec = _time_flushed(lambda: kernels.paged_decode(devt["q"], kc, vc, devt["bt"], devt["ln"], d ** -0.5, out=out,
                                                       workspace=ws), args.steps, flush)
    clocks = sampler.stop()
    h2d = sum(v.numel() * v.element_size() for v in host.values())
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    hbm_peak = peaks.get("hbm_gbs", 6650.0)
    nbytes = int(lens.sum()) * hk * d * 2 * 2 + b * hq * d * 2 * 2
    cpu = None
    if not args.no_cpu:
        cpu = c1_cpu_sample(args.seed)
    line = {"metric": "config-1 single op (KV store + paged decode, 8 seqs): ops/s", "value": round(1 / t_dev, 1),
            "unit": "ops/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(t_dev * 1e3, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded N(0,1) cache, q and new K/V)",
            "config": {"workload": "c1: BASELINE configs[0], store + decode of 8 sequences, contexts U[16,1024], "
                                   "16 Q / 8 KV heads, 64 blocks of 256",
                       "l2": "flushed before every op (512 MB read-modify-write): the 64 MB cache fits in L2"},
            "roofline": {"bound": "hbm", "achieved": round(nbytes / t_dec / 1e9, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(nbytes / t_dec / 1e9 / hbm_peak, 4), "traffic": None,
                         "kernel": "paged_decode_kernel<bf16,G=2,Hk=8>", "avg_launch_us": round(t_dec * 1e6, 2),
                         "note": "8 sequences: 17 MB per launch, latency-bound (one wave of 32 CTAs)",
                         "peak_source": "of measured (MEASURED_PEAKS.json hbm_gbs)" if peaks else "of fallback"},
            "cpu_baseline": cpu,
            "e2e": {"value": round(1 / t_e2e, 1), "unit": "ops/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": out_host.numel() * 2, "us_per_op": round(t_e2e * 1e6, 2)},
            "clocks": clocks, "gpu_launches": 2 * args.steps}
    print(json.dumps(line), flush=True)


def c1_cpu_sample(seed: int, reps: int = 20) -> dict:
    """The config-1 op on the host cores through the CPU oracle (the reference's store scatter and
    fp32 attention restatement), mean seconds per op over reps."""
    import torch

    from oracle import attention as oattn
    from oracle import kv_store

    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    b, hq, hk, d, nb, bs = 8, 16, 8, 128, 64, 256
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(16, 1025, (b,), generator=g)
    perm = torch.randperm(nb, generator=g).tolist()
    tables, off = [], 0
    for n in lens.tolist():
        k = -(-n // bs)
        tables.append(perm[off:off + k] + [-1] * (4 - k))
        off += k
    kc = torch.randn(nb, bs, hk, d, generator=g).bfloat16()
    vc = torch.randn(nb, bs, hk, d, generator=g).bfloat16()
    q = torch.randn(b, hq, d, generator=g).bfloat16()
    kn = torch.randn(b, hk, d, generator=g).bfloat16()
    vn = torch.randn(b, hk, d, generator=g).bfloat16()
    bt = torch.tensor(tables, dtype=torch.int32)
    slots = torch.tensor([t[(n - 1) // bs] * bs + (n - 1) % bs for t, n in zip(tables, lens.tolist())],
                         dtype=torch.int32)
    kv_store.store_kvcache(kn, vn, kc, vc, slots)
    oattn.paged_decode(q, kc, vc, bt, lens, d ** -0.5)
    t0 = time.perf_counter()
    for _ in range(reps):
        kv_store.store_kvcache(kn, vn, kc, vc, slots)
        oattn.paged_decode(q, kc, vc, bt, lens, d ** -0.5)
    dt = (time.perf_counter() - t0) / reps
    return {"value": round(1 / dt, 2), "unit": "ops/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{reps} ops of the config-1 store + decode through the CPU oracle (fp32 attention), "
                      f"{dt * 1e3:.2f} ms per op"}


def run_profile(args):
    """Short, self-contained cases for ncu (one GPU)."""
    import torch

    from hilda_vllm_b200 import LLM, SamplingParams, kernels

    if args.profile == "allreduce":
        allreduce_profile(args)
        return
    if args.profile == "reference-kernels":
        print(json.dumps({"profile": "reference-kernels", **reference_kernel_ab(args.seed, max(args.steps, 5))}))
        return
    torch.cuda.set_device(0)
    g = torch.Generator().manual_seed(args.seed)
    if args.profile in ("decode-kernel", "decode-kernel-tc"):
        # Config-2 shapes at mid-job: 256 sequences, contexts U[65, 1087] (mean ~576), Hq 16 / Hk 8.
        # --workload c5: the Qwen3-8B layout (Hq 32 / Hk 8, GQA 4) at its mid-job contexts (prompt
        # U[256, 1024] + 256 generated); --kv fp8 stores the cache as e4m3.
        b, hq, hk, d, bs = NUM_SEQS, 16, 8, 128, 256
        lens = torch.randint(PROMPT_LEN + 1, PROMPT_LEN + OUTPUT_LEN, (b,), generator=g)
        if args.workload == "c5":
            hq = 32
            lens = torch.randint(256 + 256, 1024 + 256 + 1, (b,), generator=g)
        if args.tp_shard > 1:  # one GPU's heads under tensor parallelism
            hq, hk = hq // args.tp_shard, hk // args.tp_shard
        fp8 = args.kv == "fp8"
        nblk = [-(-int(n) // bs) for n in lens]
        perm = torch.randperm(sum(nblk), generator=g).tolist()
        mb = max(nblk)
        tables, off = [], 0
        for n in nblk:
            tables.append(perm[off:off + n] + [-1] * (mb - n))
            off += n
        dev = torch.device("cuda", 0)
        kc = torch.randn(sum(nblk), bs, hk, d, device=dev, dtype=torch.bfloat16)
        vc = torch.randn_like(kc)
        if fp8:
            kc, vc = kc.to(torch.float8_e4m3fn), vc.to(torch.float8_e4m3fn)
        q = torch.randn(b, hq, d, device=dev, dtype=torch.bfloat16)
        bt = torch.tensor(tables, dtype=torch.int32, device=dev)
        ln = lens.to(torch.int32).to(dev)
        out = torch.empty_like(q)
        ws = kernels.make_decode_workspace(b, hq, d, mb, bs, dev)
        tc = args.profile == "decode-kernel-tc"
        for _ in range(3):
            kernels.paged_decode(q, kc, vc, bt, ln, d ** -0.5, out=out, workspace=ws, tensor_cores=tc)
        torch.cuda.synchronize()
        stream = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.profiler.start()
        e0.record(stream)
        for _ in range(args.steps):
            kernels.paged_decode(q, kc, vc, bt, ln, d ** -0.5, out=out, workspace=ws, tensor_cores=tc)
        e1.record(stream)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        elem = 1 if fp8 else 2
        nbytes = int(lens.sum()) * hk * d * elem * 2 + b * hq * d * 4
        us = e0.elapsed_time(e1) * 1e3 / args.steps
        res = {"profile": args.profile, "workload": args.workload, "kv": "fp8" if fp8 else "bf16",
               "hq": hq, "hk": hk, "launches": args.steps, "bytes_per_launch": nbytes,
               "cache_gb": round(2 * kc.numel() * elem / 1e9, 2), "us_per_launch": round(us, 2),
               "gb_per_s": round(nbytes / us / 1e3, 1)}
        print(json.dumps(res))
        return
    if args.profile == "prefill-kernel":
        # BASELINE config-4 prefill shape: 8 sequences of 4096..8192 new tokens over a 2048-token
        # cached prefix (paged), Hq 16 / Hk 8, causal; FLOPs = 4 * Hq * D * sum_i visible_keys(i).
        hq, hk, d, bs = 16, 8, 128, 256
        dev = torch.device("cuda", 0)
        chunks = [int(x) for x in torch.randint(4096, 8193, (8,), generator=g)]
        prefix = 2048
        kl = [prefix + c for c in chunks]
        nblk = [-(-n // bs) for n in kl]
        perm = torch.randperm(sum(nblk), generator=g).tolist()
        mb = max(nblk)
        tables, off = [], 0
        for n in nblk:
            tables.append(perm[off:off + n] + [-1] * (mb - n))
            off += n
        kc = torch.randn(sum(nblk), bs, hk, d, device=dev, dtype=torch.bfloat16)
        vc = torch.randn_like(kc)
        tq = sum(chunks)
        q = torch.randn(tq, hq, d, device=dev, dtype=torch.bfloat16)
        cuq = torch.tensor([0] + list(__import__("itertools").accumulate(chunks)), dtype=torch.int32, device=dev)
        cuk = torch.tensor([0] + list(__import__("itertools").accumulate(kl)), dtype=torch.int32, device=dev)
        bt = torch.tensor(tables, dtype=torch.int32, device=dev)
        flops = sum(4 * hq * d * (c * prefix + c * (c + 1) // 2) for c in chunks)
        res = {"profile": "prefill-kernel", "tokens": tq, "gflop": round(flops / 1e9, 1)}
        variants = {"tc_precise": lambda: kernels.varlen_prefill(q, kc, vc, cuq, cuk, max(chunks), max(kl), d ** -0.5,
                                                                 block_table=bt, precise_p=True),
                    "tc_bf16p": lambda: kernels.varlen_prefill(q, kc, vc, cuq, cuk, max(chunks), max(kl), d ** -0.5,
                                                               block_table=bt, precise_p=False),
                    "tc_one_head_precise": lambda: kernels.varlen_prefill(q, kc, vc, cuq, cuk, max(chunks), max(kl),
                                                                          d ** -0.5, block_table=bt,
                                                                          one_head_per_cta=True)}
        stream = torch.cuda.current_stream()
        for name, fn in variants.items():
            fn()
            torch.cuda.synchronize()
            reps = args.steps
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            if name == "tc_precise":
                torch.cuda.profiler.start()
            e0.record(stream)
            for _ in range(reps):
                fn()
            e1.record(stream)
            torch.cuda.synchronize()
            if name == "tc_precise":
                torch.cuda.profiler.stop()
            ms = e0.elapsed_time(e1) / reps
            res[name] = {"ms": round(ms, 3), "tflops": round(flops / ms / 1e9, 1)}
        print(json.dumps(res))
        return
    if args.profile == "small-kernels":
        small_kernels(args, g)
        return

    # decode-steps: the engine at the job's mid context (prompts of 576 tokens, 256 sequences).
    ctx = PROMPT_LEN + OUTPUT_LEN // 2
    prompts = [torch.randint(0, 151936, (ctx,), generator=g).tolist() for _ in range(NUM_SEQS)]
    llm = LLM(str(CFG_DIR), load_format="random", seed=args.seed, max_num_seqs=NUM_SEQS, max_model_len=MAX_MODEL_LEN,
              max_num_batched_tokens=16384, gpu_memory_utilization=0.85)
    sp = SamplingParams(greedy=True, max_tokens=args.steps + 3, ignore_eos=True)
    for p in prompts:
        llm.add_request(p, sp)
    while llm.scheduler.waiting:
        llm.step()
    llm.step()  # first decode step outside the range (full packet)
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    for _ in range(args.steps):
        llm.step()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    print(json.dumps({"profile": "decode-steps", "steps": args.steps, "context": ctx + 1}))
    llm.exit()


# ----------------------------------------------------------------------------- other workloads
def _engine_e2e(args, model_dir, prompts, params, **llm_kwargs):
    """One warm-up job, then the timed job, through LLM.generate; returns (line fields, llm)."""
    import torch
    import torch.distributed as dist

    from hilda_vllm_b200 import LLM

    world = args.gpus
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    llm = LLM(str(model_dir), load_format="random", seed=args.seed, tensor_parallel_size=world,
              distributed_executor="external" if world > 1 else "spawn", **llm_kwargs)
    if getattr(llm, "is_worker", False):
        if dist.is_initialized():
            dist.destroy_process_group()
        return None, None
    from hilda_vllm_b200.engine.scheduler import Scheduler

    warm = [p[:64] for p in prompts[:8]]
    llm.generate(warm, params[:8], use_tqdm=False)
    llm.scheduler = Scheduler(llm.config)
    llm.model_runner.call("reset_decode_state")
    llm.model_runner.io_bytes = {"h2d": 0, "d2h": 0}
    sampler = ClockSampler(local)
    sampler.start()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    outs = llm.generate(prompts, params, use_tqdm=False)
    wall = time.perf_counter() - t0
    clocks = sampler.stop()
    st = llm.last_generate_stats
    n_out = sum(len(o["token_ids"]) for o in outs)
    steps = st["decode_steps"] + 1
    fields = {"e2e": {"value": round(n_out / wall, 1), "unit": "tok/s",
                      "h2d_bytes_per_step": int(llm.model_runner.io_bytes["h2d"] / steps),
                      "d2h_bytes_per_step": int(llm.model_runner.io_bytes["d2h"] / steps),
                      "wall_s": round(wall, 3), "output_tokens": n_out,
                      "prompt_tokens": st["prompt_tokens"], "prefill_tokens": st["prefill_tokens"],
                      "prefill_s": round(st["prefill_time_s"], 3), "decode_s": round(st["decode_time_s"], 3),
                      "prefill_tok_s": round(st["prefill_throughput_toks"], 1),
                      "decode_tok_s": round(st["decode_throughput_toks"], 1),
                      "decode_steps": st["decode_steps"], "avg_decode_active_bs": round(st["avg_decode_active_bs"], 2),
                      "min_free_blocks": st["min_free_blocks_observed"], "kv_blocks": st["kv_num_blocks"],
                      "prefill_blocked_steps": st["prefill_allocation_blocked_steps"]},
              "clocks": clocks}
    return fields, llm


def run_workload(args):
    """BASELINE configs 3, 4 and 5 through the public API (e2e); value = output tok/s."""
    import torch

    from hilda_vllm_b200 import SamplingParams

    g = torch.Generator().manual_seed(args.seed)
    vocab = 151936
    if args.workload == "c3":
        # FP8 e4m3 KV with per-head scales (unit scales, the reference-compatible setting), 256 seqs,
        # prompts U[32,128], 512 greedy tokens, pool capped at 512 blocks (< 768 needed at the
        # peak) so the scheduler preempts, re-prefills and compacts the decode batch.
        prompts = [torch.randint(0, vocab, (int(torch.randint(32, 129, (1,), generator=g)),), generator=g).tolist()
                   for _ in range(256)]
        params = [SamplingParams(greedy=True, max_tokens=512, ignore_eos=True)] * 256
        kw = dict(max_num_seqs=256, max_model_len=64 + 512 + 256 + 128, max_num_batched_tokens=16384,
                  kv_cache_dtype="fp8", kvcache_block_cap=512, gpu_memory_utilization=0.85)
        cfg, desc = CFG_DIR, "qwen3-0.6b FP8 KV, 256 seqs, prompt U[32,128], 512 greedy, pool capped at 512 blocks"
    elif args.workload == "c4":
        # 64 long prompts U[4096,8192] in 8 groups sharing a 2048-token prefix (max_tokens 1, as the
        # reference's jitter benchmark), plus 128 decode sequences of prompt 64 / output 256; prefill
        # chunk budget 8192; max_model_len = max_num_batched_tokens = 8448 (config.py:40).
        prompts, params = [], []
        for grp in range(8):
            prefix = torch.randint(0, vocab, (2048,), generator=g).tolist()
            for _ in range(8):
                n = int(torch.randint(4096, 8193, (1,), generator=g))
                prompts.append(prefix + torch.randint(0, vocab, (n - 2048,), generator=g).tolist())
                params.append(SamplingParams(greedy=True, max_tokens=1, ignore_eos=True))
        for _ in range(128):
            prompts.append(torch.randint(0, vocab, (64,), generator=g).tolist())
            params.append(SamplingParams(greedy=True, max_tokens=256, ignore_eos=True))
        order = torch.randperm(len(prompts), generator=g).tolist()
        prompts = [prompts[i] for i in order]
        params = [params[i] for i in order]
        kw = dict(max_num_seqs=256, max_model_len=8448, max_num_batched_tokens=8448, chunked_prefill_size=8192,
                  gpu_memory_utilization=0.85)
        cfg, desc = CFG_DIR, "qwen3-0.6b mixed: 64 x U[4096,8192] prompts (8 groups sharing 2048-token prefixes) + 128 x (64 -> 256)"
    else:
        # Qwen3-8B shape, 256 seqs, prompts U[256,1024], 512 greedy tokens, TP over --gpus.
        prompts = [torch.randint(0, vocab, (int(torch.randint(256, 1025, (1,), generator=g)),), generator=g).tolist()
                   for _ in range(256)]
        params = [SamplingParams(greedy=True, max_tokens=512, ignore_eos=True)] * 256
        kw = dict(max_num_seqs=256, max_model_len=1024 + 512 + 256, max_num_batched_tokens=16384,
                  kv_cache_dtype="fp8" if args.kv == "fp8" else "auto", gpu_memory_utilization=0.85)
        cfg = ROOT / "hilda_vllm_b200" / "model_configs" / "qwen3-8b"
        desc = f"qwen3-8b, 256 seqs, prompt U[256,1024], 512 greedy, {'fp8' if args.kv == 'fp8' else 'bf16'} KV, tp{args.gpus}"
    fields, llm = _engine_e2e(args, cfg, prompts, params, **kw)
    if fields is None:
        return
    e2e = fields["e2e"]
    line = {"metric": f"{desc}: output tok/s", "value": e2e["value"], "unit": "tok/s", "n_gpus": args.gpus,
            "steps": 1, "warmup": 1, "ms_per_step": round(e2e["wall_s"] * 1e3, 1), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic", "config": {"workload": args.workload, "desc": desc,
                                                             "parallelism": f"tp{args.gpus}"},
            **fields}
    print(json.dumps(line), flush=True)
    llm.exit()


def main():
    args = parse()
    if args.profile:
        run_profile(args)
        return
    if args.workload == "c1":
        if args.impl == "reference":
            run_c1_reference(args)
        else:
            run_c1(args)
        return
    if args.workload != "c2" and args.impl == "ours":
        run_workload(args)
        return
    if args.impl == "reference":
        run_reference_arm(args)
        return
    run_ours(args)


if __name__ == "__main__":
    main()
