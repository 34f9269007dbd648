"""User-facing engine: LLM(model, **config) with add_request / step / generate / generate_stream.

Same API and step semantics as mini_vllm/engine/llm_engine.py:17-470 (without speculative
decoding): schedule -> run on the model runner(s) -> postprocess, the FP8 prefill->decode cache
conversion after prefill steps, and the same throughput statistics in last_generate_stats.
step() returns the reference's 13-tuple; the speculative-decoding fields are always zero.
"""
from __future__ import annotations

import atexit
import os
import socket
from dataclasses import fields
from time import perf_counter

import torch.multiprocessing as mp

from hilda_vllm_b200.config import Config
from hilda_vllm_b200.engine.model_runner import ModelRunner
from hilda_vllm_b200.engine.scheduler import Scheduler
from hilda_vllm_b200.engine.sequence import PLACEHOLDER, Sequence
from hilda_vllm_b200.sampling_params import SamplingParams
from hilda_vllm_b200.utils.tokenizer import load_tokenizer


def _free_port() -> int:
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


class LLMEngine:

    def __init__(self, model, **kwargs):
        names = {f.name for f in fields(Config)}
        config = Config(model, **{k: v for k, v in kwargs.items() if k in names})
        self.config = config
        self.ps = []
        self.events = []
        if config.tensor_parallel_size > 1 and config.distributed_executor == "spawn" \
                and "MINI_VLLM_DIST_PORT" not in os.environ:
            os.environ["MINI_VLLM_DIST_PORT"] = str(_free_port())  # inherited by the spawned ranks
        if config.distributed_executor == "external" and config.tensor_parallel_size > 1:
            import torch.distributed as dist
            rank = dist.get_rank()
            if rank != 0:
                # Worker rank: serve rank 0's calls until it exits, then return a shell.
                ModelRunner(config, rank, None)
                self.is_worker = True
                return
            self.model_runner = ModelRunner(config, 0, None)
        else:
            ctx = mp.get_context("spawn")
            for i in range(1, config.tensor_parallel_size):
                event = ctx.Event()
                process = ctx.Process(target=ModelRunner, args=(config, i, event))
                process.start()
                self.ps.append(process)
                self.events.append(event)
            self.model_runner = ModelRunner(config, 0, self.events)
        self.is_worker = False
        self.tokenizer = load_tokenizer(config.model, config.hf_config)
        config.eos = self.tokenizer.eos_token_id if self.tokenizer.eos_token_id is not None else -1
        self.scheduler = Scheduler(config)
        self._inflight = None
        self.last_generate_stats = None
        self.last_step_diagnostics = None
        atexit.register(self.exit)

    def exit(self):
        if not hasattr(self, "model_runner"):
            return
        self.model_runner.call("exit")
        del self.model_runner
        for p in self.ps:
            p.join()

    def add_request(self, prompt: str | list[int], sampling_params: SamplingParams):
        if isinstance(prompt, str):
            prompt = self.tokenizer.encode(prompt)
        seq = Sequence(prompt, sampling_params)
        self.scheduler.add(seq)
        return seq

    # ------------------------------------------------------------------ stepping
    # Overlapped decode (config.async_decode, default on): while every running sequence stops
    # by length (ignore_eos, or no EOS token), a decode step sampled on the device (greedy or
    # plain temperature) is launched before the
    # previous one's tokens are read back; its sequences get PLACEHOLDER tokens that the next
    # step() fills.  The host then schedules and packs step k+1 while the GPU runs step k.  Any
    # other step (prefill, sampling, EOS possible, a packet that needs a token still on the GPU)
    # first drains the step in flight and runs synchronously, as the reference does.
    def _drain(self) -> list:
        """Reads back the step in flight, fills its placeholders, returns its finished outputs."""
        if self._inflight is None:
            return []
        handle, pending, finished = self._inflight
        self._inflight = None
        self.scheduler.resolve_tokens(pending, self.model_runner.collect_decode(handle))
        return [(seq.seq_id, seq.completion_token_ids) for seq in finished]

    def _step_result(self, outputs, num_prefill_tokens, num_decode_tokens):
        return outputs, num_prefill_tokens, num_decode_tokens, 0, 0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0

    def step(self):
        if self.config.async_decode and self._inflight is not None and not self.scheduler.eos_cannot_stop():
            early = self._drain()
        else:
            early = []
        if self.scheduler.is_finished():
            return self._step_result(early + self._drain(), 0, 0)
        seqs, is_prefill = self.scheduler.schedule()
        if not seqs:
            return self._step_result(early + self._drain(), 0, 0)
        if (self.config.async_decode and not is_prefill and self.scheduler.eos_cannot_stop()
                and all(s.is_padding or self.model_runner.samples_on_device(s.seq) for s in seqs)):
            if not self.model_runner.can_launch_decode(seqs):
                early += self._drain()
            handle = self.model_runner.launch_decode(seqs)
            self.last_step_diagnostics = {
                "running": len(self.scheduler.running),
                "waiting": len(self.scheduler.waiting),
                "decode_batch": self.model_runner.last_decode_batch_info or {},
            }
            pending, finished = self.scheduler.postprocess_launched(seqs)
            early += self._drain()
            self._inflight = (handle, pending, finished)
            return self._step_result(early, 0, len(pending))
        early += self._drain()
        outputs, n_pre, n_dec = self._step_sync(seqs, is_prefill)
        return self._step_result(early + outputs, n_pre, n_dec)

    def _step_sync(self, seqs, is_prefill):
        token_ids = self.model_runner.run(seqs, is_prefill)
        self.last_step_diagnostics = {
            "running": len(self.scheduler.running),
            "waiting": len(self.scheduler.waiting),
            "decode_batch": None if is_prefill else (self.model_runner.last_decode_batch_info or {}),
        }
        self.scheduler.postprocess(seqs, token_ids, is_prefill)
        if is_prefill and self.config.kv_cache_dtype == "fp8":
            ready = [s.seq for s in seqs if not s.is_padding and s.seq.is_prefill_done and not s.seq.is_finished
                     and not s.seq.decode_cache_ready]
            if ready:
                self.model_runner.convert_prefill_to_decode_cache(ready)
                for seq in ready:
                    seq.decode_cache_ready = True
        outputs = [(s.seq.seq_id, s.seq.completion_token_ids) for s in seqs if not s.is_padding and s.seq.is_finished]
        if is_prefill:
            num_prefill_tokens = sum(s.token_chunk_size for s in seqs if not s.is_padding)
            num_decode_tokens = sum(1 for s, t in zip(seqs, token_ids) if not s.is_padding and t is not None)
        else:
            num_prefill_tokens = 0
            num_decode_tokens = sum(1 for s in seqs if not s.is_padding)
        return outputs, num_prefill_tokens, num_decode_tokens

    def is_finished(self):
        return self.scheduler.is_finished() and self._inflight is None

    def _add_sequences(self, prompts, sampling_params) -> list[Sequence]:
        if not isinstance(sampling_params, list):
            sampling_params = [sampling_params] * len(prompts)
        return [self.add_request(p, sp) for p, sp in zip(prompts, sampling_params)]

    def generate_stream(self, prompts, sampling_params):
        self.scheduler.reset_diagnostics()
        seqs = self._add_sequences(prompts, sampling_params)
        emitted = {seq.seq_id: 0 for seq in seqs}
        index = {seq.seq_id: i for i, seq in enumerate(seqs)}
        stats = self._init_generate_stats(seqs)
        start = perf_counter()
        while not self.is_finished():
            t = perf_counter()
            _, n_pre, n_dec, *_ = self.step()
            self._update_generate_stats(stats, n_pre, n_dec, perf_counter() - t, self.last_step_diagnostics)
            for seq in seqs:
                done = seq.completion_token_ids
                if PLACEHOLDER in done:  # tokens still on the GPU are emitted next step
                    done = done[:done.index(PLACEHOLDER)]
                prev = emitted[seq.seq_id]
                if len(done) <= prev:
                    continue
                emitted[seq.seq_id] = len(done)
                yield {"request_index": index[seq.seq_id], "seq_id": seq.seq_id, "token_ids": list(done[prev:]),
                       "completion_token_ids": list(done), "is_finished": seq.is_finished}
        self._set_last_generate_stats(stats, perf_counter() - start)

    def generate(self, prompts, sampling_params, use_tqdm: bool = True) -> list[dict]:
        self.scheduler.reset_diagnostics()
        pbar = None
        if use_tqdm:
            from tqdm.auto import tqdm
            pbar = tqdm(total=len(prompts), desc="Generating", dynamic_ncols=True)
        seqs = self._add_sequences(prompts, sampling_params)
        outputs = {}
        stats = self._init_generate_stats(seqs)
        start = perf_counter()
        while not self.is_finished():
            t = perf_counter()
            output, n_pre, n_dec, *_ = self.step()
            pre_tps, dec_tps = self._update_generate_stats(stats, n_pre, n_dec, perf_counter() - t,
                                                           self.last_step_diagnostics)
            if pbar is not None:
                pbar.set_postfix({"Prefill": f"{int(pre_tps)}tok/s", "Decode": f"{int(dec_tps)}tok/s"})
            for seq_id, token_ids in output:
                outputs[seq_id] = token_ids
                if pbar is not None:
                    pbar.update(1)
        self._set_last_generate_stats(stats, perf_counter() - start)
        if pbar is not None:
            pbar.close()
        return [{"text": self.tokenizer.decode(outputs[seq.seq_id]), "token_ids": outputs[seq.seq_id]} for seq in seqs]

    # ------------------------------------------------------------------ scoring
    def score_next_tokens(self, token_lists: list[list[int]], targets: list[int]) -> list[dict]:
        """For each token list, the model's next-token logits after its last token, summarised:
        the greedy choice (argmax, lowest id among equal maxima), the top logit and the logit of
        the given target token.  Prefill-only passes on fresh blocks (no prefix-cache reuse) run
        while the engine has no requests of its own; lists are packed into batches of at most
        max_num_batched_tokens tokens.  This is a teacher-forced check of generated tokens: feed a
        prompt plus the first s generated tokens and ask whether token s is the model's choice."""
        from hilda_vllm_b200.engine.scheduler import ScheduledSequence

        assert self.scheduler.is_finished() and self._inflight is None, "score_next_tokens needs an idle engine"
        assert len(token_lists) == len(targets)
        bm = self.scheduler.block_manager
        budget = self.config.max_num_batched_tokens
        out: list[dict] = []
        i = 0
        while i < len(token_lists):
            batch = []
            used = 0
            while i < len(token_lists) and len(batch) < self.config.max_num_seqs:
                seq = Sequence(list(token_lists[i]), SamplingParams(greedy=True, max_tokens=1))
                if used + len(seq) > budget or len(bm.free_block_ids) < seq.num_blocks:
                    break
                bm.allocate_uncached(seq)
                batch.append(ScheduledSequence(seq, len(seq)))
                used += len(seq)
                i += 1
            if not batch:
                raise RuntimeError(f"score_next_tokens: list {i} ({len(token_lists[i])} tokens) does not fit the "
                                   f"batch budget ({budget}) or the KV pool")
            try:
                res = self.model_runner.score(batch, targets[i - len(batch):i])
            finally:
                for sched in batch:
                    bm.deallocate(sched.seq)
            out.extend(res)
        return out

    # ------------------------------------------------------------------ statistics
    @staticmethod
    def _init_generate_stats(seqs):
        return {
            "num_requests": len(seqs), "prompt_tokens": sum(s.num_prompt_tokens for s in seqs),
            "prefill_tokens": 0, "decode_tokens": 0, "prefill_time_s": 0.0, "decode_time_s": 0.0,
            "decode_steps": 0, "decode_scheduled_bs_sum": 0, "decode_active_bs_sum": 0, "decode_graph_bs_sum": 0,
            "decode_padded_slots_sum": 0, "decode_active_bs_max": 0, "running_max": 0, "waiting_max": 0,
        }

    @staticmethod
    def _update_generate_stats(stats, n_prefill, n_decode, elapsed, diag=None):
        pre_tps = dec_tps = 0.0
        if n_prefill > 0:
            stats["prefill_tokens"] += n_prefill
            stats["prefill_time_s"] += elapsed
            pre_tps = n_prefill / elapsed if elapsed else 0.0
        if n_decode > 0:
            stats["decode_tokens"] += n_decode
            stats["decode_time_s"] += elapsed
            dec_tps = n_decode / elapsed if elapsed else 0.0
        if diag:
            stats["running_max"] = max(stats["running_max"], diag.get("running", 0))
            stats["waiting_max"] = max(stats["waiting_max"], diag.get("waiting", 0))
            batch = diag.get("decode_batch")
            if batch is not None:
                active = batch.get("active_seqs", 0)
                stats["decode_steps"] += 1
                stats["decode_scheduled_bs_sum"] += batch.get("scheduled_bs", 0)
                stats["decode_active_bs_sum"] += active
                stats["decode_graph_bs_sum"] += batch.get("graph_bs", 0)
                stats["decode_padded_slots_sum"] += batch.get("padded_slots", 0)
                stats["decode_active_bs_max"] = max(stats["decode_active_bs_max"], active)
        return pre_tps, dec_tps

    def _set_last_generate_stats(self, stats, total_time):
        out = stats["decode_tokens"]
        steps = stats["decode_steps"]
        res = {
            "num_requests": stats["num_requests"], "prompt_tokens": stats["prompt_tokens"], "output_tokens": out,
            "prefill_tokens": stats["prefill_tokens"], "decode_tokens": stats["decode_tokens"],
            "prefill_time_s": stats["prefill_time_s"], "decode_time_s": stats["decode_time_s"],
            "total_time_s": total_time,
            "prefill_throughput_toks": stats["prefill_tokens"] / stats["prefill_time_s"] if stats["prefill_time_s"] else 0.0,
            "decode_throughput_toks": stats["decode_tokens"] / stats["decode_time_s"] if stats["decode_time_s"] else 0.0,
            "total_throughput_toks": out / total_time if total_time else 0.0,
            "decode_steps": steps,
        }
        for key in ("scheduled_bs", "active_bs", "graph_bs", "padded_slots"):
            res[f"avg_decode_{key}"] = stats[f"decode_{key}_sum"] / steps if steps else 0.0
        res.update({"decode_active_bs_max": stats["decode_active_bs_max"], "running_max": stats["running_max"],
                    "waiting_max": stats["waiting_max"]})
        res.update(self.scheduler.get_diagnostics())
        self.last_generate_stats = res
