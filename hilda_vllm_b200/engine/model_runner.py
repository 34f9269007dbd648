"""Per-GPU model runner: KV pool, batch preparation, decode CUDA graphs, TP control plane.

Mirrors mini_vllm/engine/model_runner.py (ModelRunner) for the non-speculative path:
  - allocate_kv_cache (:141-220): the pool [2, L, NB, BS, Hk/tp, D] (plus the FP8 twin) sized
    from free memory, per-layer views handed to each Attention module;
  - prepare_prefill (:614-650): varlen metadata and slot mapping for the scheduled chunks;
  - prepare_decode (:652-720): replaced by DecodePacker + the hl_pack_decode_batch kernel, so
    the host sends one small packet per step instead of rewriting every slot;
  - capture_cudagraph / run_model (:735-832): one graph per batch bucket [1,2,4,8,16,...,512];
    each graph holds the pack kernel, the whole model, the LM head and the device sampler
    (greedy argmax, Gumbel-max temperature sampling, and on one GPU the top-k / top-p filters
    of hl_sample_filtered; under tensor parallelism top-k / top-p rows gather their logits to
    rank 0, which samples them with the same kernel), so a decode step is: one packet copy,
    one graph replay, one token copy back;
  - convert_prefill_to_decode_cache (:483-502): one launch for all layers;
  - the tensor-parallel RPC through shared memory (:82-130) with rank 0 driving.
"""
from __future__ import annotations

import os
import pickle
import time
from multiprocessing.shared_memory import SharedMemory

import numpy as np
import torch
import torch.distributed as dist

from hilda_vllm_b200 import kernels
from hilda_vllm_b200.engine.control_plane import ShmChannel
from hilda_vllm_b200.engine.decode_packer import DecodePacker, packet_capacity_bytes
from hilda_vllm_b200.engine.scheduler import ScheduledSequence
from hilda_vllm_b200.engine.sequence import Sequence
from hilda_vllm_b200.layers import nvlink_allreduce
from hilda_vllm_b200.layers.attention import Attention
from hilda_vllm_b200.layers.nvlink_allreduce import NvlinkAllReduce
from hilda_vllm_b200.models.qwen3 import Qwen3ForCausalLM
from hilda_vllm_b200.utils.context import reset_context, set_context
from hilda_vllm_b200.utils.loader import has_checkpoint, load_model, random_init

MODEL_REGISTRY = {"qwen3": Qwen3ForCausalLM}
MAX_GRAPH_BS = 512


def sampling_settings(seqs: list[Sequence]):
    """None when every sequence samples greedily, else the per-row sampler inputs."""
    if all(getattr(s, "greedy", False) for s in seqs):
        return None
    return ([s.temperature for s in seqs], [s.top_k for s in seqs], [s.top_p for s in seqs],
            [bool(getattr(s, "greedy", False)) for s in seqs])


def device_sampleable(seq, filters: bool = False) -> bool:
    """Whether the decode graph samples this sequence on the device: greedy and plain temperature
    sampling always (hl_sample), top-k / top-p too when `filters` (one GPU holds the whole
    vocabulary: hl_sample_filtered)."""
    return bool(getattr(seq, "greedy", False)) or filters or (seq.top_k == -1 and seq.top_p >= 1.0)


def decode_sampling(scheduled_seqs, filters: bool = False) -> np.ndarray | None:
    """Per-row device sampler settings as one float32 [3, n] array — temperature (0: greedy argmax,
    also for padding rows), top_k (int32 bits; 0 = no filter), top_p (1 = no filter) — or None when
    some row needs the host sampler."""
    n = len(scheduled_seqs)
    out = np.zeros((3, n), np.float32)
    out[2] = 1.0
    ks = out[1].view(np.int32)
    for i, sched in enumerate(scheduled_seqs):
        seq = sched.seq
        if seq is None:
            continue
        if not device_sampleable(seq, filters):
            return None
        if not getattr(seq, "greedy", False):
            out[0, i] = seq.temperature
            ks[i] = max(int(seq.top_k), 0)
            out[2, i] = seq.top_p
    return out


def decode_temperatures(scheduled_seqs) -> np.ndarray | None:
    """Per-row temperature for hl_sample (0: greedy argmax, also for padding rows), or None when
    some row needs top-k / top-p."""
    samp = decode_sampling(scheduled_seqs)
    return None if samp is None else samp[0].copy()


def merge_shard_argmax(all_val: torch.Tensor, all_idx: torch.Tensor) -> torch.Tensor:
    """Global greedy token from per-shard (max value, global index) pairs, shards ordered by
    vocabulary range ([tp, n] each): the first shard holding the maximum wins, which is the
    lowest vocabulary id among equal maxima, as a single argmax over all logits would pick."""
    best = all_val.argmax(0, keepdim=True)
    return all_idx.gather(0, best).squeeze(0)


def graph_batch_sizes(max_bs: int) -> list[int]:
    max_bs = min(max_bs, MAX_GRAPH_BS)
    return [b for b in (1, 2, 4, 8) if b <= max_bs] + list(range(16, max_bs + 1, 16))


def prefill_metadata(seqs: list[ScheduledSequence], block_size: int) -> dict:
    """Host-side prefill batch description, as the reference's prepare_prefill builds it
    (mini_vllm/engine/model_runner.py:614-650): concatenated chunk tokens and positions,
    cu_seqlens_q / cu_seqlens_k (keys = prefix + chunk), their maxima, the slot of every chunk
    token (block_table[pos // BS] * BS + pos % BS, only for sequences with a block table) and,
    when any chunk starts after position 0, the -1 padded block tables of all sequences."""
    ids, pos, slots = [], [], []
    cu_q, cu_k = [0], [0]
    max_q = max_k = 0
    has_prefix = False
    for sched in seqs:
        seq = sched.seq
        start = seq.num_computed_tokens
        end = start + sched.token_chunk_size
        ids.extend(seq.token_ids[start:end])
        p = np.arange(start, end, dtype=np.int64)
        pos.append(p)
        cu_q.append(cu_q[-1] + end - start)
        cu_k.append(cu_k[-1] + end)
        max_q = max(max_q, end - start)
        max_k = max(max_k, end)
        has_prefix = has_prefix or start > 0
        if seq.block_table:
            table = np.asarray(seq.block_table, dtype=np.int64)
            slots.append(table[p // block_size] * block_size + p % block_size)
    block_tables = None
    if has_prefix:
        width = max(len(s.seq.block_table) for s in seqs)
        block_tables = np.full((len(seqs), width), -1, dtype=np.int32)
        for i, s in enumerate(seqs):
            block_tables[i, : len(s.seq.block_table)] = s.seq.block_table
    return {
        "input_ids": np.asarray(ids, dtype=np.int64),
        "positions": np.concatenate(pos) if pos else np.zeros(0, np.int64),
        "cu_seqlens_q": np.asarray(cu_q, dtype=np.int32),
        "cu_seqlens_k": np.asarray(cu_k, dtype=np.int32),
        "max_seqlen_q": max_q,
        "max_seqlen_k": max_k,
        "slot_mapping": (np.concatenate(slots) if slots else np.zeros(0, np.int64)).astype(np.int32),
        "block_tables": block_tables,
    }


class ModelRunner:

    def __init__(self, config, rank: int, event=None):
        self.config = config
        hf = config.hf_config
        self.block_size = config.kvcache_block_size
        self.max_num_decode_blocks = (config.max_model_len + self.block_size - 1) // self.block_size
        self.enforce_eager = config.enforce_eager
        self.world_size = config.tensor_parallel_size
        self.rank = rank
        self.event = event
        self.use_fp8_kv_cache = config.kv_cache_dtype == "fp8"
        self.last_decode_batch_info = None
        self.graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self.graph_pool = None

        self.external = getattr(config, "distributed_executor", "spawn") == "external"
        self.io_bytes = {"h2d": 0, "d2h": 0}
        # Seconds the host spent blocked on the GPU for a step's tokens (rank 0); the rest of a
        # job's wall time is host work (scheduling, packets, control plane) or idle GPU.
        self.gpu_wait_s = 0.0
        self.recording: list[torch.Tensor] | None = None
        if self.world_size > 1 and not dist.is_initialized():
            port = int(os.getenv("MINI_VLLM_DIST_PORT", "2333"))
            dist.init_process_group("nccl", f"tcp://127.0.0.1:{port}", world_size=self.world_size, rank=rank,
                                    device_id=torch.device("cuda", int(os.getenv("LOCAL_RANK", rank))))
        self.rpc_group = None
        self.chan = None
        if self.world_size > 1 and self.external:
            # Ranks launched by torchrun: the control plane is a shared-memory channel polled by
            # the ranks (ShmChannel) instead of the spawn mode's block + inherited events; a gloo
            # group carries its name once.
            self.rpc_group = dist.new_group(backend="gloo")
        local = int(os.getenv("LOCAL_RANK", rank))
        torch.cuda.set_device(local)
        self.device = torch.device("cuda", local)
        self.allreduce = None
        if self.world_size > 1 and getattr(config, "custom_allreduce", True):
            # Peer-mapped buffers for the decode batches (up to the largest CUDA-graph batch).
            max_rows = graph_batch_sizes(config.max_num_seqs)[-1]
            self.allreduce = NvlinkAllReduce(rank, self.world_size, max_rows, hf.hidden_size, self.device)
            nvlink_allreduce.set_active(self.allreduce)
        default_dtype = torch.get_default_dtype()
        torch.set_default_dtype(torch.bfloat16)
        torch.set_default_device(self.device)
        try:
            cls = MODEL_REGISTRY.get(hf.model_type, Qwen3ForCausalLM)
            self.model = cls(hf)
            if config.load_format == "auto" and has_checkpoint(config.model):
                load_model(self.model, config.model)
            else:
                random_init(self.model, hf, seed=config.seed, std=config.init_std, device=self.device)
            self.vocab_size = hf.vocab_size
            self.warmup_model()
            self.allocate_kv_cache()
            self.allocate_decode_runtime_buffers()
            if not self.enforce_eager:
                self.capture_cudagraph()
        finally:
            torch.set_default_device("cpu")
            torch.set_default_dtype(default_dtype)

        if self.world_size > 1 and not self.external:
            if rank == 0:
                self.shm = SharedMemory(name="hilda_b200", create=True, size=2 ** 20)
                dist.barrier()
            else:
                dist.barrier()
                self.shm = SharedMemory(name="hilda_b200")
                self.loop()
        elif self.world_size > 1:
            box = [None]
            if rank == 0:
                self.chan = ShmChannel.create(self.world_size)
                box = [self.chan.name]
            dist.broadcast_object_list(box, src=0, group=self.rpc_group)
            if rank > 0:
                self.chan = ShmChannel.attach(box[0], rank, self.world_size)
            dist.barrier(group=self.rpc_group)
            if rank > 0:
                self.loop()

    # ------------------------------------------------------------------ TP control plane
    def exit(self):
        if self.world_size > 1 and not self.external:
            self.shm.close()
            dist.barrier()
            if self.rank == 0:
                self.shm.unlink()
        if self.chan is not None:
            self.chan.close()  # rank 0 removes the segment; mapped views stay valid
            self.chan = None
        self.graphs = {}
        self.graph_pool = None
        torch.cuda.synchronize()
        if self.allreduce is not None:
            nvlink_allreduce.set_active(None)
            dist.barrier()  # no peer may still read this rank's buffers
            self.allreduce.close()
            self.allreduce = None
        if self.world_size > 1 and dist.is_initialized():
            dist.destroy_process_group()

    def loop(self):
        while True:
            method, args = self.read_shm()
            self.call(method, *args)
            if method == "exit":
                break

    def read_shm(self):
        assert self.world_size > 1 and self.rank > 0
        if self.external:
            return self.chan.recv()
        self.event.wait()
        n = int.from_bytes(self.shm.buf[0:4], "little")
        method, *args = pickle.loads(self.shm.buf[4:n + 4])
        self.event.clear()
        return method, args

    def write_shm(self, method, *args):
        assert self.world_size > 1 and self.rank == 0
        if self.external:
            self.chan.send(method, *args)
            return
        data = pickle.dumps([method, *args])
        self.shm.buf[0:4] = len(data).to_bytes(4, "little")
        self.shm.buf[4:len(data) + 4] = data
        for ev in self.event:
            ev.set()

    def call(self, method, *args):
        if self.world_size > 1 and self.rank == 0:
            self.write_shm(method, *args)
        return getattr(self, method)(*args)

    # ------------------------------------------------------------------ memory
    def attention_layers(self) -> list[Attention]:
        return [m for m in self.model.modules() if isinstance(m, Attention)]

    @torch.inference_mode()
    def warmup_model(self):
        """Largest prefill (max_num_batched_tokens tokens) before the KV pool exists, so the
        activation peak is known when the pool is sized (model_runner.py:132-139)."""
        torch.cuda.empty_cache()
        torch.cuda.reset_peak_memory_stats()
        max_tokens, max_len = self.config.max_num_batched_tokens, self.config.max_model_len
        num_seqs = max(1, min(max_tokens // max_len, self.config.max_num_seqs))
        seqs = [ScheduledSequence(Sequence([0] * max_len), max_len) for _ in range(num_seqs)]
        input_ids, positions = self.prepare_prefill(seqs)
        self.model.compute_logits(self.model(input_ids, positions))
        reset_context()
        torch.cuda.synchronize()
        torch.cuda.empty_cache()

    def kv_block_bytes(self) -> int:
        hf = self.config.hf_config
        hk = hf.num_key_value_heads // self.world_size
        d = getattr(hf, "head_dim", None) or hf.hidden_size // hf.num_attention_heads
        per_elem = 2 + (1 if self.use_fp8_kv_cache else 0)
        return 2 * hf.num_hidden_layers * self.block_size * hk * d * per_elem

    def allocate_kv_cache(self):
        config = self.config
        hf = config.hf_config
        free, total = torch.cuda.mem_get_info()
        used = total - free
        stats = torch.cuda.memory_stats()
        peak, current = stats["allocated_bytes.all.peak"], stats["allocated_bytes.all.current"]
        # Room for the decode buffers, graph pool and workspace that are allocated afterwards.
        reserve = 2 << 30
        budget = int(total * config.gpu_memory_utilization - used - peak + current) - reserve
        num_blocks = budget // self.kv_block_bytes()
        if config.kvcache_block_cap > 0:
            num_blocks = min(num_blocks, config.kvcache_block_cap)
        if self.world_size > 1:  # rank 0 schedules for every rank: use the smallest pool
            t = torch.tensor([num_blocks], dtype=torch.int64, device=self.device)
            dist.all_reduce(t, op=dist.ReduceOp.MIN)
            num_blocks = int(t.item())
        config.num_kvcache_blocks = int(num_blocks)
        assert config.num_kvcache_blocks > 0, "no memory left for the KV cache"
        hk = hf.num_key_value_heads // self.world_size
        d = getattr(hf, "head_dim", None) or hf.hidden_size // hf.num_attention_heads
        shape = (2, hf.num_hidden_layers, config.num_kvcache_blocks, self.block_size, hk, d)
        layers = self.attention_layers()
        if self.use_fp8_kv_cache:
            self.prefill_kv_cache = torch.zeros(shape, dtype=torch.bfloat16)
            self.decode_kv_cache = torch.zeros(shape, dtype=torch.float8_e4m3fn)
            self.kv_scales = torch.full((2, hf.num_hidden_layers, hk), float(config.kv_cache_scale),
                                        dtype=torch.float32)
        else:
            self.kv_cache = torch.zeros(shape, dtype=torch.bfloat16)
        for layer_id, module in enumerate(layers):
            module.kv_cache_dtype = config.kv_cache_dtype
            if self.use_fp8_kv_cache:
                module.prefill_k_cache = self.prefill_kv_cache[0, layer_id]
                module.prefill_v_cache = self.prefill_kv_cache[1, layer_id]
                module.decode_k_cache = self.decode_kv_cache[0, layer_id]
                module.decode_v_cache = self.decode_kv_cache[1, layer_id]
                module.k_cache = module.prefill_k_cache
                module.v_cache = module.prefill_v_cache
                module.k_scale = self.kv_scales[0, layer_id]
                module.v_scale = self.kv_scales[1, layer_id]
            else:
                module.k_cache = self.kv_cache[0, layer_id]
                module.v_cache = self.kv_cache[1, layer_id]

    def convert_prefill_to_decode_cache(self, seqs: list[Sequence]):
        """FP8 mode (rank 0): quantise the BF16 prefill-cache rows of every cached token of
        `seqs` into the FP8 decode cache on all ranks, all layers in one launch
        (model_runner.py:483-502).

        Departure from the reference, on purpose: it copies positions [0, num_prompt_tokens)
        (model_runner.py:488-491), which after a preemption misses the completion tokens that
        the re-prefill recomputed into the BF16 cache; here every position whose KV the prefill
        wrote, [0, num_computed_tokens), is copied (identical for sequences never preempted)."""
        if not self.use_fp8_kv_cache or not seqs:
            return
        bs = self.block_size
        slots = []
        for seq in seqs:
            table = np.asarray(seq.block_table, dtype=np.int64)
            pos = np.arange(seq.num_computed_tokens, dtype=np.int64)
            slots.append(table[pos // bs] * bs + pos % bs)
        self.call("copy_to_decode_cache", np.concatenate(slots).astype(np.int32))

    @torch.inference_mode()
    def copy_to_decode_cache(self, slots: np.ndarray):
        slot_mapping = torch.from_numpy(slots).pin_memory().to(self.device, non_blocking=True)
        kernels.copy_kvcache_fp8_layers(self.prefill_kv_cache[0], self.prefill_kv_cache[1],
                                        self.decode_kv_cache[0], self.decode_kv_cache[1], slot_mapping,
                                        self.kv_scales[0], self.kv_scales[1])

    @torch.inference_mode()
    def allocate_decode_runtime_buffers(self):
        hf = self.config.hf_config
        self.max_bs = max_bs = self.config.max_num_seqs
        mb = self.max_num_decode_blocks
        dev = self.device
        # Persistent decode buffers: read by the captured graphs, written by the pack kernel.
        self.graph_vars = dict(
            input_ids=torch.zeros(max_bs, dtype=torch.int64, device=dev),
            positions=torch.zeros(max_bs, dtype=torch.int64, device=dev),
            slot_mapping=torch.full((max_bs,), -1, dtype=torch.int32, device=dev),
            context_lens=torch.zeros(max_bs, dtype=torch.int32, device=dev),
            block_tables=torch.full((max_bs, mb), -1, dtype=torch.int32, device=dev),
            next_tokens=torch.zeros(max_bs, dtype=torch.int64, device=dev),
            slot_seq_ids=torch.full((max_bs,), -1, dtype=torch.int64, device=dev),
            slot_bt_lens=torch.zeros(max_bs, dtype=torch.int32, device=dev),
        )
        cap = packet_capacity_bytes(max_bs, mb)
        cap = (cap + 15) & ~15
        self.packet_dev = torch.zeros(cap, dtype=torch.uint8, device=dev)
        # Two pinned packet and token buffers: an overlapped decode step (launch_decode) uses one
        # while the previous step's copies may still be pending on the other.
        self.packet_bufs = [torch.zeros(cap, dtype=torch.uint8, device="cpu", pin_memory=True) for _ in range(2)]
        self.tokens_bufs = [torch.zeros(max_bs, dtype=torch.int64, device="cpu", pin_memory=True) for _ in range(2)]
        self.done_events = [torch.cuda.Event(), torch.cuda.Event()]
        self.launch_parity = 0
        self.packet_host = self.packet_bufs[0]
        self.tokens_host = self.tokens_bufs[0]
        self.packer = DecodePacker(max_bs, mb, self.packet_host.numpy())
        self.copy_done = self.done_events[0]
        hq = hf.num_attention_heads // self.world_size
        d = getattr(hf, "head_dim", None) or hf.hidden_size // hf.num_attention_heads
        self.decode_workspace = kernels.make_decode_workspace(max_bs, hq, d, mb, self.block_size, dev)
        # Device sampler: per-slot [temperature (0 = greedy); top_k (int32 bits, 0 = none); top_p],
        # noise seed and launch counter.  samp_host mirrors what the device holds.
        self.graph_vars["samp"] = torch.zeros(3, max_bs, dtype=torch.float32, device=dev)
        self.graph_vars["samp"][2].fill_(1.0)
        self.graph_vars["temps"] = self.graph_vars["samp"][0]
        self.samp_bufs = [torch.zeros(3, max_bs, dtype=torch.float32, device="cpu", pin_memory=True) for _ in range(2)]
        self.samp_host = np.zeros((3, max_bs), np.float32)
        self.samp_host[2] = 1.0
        self.device_filters = self.world_size == 1  # top-k / top-p need the whole vocabulary
        self.sample_seed = (int(getattr(self.config, "seed", 0)) * 0x9E3779B1 + 0x5EED) & 0xFFFFFFFFFFFFFFFF
        self.sample_state = torch.zeros(2, dtype=torch.int64, device=dev)
        self.prefill_sample_state = torch.zeros(2, dtype=torch.int64, device=dev)  # rank 0's prefill rows
        # Per-rank greedy reduction buffers (tensor parallelism).
        tp = self.world_size
        self.tp_idx = torch.zeros(max_bs, dtype=torch.int64, device=dev)
        self.tp_val = torch.zeros(max_bs, dtype=torch.float32, device=dev)
        self.tp_all_idx = torch.zeros(tp, max_bs, dtype=torch.int64, device=dev)
        self.tp_all_val = torch.zeros(tp, max_bs, dtype=torch.float32, device=dev)
        for module in self.attention_layers():
            module.decode_workspace = self.decode_workspace
        self.logits_buf = None
        # Error words of the attention kernels (decode: word 0 of its workspace, prefill: the
        # library's device word), copied to the host with each step's tokens and checked after
        # the step's synchronisation: a bounded wait that gave up or a block id outside the pool
        # leaves output rows unwritten, so the step must not return tokens.
        self.err_bufs = [torch.zeros(2, dtype=torch.int32, device="cpu", pin_memory=True) for _ in range(2)]
        self.decode_err_word = self.decode_workspace[:4].view(torch.int32)

    # ------------------------------------------------------------------ batch preparation
    def prepare_prefill(self, seqs: list[ScheduledSequence]):
        """Varlen metadata for the scheduled prefill chunks (model_runner.py:614-650)."""
        return self._upload_prefill(prefill_metadata(seqs, self.block_size))

    def _upload_prefill(self, meta: dict):
        dev = self.device

        def h2d(arr):
            self.io_bytes["h2d"] += arr.nbytes
            return torch.from_numpy(arr).pin_memory().to(dev, non_blocking=True)

        input_ids = h2d(meta["input_ids"])
        positions = h2d(meta["positions"])
        bt = meta["block_tables"]
        set_context(True, h2d(meta["cu_seqlens_q"]), h2d(meta["cu_seqlens_k"]), meta["max_seqlen_q"],
                    meta["max_seqlen_k"], h2d(meta["slot_mapping"]), None, None if bt is None else h2d(bt))
        return input_ids, positions

    def _decode_graph_batch_size(self, bs: int) -> int:
        if self.enforce_eager or bs > MAX_GRAPH_BS:
            return bs
        return next(g for g in self.graph_bs if g >= bs)

    def _set_decode_context(self, n: int):
        gv = self.graph_vars
        set_context(False, slot_mapping=gv["slot_mapping"][:n], context_lens=gv["context_lens"][:n],
                    block_tables=gv["block_tables"][:n])

    def _decode_body(self, n: int, greedy: bool):
        """Pack kernel + model + LM head (+ the device sampler) over the first n decode slots;
        greedy=False leaves the logits for the host sampler."""
        gv = self.graph_vars
        kernels.pack_decode_batch(self.packet_dev, n, self.block_size, gv["slot_seq_ids"], gv["slot_bt_lens"],
                                  gv["next_tokens"], gv["input_ids"], gv["positions"], gv["slot_mapping"],
                                  gv["context_lens"], gv["block_tables"])
        self._set_decode_context(n)
        hidden = self.model(gv["input_ids"][:n], gv["positions"][:n])
        logits = self.logits_buf[:n]
        torch.matmul(hidden, self.model.lm_head.weight.t(), out=logits)
        if greedy:
            self._device_tokens(logits, gv["next_tokens"][:n])
        return logits

    def _device_tokens(self, logits: torch.Tensor, out: torch.Tensor):
        """Token per row into `out` (device), on every rank: the greedy argmax, or for rows with a
        temperature in graph_vars["temps"] a Gumbel-max sample (hl_sample).  Under tensor
        parallelism each rank reduces its vocabulary shard to (max, index) — the noise is a
        function of the global index, so the shards draw disjoint parts of one noise field —
        and the ranks all-gather those pairs (2 x 12 bytes per row instead of the logits); the
        lowest rank wins ties, which is the lowest global index because shards are ordered."""
        n = logits.shape[0]
        temps = self.graph_vars["temps"][:n]
        if self.world_size == 1:
            samp = self.graph_vars["samp"]
            kernels.sample_filtered(logits, temps, samp[1].view(torch.int32)[:n], samp[2][:n], self.sample_seed,
                                    self.sample_state, out=out)
            return
        head = self.model.lm_head
        idx = self.tp_idx[:n]
        val = self.tp_val[:n]
        kernels.sample(logits, temps, self.sample_seed, self.sample_state, out=idx, index_offset=head.vocab_start_idx,
                       out_values=val)
        all_val = self.tp_all_val.view(-1)[: self.world_size * n].view(self.world_size, n)
        all_idx = self.tp_all_idx.view(-1)[: self.world_size * n].view(self.world_size, n)
        dist.all_gather_into_tensor(all_val, val)
        dist.all_gather_into_tensor(all_idx, idx)
        out.copy_(merge_shard_argmax(all_val, all_idx))

    def _ensure_logits_buf(self, rows: int):
        vocab_local = self.model.lm_head.num_embeddings_per_partition
        if self.logits_buf is None or self.logits_buf.shape[0] < rows:
            self.logits_buf = torch.zeros(rows, vocab_local, dtype=torch.bfloat16, device=self.device)

    # ------------------------------------------------------------------ running
    # Rank 0 turns the scheduler's decision into small arrays — the prefill metadata, or the
    # decode packet — plus the sampling settings, and only those cross to the other ranks
    # (the reference pickles every scheduled Sequence to every rank each step,
    # model_runner.py:117-124); every rank then executes the same step.
    @torch.inference_mode()
    def run(self, scheduled_seqs: list[ScheduledSequence], is_prefill: bool) -> list[int | None]:
        if is_prefill:
            meta = prefill_metadata(scheduled_seqs, self.block_size)
            rows = [i for i, s in enumerate(scheduled_seqs) if s.requires_sampling]
            samp = sampling_settings([scheduled_seqs[i].seq for i in rows])
            return self.call("execute_prefill", meta, len(scheduled_seqs), rows, samp)
        bs = len(scheduled_seqs)
        graph_bs = self._decode_graph_batch_size(bs)
        self.packer.buffer = self.packet_host.numpy()
        nbytes = self.packer.build(scheduled_seqs, graph_bs)
        real = [i for i, s in enumerate(scheduled_seqs) if not s.is_padding]
        temps = decode_sampling(scheduled_seqs, self.device_filters)
        samp = None if temps is not None else sampling_settings([scheduled_seqs[i].seq for i in real])
        temps = self._temps_change(temps, graph_bs)
        self.last_decode_batch_info = {"scheduled_bs": bs, "graph_bs": graph_bs, "active_seqs": len(real),
                                       "padded_slots": bs - len(real), "pack_events": self.packer.last_num_events}
        packet = self.packet_host[:nbytes].numpy()
        tokens = self.call("execute_decode", packet, bs, graph_bs, real, samp, temps)
        self.packer.note_sampled(bs, tokens)
        out: list[int | None] = [None] * bs
        for i in real:
            out[i] = tokens[i]
        return out

    def _temps_change(self, samp: np.ndarray | None, graph_bs: int) -> np.ndarray | None:
        """The [3, max_bs] sampler settings to upload this step (slots [0, graph_bs) from `samp`,
        padding slots greedy and unfiltered), or None if the device already holds them."""
        if samp is None:
            return None
        full = self.samp_host.copy()
        full[:, :graph_bs] = 0.0
        full[2, :graph_bs] = 1.0
        full[:, : samp.shape[1]] = samp
        if np.array_equal(full.view(np.uint32), self.samp_host.view(np.uint32)):
            return None
        self.samp_host[:] = full
        return full

    def _upload_temps(self, samp: np.ndarray | None, par: int) -> None:
        """Copies a whole settings block (what _temps_change returned) to the device; the other
        ranks receive it with the step and keep their own mirror."""
        if samp is None:
            return
        self.samp_bufs[par].numpy()[:] = samp
        self.graph_vars["samp"].copy_(self.samp_bufs[par], non_blocking=True)
        self.samp_host[:] = samp

    # ------------------------------------------------------------------ overlapped decode
    # A greedy decode step launched without waiting for its tokens: the argmax leaves them in
    # next_tokens on the device (where the next step's pack kernel reads them) and one
    # asynchronous device->host copy brings them to a pinned buffer that collect_decode() reads
    # after the next step has been launched.
    def samples_on_device(self, seq) -> bool:
        return device_sampleable(seq, self.device_filters)

    def can_launch_decode(self, scheduled_seqs) -> bool:
        return (decode_sampling(scheduled_seqs, self.device_filters) is not None
                and not self.packer.needs_host_tokens(scheduled_seqs))

    @torch.inference_mode()
    def launch_decode(self, scheduled_seqs: list[ScheduledSequence]):
        bs = len(scheduled_seqs)
        graph_bs = self._decode_graph_batch_size(bs)
        par = self.launch_parity
        self.launch_parity ^= 1
        self.packer.buffer = self.packet_bufs[par].numpy()
        nbytes = self.packer.build(scheduled_seqs, graph_bs)
        temps = self._temps_change(decode_sampling(scheduled_seqs, self.device_filters), graph_bs)
        real = sum(1 for s in scheduled_seqs if not s.is_padding)
        self.last_decode_batch_info = {"scheduled_bs": bs, "graph_bs": graph_bs, "active_seqs": real,
                                       "padded_slots": bs - real, "pack_events": self.packer.last_num_events}
        self.call("execute_decode_launch", self.packet_bufs[par][:nbytes].numpy(), bs, graph_bs, par, temps)
        self.packer.note_launched(bs, scheduled_seqs)
        return par, bs

    @torch.inference_mode()
    def execute_decode_launch(self, packet: np.ndarray, bs: int, graph_bs: int, par: int, temps=None):
        self._upload_temps(temps, par)
        nbytes = packet.nbytes
        host = self.packet_bufs[par].numpy()
        if packet.ctypes.data != host.ctypes.data:
            host[:nbytes] = packet
        self.packet_dev[:nbytes].copy_(self.packet_bufs[par][:nbytes], non_blocking=True)
        self.io_bytes["h2d"] += nbytes
        if self.recording is not None:
            self.recording.append(self.packet_dev[:nbytes].clone())
        if graph_bs in self.graphs:
            self.graphs[graph_bs].replay()
        else:
            self._ensure_logits_buf(graph_bs)
            self._decode_body(graph_bs, greedy=True)
        self.tokens_bufs[par][:bs].copy_(self.graph_vars["next_tokens"][:bs], non_blocking=True)
        self.io_bytes["d2h"] += 8 * bs
        if self.allreduce is not None:
            self.allreduce.copy_error_word()
        self._queue_error_words(par)
        self.done_events[par].record()
        reset_context()

    def collect_decode(self, handle) -> list[int]:
        par, bs = handle
        t0 = time.perf_counter()
        self.done_events[par].synchronize()
        self.gpu_wait_s += time.perf_counter() - t0
        if self.allreduce is not None:
            self.allreduce.check_errors()
        self._check_error_words(par)
        return self.tokens_bufs[par][:bs].tolist()

    def _queue_error_words(self, par: int) -> None:
        """Queues device->host copies of the decode and prefill error words on the current stream."""
        buf = self.err_bufs[par]
        buf[0:1].copy_(self.decode_err_word, non_blocking=True)
        kernels.copy_prefill_errors_async(buf[1:2])

    def _check_error_words(self, par: int) -> None:
        """Raises if an attention kernel recorded an error (after _queue_error_words and a sync)."""
        dec, pre = (int(x) for x in self.err_bufs[par].tolist())
        if dec or pre:
            what = []
            if (dec | pre) & 1:
                what.append("a bounded wait for a tile copy timed out")
            if (dec | pre) & 2:
                what.append("a block table entry was outside the KV pool")
            raise RuntimeError(f"attention kernel error on rank {self.rank} (decode word {dec}, prefill word {pre}): "
                               + "; ".join(what) + "; outputs of that step are invalid")

    def _sample_rows(self, logits: torch.Tensor, samp) -> list[int]:
        """Tokens for rows of full-vocabulary logits (rank 0): greedy argmax, or a device draw with
        the request's temperature, top-k and top-p (hl_sample_filtered)."""
        if samp is None:
            return kernels.argmax(logits).tolist()
        temps, ks, ps, greedy = samp
        dev = self.device
        t = torch.tensor([0.0 if g else x for g, x in zip(greedy, temps)], dtype=torch.float32, device=dev)
        k = torch.tensor([0 if g else max(int(x), 0) for g, x in zip(greedy, ks)], dtype=torch.int32, device=dev)
        p = torch.tensor([1.0 if g else x for g, x in zip(greedy, ps)], dtype=torch.float32, device=dev)
        return kernels.sample_filtered(logits, t, k, p, self.sample_seed ^ 0xA5A5, self.prefill_sample_state).tolist()

    def _gather_logits(self, logits: torch.Tensor) -> torch.Tensor | None:
        if self.world_size == 1:
            return logits
        parts = [torch.empty_like(logits) for _ in range(self.world_size)] if self.rank == 0 else None
        dist.gather(logits, parts, 0)
        return torch.cat(parts, -1) if self.rank == 0 else None

    @torch.inference_mode()
    def execute_prefill(self, meta: dict, n_sched: int, rows: list[int], samp):
        input_ids, positions = self._upload_prefill(meta)
        hidden = self.model(input_ids, positions)
        logits = self._gather_logits(self.model.lm_head.local_logits(hidden))
        token_ids = None
        if self.rank == 0:
            token_ids = [None] * n_sched
            if rows:
                self._queue_error_words(0)
                sub = logits[rows] if len(rows) != logits.shape[0] else logits
                for i, t in zip(rows, self._sample_rows(sub.contiguous(), samp)):  # synchronises
                    token_ids[i] = t
                self._check_error_words(0)
        reset_context()
        return token_ids

    def score(self, scheduled_seqs: list[ScheduledSequence], targets: list[int]) -> list[dict]:
        """One prefill pass over whole sequences; per sequence the greedy token, the top logit and
        the target token's logit at the last position (LLMEngine.score_next_tokens)."""
        meta = prefill_metadata(scheduled_seqs, self.block_size)
        return self.call("execute_score", meta, list(targets))

    @torch.inference_mode()
    def execute_score(self, meta: dict, targets: list[int]):
        input_ids, positions = self._upload_prefill(meta)
        hidden = self.model(input_ids, positions)
        logits = self._gather_logits(self.model.lm_head.local_logits(hidden))
        res = None
        if self.rank == 0:
            logits = logits.float()
            top, arg = logits.max(-1)
            tgt = logits.gather(1, torch.tensor(targets, dtype=torch.int64, device=logits.device).view(-1, 1))
            self._queue_error_words(0)
            res = [{"argmax": int(a), "top_logit": float(t), "target_logit": float(x)}
                   for a, t, x in zip(kernels.argmax(logits.bfloat16()).tolist(), top.tolist(), tgt.view(-1).tolist())]
            self._check_error_words(0)
        reset_context()
        return res

    @torch.inference_mode()
    def execute_decode(self, packet: np.ndarray, bs: int, graph_bs: int, real: list[int], samp, temps=None):
        self._upload_temps(temps, 0)
        nbytes = packet.nbytes
        host = self.packet_host.numpy()
        if packet.ctypes.data != host.ctypes.data:
            host[:nbytes] = packet
        self.packet_dev[:nbytes].copy_(self.packet_host[:nbytes], non_blocking=True)
        self.io_bytes["h2d"] += nbytes
        if self.recording is not None:
            self.recording.append(self.packet_dev[:nbytes].clone())
        gv = self.graph_vars
        if samp is None:
            # Greedy: tokens are picked on the device (inside the graph when there is one) on
            # every rank, so nothing but the packet crossed the host.
            if graph_bs in self.graphs:
                self.graphs[graph_bs].replay()
            else:
                self._ensure_logits_buf(graph_bs)
                self._decode_body(graph_bs, greedy=True)
        else:
            if graph_bs in self.graphs:
                self.graphs[graph_bs].replay()
                logits = self.logits_buf[:graph_bs]
            else:
                self._ensure_logits_buf(graph_bs)
                logits = self._decode_body(graph_bs, greedy=False)
            logits = self._gather_logits(logits)
            if self.rank == 0 and real:
                sampled = torch.tensor(self._sample_rows(logits[real].contiguous(), samp), dtype=torch.int64)
                toks = torch.zeros(bs, dtype=torch.int64)
                toks[real] = sampled
                gv["next_tokens"][:bs].copy_(toks.pin_memory(), non_blocking=True)
            if self.world_size > 1:
                dist.broadcast(gv["next_tokens"][:bs], 0)
        # One device->host copy of the step's tokens (and, under TP, of the all-reduce's error word).
        self.tokens_host[:bs].copy_(gv["next_tokens"][:bs], non_blocking=True)
        self.io_bytes["d2h"] += 8 * bs
        if self.allreduce is not None:
            self.allreduce.copy_error_word()
        self._queue_error_words(0)
        self.copy_done.record()
        t0 = time.perf_counter()
        self.copy_done.synchronize()
        self.gpu_wait_s += time.perf_counter() - t0
        if self.allreduce is not None:
            self.allreduce.check_errors()
        self._check_error_words(0)
        reset_context()
        return self.tokens_host[:bs].tolist()

    @torch.inference_mode()
    def capture_cudagraph(self):
        self.graph_bs = graph_batch_sizes(self.config.max_num_seqs)
        greedy = True
        self._ensure_logits_buf(self.graph_bs[-1])
        # The packet is all zeros during capture: batch 0, every slot padding.
        self.packet_dev.zero_()
        for bs in reversed(self.graph_bs):
            graph = torch.cuda.CUDAGraph()
            self._decode_body(bs, greedy)  # warm-up outside the graph
            torch.cuda.synchronize()
            with torch.cuda.graph(graph, self.graph_pool):
                self._decode_body(bs, greedy)
            if self.graph_pool is None:
                self.graph_pool = graph.pool()
            self.graphs[bs] = graph
            torch.cuda.synchronize()
            reset_context()
        # Capture ran the pack kernel on an empty packet: reset the device-side slot state.
        gv = self.graph_vars
        gv["slot_seq_ids"].fill_(-1)
        gv["slot_bt_lens"].zero_()
        gv["block_tables"].fill_(-1)
        gv["context_lens"].zero_()
        gv["slot_mapping"].fill_(-1)
        self.packer.forget_tokens()
        torch.cuda.synchronize()

    # ------------------------------------------------------------------ benchmarking support
    def record_packets(self, enable: bool):
        """Start (or stop) keeping a device copy of every decode packet sent."""
        self.recording = [] if enable else None

    def take_recording(self) -> list[torch.Tensor]:
        rec, self.recording = self.recording or [], None
        self.recorded_packets = rec
        return rec

    @torch.inference_mode()
    def reset_decode_state(self):
        """Forget every decode slot (device buffers and the host mirror)."""
        gv = self.graph_vars
        gv["slot_seq_ids"].fill_(-1)
        gv["slot_bt_lens"].zero_()
        gv["block_tables"].fill_(-1)
        gv["context_lens"].zero_()
        gv["slot_mapping"].fill_(-1)
        gv["positions"].zero_()
        gv["samp"].zero_()
        gv["samp"][2].fill_(1.0)
        self.samp_host[:] = 0.0
        self.samp_host[2] = 1.0
        self.packer = DecodePacker(self.max_bs, self.max_num_decode_blocks, self.packet_host.numpy())

    @torch.inference_mode()
    def replay_recorded(self, bs: int, probe_every: int = 0):
        """Replays the recorded decode packets back to back on the device (each: a device-to-
        device packet copy + one graph replay, tokens fed back through next_tokens).  Returns
        the elapsed seconds measured with CUDA events on the launching stream, and, when
        probe_every > 0, (algorithmic bytes, seconds) samples of the layer-0 decode kernel timed
        on its own between steps."""
        graph = self.graphs[self._decode_graph_batch_size(bs)]
        stream = torch.cuda.current_stream()
        samples = []
        if self.world_size > 1:
            dist.barrier()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for i, pkt in enumerate(self.recorded_packets):
            self.packet_dev[: pkt.numel()].copy_(pkt, non_blocking=True)
            graph.replay()
            if probe_every and i % probe_every == probe_every // 2:
                samples.append(self._probe_decode(bs))
        end.record(stream)
        torch.cuda.synchronize()
        elapsed = start.elapsed_time(end) / 1e3
        if self.world_size > 1:  # the job is as slow as its slowest rank
            t = torch.tensor([elapsed], device=self.device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            elapsed = float(t.item())
        return elapsed, samples

    def _probe_decode(self, bs: int):
        hf = self.config.hf_config
        hq = hf.num_attention_heads // self.world_size
        hk = hf.num_key_value_heads // self.world_size
        d = getattr(hf, "head_dim", None) or hf.hidden_size // hf.num_attention_heads
        layer = self.attention_layers()[0]
        gv = self.graph_vars
        q = torch.randn(bs, hq, d, dtype=torch.bfloat16, device=self.device)
        out = torch.empty_like(q)
        ctx, bt = gv["context_lens"][:bs], gv["block_tables"][:bs]
        k_cache = layer.decode_k_cache if self.use_fp8_kv_cache else layer.k_cache
        v_cache = layer.decode_v_cache if self.use_fp8_kv_cache else layer.v_cache
        elem = 1 if self.use_fp8_kv_cache else 2

        def launch():
            kernels.paged_decode(q, k_cache, v_cache, bt, ctx, layer.scale, out=out, workspace=self.decode_workspace,
                                 k_scale=layer.k_scale, v_scale=layer.v_scale)

        for _ in range(3):
            launch()
        reps = 20
        # The launches replay from a CUDA graph, as in a decode step: issued from Python one by
        # one, a launch of a few tens of microseconds (one GPU's heads under tensor parallelism)
        # would be timed at the host's issue rate instead.
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(reps):
                launch()
        graph.replay()
        stream = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        # Nothing in flight before the start event: the decode kernel is a programmatic dependent
        # launch and would otherwise begin under the previous launch's tail.
        torch.cuda.synchronize()
        e0.record(stream)
        graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        del graph
        lens = ctx.tolist()
        nbytes = sum(lens) * hk * d * elem * 2 + bs * hq * d * 2 * 2
        return nbytes, e0.elapsed_time(e1) / 1e3 / reps
