"""Engine configuration: the fields and checks of mini_vllm/config.py:6-45, plus a few
options this build adds (marked below).  Speculative decoding is outside this build's scope,
so a non-empty ``spec_decode_model`` is rejected."""
import os
from dataclasses import dataclass

from transformers import AutoConfig


@dataclass
class Config:
    model: str
    max_num_batched_tokens: int = 16384
    max_num_seqs: int = 512
    max_model_len: int = 4096
    enable_chunked_prefill: bool = True
    chunked_prefill_size: int = 512
    chunked_prefill_min_size: int = 128
    chunked_prefill_tile_size: int = 128
    gpu_memory_utilization: float = 0.9
    tensor_parallel_size: int = 1
    enforce_eager: bool = False
    hf_config: AutoConfig | None = None
    eos: int = -1
    kvcache_block_size: int = 256
    num_kvcache_blocks: int = -1
    kv_cache_dtype: str = "auto"
    spec_decode_model: str = ""
    spec_decode_gamma: int = 5
    spec_decode_max_batch_size: int = 16
    # --- added by this build ---
    # "auto": load *.safetensors from `model` when present, else seeded random init;
    # "random": always seeded random init (Linear/Embedding N(0, init_std), norms = 1).
    load_format: str = "auto"
    seed: int = 0
    init_std: float = 0.02
    # Upper bound on the KV pool (blocks); -1 = size the pool from free memory only.
    kvcache_block_cap: int = -1
    # Per-KV-head FP8 scale used for every layer (1.0 reproduces the reference's unscaled store).
    kv_cache_scale: float = 1.0
    # "spawn": rank 0 starts ranks 1..tp-1 itself (the reference's way, shared-memory RPC);
    # "external": every rank is already running (torchrun) and calls LLM(...) itself; rank 0
    # drives, the others serve the model-runner loop inside the constructor (calls through a
    # polled shared-memory segment whose name crosses once over gloo).
    distributed_executor: str = "spawn"
    # Tensor parallelism: reduce decode-sized o_proj / down_proj outputs with the fused NVLink
    # all-reduce + add + RMSNorm kernel (False: NCCL all-reduce as the reference does).
    custom_allreduce: bool = True
    # Overlap the host side of decode step k+1 with the GPU running step k while no running
    # sequence can stop on EOS (see LLMEngine.step); False runs every step synchronously.
    async_decode: bool = True
    # The reference appends a padding row's token to a sequence preempted as a victim after it
    # was put in the same decode batch (scheduler.py:326-340); True drops that token instead
    # (correct outputs; block decisions then differ from the reference in that case).
    drop_preempted_decode_token: bool = False
    # When nothing can run because the head of the waiting queue cannot get its blocks, let
    # chunked prefills further back that already hold blocks proceed (the reference raises
    # "no runnable prefill or decode work" there); False reproduces the reference.
    unblock_prefill_head: bool = True

    def __post_init__(self):
        assert os.path.isdir(self.model)
        assert self.chunked_prefill_size > 0
        assert self.chunked_prefill_min_size > 0
        assert self.chunked_prefill_tile_size > 0
        assert self.chunked_prefill_min_size <= self.chunked_prefill_size
        assert self.kvcache_block_size % 256 == 0
        assert 1 <= self.tensor_parallel_size <= 8
        assert self.kv_cache_dtype in {"auto", "fp8"}
        assert self.spec_decode_gamma >= 1
        assert self.load_format in {"auto", "random"}
        assert self.kv_cache_scale > 0
        assert self.distributed_executor in {"spawn", "external"}
        if self.spec_decode_model:
            raise NotImplementedError("speculative decoding is not part of this build")
        self.hf_config = AutoConfig.from_pretrained(self.model)
        self.max_model_len = min(self.max_model_len, self.hf_config.max_position_embeddings)
        assert self.max_num_batched_tokens >= self.max_model_len
        self.draft_hf_config = None
