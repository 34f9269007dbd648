"""hilda_vllm_b200: B200 (sm_100a) continuous-batching paged-attention engine with the
mini_vllm API (LLM, SamplingParams).  The attention hot path runs on hand-written CUDA
kernels behind the C ABI in include/hilda_b200.h (libhilda_b200.so, built in-tree)."""
from hilda_vllm_b200.sampling_params import SamplingParams


def __getattr__(name):
    # LLM pulls in torch.distributed and the model runner; import it on first use.
    if name == "LLM":
        from hilda_vllm_b200.llm import LLM
        return LLM
    raise AttributeError(name)


__all__ = ["LLM", "SamplingParams"]
