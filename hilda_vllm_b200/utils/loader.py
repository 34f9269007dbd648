"""Weight loading: safetensors checkpoints (mini_vllm/utils/loader.py:12-28 mapping rules) or a
seeded random initialisation that goes through the same per-parameter weight loaders, so a
tensor-parallel rank holds exactly its shard of the single-GPU model's weights."""
import os
import zlib
from glob import glob

import torch
from torch import nn


def default_weight_loader(param: nn.Parameter, loaded_weight: torch.Tensor):
    param.data.copy_(loaded_weight)


def _dispatch(model: nn.Module, weight_name: str, tensor: torch.Tensor) -> None:
    mapping = getattr(model, "packed_modules_mapping", {})
    for key, (target, shard_id) in mapping.items():
        if key in weight_name:
            param = model.get_parameter(weight_name.replace(key, target))
            param.weight_loader(param, tensor, shard_id)
            return
    param = model.get_parameter(weight_name)
    getattr(param, "weight_loader", default_weight_loader)(param, tensor)


def has_checkpoint(path: str) -> bool:
    return bool(glob(os.path.join(path, "*.safetensors")))


def load_model(model: nn.Module, path: str) -> None:
    from safetensors import safe_open

    tied = getattr(model, "tie_word_embeddings", False)
    for file in sorted(glob(os.path.join(path, "*.safetensors"))):
        with safe_open(file, "pt", "cpu") as f:
            for name in f.keys():
                if tied and name.startswith("lm_head."):
                    continue
                _dispatch(model, name, f.get_tensor(name))
    if tied and hasattr(model, "tie_weights"):
        model.tie_weights()


def checkpoint_tensor_shapes(hf_config) -> list[tuple[str, tuple[int, ...], bool]]:
    """(name, full shape, is_norm) of every tensor of a Hugging Face Qwen3 checkpoint."""
    h = hf_config.hidden_size
    hq = hf_config.num_attention_heads
    hk = hf_config.num_key_value_heads
    d = getattr(hf_config, "head_dim", None) or h // hq
    inter = hf_config.intermediate_size
    vocab = hf_config.vocab_size
    out = [("model.embed_tokens.weight", (vocab, h), False)]
    for i in range(hf_config.num_hidden_layers):
        p = f"model.layers.{i}."
        out += [
            (p + "input_layernorm.weight", (h,), True),
            (p + "self_attn.q_proj.weight", (hq * d, h), False),
            (p + "self_attn.k_proj.weight", (hk * d, h), False),
            (p + "self_attn.v_proj.weight", (hk * d, h), False),
            (p + "self_attn.q_norm.weight", (d,), True),
            (p + "self_attn.k_norm.weight", (d,), True),
            (p + "self_attn.o_proj.weight", (h, hq * d), False),
            (p + "post_attention_layernorm.weight", (h,), True),
            (p + "mlp.gate_proj.weight", (inter, h), False),
            (p + "mlp.up_proj.weight", (inter, h), False),
            (p + "mlp.down_proj.weight", (h, inter), False),
        ]
    out.append(("model.norm.weight", (h,), True))
    if not getattr(hf_config, "tie_word_embeddings", False):
        out.append(("lm_head.weight", (vocab, h), False))
    return out


def random_weights(hf_config, seed: int = 0, std: float = 0.02, device="cpu", dtype=torch.bfloat16):
    """Yields (checkpoint name, full tensor) of the seeded random initialisation:
    Linear/Embedding ~ N(0, std) drawn in fp32 and rounded to `dtype`, RMSNorm gains = 1.
    Each tensor has its own generator seeded from (seed, crc32(name)), so the values do not
    depend on the order of loading or on the tensor-parallel layout."""
    for name, shape, is_norm in checkpoint_tensor_shapes(hf_config):
        if is_norm:
            yield name, torch.ones(shape, dtype=dtype, device=device)
            continue
        g = torch.Generator(device=device)
        g.manual_seed((seed * 1_000_003 + zlib.crc32(name.encode())) & 0x7FFF_FFFF_FFFF_FFFF)
        yield name, (torch.randn(shape, generator=g, device=device, dtype=torch.float32) * std).to(dtype)


def random_init(model: nn.Module, hf_config, seed: int = 0, std: float = 0.02, device=None) -> None:
    """Loads random_weights() into `model` through its weight loaders (so each tensor-parallel
    rank keeps its shard of the single-GPU weights)."""
    device = device or next(model.parameters()).device
    dtype = next(model.parameters()).dtype
    for name, tensor in random_weights(hf_config, seed, std, device, dtype):
        _dispatch(model, name, tensor)
        del tensor
    if getattr(model, "tie_word_embeddings", False) and hasattr(model, "tie_weights"):
        model.tie_weights()
