"""KV store restatements (TEST ORACLE ONLY).

store_kvcache: mini_vllm/layers/attention.py:59-90 — for every token i whose slot is not -1,
the num_kv_heads*head_dim contiguous elements of key[i] / value[i] land in row `slot` of the
cache viewed as [num_blocks*block_size, num_kv_heads*head_dim].
store_kvcache_fp8 / copy_kvcache_fp8: attention.py:51-56 (kernels not in the reference tree):
the same scatter with e4m3 quantisation round-to-nearest-even(x / scale[h]) saturated at 448.
"""
from __future__ import annotations

import numpy as np
import torch

from oracle import build as _build


def store_kvcache(key, value, k_cache, v_cache, slot_mapping):
    """In place on k_cache / v_cache (CPU tensors)."""
    n, hk, d = key.shape
    kf = k_cache.view(-1, hk * d)
    vf = v_cache.view(-1, hk * d)
    for i, slot in enumerate(slot_mapping.tolist()):
        if slot == -1:
            continue
        kf[slot] = key[i].reshape(-1)
        vf[slot] = value[i].reshape(-1)


def quantize_e4m3(x_bf16: torch.Tensor, scale: torch.Tensor | None) -> torch.Tensor:
    """[..., Hk, D] bf16 -> uint8 e4m3 bytes, per-head scale (None = 1), via the C oracle."""
    lib = _build.load()
    shape = x_bf16.shape
    hk, d = shape[-2], shape[-1]
    src = np.ascontiguousarray(x_bf16.contiguous().view(torch.int16).numpy().reshape(-1, hk * d))
    out = np.zeros(src.shape, np.uint8)
    sc = None if scale is None else np.ascontiguousarray(scale.float().numpy().astype(np.float32))
    lib.oracle_quantize_rows(src.ctypes.data, src.shape[0], hk, d, None if sc is None else sc.ctypes.data,
                             out.ctypes.data)
    return torch.from_numpy(out).reshape(shape)


def quantize_e4m3_torch(x_bf16: torch.Tensor, scale: torch.Tensor | None) -> torch.Tensor:
    """quantize_e4m3 in torch on any device: clamp(x / scale[h], -448, 448) cast to e4m3 (round to
    nearest even), as uint8 bytes.  The clamp is what saturates: a plain cast turns overflow into
    NaN.  Equal to the C restatement on every finite bf16 input (checked exhaustively on the CPU),
    so a GPU-resident oracle can quantise without a host round trip."""
    x = x_bf16.float()
    if scale is not None:
        x = x / scale.float().to(x.device).view(*([1] * (x.dim() - 2)), -1, 1)
    return torch.clamp(x, -448.0, 448.0).to(torch.float8_e4m3fn).view(torch.uint8)


def dequantize_e4m3(q_u8: torch.Tensor, scale: torch.Tensor | None) -> torch.Tensor:
    """uint8 e4m3 bytes [..., Hk, D] -> fp32 value * scale[h]."""
    x = q_u8.view(torch.float8_e4m3fn).float()
    if scale is not None:
        x = x * scale.float().view(*([1] * (x.dim() - 2)), -1, 1)
    return x


def store_kvcache_fp8(key, value, k_cache_u8, v_cache_u8, slot_mapping, k_scale=None, v_scale=None):
    """In place on uint8 caches."""
    n, hk, d = key.shape
    kq = quantize_e4m3(key, k_scale)
    vq = quantize_e4m3(value, v_scale)
    kf = k_cache_u8.view(-1, hk * d)
    vf = v_cache_u8.view(-1, hk * d)
    for i, slot in enumerate(slot_mapping.tolist()):
        if slot == -1:
            continue
        kf[slot] = kq[i].reshape(-1)
        vf[slot] = vq[i].reshape(-1)


def copy_kvcache_fp8(src_k, src_v, dst_k_u8, dst_v_u8, slot_mapping, k_scale=None, v_scale=None):
    nb, bs, hk, d = src_k.shape
    slots = torch.as_tensor(slot_mapping).long()
    slots = slots[slots >= 0]
    sk = src_k.view(-1, hk, d)[slots]
    sv = src_v.view(-1, hk, d)[slots]
    dst_k_u8.view(-1, hk, d)[slots] = quantize_e4m3(sk, k_scale)
    dst_v_u8.view(-1, hk, d)[slots] = quantize_e4m3(sv, v_scale)
