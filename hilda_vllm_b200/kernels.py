"""PyTorch-facing wrappers of the C ABI (include/hilda_b200.h).

Each wrapper validates shapes the way the reference does (mini_vllm/layers/attention.py:83-90
asserts strides), passes raw device pointers and the current CUDA stream to the library and
raises HildaKernelError on a non-zero status.  Tensors must live on a CUDA device; there is
no CPU path.  Every call only launches kernels on the current stream, so all of them can be
captured in a CUDA graph (workspaces are caller-provided or created before capture).
"""
from __future__ import annotations

import ctypes

import torch

from hilda_vllm_b200 import _lib
from hilda_vllm_b200._lib import HlPackEvent, HlPackHeader, check

KV_BF16 = 0
KV_FP8_E4M3 = 1

# Flags of hl_pack_event (include/hilda_b200.h).
EV_SCALARS = 1
EV_ROW = 2
EV_ROW_FILL = 4
EV_CLEAR = 8


def _cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("hilda_vllm_b200 kernels need CUDA tensors (there is no CPU fallback)")


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _p(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


# ----------------------------------------------------------------------------- KV store
def _check_store_args(key, value, k_cache, v_cache, slot_mapping):
    n, num_heads, head_dim = key.shape
    d = num_heads * head_dim
    assert key.stride(-1) == 1 and value.stride(-1) == 1
    assert key.stride(1) == head_dim and value.stride(1) == head_dim
    assert k_cache.stride(1) == d and v_cache.stride(1) == d
    assert slot_mapping.numel() == n
    assert slot_mapping.dtype == torch.int32 and slot_mapping.is_contiguous()
    assert key.dtype == torch.bfloat16 and value.dtype == torch.bfloat16
    _cuda(key, value, k_cache, v_cache, slot_mapping)
    return n, num_heads, head_dim


def store_kvcache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                  slot_mapping: torch.Tensor) -> None:
    """BF16 scatter of key/value [N, Hk, D] into k_cache/v_cache [NB, BS, Hk, D] by slot_mapping
    (slot -1 skipped).  Same contract as mini_vllm/layers/attention.py:83-90."""
    n, hk, hd = _check_store_args(key, value, k_cache, v_cache, slot_mapping)
    assert k_cache.dtype == torch.bfloat16 and v_cache.dtype == torch.bfloat16
    if n == 0:
        return
    num_slots = k_cache.shape[0] * k_cache.shape[1]
    lib = _lib.load()
    check(lib.hl_store_kv_bf16(key.data_ptr(), value.data_ptr(), key.stride(0), value.stride(0),
                               k_cache.data_ptr(), v_cache.data_ptr(), slot_mapping.data_ptr(), n, num_slots,
                               hk, hd, _stream(key)), "hl_store_kv_bf16")


def store_kvcache_fp8(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                      slot_mapping: torch.Tensor, k_scale: torch.Tensor | None = None,
                      v_scale: torch.Tensor | None = None) -> None:
    """BF16 -> FP8 e4m3 quantising store with per-KV-head fp32 scales (None = unit scale,
    the reference's hilda_store_kvcache_fp8 signature, attention.py:51-52)."""
    n, hk, hd = _check_store_args(key, value, k_cache, v_cache, slot_mapping)
    assert k_cache.dtype == torch.float8_e4m3fn and v_cache.dtype == torch.float8_e4m3fn
    for s in (k_scale, v_scale):
        if s is not None:
            assert s.dtype == torch.float32 and s.numel() == hk and s.is_contiguous()
    _cuda(k_scale, v_scale)
    if n == 0:
        return
    num_slots = k_cache.shape[0] * k_cache.shape[1]
    lib = _lib.load()
    check(lib.hl_store_kv_fp8(key.data_ptr(), value.data_ptr(), key.stride(0), value.stride(0),
                              k_cache.data_ptr(), v_cache.data_ptr(), slot_mapping.data_ptr(), n, num_slots,
                              hk, hd, _p(k_scale), _p(v_scale), _stream(key)), "hl_store_kv_fp8")


def copy_kvcache_fp8(src_k_cache: torch.Tensor, src_v_cache: torch.Tensor, dst_k_cache: torch.Tensor,
                     dst_v_cache: torch.Tensor, slot_mapping: torch.Tensor, k_scale: torch.Tensor | None = None,
                     v_scale: torch.Tensor | None = None) -> None:
    """One layer: dst[slot] = fp8(src[slot] / scale) for every slot in slot_mapping
    (the reference's copy_kvcache_fp8, attention.py:55-56)."""
    copy_kvcache_fp8_layers(src_k_cache.unsqueeze(0), src_v_cache.unsqueeze(0), dst_k_cache.unsqueeze(0),
                            dst_v_cache.unsqueeze(0), slot_mapping,
                            None if k_scale is None else k_scale.view(1, -1),
                            None if v_scale is None else v_scale.view(1, -1))


def copy_kvcache_fp8_layers(src_k: torch.Tensor, src_v: torch.Tensor, dst_k: torch.Tensor, dst_v: torch.Tensor,
                            slot_mapping: torch.Tensor, k_scales: torch.Tensor | None = None,
                            v_scales: torch.Tensor | None = None) -> None:
    """All layers in one launch: src_* [L, NB, BS, Hk, D] bf16, dst_* same shape e4m3,
    k_scales/v_scales [L, Hk] fp32 (or None)."""
    _cuda(src_k, src_v, dst_k, dst_v, slot_mapping, k_scales, v_scales)
    num_layers, nb, bs, hk, hd = src_k.shape
    assert src_k.dtype == torch.bfloat16 and dst_k.dtype == torch.float8_e4m3fn
    assert src_k.stride() == src_v.stride() and dst_k.stride() == dst_v.stride()
    assert src_k.stride(1) == bs * hk * hd and dst_k.stride(1) == bs * hk * hd
    assert src_k.stride()[2:] == (hk * hd, hd, 1) and dst_k.stride()[2:] == (hk * hd, hd, 1)
    assert slot_mapping.dtype == torch.int32 and slot_mapping.is_contiguous()
    scale_stride = 0
    for s in (k_scales, v_scales):
        if s is not None:
            assert s.dtype == torch.float32 and s.shape == (num_layers, hk) and s.is_contiguous()
            scale_stride = hk
    n = slot_mapping.numel()
    if n == 0:
        return
    lib = _lib.load()
    check(lib.hl_copy_kv_bf16_to_fp8(src_k.data_ptr(), src_v.data_ptr(), dst_k.data_ptr(), dst_v.data_ptr(),
                                     slot_mapping.data_ptr(), n, nb * bs, hk, hd, _p(k_scales), _p(v_scales),
                                     num_layers, src_k.stride(0), dst_k.stride(0), scale_stride,
                                     _stream(src_k)), "hl_copy_kv_bf16_to_fp8")


# ------------------------------------------------------------------------ decode attention
def decode_workspace_bytes(batch: int, num_q_heads: int, head_dim: int, max_blocks_per_seq: int,
                           block_size: int) -> int:
    n = _lib.load().hl_paged_decode_workspace_size(batch, num_q_heads, head_dim, max_blocks_per_seq, block_size)
    if n < 0:
        raise ValueError("bad decode workspace shape")
    return int(n)


def make_decode_workspace(batch: int, num_q_heads: int, head_dim: int, max_blocks_per_seq: int,
                          block_size: int, device) -> torch.Tensor:
    """Zero-filled workspace for paged_decode (its tickets must start at zero)."""
    n = decode_workspace_bytes(batch, num_q_heads, head_dim, max_blocks_per_seq, block_size)
    return torch.zeros(n, dtype=torch.uint8, device=device)


def paged_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_tables: torch.Tensor,
                 context_lens: torch.Tensor, softmax_scale: float, out: torch.Tensor | None = None,
                 workspace: torch.Tensor | None = None, k_scale: torch.Tensor | None = None,
                 v_scale: torch.Tensor | None = None, tensor_cores: bool = False) -> torch.Tensor:
    """Decode attention for one new token per sequence over the paged cache.

    q [B, Hq, D] (or [B, 1, Hq, D]) bf16; k_cache/v_cache [NB, BS, Hk, D] bf16 or e4m3;
    block_tables [B, >= max_blocks] int32; context_lens [B] int32.  Returns out [B, Hq, D].
    The semantics are flash_attn_with_kvcache's for a single causal query token
    (mini_vllm/layers/attention.py:162-170).  The library picks the kernel (the tcgen05 one for
    GQA ratios >= 4); tensor_cores=True forces the tcgen05 variant (hl_paged_decode_tc) for any
    ratio it supports."""
    if q.dim() == 4:
        assert q.shape[1] == 1
        q = q.squeeze(1)
    _cuda(q, k_cache, v_cache, block_tables, context_lens, out, workspace, k_scale, v_scale)
    b, hq, hd = q.shape
    nb, bsz, hk, hd2 = k_cache.shape
    assert hd == hd2 and q.stride(2) == 1 and q.stride(1) == hd
    assert k_cache.is_contiguous() and v_cache.is_contiguous() and v_cache.shape == k_cache.shape
    assert block_tables.dtype == torch.int32 and block_tables.stride(1) == 1 and block_tables.shape[0] >= b
    assert context_lens.dtype == torch.int32 and context_lens.is_contiguous() and context_lens.numel() >= b
    if k_cache.dtype == torch.bfloat16:
        kv_dtype = KV_BF16
    elif k_cache.dtype == torch.float8_e4m3fn:
        kv_dtype = KV_FP8_E4M3
    else:
        raise TypeError(f"unsupported cache dtype {k_cache.dtype}")
    if out is None:
        out = torch.empty(b, hq, hd, dtype=torch.bfloat16, device=q.device)
    assert out.dtype == torch.bfloat16 and out.stride(2) == 1 and out.stride(1) == hd
    if b == 0:
        return out
    max_blocks = block_tables.shape[1]
    if workspace is None:
        workspace = make_decode_workspace(b, hq, hd, max_blocks, bsz, q.device)
    lib = _lib.load()
    fn = lib.hl_paged_decode_tc if tensor_cores else lib.hl_paged_decode
    check(fn(q.data_ptr(), q.stride(0), k_cache.data_ptr(), v_cache.data_ptr(), kv_dtype,
             _p(k_scale), _p(v_scale), block_tables.data_ptr(), block_tables.stride(0),
             max_blocks, context_lens.data_ptr(), b, hq, hk, hd, bsz, nb, float(softmax_scale),
             out.data_ptr(), out.stride(0), workspace.data_ptr(), workspace.numel(),
             _stream(q)), "hl_paged_decode")
    return out


def decode_errors(workspace: torch.Tensor) -> int:
    """Error bits the decode kernel recorded in its workspace (synchronises the stream)."""
    val = ctypes.c_int32(0)
    check(_lib.load().hl_paged_decode_read_errors(workspace.data_ptr(), ctypes.addressof(val), _stream(workspace)),
          "hl_paged_decode_read_errors")
    return int(val.value)


# ------------------------------------------------------------------------ prefill attention
def varlen_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens_q: torch.Tensor,
                   cu_seqlens_k: torch.Tensor, max_seqlen_q: int, max_seqlen_k: int, softmax_scale: float,
                   block_table: torch.Tensor | None = None, out: torch.Tensor | None = None,
                   precise_p: bool = True, one_head_per_cta: bool = False) -> torch.Tensor:
    """Causal varlen attention with a bottom-right-aligned mask on the tcgen05/TMEM kernel.

    Same arguments as the reference's flash_attn_varlen_func call
    (mini_vllm/layers/attention.py:149-160): q [Tq, Hq, D]; with block_table, k/v are the paged
    caches [NB, BS, Hk, D]; without, k/v are [Tk, Hk, D].  Returns [Tq, Hq, D] bf16.
    precise_p feeds P to the P.V MMA as bf16 hi + lo terms (see hl_varlen_prefill);
    one_head_per_cta forces the one-query-head-per-CTA kernel instead of the head-pair kernel."""
    _cuda(q, k, v, cu_seqlens_q, cu_seqlens_k, block_table, out)
    tq, hq, hd = q.shape
    assert q.stride(2) == 1 and q.stride(1) == hd
    assert cu_seqlens_q.dtype == torch.int32 and cu_seqlens_k.dtype == torch.int32
    num_seqs = cu_seqlens_q.numel() - 1
    if block_table is not None:
        nb, bsz, hk, _ = k.shape
        assert k.is_contiguous() and v.is_contiguous()
        assert block_table.dtype == torch.int32 and block_table.stride(1) == 1
        bt_ptr, bt_stride, k_rs, v_rs, total_k = block_table.data_ptr(), block_table.stride(0), 0, 0, 0
    else:
        total_k, hk, _ = k.shape
        assert k.stride(2) == 1 and k.stride(1) == hd and v.stride(2) == 1 and v.stride(1) == hd
        nb, bsz = 0, 0
        bt_ptr, bt_stride, k_rs, v_rs = None, 0, k.stride(0), v.stride(0)
    if out is None:
        out = torch.empty(tq, hq, hd, dtype=torch.bfloat16, device=q.device)
    if num_seqs <= 0 or tq == 0:
        return out
    lib = _lib.load()
    check(lib.hl_varlen_prefill(q.data_ptr(), q.stride(0), tq, k.data_ptr(), v.data_ptr(), k_rs, v_rs, total_k,
                                   cu_seqlens_q.data_ptr(), cu_seqlens_k.data_ptr(), bt_ptr, bt_stride, num_seqs,
                                   int(max_seqlen_q), hq, hk, hd, bsz, nb, float(softmax_scale), out.data_ptr(),
                                   out.stride(0), (1 if precise_p else 0) | (2 if one_head_per_cta else 0),
                                   _stream(q)), "hl_varlen_prefill")
    return out


def prefill_errors() -> int:
    """Error bits of the tensor-core prefill kernel (synchronous)."""
    val = ctypes.c_int32(0)
    check(_lib.load().hl_varlen_prefill_read_errors(ctypes.addressof(val)), "hl_varlen_prefill_read_errors")
    return int(val.value)


def copy_prefill_errors_async(dst: torch.Tensor) -> None:
    """Queues a copy of the prefill kernel's error word into dst (an int32 element of pinned host
    or device memory) on the current stream."""
    assert dst.dtype == torch.int32 and dst.numel() >= 1
    check(_lib.load().hl_varlen_prefill_copy_errors_async(dst.data_ptr(), torch.cuda.current_stream().cuda_stream),
          "hl_varlen_prefill_copy_errors_async")


# ------------------------------------------------------------------------ decode packing
def pack_decode_batch(packet: torch.Tensor, graph_batch: int, block_size: int, slot_seq_ids: torch.Tensor,
                      slot_bt_lens: torch.Tensor, next_tokens: torch.Tensor, input_ids: torch.Tensor,
                      positions: torch.Tensor, slot_mapping: torch.Tensor, context_lens: torch.Tensor,
                      block_tables: torch.Tensor) -> None:
    """Rebuilds the persistent decode buffers on the device from the packet (a device uint8
    buffer: hl_pack_header, events, block-id pool; see hl_pack_decode_batch)."""
    _cuda(packet, slot_seq_ids, slot_bt_lens, next_tokens, input_ids, positions, slot_mapping, context_lens,
          block_tables)
    assert packet.dtype == torch.uint8 and packet.is_contiguous()
    assert block_tables.dtype == torch.int32 and block_tables.stride(1) == 1
    assert slot_seq_ids.dtype == torch.int64 and slot_bt_lens.dtype == torch.int32
    assert input_ids.dtype == torch.int64 and positions.dtype == torch.int64 and next_tokens.dtype == torch.int64
    assert slot_mapping.dtype == torch.int32 and context_lens.dtype == torch.int32
    lib = _lib.load()
    check(lib.hl_pack_decode_batch(packet.data_ptr(), packet.numel(), int(graph_batch), int(block_size),
                                   slot_seq_ids.data_ptr(), slot_bt_lens.data_ptr(), next_tokens.data_ptr(),
                                   input_ids.data_ptr(), positions.data_ptr(), slot_mapping.data_ptr(),
                                   context_lens.data_ptr(), block_tables.data_ptr(), block_tables.stride(0),
                                   block_tables.shape[1], _stream(block_tables)), "hl_pack_decode_batch")


PACK_EVENT_BYTES = ctypes.sizeof(HlPackEvent)
PACK_HEADER_BYTES = ctypes.sizeof(HlPackHeader)


# ------------------------------------------------------------------------ layer kernels
def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, residual: torch.Tensor | None = None,
            out: torch.Tensor | None = None):
    """RMSNorm (residual None) or add+RMSNorm updating `residual` in place; returns out or
    (out, residual) like RMSNorm.forward (mini_vllm/layers/layernorm.py:44-52)."""
    _cuda(x, weight, residual, out)
    rows, hidden = x.shape
    assert x.stride(1) == 1 and weight.is_contiguous()
    if out is None:
        out = torch.empty(rows, hidden, dtype=x.dtype, device=x.device)
    if residual is not None:
        assert residual.is_contiguous() and residual.shape == x.shape
    lib = _lib.load()
    check(lib.hl_rmsnorm(x.data_ptr(), x.stride(0), _p(residual), weight.data_ptr(), out.data_ptr(), out.stride(0),
                         rows, hidden, float(eps), _stream(x)), "hl_rmsnorm")
    return out if residual is None else (out, residual)


def qk_norm_rope(qkv: torch.Tensor, num_q_heads: int, num_kv_heads: int, head_dim: int, q_weight: torch.Tensor,
                 k_weight: torch.Tensor, cos_sin: torch.Tensor, positions: torch.Tensor, eps: float) -> None:
    """In place on qkv [T, (Hq+2Hk)*D]: per-head RMSNorm of q and k, then NeoX RoPE."""
    _cuda(qkv, q_weight, k_weight, cos_sin, positions)
    assert qkv.stride(1) == 1 and cos_sin.dtype == torch.float32 and cos_sin.is_contiguous()
    assert positions.dtype == torch.int64 and positions.is_contiguous()
    lib = _lib.load()
    check(lib.hl_qk_norm_rope(qkv.data_ptr(), qkv.stride(0), qkv.shape[0], num_q_heads, num_kv_heads, head_dim,
                              q_weight.data_ptr(), k_weight.data_ptr(), cos_sin.data_ptr(), positions.data_ptr(),
                              float(eps), _stream(qkv)), "hl_qk_norm_rope")


def qk_norm_rope_store(qkv: torch.Tensor, num_q_heads: int, num_kv_heads: int, head_dim: int,
                       q_weight: torch.Tensor, k_weight: torch.Tensor, cos_sin: torch.Tensor, positions: torch.Tensor,
                       eps: float, k_cache: torch.Tensor, v_cache: torch.Tensor, slot_mapping: torch.Tensor,
                       k_scale: torch.Tensor | None = None, v_scale: torch.Tensor | None = None,
                       k_mirror: torch.Tensor | None = None, v_mirror: torch.Tensor | None = None) -> None:
    """qk_norm_rope plus the KV-cache store of the rotated k heads and the v heads, in one
    launch.  Caches are [NB, BS, Hk, D] bf16 (store_kvcache) or float8_e4m3fn (the FP8 store,
    per-head scales optional); slot -1 skips a token.  With an FP8 store, k_mirror / v_mirror
    (bf16 caches of the same shape) receive the bf16 rows in the same launch."""
    _cuda(qkv, q_weight, k_weight, cos_sin, positions, k_cache, v_cache, slot_mapping, k_scale, v_scale, k_mirror,
          v_mirror)
    assert qkv.stride(1) == 1 and cos_sin.dtype == torch.float32 and cos_sin.is_contiguous()
    assert positions.dtype == torch.int64 and positions.is_contiguous()
    assert slot_mapping.dtype == torch.int32 and slot_mapping.is_contiguous() and slot_mapping.numel() >= qkv.shape[0]
    assert k_cache.is_contiguous() and v_cache.is_contiguous() and k_cache.shape == v_cache.shape
    assert k_cache.dtype == v_cache.dtype and k_cache.shape[-2:] == (num_kv_heads, head_dim)
    if k_cache.dtype == torch.bfloat16:
        kv_dtype = 0
    else:
        assert k_cache.dtype == torch.float8_e4m3fn
        kv_dtype = 1
    for sc in (k_scale, v_scale):
        assert sc is None or (sc.dtype == torch.float32 and sc.is_contiguous() and sc.numel() == num_kv_heads)
    num_slots = k_cache.numel() // (num_kv_heads * head_dim)
    lib = _lib.load()
    if k_mirror is None and v_mirror is None:
        check(lib.hl_qk_norm_rope_store(qkv.data_ptr(), qkv.stride(0), qkv.shape[0], num_q_heads, num_kv_heads,
                                        head_dim, q_weight.data_ptr(), k_weight.data_ptr(), cos_sin.data_ptr(),
                                        positions.data_ptr(), float(eps), k_cache.data_ptr(), v_cache.data_ptr(),
                                        kv_dtype, slot_mapping.data_ptr(), num_slots, _p(k_scale), _p(v_scale),
                                        _stream(qkv)), "hl_qk_norm_rope_store")
        return
    assert kv_dtype == 1 and k_mirror is not None and v_mirror is not None
    for m in (k_mirror, v_mirror):
        assert m.dtype == torch.bfloat16 and m.is_contiguous() and m.shape == k_cache.shape
    check(lib.hl_qk_norm_rope_store_mirrored(qkv.data_ptr(), qkv.stride(0), qkv.shape[0], num_q_heads, num_kv_heads,
                                             head_dim, q_weight.data_ptr(), k_weight.data_ptr(), cos_sin.data_ptr(),
                                             positions.data_ptr(), float(eps), k_cache.data_ptr(), v_cache.data_ptr(),
                                             kv_dtype, slot_mapping.data_ptr(), num_slots, _p(k_scale), _p(v_scale),
                                             k_mirror.data_ptr(), v_mirror.data_ptr(), _stream(qkv)),
          "hl_qk_norm_rope_store_mirrored")


def sample(logits: torch.Tensor, temperatures: torch.Tensor | None, seed: int, step_state: torch.Tensor | None,
           out: torch.Tensor | None = None, index_offset: int = 0,
           out_values: torch.Tensor | None = None) -> torch.Tensor:
    """Per row: Gumbel-max temperature sample (temperatures[row] > 0) or greedy argmax of bf16
    logits [rows, V] (hl_sample).  step_state: int64 [2] device counter advanced per launch."""
    _cuda(logits, temperatures, step_state, out, out_values)
    rows, vocab = logits.shape
    assert logits.dtype == torch.bfloat16 and logits.stride(1) == 1
    if temperatures is not None:
        assert temperatures.dtype == torch.float32 and temperatures.is_contiguous() and temperatures.numel() >= rows
    if step_state is not None:
        assert step_state.dtype == torch.int64 and step_state.numel() >= 2
    if out is None:
        out = torch.empty(rows, dtype=torch.int64, device=logits.device)
    lib = _lib.load()
    check(lib.hl_sample(logits.data_ptr(), logits.stride(0), rows, vocab, int(index_offset), _p(temperatures),
                        int(seed) & 0xFFFFFFFFFFFFFFFF, _p(step_state), out.data_ptr(), _p(out_values),
                        _stream(logits)), "hl_sample")
    return out


def sample_filtered(logits: torch.Tensor, temperatures: torch.Tensor | None, top_ks: torch.Tensor | None,
                    top_ps: torch.Tensor | None, seed: int, step_state: torch.Tensor | None,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """hl_sample with the reference's top-k / top-p filters (mini_vllm/layers/sampler.py:13-49):
    per row a Gumbel-max draw from softmax(logits / T) restricted to the top-k, then top-p, set
    (top_ks int32, <= 0 or >= V: no filter; top_ps float32, >= 1: no filter); greedy argmax where
    T <= 0.  Rows without filters get exactly sample()'s token for the same seed and step."""
    _cuda(logits, temperatures, top_ks, top_ps, step_state, out)
    rows, vocab = logits.shape
    assert logits.dtype == torch.bfloat16 and logits.stride(1) == 1
    for t, dt in ((temperatures, torch.float32), (top_ks, torch.int32), (top_ps, torch.float32)):
        if t is not None:
            assert t.dtype == dt and t.is_contiguous() and t.numel() >= rows
    if step_state is not None:
        assert step_state.dtype == torch.int64 and step_state.numel() >= 2
    if out is None:
        out = torch.empty(rows, dtype=torch.int64, device=logits.device)
    lib = _lib.load()
    check(lib.hl_sample_filtered(logits.data_ptr(), logits.stride(0), rows, vocab, _p(temperatures), _p(top_ks),
                                 _p(top_ps), int(seed) & 0xFFFFFFFFFFFFFFFF, _p(step_state), out.data_ptr(),
                                 _stream(logits)), "hl_sample_filtered")
    return out


def silu_mul(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    _cuda(x, out)
    rows, two_i = x.shape
    inter = two_i // 2
    assert x.stride(1) == 1
    if out is None:
        out = torch.empty(rows, inter, dtype=x.dtype, device=x.device)
    lib = _lib.load()
    check(lib.hl_silu_mul(x.data_ptr(), x.stride(0), out.data_ptr(), out.stride(0), rows, inter, _stream(x)),
          "hl_silu_mul")
    return out


def argmax(logits: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    _cuda(logits, out)
    rows, vocab = logits.shape
    assert logits.dtype == torch.bfloat16 and logits.stride(1) == 1
    if out is None:
        out = torch.empty(rows, dtype=torch.int64, device=logits.device)
    lib = _lib.load()
    check(lib.hl_argmax(logits.data_ptr(), logits.stride(0), rows, vocab, out.data_ptr(), _stream(logits)),
          "hl_argmax")
    return out


def argmax_shard(logits: torch.Tensor, index_offset: int, out_tokens: torch.Tensor, out_values: torch.Tensor):
    """Per-row (max value, index + index_offset) of one vocabulary shard (hl_argmax_shard)."""
    _cuda(logits, out_tokens, out_values)
    rows, vocab = logits.shape
    assert logits.dtype == torch.bfloat16 and logits.stride(1) == 1
    assert out_tokens.dtype == torch.int64 and out_values.dtype == torch.float32
    lib = _lib.load()
    check(lib.hl_argmax_shard(logits.data_ptr(), logits.stride(0), rows, vocab, int(index_offset),
                              out_tokens.data_ptr(), out_values.data_ptr(), _stream(logits)), "hl_argmax_shard")
