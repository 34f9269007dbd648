"""Loads libhilda_b200.so (the sm_100a kernels behind the C ABI in include/hilda_b200.h).

There is no fallback: if the library is missing or cannot be loaded, every kernel call
raises.  Build it with ``python -m hilda_vllm_b200.csrc.build`` (``__graft_entry__.build()``
does the same).
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libhilda_b200.so"

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None

c_int = ctypes.c_int
c_i64 = ctypes.c_int64
c_f32 = ctypes.c_float
c_vp = ctypes.c_void_p
c_char_p = ctypes.c_char_p


class HlPackHeader(ctypes.Structure):
    """Mirror of hl_pack_header (include/hilda_b200.h)."""

    _fields_ = [
        ("num_events", ctypes.c_int32),
        ("batch", ctypes.c_int32),
        ("pool_offset", ctypes.c_int32),
        ("pool_len", ctypes.c_int32),
    ]


class HlPackEvent(ctypes.Structure):
    """Mirror of hl_pack_event (include/hilda_b200.h)."""

    _fields_ = [
        ("flags", ctypes.c_int32),
        ("slot", ctypes.c_int32),
        ("ctx_len", ctypes.c_int32),
        ("bt_len", ctypes.c_int32),
        ("seq_id", ctypes.c_int64),
        ("token", ctypes.c_int64),
        ("row_start", ctypes.c_int32),
        ("row_count", ctypes.c_int32),
        ("pool_off", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


# Function name -> (restype, argtypes).  Kept in the order of include/hilda_b200.h.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "hl_last_error_string": (c_char_p, []),
    "hl_version": (c_int, []),
    "hl_store_kv_bf16": (c_int, [c_vp, c_vp, c_i64, c_i64, c_vp, c_vp, c_vp, c_i64, c_i64, c_int, c_int, c_vp]),
    "hl_store_kv_fp8": (
        c_int,
        [c_vp, c_vp, c_i64, c_i64, c_vp, c_vp, c_vp, c_i64, c_i64, c_int, c_int, c_vp, c_vp, c_vp],
    ),
    "hl_copy_kv_bf16_to_fp8": (
        c_int,
        [c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_int, c_int, c_vp, c_vp, c_int, c_i64, c_i64, c_i64, c_vp],
    ),
    "hl_paged_decode_workspace_size": (c_i64, [c_int, c_int, c_int, c_int, c_int]),
    "hl_paged_decode": (
        c_int,
        [
            c_vp, c_i64, c_vp, c_vp, c_int, c_vp, c_vp, c_vp, c_i64, c_int, c_vp, c_int,
            c_int, c_int, c_int, c_int, c_i64, c_f32, c_vp, c_i64, c_vp, c_i64, c_vp,
        ],
    ),
    "hl_paged_decode_tc": (
        c_int,
        [
            c_vp, c_i64, c_vp, c_vp, c_int, c_vp, c_vp, c_vp, c_i64, c_int, c_vp, c_int,
            c_int, c_int, c_int, c_int, c_i64, c_f32, c_vp, c_i64, c_vp, c_i64, c_vp,
        ],
    ),
    "hl_paged_decode_noalloc": (
        c_int,
        [
            c_vp, c_i64, c_vp, c_vp, c_int, c_vp, c_vp, c_vp, c_i64, c_int, c_vp, c_int,
            c_int, c_int, c_int, c_int, c_i64, c_f32, c_vp, c_i64, c_vp,
        ],
    ),
    "hl_paged_decode_noalloc_capacity": (c_i64, []),
    "hl_paged_decode_noalloc_read_errors": (c_int, [c_vp, c_vp]),
    "hl_paged_decode_read_errors": (c_int, [c_vp, c_vp, c_vp]),
    "hl_varlen_prefill": (
        c_int,
        [
            c_vp, c_i64, c_i64, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp, c_i64, c_int, c_int,
            c_int, c_int, c_int, c_int, c_i64, c_f32, c_vp, c_i64, c_int, c_vp,
        ],
    ),
    "hl_varlen_prefill_read_errors": (c_int, [c_vp]),
    "hl_varlen_prefill_copy_errors_async": (c_int, [c_vp, c_vp]),
    "hl_varlen_prefill_clear_errors": (c_int, [c_vp]),
    "hl_pack_decode_batch": (
        c_int,
        [c_vp, c_i64, c_int, c_int, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_int, c_vp],
    ),
    "hl_rmsnorm": (c_int, [c_vp, c_i64, c_vp, c_vp, c_vp, c_i64, c_int, c_int, c_f32, c_vp]),
    "hl_qk_norm_rope": (c_int, [c_vp, c_i64, c_int, c_int, c_int, c_int, c_vp, c_vp, c_vp, c_vp, c_f32, c_vp]),
    "hl_qk_norm_rope_store": (c_int, [c_vp, c_i64, c_int, c_int, c_int, c_int, c_vp, c_vp, c_vp, c_vp, c_f32, c_vp,
                                      c_vp, c_int, c_vp, c_i64, c_vp, c_vp, c_vp]),
    "hl_qk_norm_rope_store_mirrored": (c_int, [c_vp, c_i64, c_int, c_int, c_int, c_int, c_vp, c_vp, c_vp, c_vp,
                                               c_f32, c_vp, c_vp, c_int, c_vp, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "hl_device_alloc": (c_int, [c_i64, c_vp]),
    "hl_device_free": (c_int, [c_vp]),
    "hl_ipc_get_handle": (c_int, [c_vp, c_vp]),
    "hl_ipc_open_handle": (c_int, [c_vp, c_vp]),
    "hl_ipc_close_handle": (c_int, [c_vp]),
    "hl_allreduce_signal_bytes": (c_i64, []),
    "hl_allreduce_add_rmsnorm": (c_int, [c_vp, c_vp, c_int, c_int, c_int, c_int, c_vp, c_vp, c_vp, c_i64, c_f32,
                                         c_vp, c_vp, c_i64, c_vp]),
    "hl_allreduce_add_rmsnorm_2shot": (c_int, [c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_vp, c_vp, c_vp, c_i64,
                                               c_f32, c_vp, c_vp, c_i64, c_vp]),
    "hl_silu_mul": (c_int, [c_vp, c_i64, c_vp, c_i64, c_int, c_int, c_vp]),
    "hl_sample": (c_int, [c_vp, c_i64, c_int, c_int, c_i64, c_vp, ctypes.c_uint64, c_vp, c_vp, c_vp, c_vp]),
    "hl_sample_filtered": (c_int, [c_vp, c_i64, c_int, c_int, c_vp, c_vp, c_vp, ctypes.c_uint64, c_vp, c_vp,
                                   c_vp]),
    "hl_argmax": (c_int, [c_vp, c_i64, c_int, c_int, c_vp, c_vp]),
    "hl_argmax_shard": (c_int, [c_vp, c_i64, c_int, c_int, c_i64, c_vp, c_vp, c_vp]),
}


class HildaKernelError(RuntimeError):
    """A C-ABI call returned a non-zero hl_status."""


def load() -> ctypes.CDLL:
    """Returns the loaded library, loading it on first use.  Raises if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH.name} is not built; run `python -m hilda_vllm_b200.csrc.build` "
                "(there is no CPU or Triton fallback for these kernels)"
            )
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def check(status: int, name: str) -> None:
    if status != 0:
        msg = load().hl_last_error_string()
        text = msg.decode() if msg else ""
        raise HildaKernelError(f"{name} failed with status {status}: {text}")
