"""The C-ABI library loads on the CPU host, exports exactly what include/hilda_b200.h declares,
and rejects bad arguments with HL_ERR_INVALID before touching the GPU."""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from hilda_vllm_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "hilda_b200.h"


def declared_functions() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*(hl_[a-z_0-9]+)\s*\(", text, re.M))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 14
    for n in names:
        assert hasattr(lib, n), n
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (hl_[a-z_0-9]+)$", out, re.M))
    assert names == exported


def test_ctypes_signatures_cover_the_header():
    assert declared_functions() == set(_lib.SIGNATURES)


def test_struct_layouts_match_header():
    assert ctypes.sizeof(_lib.HlPackHeader) == 16
    assert ctypes.sizeof(_lib.HlPackEvent) == 48
    from hilda_vllm_b200.engine.decode_packer import EVENT_DTYPE, HEADER_DTYPE
    for (name, _), field in zip(_lib.HlPackEvent._fields_, EVENT_DTYPE.names):
        assert name == field
        assert getattr(_lib.HlPackEvent, name).offset == EVENT_DTYPE.fields[field][1]
    for (name, _), field in zip(_lib.HlPackHeader._fields_, HEADER_DTYPE.names):
        assert getattr(_lib.HlPackHeader, name).offset == HEADER_DTYPE.fields[field][1]


def test_invalid_arguments_are_rejected_without_gpu():
    lib = _lib.load()
    assert lib.hl_version() == 1
    # negative token count
    assert lib.hl_store_kv_bf16(None, None, 0, 0, None, None, None, -1, 0, 8, 128, None) == 1
    assert b"num_tokens" in lib.hl_last_error_string()
    # empty batch is a no-op success
    assert lib.hl_store_kv_bf16(None, None, 0, 0, None, None, None, 0, 0, 8, 128, None) == 0
    assert lib.hl_last_error_string() == b""
    # decode: unsupported head_dim and missing workspace
    p = ctypes.c_void_p(16)
    rc = lib.hl_paged_decode(p, 2048, p, p, 0, None, None, p, 4, 4, p, 8, 16, 8, 64, 256, 64, 0.1, p, 2048, p, 1 << 30,
                             None)
    assert rc == 1 and b"head_dim" in lib.hl_last_error_string()
    rc = lib.hl_paged_decode(p, 2048, p, p, 0, None, None, p, 4, 4, p, 8, 16, 8, 128, 256, 64, 0.1, p, 2048, p, 10, None)
    assert rc == 4 and b"workspace" in lib.hl_last_error_string()
    assert lib.hl_paged_decode_workspace_size(0, 16, 128, 4, 256) == -1
    assert lib.hl_paged_decode_workspace_size(256, 16, 128, 5, 256) > 0
    rc = lib.hl_varlen_prefill(p, 2048, 100, p, p, 0, 0, 100, p, p, None, 0, 2, 8, 16, 8, 64, 256, 0, 0.1, p, 2048, 1,
                               None)
    assert rc == 1 and b"head_dim" in lib.hl_last_error_string()
    assert lib.hl_pack_decode_batch(p, 8, 16, 256, p, p, p, p, p, p, p, p, 4, 4, None) == 1  # packet too small
    assert lib.hl_pack_decode_batch(p, 64, 2000, 256, p, p, p, p, p, p, p, p, 4, 4, None) == 1  # graph batch too big
    assert lib.hl_rmsnorm(p, 1000, None, p, p, 1000, 4, 1000, 1e-6, None) == 1  # hidden not multiple of 256


def test_kernel_wrappers_refuse_cpu_tensors():
    import torch

    from hilda_vllm_b200 import kernels
    k = torch.zeros(2, 8, 128, dtype=torch.bfloat16)
    cache = torch.zeros(2, 256, 8, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="no CPU fallback"):
        kernels.store_kvcache(k, k, cache, cache, torch.zeros(2, dtype=torch.int32))
