"""The allocation-free decode entry point, hl_paged_decode_noalloc.

It exists for callers that cannot allocate device memory themselves (a host binding the library
through an FFI without a device allocator, or a serving loop whose memory is all reserved up
front and must not call cudaMalloc): its split-K scratch is a fixed device array inside the
library.  This file is collected last on purpose, so a failure here comes after every other
test has run; it also passes on its own in a fresh process.
"""
import ctypes

import pytest
import torch

from hilda_vllm_b200 import _lib, kernels

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = dict(rtol=2e-2, atol=2e-3)  # the BF16 attention tolerance used by the other decode tests


def _case(seed, lens, hq=16, hk=8, d=128, bs=256):
    g = torch.Generator().manual_seed(seed)
    nblk = [max(1, -(-n // bs)) for n in lens]
    mb = max(nblk)
    perm = torch.randperm(sum(nblk), generator=g).tolist()
    tables, off = [], 0
    for n in nblk:
        tables.append(perm[off:off + n] + [-1] * (mb - n))
        off += n
    k = torch.randn(sum(nblk), bs, hk, d, generator=g).bfloat16().to(DEV)
    v = torch.randn(sum(nblk), bs, hk, d, generator=g).bfloat16().to(DEV)
    q = torch.randn(len(lens), hq, d, generator=g).bfloat16().to(DEV)
    bt = torch.tensor(tables, dtype=torch.int32, device=DEV)
    ln = torch.tensor(lens, dtype=torch.int32, device=DEV)
    return q, k, v, bt, ln


def _noalloc(q, k, v, bt, ln, scale):
    lib = _lib.load()
    b, hq, d = q.shape
    out = torch.empty_like(q)
    rc = lib.hl_paged_decode_noalloc(q.data_ptr(), q.stride(0), k.data_ptr(), v.data_ptr(), 0, None, None,
                                     bt.data_ptr(), bt.stride(0), bt.shape[1], ln.data_ptr(), b, hq, k.shape[2], d,
                                     k.shape[1], k.shape[0], ctypes.c_float(scale), out.data_ptr(), out.stride(0),
                                     torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.hl_last_error_string()
    return out


def test_noalloc_decode_matches_workspace_decode_twice_in_a_row():
    scale = 128 ** -0.5
    # Two calls in a row on different inputs: the second reuses the scratch the first left
    # behind (multi-split sequences exercise the tickets and partials).
    for seed, lens in ((31, [1, 130, 700, 0, 1024, 300]), (32, [2048, 5, 257, 129, 0, 900, 64, 1500])):
        q, k, v, bt, ln = _case(seed, lens)
        want = kernels.paged_decode(q, k, v, bt, ln, scale)
        got = _noalloc(q, k, v, bt, ln, scale)
        torch.cuda.synchronize()
        err = (got.float() - want.float()).abs()
        assert bool((err <= TOL["atol"] + TOL["rtol"] * want.float().abs()).all()), float(err.max())


def test_noalloc_rejects_shapes_beyond_its_scratch():
    lib = _lib.load()
    cap = lib.hl_paged_decode_noalloc_capacity()
    assert cap == 32 << 20
    # 4096 sequences x 64 pages of 256 tokens needs far more than the built-in scratch.
    p = ctypes.c_void_p(256)
    rc = lib.hl_paged_decode_noalloc(p, 2048, p, p, 0, None, None, p, 64, 64, p, 4096, 16, 8, 128, 256, 1 << 20,
                                     ctypes.c_float(0.1), p, 2048, None)
    assert rc == 3
    assert b"more than the built-in" in lib.hl_last_error_string()
