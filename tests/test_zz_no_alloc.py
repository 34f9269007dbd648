"""The allocation-free decode entry point, hl_paged_decode_noalloc.

It exists for callers that cannot allocate device memory themselves (a host binding the library
through an FFI without a device allocator, or a serving loop whose memory is all reserved up
front and must not call cudaMalloc): its split-K scratch is a fixed device array inside the
library.  This file is collected last on purpose, so a failure here comes after every other
test has run; it also passes on its own in a fresh process.

Both decode kernels are covered: the CUDA-core kernel (GQA ratio 2, BF16 and e4m3) and the
tcgen05 kernel that hl_paged_decode picks for GQA ratios 4 and 8, whose tickets and partials sit
further into the scratch.  Each case makes two calls in a row with multi-split sequences (the
second call finds the first one's tickets and partials in the array) and asserts that the output
is bit-identical to hl_paged_decode with a caller-provided workspace (same kernel, fixed merge
order) and within the attention tolerance of the fp32 oracle.
"""
import ctypes

import pytest
import torch

from hilda_vllm_b200 import _lib, kernels
from oracle import attention as oattn
from oracle import kv_store

pytestmark = pytest.mark.gpu
DEV = "cuda"
BF16_TOL = dict(rtol=2e-2, atol=2e-3)  # the BF16 attention tolerance of the other decode tests
FP8_TOL = dict(rtol=2e-2, atol=6e-2)   # the FP8-KV tolerance of the other decode tests


def _case(seed, lens, hq, hk, fp8, d=128, bs=256):
    g = torch.Generator().manual_seed(seed)
    nblk = [max(1, -(-n // bs)) for n in lens]
    mb = max(nblk)
    perm = torch.randperm(sum(nblk), generator=g).tolist()
    tables, off = [], 0
    for n in nblk:
        tables.append(perm[off:off + n] + [-1] * (mb - n))
        off += n
    k = torch.randn(sum(nblk), bs, hk, d, generator=g).bfloat16()
    v = torch.randn(sum(nblk), bs, hk, d, generator=g).bfloat16()
    ks = vs = None
    if fp8:
        ks = torch.rand(hk, generator=g) + 0.5
        vs = torch.rand(hk, generator=g) + 0.5
        k = kv_store.quantize_e4m3(k, ks)
        v = kv_store.quantize_e4m3(v, vs)
    q = torch.randn(len(lens), hq, d, generator=g).bfloat16()
    bt = torch.tensor(tables, dtype=torch.int32)
    ln = torch.tensor(lens, dtype=torch.int32)
    return q, k, v, bt, ln, ks, vs


def _noalloc(q, k, v, bt, ln, scale, ks=None, vs=None):
    lib = _lib.load()
    b, hq, d = q.shape
    out = torch.empty_like(q)
    fp8 = k.dtype == torch.uint8
    rc = lib.hl_paged_decode_noalloc(q.data_ptr(), q.stride(0), k.data_ptr(), v.data_ptr(), 1 if fp8 else 0,
                                     None if ks is None else ks.data_ptr(), None if vs is None else vs.data_ptr(),
                                     bt.data_ptr(), bt.stride(0), bt.shape[1], ln.data_ptr(), b, hq, k.shape[2], d,
                                     k.shape[1], k.shape[0], ctypes.c_float(scale), out.data_ptr(), out.stride(0),
                                     torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.hl_last_error_string()
    return out


def _noalloc_errors():
    lib = _lib.load()
    val = ctypes.c_int32(-1)
    rc = lib.hl_paged_decode_noalloc_read_errors(ctypes.addressof(val), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.hl_last_error_string()
    return int(val.value)


@pytest.mark.parametrize("hq,hk,fp8", [(16, 8, False), (32, 8, False), (64, 8, False),
                                       (16, 8, True), (32, 8, True), (64, 8, True)])
def test_noalloc_decode_matches_workspace_decode_twice_in_a_row(hq, hk, fp8):
    scale = 128 ** -0.5
    tol = FP8_TOL if fp8 else BF16_TOL
    # Two calls in a row on different inputs: the second reuses the scratch the first left
    # behind.  Lengths above 1024 give several splits (CUDA-core kernel) and several units per
    # (sequence, head) cut across CTAs (tcgen05 kernel), so tickets and partials are used.
    for seed, lens in ((31 + hq, [1, 130, 700, 0, 1024, 300, 2000]),
                       (32 + hq, [2048, 5, 257, 129, 0, 900, 64, 1500])):
        q, k, v, bt, ln, ks, vs = _case(seed, lens, hq, hk, fp8)
        qd, kd, vd, btd, lnd = (t.to(DEV) for t in (q, k, v, bt, ln))
        ksd = None if ks is None else ks.to(DEV)
        vsd = None if vs is None else vs.to(DEV)
        kview = kd.view(torch.float8_e4m3fn) if fp8 else kd
        vview = vd.view(torch.float8_e4m3fn) if fp8 else vd
        want = kernels.paged_decode(qd, kview, vview, btd, lnd, scale, k_scale=ksd, v_scale=vsd)
        got = _noalloc(qd, kd, vd, btd, lnd, scale, ksd, vsd)
        torch.cuda.synchronize()
        assert _noalloc_errors() == 0
        assert torch.equal(got.view(torch.int16), want.view(torch.int16)), \
            f"noalloc differs from the workspace path (max {float((got.float() - want.float()).abs().max()):.3e})"
        ref = oattn.paged_decode(q, k, v, bt, ln, scale, ks, vs, fp8=fp8)
        err = (got.float().cpu() - ref).abs()
        assert bool((err <= tol["atol"] + tol["rtol"] * ref.abs()).all()), float(err.max())


@pytest.mark.parametrize("hq", [16, 32])
def test_noalloc_error_word_reports_a_bad_block_then_clears(hq):
    """A block id beyond the pool is caught by the kernel's bounds check (no load from it): the call
    still returns HL_OK, the error word read back afterwards has bit 1 set, and the next clean call
    starts from zero again."""
    scale = 128 ** -0.5
    q, k, v, bt, ln, _, _ = _case(40 + hq, [300, 600], hq, 8, False)
    bad = bt.clone()
    bad[1, 1] = k.shape[0] + 3
    qd, kd, vd, lnd = q.to(DEV), k.to(DEV), v.to(DEV), ln.to(DEV)
    _noalloc(qd, kd, vd, bad.to(DEV), lnd, scale)
    assert _noalloc_errors() & 2
    _noalloc(qd, kd, vd, bt.to(DEV), lnd, scale)
    assert _noalloc_errors() == 0


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
