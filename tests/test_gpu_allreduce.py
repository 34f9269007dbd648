"""The fused NVLink all-reduce + add + RMSNorm (hl_allreduce_add_rmsnorm).

* one rank: the kernel reduces to add + RMSNorm and must equal hl_rmsnorm bit for bit;
* a peer that never arrives (its flag is never set): the bounded wait expires, the error word
  says HL_AR_TIMEOUT, the context stays usable;
* two or more GPUs (skipped with fewer): one process per GPU, several alternating calls, outputs
  bit-identical on every rank and equal to bf16(sum of partials) + add + RMSNorm, for the one-shot
  and the two-shot kernel.
"""
import ctypes
import os
import socket

import pytest
import torch

from hilda_vllm_b200 import _lib, kernels
from hilda_vllm_b200.layers.nvlink_allreduce import NvlinkAllReduce

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _reference(partials, residual, weight, eps):
    """bf16(fp32 sum in rank order) then the add + RMSNorm kernel."""
    acc = torch.zeros_like(partials[0], dtype=torch.float32)
    for p in partials:
        acc = acc + p.float()
    res = residual.clone()
    y, res = kernels.rmsnorm(acc.bfloat16(), weight, eps, residual=res)
    return y, res


@pytest.mark.parametrize("two_shot", [False, True])
@pytest.mark.parametrize("rows,hidden", [(1, 1024), (256, 1024), (300, 4096), (37, 2560), (512, 8192)])
def test_single_rank_equals_add_rmsnorm(rows, hidden, two_shot):
    g = torch.Generator().manual_seed(rows + hidden)
    ar = NvlinkAllReduce(0, 1, 512, hidden, torch.device(DEV))
    ar.force_two_shot = two_shot
    try:
        w = (torch.rand(hidden, generator=g) + 0.5).bfloat16().to(DEV)
        for slot in (0, 1, 0):
            x = torch.randn(rows, hidden, generator=g).bfloat16().to(DEV)
            res = torch.randn(rows, hidden, generator=g).bfloat16().to(DEV)
            ar.output(slot, rows).copy_(x)
            want_y, want_r = _reference([x], res, w, 1e-6)
            got_y, got_r = ar.add_rmsnorm(slot, rows, res, w, 1e-6)
            torch.cuda.synchronize()
            assert torch.equal(got_y.view(torch.int16), want_y.view(torch.int16))
            assert torch.equal(got_r.view(torch.int16), want_r.view(torch.int16))
        ar.copy_error_word()
        torch.cuda.synchronize()
        ar.check_errors()
    finally:
        ar.close()


def test_missing_peer_times_out_with_error_word():
    """world=2 in one process: the 'peer' signal area is a local buffer nobody writes, so the
    wait for rank 1 must give up after the (50 ms) limit and report it."""
    lib = _lib.load()
    rows, hidden = 4, 1024
    data = torch.randn(rows, hidden, device=DEV).bfloat16()
    sig_bytes = int(lib.hl_allreduce_signal_bytes())
    sig = [torch.zeros(sig_bytes // 4, dtype=torch.int32, device=DEV) for _ in range(2)]
    epochs = torch.zeros(128, dtype=torch.int32, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    res = torch.randn(rows, hidden, device=DEV).bfloat16()
    out = torch.empty_like(res)
    w = torch.ones(hidden, device=DEV).bfloat16()
    arr = ctypes.c_void_p * 2
    peer_data = arr(data.data_ptr(), data.data_ptr())
    peer_sig = arr(sig[0].data_ptr(), sig[1].data_ptr())
    stream = torch.cuda.current_stream().cuda_stream
    kernels.check(lib.hl_allreduce_add_rmsnorm(ctypes.addressof(peer_data), ctypes.addressof(peer_sig), 2, 0, rows,
                                               hidden, res.data_ptr(), w.data_ptr(), out.data_ptr(), out.stride(0),
                                               1e-6, epochs.data_ptr(), err.data_ptr(), 50_000_000, stream),
                  "hl_allreduce_add_rmsnorm")
    torch.cuda.synchronize()
    assert int(err.item()) == 1  # HL_AR_TIMEOUT
    # Rank 0 announced itself in the peer's area; the context is still usable.
    assert int(sig[1][0 * 8 + 0].item()) == 1
    assert torch.isfinite(out.float()).all()
    assert float((torch.ones(3, device=DEV) * 2).sum()) == 6.0


@pytest.mark.parametrize("two_shot", [False, True])
@pytest.mark.parametrize("world,rank,hidden,rows", [(4, 1, 1024, 256), (8, 3, 1024, 256), (8, 5, 4096, 256),
                                                    (8, 0, 2560, 37), (4, 2, 4096, 300)])
def test_emulated_ranks_on_one_gpu(two_shot, world, rank, hidden, rows):
    """`world` ranks emulated in one process on one GPU: every peer's partial sums, flags and
    result buffer are local buffers, and this rank's own flag area is set in advance so that no
    wait blocks (nothing waits on another kernel).  The kernel's multi-rank arithmetic (the sum in
    rank order over all ranks, the two-shot kernel's owned rows and pushes) must give
    bf16(sum of partials) + add + RMSNorm bit for bit; the two-shot kernel reads the rows other
    ranks own from this rank's result buffer, which the test fills with the expected sums."""
    lib = _lib.load()
    g = torch.Generator().manual_seed(world * 1000 + hidden + rows)
    partials = [torch.randn(rows, hidden, generator=g).bfloat16().to(DEV) for _ in range(world)]
    res = torch.randn(rows, hidden, generator=g).bfloat16().to(DEV)
    w = (torch.rand(hidden, generator=g) + 0.5).bfloat16().to(DEV)
    want_y, want_r = _reference(partials, res, w, 1e-6)
    sums = torch.zeros(rows, hidden, dtype=torch.float32, device=DEV)
    for p in partials:
        sums += p.float()
    sums = sums.bfloat16()
    owned = torch.tensor([r % world == rank for r in range(rows)], device=DEV)
    sig_bytes = int(lib.hl_allreduce_signal_bytes())
    sig = [torch.zeros(sig_bytes // 4, dtype=torch.int32, device=DEV) for _ in range(world)]
    sig[rank].fill_(1 << 30)  # every peer "arrived" long ago, on both flag banks
    results = [torch.zeros(rows, hidden, dtype=torch.bfloat16, device=DEV) for _ in range(world)]
    results[rank][~owned] = sums[~owned]
    epochs = torch.zeros(128, dtype=torch.int32, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = torch.empty_like(res)
    arr = ctypes.c_void_p * world
    peer_data = arr(*[p.data_ptr() for p in partials])
    peer_sig = arr(*[x.data_ptr() for x in sig])
    peer_res = arr(*[x.data_ptr() for x in results])
    stream = torch.cuda.current_stream().cuda_stream
    if two_shot:
        rc = lib.hl_allreduce_add_rmsnorm_2shot(ctypes.addressof(peer_data), ctypes.addressof(peer_res),
                                                ctypes.addressof(peer_sig), world, rank, rows, hidden, res.data_ptr(),
                                                w.data_ptr(), out.data_ptr(), out.stride(0), 1e-6, epochs.data_ptr(),
                                                err.data_ptr(), 2_000_000_000, stream)
    else:
        rc = lib.hl_allreduce_add_rmsnorm(ctypes.addressof(peer_data), ctypes.addressof(peer_sig), world, rank, rows,
                                          hidden, res.data_ptr(), w.data_ptr(), out.data_ptr(), out.stride(0), 1e-6,
                                          epochs.data_ptr(), err.data_ptr(), 2_000_000_000, stream)
    kernels.check(rc, "hl_allreduce_add_rmsnorm")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(out.view(torch.int16), want_y.view(torch.int16))
    assert torch.equal(res.view(torch.int16), want_r.view(torch.int16))
    if two_shot:  # this rank pushed exactly its own rows' sums to every rank
        for r in range(world):
            assert torch.equal(results[r][owned].view(torch.int16), sums[owned].view(torch.int16))
            if r != rank:
                assert not (results[r][~owned].float() != 0).any()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q, two_shot, hidden, rows):
    import torch.distributed as dist
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                device_id=torch.device("cuda", rank))
        ar = NvlinkAllReduce(rank, world, 512, hidden, torch.device("cuda", rank), timeout_s=10.0)
        ar.force_two_shot = two_shot
        w = (torch.arange(hidden, device="cuda") % 7 + 1).bfloat16() / 4
        results = []
        for call in range(6):
            slot = call % 2
            g = torch.Generator().manual_seed(1000 * call + rank)
            x = torch.randn(rows, hidden, generator=g).bfloat16().cuda()
            g2 = torch.Generator().manual_seed(77 + call)
            res = torch.randn(rows, hidden, generator=g2).bfloat16().cuda()
            ar.output(slot, rows).copy_(x)
            y, r = ar.add_rmsnorm(slot, rows, res, w, 1e-6)
            parts = [torch.empty_like(x) for _ in range(world)]
            dist.all_gather(parts, x)  # every rank's partials, to build the reference
            res2 = torch.randn(rows, hidden, generator=torch.Generator().manual_seed(77 + call)).bfloat16().cuda()
            want_y, want_r = _reference(parts, res2, w, 1e-6)
            results.append((torch.equal(y.view(torch.int16), want_y.view(torch.int16)),
                            torch.equal(r.view(torch.int16), want_r.view(torch.int16)),
                            int(y.view(torch.int16).long().sum().item())))
        ar.copy_error_word()
        torch.cuda.synchronize()
        dist.barrier()
        q.put((rank, results, int(ar.error_host[0])))
        ar.close()
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e), -1))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("two_shot,hidden,rows", [(False, 1024, 256), (True, 1024, 256), (True, 4096, 300),
                                                   (False, 4096, 256), (False, 2560, 37), (True, 2560, 37)])
def test_ranks_bit_exact_and_identical(two_shot, hidden, rows):
    """All GPUs of the box (up to 8) as ranks, one-shot and two-shot kernels: every rank's output
    and residual equal bf16(sum of partials in rank order) + add + RMSNorm bit for bit."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    world = min(torch.cuda.device_count(), 8)
    env_backup = os.environ.get("NCCL_NVLS_ENABLE")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        procs = [ctx.Process(target=_worker, args=(r, world, port, q, two_shot, hidden, rows)) for r in range(world)]
        for p in procs:
            p.start()
        out = [q.get(timeout=300) for _ in range(world)]
        for p in procs:
            p.join(timeout=60)
    finally:
        if env_backup is None:
            os.environ.pop("NCCL_NVLS_ENABLE", None)
        else:
            os.environ["NCCL_NVLS_ENABLE"] = env_backup
    out.sort()
    for rank, results, err in out:
        assert err == 0, (rank, results)
        assert all(ok_y and ok_r for ok_y, ok_r, _ in results), (rank, results)
    for other in out[1:]:
        assert [c for *_, c in out[0][1]] == [c for *_, c in other[1]]  # identical on every rank
