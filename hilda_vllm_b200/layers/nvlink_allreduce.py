"""Tensor-parallel all-reduce over NVLink peer memory, fused with the add + RMSNorm after it.

The reference sums the row-parallel partial outputs (o_proj, down_proj) with
dist.all_reduce (mini_vllm/layers/linear.py:176-178) and then runs add + RMSNorm
(layers/layernorm.py:30-42).  With this module active, RowParallelLinear writes its partial
output straight into a buffer every peer has mapped (CUDA IPC), and the next RMSNorm runs
hl_allreduce_add_rmsnorm: one kernel that meets the peers at a flag barrier, reads the rows of
all ranks over NVLink, sums them in rank order and applies the add + RMSNorm.  Two buffers
alternate (o_proj -> slot 0, down_proj -> slot 1), which is what lets the kernel use a single
barrier per call.  From three ranks on, wide rows take hl_allreduce_add_rmsnorm_2shot instead
(each rank reduces 1/world of the rows, pushes them to every rank, second barrier).  Batches
larger than the buffers (prefill) keep NCCL.

All ranks must make the same calls in the same order; the decision to use the buffers depends
only on the row count, which is identical on every rank.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from hilda_vllm_b200 import _lib
from hilda_vllm_b200.kernels import check

_ACTIVE: "NvlinkAllReduce | None" = None
HANDLE_BYTES = 64  # sizeof(cudaIpcMemHandle_t)
MAX_BLOCKS = 128   # per-CTA flag slots / call counters in the kernel


def active() -> "NvlinkAllReduce | None":
    return _ACTIVE


def set_active(ar: "NvlinkAllReduce | None") -> None:
    global _ACTIVE
    _ACTIVE = ar


def prefer_two_shot(world: int, rows: int, hidden: int) -> bool:
    """True when the one-shot kernel would pull more than 10 MiB of bf16 partial sums from its
    peers, counting at least 128 rows (see NvlinkAllReduce.two_shot for the measurements)."""
    return world > 2 and (world - 1) * max(rows, 128) * hidden * 2 > (10 << 20)


class _DeviceArray:
    """Exposes a raw device allocation to torch.as_tensor (__cuda_array_interface__ v3)."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None, "stream": None}


class NvlinkAllReduce:

    def __init__(self, rank: int, world: int, max_rows: int, hidden: int, device: torch.device,
                 group=None, timeout_s: float = 20.0):
        assert 1 <= world <= 8 and hidden % 256 == 0 and hidden <= 8192
        self.lib = _lib.load()
        self.rank, self.world, self.max_rows, self.hidden = rank, world, max_rows, hidden
        self.device = device
        self.timeout_ns = int(timeout_s * 1e9)
        self.stats = {"calls": 0}
        nbytes = max_rows * hidden * 2
        sig_bytes = int(self.lib.hl_allreduce_signal_bytes())
        self._owned: list[int] = []
        self._opened: list[int] = []
        # [partials slot 0, partials slot 1, flags, reduced rows (two-shot)]
        own = [self._alloc(nbytes), self._alloc(nbytes), self._alloc(sig_bytes), self._alloc(nbytes)]
        self._epochs = self._alloc(MAX_BLOCKS * 4)
        self._error = self._alloc(256)
        handles = b""
        for ptr in own:
            h = ctypes.create_string_buffer(HANDLE_BYTES)
            check(self.lib.hl_ipc_get_handle(ctypes.c_void_p(ptr), h), "hl_ipc_get_handle")
            handles += h.raw
        gathered: list = [None] * world
        if world > 1:
            dist.all_gather_object(gathered, handles, group=group)
        else:
            gathered[0] = handles
        ptrs = [[0] * world for _ in range(4)]  # [data0, data1, signal, result][rank]
        for p in range(world):
            for i in range(4):
                if p == rank:
                    ptrs[i][p] = own[i]
                    continue
                out = ctypes.c_void_p()
                blob = gathered[p][i * HANDLE_BYTES:(i + 1) * HANDLE_BYTES]
                check(self.lib.hl_ipc_open_handle(blob, ctypes.byref(out)), "hl_ipc_open_handle")
                self._opened.append(out.value)
                ptrs[i][p] = out.value
        arr = ctypes.c_void_p * world
        self._peer_data = [arr(*ptrs[0]), arr(*ptrs[1])]
        self._peer_signal = arr(*ptrs[2])
        self._peer_result = arr(*ptrs[3])
        self._buf_ptrs = own[:2]
        self.force_two_shot: bool | None = None
        self.buffers = [torch.as_tensor(_DeviceArray(p, (max_rows, hidden), "<i2"), device=device).view(torch.bfloat16)
                        for p in own[:2]]
        self.error_host = torch.zeros(1, dtype=torch.int32, pin_memory=True, device="cpu")
        self._error_dev = torch.as_tensor(_DeviceArray(self._error, (1,), "<i4"), device=device)

    def _alloc(self, nbytes: int) -> int:
        ptr = ctypes.c_void_p()
        check(self.lib.hl_device_alloc(nbytes, ctypes.byref(ptr)), "hl_device_alloc")
        self._owned.append(ptr.value)
        return ptr.value

    # ------------------------------------------------------------------ use
    def fits(self, rows: int) -> bool:
        """Whether this batch takes the fused path (decode batches up to the buffers' rows).  On
        B200 (56 calls in a graph) the faster fused kernel beats NCCL + RMSNorm at every measured
        shape: two ranks, 256 rows: 7.8 vs 18.3 us (hidden 1024), 14.9 vs 27.8 (hidden 4096);
        eight ranks: see two_shot()."""
        return 0 < rows <= min(self.max_rows, 512)

    def two_shot(self, rows: int) -> bool:
        """The two-shot kernel (each rank reduces 1/world of the rows and pushes them to all) once
        the one-shot kernel would pull more than 10 MiB from its peers, counting at least 128 rows:
        the one-shot kernel's traffic grows with world - 1, the two-shot kernel's does not, but it
        waits on a second barrier.  B200, 8 ranks, us per call in a graph of 56 calls (one-shot /
        two-shot / NCCL all-reduce + RMSNorm):
          hidden 1024  rows  64: 10.1 / 16.2 / 32.0     hidden 4096  rows  64: 17.9 / 22.6 / 36.1
          hidden 1024  rows 256: 14.6 / 16.7 / 34.0     hidden 4096  rows 256: 37.2 / 35.1 / 40.7
        `force_two_shot` (None, True or False) overrides the choice, for tests and profiles."""
        if self.force_two_shot is not None:
            return self.force_two_shot
        return prefer_two_shot(self.world, rows, self.hidden)

    def output(self, slot: int, rows: int) -> torch.Tensor:
        """Where the row-parallel GEMM of `slot` writes its partial sums for `rows` rows."""
        return self.buffers[slot][:rows]

    def slot_of(self, t: torch.Tensor) -> int | None:
        """The slot whose buffer `t` is (from its first row), else None."""
        if t.dim() != 2 or not t.is_contiguous():
            return None
        ptr = t.data_ptr()
        for i, base in enumerate(self._buf_ptrs):
            if ptr == base:
                return i
        return None

    def add_rmsnorm(self, slot: int, rows: int, residual: torch.Tensor, weight: torch.Tensor, eps: float,
                    out: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        """out = RMSNorm(all_reduce(partials) + residual) with residual updated in place."""
        assert residual.is_contiguous() and residual.shape == (rows, self.hidden)
        if out is None:
            out = torch.empty_like(residual)
        stream = torch.cuda.current_stream(residual.device).cuda_stream
        self.stats["calls"] += 1
        if self.two_shot(rows):
            check(self.lib.hl_allreduce_add_rmsnorm_2shot(
                ctypes.addressof(self._peer_data[slot]), ctypes.addressof(self._peer_result),
                ctypes.addressof(self._peer_signal), self.world, self.rank, rows, self.hidden, residual.data_ptr(),
                weight.data_ptr(), out.data_ptr(), out.stride(0), float(eps), ctypes.c_void_p(self._epochs),
                ctypes.c_void_p(self._error), self.timeout_ns, stream), "hl_allreduce_add_rmsnorm_2shot")
            return out, residual
        check(self.lib.hl_allreduce_add_rmsnorm(
            ctypes.addressof(self._peer_data[slot]), ctypes.addressof(self._peer_signal), self.world, self.rank, rows,
            self.hidden, residual.data_ptr(), weight.data_ptr(), out.data_ptr(), out.stride(0), float(eps),
            ctypes.c_void_p(self._epochs), ctypes.c_void_p(self._error), self.timeout_ns, stream),
            "hl_allreduce_add_rmsnorm")
        return out, residual

    def copy_error_word(self) -> None:
        """Queues a device->host copy of the error word on the current stream."""
        self.error_host.copy_(self._error_dev, non_blocking=True)

    def check_errors(self) -> None:
        """Raises if a previous call timed out waiting for a peer (after copy_error_word and a sync)."""
        if int(self.error_host[0]):
            raise RuntimeError("NVLink all-reduce: a peer rank did not arrive within the timeout "
                               f"(error word {int(self.error_host[0])})")

    def close(self) -> None:
        self.buffers = []
        self._error_dev = None
        for ptr in self._opened:
            self.lib.hl_ipc_close_handle(ctypes.c_void_p(ptr))
        self._opened = []
        for ptr in self._owned:
            self.lib.hl_device_free(ctypes.c_void_p(ptr))
        self._owned = []
