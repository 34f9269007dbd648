"""RMSNorm (mini_vllm/layers/layernorm.py:6-52) on the hl_rmsnorm kernel.

forward(x) returns RMSNorm(x); forward(x, residual) returns (RMSNorm(x + residual),
x + residual) like add_rms_forward, updating `residual` in place.  When x is a tensor-parallel
partial sum left in an NVLink all-reduce buffer, the all-reduce is fused into the same kernel.
"""
import torch
from torch import nn

from hilda_vllm_b200 import kernels
from hilda_vllm_b200.layers import nvlink_allreduce


class RMSNorm(nn.Module):

    def __init__(self, hidden_size: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(hidden_size))

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None):
        if residual is None:
            return kernels.rmsnorm(x, self.weight, self.eps)
        ar = nvlink_allreduce.active()
        if ar is not None:
            slot = ar.slot_of(x)
            if slot is not None:
                # x holds this rank's partial sums in a peer-mapped buffer: all-reduce + add +
                # RMSNorm in one kernel.
                return ar.add_rmsnorm(slot, x.shape[0], residual, self.weight, self.eps)
        return kernels.rmsnorm(x, self.weight, self.eps, residual=residual)
