"""RMSNorm (mini_vllm/layers/layernorm.py:6-52) on the hl_rmsnorm kernel.

forward(x) returns RMSNorm(x); forward(x, residual) returns (RMSNorm(x + residual),
x + residual) like add_rms_forward, updating `residual` in place.
"""
import torch
from torch import nn

from hilda_vllm_b200 import kernels


class RMSNorm(nn.Module):

    def __init__(self, hidden_size: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(hidden_size))

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None):
        if residual is None:
            return kernels.rmsnorm(x, self.weight, self.eps)
        return kernels.rmsnorm(x, self.weight, self.eps, residual=residual)
