"""SiluAndMul (mini_vllm/layers/activation.py:6-16) on the hl_silu_mul kernel."""
import torch
from torch import nn

from hilda_vllm_b200 import kernels


class SiluAndMul(nn.Module):

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return kernels.silu_mul(x)
