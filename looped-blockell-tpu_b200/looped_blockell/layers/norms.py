"""RMSNorm (reference looped_blockell/layers/norms.py:8-15): ``x / sqrt(mean(x^2)
+ eps) * scale`` with eps 1e-5; bf16 inputs run the sm_100a kernel."""

import torch
import torch.nn as nn


class RMSNorm(nn.Module):
    def __init__(self, d: int, eps: float = 1e-5, device=None):
        super().__init__()
        self.eps = eps
        self.scale = nn.Parameter(torch.ones(d, device=device))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        from ..kernels.ops import rmsnorm
        return rmsnorm(x.to(torch.bfloat16), self.scale.detach().to(torch.bfloat16), self.eps)
