"""RMSNorm (reference looped_blockell/layers/norms.py:8-15): ``x / sqrt(mean(x^2)
+ eps) * scale`` with eps 1e-5 and a learnable ``scale``.

The forward runs the sm_100a kernel in the input's precision: bf16 inputs
(fp32 math, bf16 out) or fp32 inputs (fp32 throughout, as the reference
layer computes them).  The backward is the closed form of the same function,
evaluated with tensor ops on the device.
"""

import torch
import torch.nn as nn


class _RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x2, scale, eps):
        from ..kernels.ops import rmsnorm
        y = rmsnorm(x2, scale.detach().to(x2.dtype), eps)
        ctx.save_for_backward(x2, scale)
        ctx.eps = eps
        return y

    @staticmethod
    def backward(ctx, dy):
        x2, scale = ctx.saved_tensors
        xf, dyf = x2.float(), dy.float()
        r = torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + ctx.eps)
        g = dyf * scale.float()
        dx = r * g - xf * r.pow(3) * (g * xf).mean(dim=-1, keepdim=True)
        dscale = (dyf * xf * r).sum(dim=0).to(scale.dtype)
        return dx.to(x2.dtype), dscale, None


class RMSNorm(nn.Module):
    def __init__(self, d: int, eps: float = 1e-5, device=None):
        super().__init__()
        self.eps = eps
        self.scale = nn.Parameter(torch.ones(d, device=device))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.dtype not in (torch.bfloat16, torch.float32):
            x = x.to(torch.float32)
        lead = x.shape[:-1]
        y = _RMSNormFn.apply(x.reshape(-1, x.shape[-1]).contiguous(), self.scale, self.eps)
        return y.reshape(*lead, x.shape[-1])
