"""Block-ELL MLP layers — the reference's Flax modules as torch.nn.Modules.

``BlockELLLinear`` and ``MLPBlock`` keep the constructor arguments and the
parameter / topology layout of looped_blockell/layers/mlp.py:28-168:
``values [R, K, B, B]`` ~ N(0, 0.02), ``bias`` zeros, topology buffers
``col_indices [R, K]`` and ``alive_mask [R, K]``; K = max(1, int(C * density));
topology seeded from (out_features, in_features), so gate and up share it as
in the reference (mlp.py:84-95).  Dead tiles (alive_mask False) are passed to
the kernel as column -1 and skipped, which equals zeroing them (mlp.py:73-77).
The SwiGLU branch runs the fused sm_100a kernel; like the PyTorch mirror
(interop/pt_model.py:862-867) its projections carry no bias.

Both modules are trainable, as the reference's are: the forward and backward
run on this package's kernels through the autograd nodes of
``kernels.autograd`` (tile gradients summed in fp32).  The kernels read a
bf16 copy of each ``values`` parameter; the copy (and the -1-masked column
indices) is rebuilt only when the parameter or the topology buffers change,
which in-place updates such as an optimizer step report through the tensor's
version counter.  Writes through ``.data`` bypass that counter: call
``refresh()`` after them.
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from .block_ell import BlockELLConfig, BlockELLTensor, create_random_topology


def _topology_seed(out_features: int, in_features: int) -> int:
    return hash((out_features, in_features)) % 2 ** 31


class BlockELLLinear(nn.Module):
    """Single Block-ELL linear layer (reference mlp.py:28-95)."""

    def __init__(self, out_features: int, in_features: int, tile_size: int = 16, density: float = 1.0,
                 dtype: torch.dtype = torch.bfloat16, bias: bool = True, device=None):
        super().__init__()
        B = tile_size
        if out_features % B or in_features % B:
            raise ValueError(f"features ({out_features}, {in_features}) must be divisible by tile_size {B}")
        self.out_features, self.in_features, self.tile_size, self.density = out_features, in_features, B, density
        self.dtype = dtype
        self.R, self.C = out_features // B, in_features // B
        self.K = max(1, int(self.C * density))
        self.values = nn.Parameter(torch.randn(self.R, self.K, B, B, device=device) * 0.02)
        self.bias = nn.Parameter(torch.zeros(out_features, device=device)) if bias else None
        self.register_buffer("col_indices", self._init_topology().to(device))
        self.register_buffer("alive_mask", torch.ones(self.R, self.K, dtype=torch.bool, device=device))

    def _init_topology(self) -> torch.Tensor:
        if self.density >= 1.0:
            return torch.arange(self.C, dtype=torch.int32).repeat(self.R, 1)[:, :self.K].contiguous()
        return create_random_topology(self.R, self.C, self.K, _topology_seed(self.out_features, self.in_features))

    @property
    def config(self) -> BlockELLConfig:
        return BlockELLConfig(R=self.R, C=self.C, K=self.K, B=self.tile_size)

    def refresh(self) -> None:
        """Drop the cached kernel copies (after writes through ``.data``)."""
        self._kcache = {}

    def _cached(self, name, key, make):
        cache = self.__dict__.setdefault("_kcache", {})
        hit = cache.get(name)
        if hit is None or hit[0] != key:
            hit = (key, make())
            cache[name] = hit
        return hit[1]

    def effective_col_indices(self) -> torch.Tensor:
        """col_indices with dead slots set to -1 (skipped by the kernel)."""
        ci, am = self.col_indices, self.alive_mask
        key = (ci.data_ptr(), ci._version, am.data_ptr(), am._version)
        return self._cached("cols", key, lambda: torch.where(am, ci, torch.full_like(ci, -1)).to(torch.int32)
                            .contiguous())

    def kernel_values(self) -> torch.Tensor:
        """The tiles the kernels read (``values`` in the compute dtype)."""
        v = self.values
        if v.dtype == self.dtype and v.is_contiguous():
            return v.detach()
        key = (v.data_ptr(), v._version, v.dtype)
        return self._cached("values", key, lambda: v.detach().to(self.dtype).contiguous())

    def as_block_ell(self) -> BlockELLTensor:
        return BlockELLTensor(values=self.kernel_values(), col_indices=self.effective_col_indices(), config=self.config)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        x2 = x.reshape(-1, self.in_features).to(self.dtype)
        if self.dtype == torch.bfloat16:
            from ..kernels.autograd import block_ell_linear_ad
            y = block_ell_linear_ad(x2, self.values, self.effective_col_indices(), compute=self.kernel_values())
        else:  # fp32 accuracy path
            from ..kernels.autograd import block_ell_linear_f32_ad
            y = block_ell_linear_f32_ad(x2, self.values, self.effective_col_indices(), compute=self.kernel_values())
        if self.bias is not None:
            y = y + self.bias.to(y.dtype)
        return y.reshape(*lead, self.out_features)


class MLPBlock(nn.Module):
    """MLP block on Block-ELL weights (reference mlp.py:98-168).

    SwiGLU: ``w_down(silu(w_gate(x)) * w_up(x))`` as one fused forward;
    otherwise the GELU MLP ``fc2(gelu(fc1(x)))``.
    """

    def __init__(self, d_model: int, d_ff: int, use_swiglu: bool = False, dropout: float = 0.0, tile_size: int = 16,
                 density: float = 1.0, dtype: torch.dtype = torch.bfloat16, device=None):
        super().__init__()
        self.d_model, self.d_ff, self.use_swiglu, self.dropout = d_model, d_ff, use_swiglu, dropout
        self.tile_size, self.density, self.dtype = tile_size, density, dtype
        kw = dict(tile_size=tile_size, density=density, dtype=dtype, device=device)
        if use_swiglu:
            self.w_gate = BlockELLLinear(d_ff, d_model, bias=False, **kw)
            self.w_up = BlockELLLinear(d_ff, d_model, bias=False, **kw)
            self.w_down = BlockELLLinear(d_model, d_ff, bias=False, **kw)
            # gate and up are seeded alike, so their topologies start identical (reference
            # mlp.py:84-95); code that edits one topology should clear this hint
            self.gate_up_shared = bool(torch.equal(self.w_gate.col_indices, self.w_up.col_indices))
        else:
            self.fc1 = BlockELLLinear(d_ff, d_model, **kw)
            self.fc2 = BlockELLLinear(d_model, d_ff, **kw)

    def forward(self, x: torch.Tensor, deterministic: bool = True, residual: bool = False) -> torch.Tensor:
        if self.use_swiglu:
            lead = x.shape[:-1]
            x2 = x.reshape(-1, self.d_model).to(self.dtype)
            g, u, d = self.w_gate, self.w_up, self.w_down
            if self.dtype == torch.bfloat16:
                from ..kernels.autograd import block_ell_swiglu_ad
                out = block_ell_swiglu_ad(x2, g.values, g.kernel_values(), g.effective_col_indices(), u.values,
                                          u.kernel_values(), u.effective_col_indices(), d.values, d.kernel_values(),
                                          d.effective_col_indices(), add_residual=residual,
                                          shared_topology=self.gate_up_shared)
            elif torch.is_grad_enabled() and (x2.requires_grad or any(w.values.requires_grad for w in (g, u, d))):
                # fp32 training: the three differentiable fp32 projections
                # (the fused fp32 kernel has no backward of its own)
                hh = F.silu(g(x2)) * u(x2)
                out = d(hh) + (x2 if residual else 0)
            else:  # fp32 inference: the fused fp32 kernel
                from ..kernels.ops import block_ell_swiglu_fwd
                out = block_ell_swiglu_fwd(x2.contiguous(), g.kernel_values(), g.effective_col_indices(),
                                           u.kernel_values(), u.effective_col_indices(), d.kernel_values(),
                                           d.effective_col_indices(), add_residual=residual)
            out = out.reshape(*lead, self.d_model)
        else:
            out = self.fc2(F.gelu(self.fc1(x)))
            if residual:
                out = out + x
        if self.dropout > 0.0 and not deterministic:
            out = F.dropout(out, p=self.dropout, training=True)
        return out
