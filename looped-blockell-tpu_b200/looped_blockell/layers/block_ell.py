"""Block-ELL sparse format — the reference's op surface, in PyTorch.

Same names and meaning as looped_blockell/layers/block_ell.py of the
reference: ``values [R, K, B, B]`` dense tiles, ``col_indices [R, K]`` int32,
logical weight ``[out_features, in_features] = [R*B, C*B]``, tiles stored
``[B_in, B_out]`` (the JAX/Flax convention, block_ell.py:96-99).  A column
index of -1 is a dead slot (looped_blockell/opt/column_reorder.py:131-136).

``block_ell_matmul`` runs the sm_100a kernel; CUDA tensors only.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Union

import torch


@dataclass
class BlockELLConfig:
    """Reference block_ell.py:19-50."""
    R: int
    C: int
    K: int
    B: int = 16

    def __post_init__(self) -> None:
        if self.K > self.C:
            raise ValueError(f"K ({self.K}) cannot exceed C ({self.C})")
        if any(v < 1 for v in (self.R, self.C, self.K, self.B)):
            raise ValueError("R, C, K, B must all be >= 1")

    @property
    def out_features(self) -> int:
        return self.R * self.B

    @property
    def in_features(self) -> int:
        return self.C * self.B

    @property
    def total_blocks(self) -> int:
        return self.R * self.K

    @property
    def total_parameters(self) -> int:
        return self.R * self.K * self.B * self.B

    @property
    def density(self) -> float:
        return self.K / self.C


@dataclass
class BlockELLTensor:
    """Reference block_ell.py:53-66 (shape validation included)."""
    values: torch.Tensor       # [R, K, B, B]
    col_indices: torch.Tensor  # [R, K] int32
    config: BlockELLConfig

    def __post_init__(self) -> None:
        cfg = self.config
        expected_v = (cfg.R, cfg.K, cfg.B, cfg.B)
        expected_i = (cfg.R, cfg.K)
        if tuple(self.values.shape) != expected_v:
            raise ValueError(f"values shape {tuple(self.values.shape)} != expected {expected_v}")
        if tuple(self.col_indices.shape) != expected_i:
            raise ValueError(f"col_indices shape {tuple(self.col_indices.shape)} != expected {expected_i}")


def create_random_topology(R: int, C: int, K: int, key: Union[int, torch.Generator, None] = None,
                           device: Union[str, torch.device] = "cpu", sort: bool = False) -> torch.Tensor:
    """col_indices [R, K] int32 with K unique columns per row (reference
    block_ell.py:69-76).  ``key`` is a seed or a torch.Generator (the JAX
    PRNGKey's role); ``sort=True`` sorts each row."""
    if K > C:
        raise ValueError(f"K ({K}) cannot exceed C ({C})")
    g = key if isinstance(key, torch.Generator) else torch.Generator().manual_seed(int(key or 0))
    cols = torch.argsort(torch.rand(R, C, generator=g), dim=1)[:, :K].to(torch.int32)
    if sort:
        cols = torch.sort(cols, dim=1).values
    return cols.to(device)


def create_block_ell_from_dense(dense: torch.Tensor, tile_size: int = 16, density: float = 0.5) -> BlockELLTensor:
    """Dense ``[out, in]`` -> Block-ELL keeping the top-K Frobenius-norm tiles
    per block-row, columns sorted (reference block_ell.py:79-116).

    A CUDA bf16/fp32 matrix with the kernels' tile sizes (64, 128) is
    converted by ``kernels.convert.dense_to_block_ell`` (two sm_100a
    launches).  Other tile sizes and host tensors — the reference's JAX code
    runs this step wherever the weights live — use the tensor expression
    below, which computes the same thing."""
    out_f, in_f = dense.shape
    B = tile_size
    if out_f % B != 0 or in_f % B != 0:
        raise ValueError(f"Dimensions ({out_f}, {in_f}) must be divisible by tile_size {B}")
    R, C = out_f // B, in_f // B
    K = max(1, int(C * density))
    if dense.is_cuda and B in (64, 128) and dense.dtype in (torch.bfloat16, torch.float32) and C <= 2048:
        from ..kernels.convert import dense_to_block_ell
        values, cols, _ = dense_to_block_ell(dense, B, K=K)
        return BlockELLTensor(values=values, col_indices=cols, config=BlockELLConfig(R=R, C=C, K=K, B=B))
    blocks = dense.reshape(R, B, C, B).permute(0, 2, 3, 1)  # [R, C, B_in, B_out]
    norms = blocks.float().pow(2).sum(dim=(2, 3)).sqrt()
    top = torch.argsort(-norms, dim=1, stable=True)[:, :K]
    cols = torch.sort(top, dim=1).values
    values = torch.gather(blocks, 1, cols[:, :, None, None].expand(R, K, B, B)).contiguous()
    return BlockELLTensor(values=values, col_indices=cols.to(torch.int32), config=BlockELLConfig(R=R, C=C, K=K, B=B))


def block_ell_to_dense(block_ell: BlockELLTensor) -> torch.Tensor:
    """Scatter to dense ``[out, in]`` (reference block_ell.py:118-146);
    dead slots are skipped."""
    cfg = block_ell.config
    R, K, B, C = cfg.R, cfg.K, cfg.B, cfg.C
    v = block_ell.values
    dense = torch.zeros(R, C, B, B, dtype=v.dtype, device=v.device)  # [R, C, B_out, B_in]
    cols = block_ell.col_indices.long()
    live = cols >= 0
    r_idx = torch.arange(R, device=v.device)[:, None].expand(R, K)[live]
    dense.index_put_((r_idx, cols[live]), v.transpose(-1, -2)[live], accumulate=True)
    return dense.permute(0, 2, 1, 3).reshape(R * B, C * B)


def block_ell_matmul(x: torch.Tensor, block_ell: BlockELLTensor, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``x [..., in_features] -> [..., out_features]`` on the sm_100a kernel
    (reference block_ell.py:149-182: ``y = x @ W^T`` over the live tiles).

    Differentiable in ``x``, ``block_ell.values`` and ``residual``, as the
    reference's is (tests/test_block_ell.py:57-72): the backward runs the
    transposed Block-ELL product and the tile-gradient kernel, and the values'
    gradient comes back in their own dtype."""
    cfg = block_ell.config
    lead = x.shape[:-1]
    if x.shape[-1] != cfg.in_features:
        raise ValueError(f"x last dim {x.shape[-1]} != in_features {cfg.in_features}")
    x2 = x.reshape(-1, cfg.in_features)
    res2 = None if residual is None else residual.reshape(-1, cfg.out_features).to(x.dtype)
    cols = block_ell.col_indices.to(torch.int32)
    if x.dtype == torch.bfloat16:
        from ..kernels.autograd import block_ell_linear_ad
        y = block_ell_linear_ad(x2.contiguous(), block_ell.values, cols, residual=res2)
    else:
        from ..kernels.autograd import block_ell_linear_f32_ad
        y = block_ell_linear_f32_ad(x2.contiguous(), block_ell.values, cols, residual=res2)
    return y.reshape(*lead, cfg.out_features)
