"""Weights from the reference's checkpoints into the Block-ELL container.

The reference converts checkpoints between its PyTorch and JAX models
(interop/convert_checkpoint.py); the MLP weights pass through
``_dense_to_block_ell`` (density 1.0, :114-131) and ``_block_ell_to_dense``
(:134-148).  Its PyTorch MLP (interop/pt_model.py:858-870) keeps
``w_gate / w_up / w_down`` as dense ``[out, in]`` weights, with a
``tile_mask [R, C]`` of alive tiles when prunable (:602-636).  These helpers
load such weights straight into the ``(values, col_indices)`` triple the
forward takes, on the weights' device: CUDA weights go through the GPU
conversion kernels (``kernels.convert``) at tile sizes 64 and 128.
"""

from __future__ import annotations

from typing import Dict, Mapping, Optional, Tuple

import torch

from .layers.block_ell import block_ell_to_dense, BlockELLConfig, BlockELLTensor, create_block_ell_from_dense

TILE_IN_OUT = 0
TILE_OUT_IN = 1


def dense_to_block_ell_full(weight: torch.Tensor, tile_size: int = 16) -> Tuple[torch.Tensor, torch.Tensor]:
    """Every tile of ``weight [out, in]``, columns in order (density 1.0):
    ``values [R, C, B_in, B_out]``, ``col_indices [R, C]`` — reference
    ``_dense_to_block_ell`` (convert_checkpoint.py:114-131)."""
    out_f, in_f = weight.shape
    be = create_block_ell_from_dense(weight, tile_size=tile_size, density=1.0)
    return be.values, be.col_indices


def block_ell_to_dense_weight(values: torch.Tensor, col_indices: torch.Tensor, out_features: int,
                              in_features: int) -> torch.Tensor:
    """Dense ``[out, in]`` from ``[B_in, B_out]`` tiles — reference
    ``_block_ell_to_dense`` (convert_checkpoint.py:134-148); dead slots (-1)
    are skipped, duplicate columns add."""
    R, K, B, _ = values.shape
    if out_features != R * B or in_features % B:
        raise ValueError("shape mismatch between the tiles and [out_features, in_features]")
    t = BlockELLTensor.__new__(BlockELLTensor)  # K may exceed C when columns repeat
    cfg = BlockELLConfig.__new__(BlockELLConfig)
    cfg.R, cfg.C, cfg.K, cfg.B = R, in_features // B, K, B
    t.values, t.col_indices, t.config = values, col_indices, cfg
    return block_ell_to_dense(t)


def masked_dense_to_block_ell(weight: torch.Tensor, tile_mask: torch.Tensor,
                              tile_size: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """The alive tiles of a pruned dense weight (``tile_mask [R, C]`` True =
    alive, as PrunableLinear keeps it, pt_model.py:630): per block-row the
    alive columns in ascending order, K = the largest alive count (>= 1),
    shorter rows padded with dead slots (-1, zero tiles)."""
    out_f, in_f = weight.shape
    B = tile_size
    R, C = out_f // B, in_f // B
    mask = tile_mask.to(torch.bool).to(weight.device)
    if tuple(mask.shape) != (R, C):
        raise ValueError(f"tile_mask shape {tuple(mask.shape)} != {(R, C)}")
    K = max(1, int(mask.sum(dim=1).max().item()) if R else 1)
    order = torch.argsort((~mask).to(torch.int8), dim=1, stable=True)[:, :K]  # alive columns first, ascending
    alive = torch.gather(mask, 1, order)
    cols = torch.where(alive, order, torch.full_like(order, -1)).to(torch.int32)
    blocks = weight.reshape(R, B, C, B).permute(0, 2, 3, 1)  # [R, C, B_in, B_out]
    vals = torch.gather(blocks, 1, order[:, :, None, None].expand(R, K, B, B))
    vals = torch.where(alive[:, :, None, None], vals, torch.zeros_like(vals)).contiguous()
    return vals, cols


def swiglu_from_state_dict(state_dict: Mapping[str, torch.Tensor], prefix: str = "", tile_size: int = 64,
                           density: Optional[float] = None, device=None, dtype=torch.bfloat16,
                           layout: int = TILE_IN_OUT) -> Dict[str, torch.Tensor]:
    """``{vg, cg, vu, cu, vd, cd}`` for ``block_ell_swiglu_fwd`` from the
    reference PyTorch MLP's ``{prefix}w_gate.weight`` / ``w_up`` / ``w_down``
    (pt_model.py:861-867).  A ``{name}.tile_mask`` in the state dict selects
    the alive tiles; otherwise ``density`` keeps the top-K tiles by norm
    (None: every tile).  Tiles come out in ``layout``."""
    out = {}
    for short, key in (("g", "w_gate"), ("u", "w_up"), ("d", "w_down")):
        w = state_dict[f"{prefix}{key}.weight"]
        w = w.to(device=device or w.device, dtype=dtype)
        mask = state_dict.get(f"{prefix}{key}.tile_mask")
        if mask is not None:
            v, c = masked_dense_to_block_ell(w, mask, tile_size)
        elif density is None:
            v, c = dense_to_block_ell_full(w, tile_size)
        else:
            be = create_block_ell_from_dense(w, tile_size=tile_size, density=density)
            v, c = be.values, be.col_indices
        if layout == TILE_OUT_IN:
            v = v.transpose(-1, -2).contiguous()
        out["v" + short], out["c" + short] = v, c
    return out
