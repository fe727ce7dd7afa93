"""Dense weight -> Block-ELL on the GPU (``bell_dense_to_ell``).

Reference: ``create_block_ell_from_dense`` (looped_blockell/layers/block_ell.py:
79-116) keeps, per block-row, the K = max(1, int(C * density)) tiles of largest
Frobenius norm, kept columns ascending.  Two launches of this package's
kernels: the tile norms (one streaming pass over the matrix) and, per
block-row, the ranking and the copy of the kept tiles in the requested layout.
"""

from __future__ import annotations

import ctypes as C
from typing import Tuple

import torch

from . import _lib
from .ops import TILE_IN_OUT, _check_cuda, _stream


def dense_to_block_ell(dense: torch.Tensor, tile_size: int, density: float = 0.5, layout: int = TILE_IN_OUT,
                       K: int = 0) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Returns ``(values [R, K, B, B], col_indices [R, K] int32, norms [R, C] f32)``.

    ``dense`` is ``[out_features, in_features]`` (bf16 or fp32, CUDA); B is 64
    or 128.  ``K`` overrides ``max(1, int(C * density))`` when positive.
    Ties in norm keep the lower column (a stable descending sort)."""
    _check_cuda("dense", dense)
    if dense.dim() != 2:
        raise RuntimeError("dense must be 2D [out_features, in_features]")
    if dense.dtype not in (torch.bfloat16, torch.float32):
        raise RuntimeError("dense must be bf16 or fp32")
    out_f, in_f = dense.shape
    B = int(tile_size)
    if out_f % B or in_f % B:
        raise ValueError(f"Dimensions ({out_f}, {in_f}) must be divisible by tile_size {B}")
    R, Cb = out_f // B, in_f // B
    K = int(K) if K > 0 else max(1, int(Cb * density))
    dense = dense.contiguous()
    values = torch.empty((R, K, B, B), dtype=dense.dtype, device=dense.device)
    cols = torch.empty((R, K), dtype=torch.int32, device=dense.device)
    norms = torch.empty((R, Cb), dtype=torch.float32, device=dense.device)
    d = _lib.BellDenseToEllDesc()
    d.dense = dense.data_ptr()
    d.dtype = _lib.BELL_DTYPE_BF16 if dense.dtype == torch.bfloat16 else _lib.BELL_DTYPE_F32
    d.out_features, d.in_features, d.B, d.K, d.layout = out_f, in_f, B, K, layout
    d.values, d.col_indices, d.norms = values.data_ptr(), cols.data_ptr(), norms.data_ptr()
    with torch.cuda.device(dense.device):
        _lib.check(_lib.load().bell_dense_to_ell(C.byref(d), _stream()), "dense_to_block_ell")
    return values, cols, norms
