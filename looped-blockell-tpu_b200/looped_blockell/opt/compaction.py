"""Physical compaction of a Block-ELL layer: pack the alive tiles of each
block-row to the front and shrink K (reference looped_blockell/opt/compaction.py:
31-61, ``compact_single_layer``)."""

from __future__ import annotations

from typing import Tuple

import torch


def compact_single_layer(values: torch.Tensor, col_indices: torch.Tensor,
                         alive_mask: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, int]:
    """Returns ``(new_values, new_col_indices, new_alive_mask, K_new)``.

    Per row, alive slots move to the front in their original order (a stable
    sort on "not alive"), then every row is cut to ``K_new`` = the largest
    alive count (at least 1).  As in the reference, a dead slot that survives
    the cut keeps its column index and tile; ``new_alive_mask`` marks it.
    """
    R, K_old = col_indices.shape
    alive = alive_mask.to(torch.bool)
    K_new = max(1, int(alive.sum(dim=1).max().item()) if R else 1)
    order = torch.argsort((~alive).to(torch.int8), dim=1, stable=True)[:, :K_new]
    new_values = torch.gather(values, 1, order[:, :, None, None].expand(R, K_new, *values.shape[2:]))
    new_cols = torch.gather(col_indices, 1, order)
    new_alive = torch.gather(alive, 1, order)
    return new_values.contiguous(), new_cols.contiguous(), new_alive.contiguous(), K_new
