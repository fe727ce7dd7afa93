"""Permutation of the internal d_ff dimension of an MLP so that alive tiles
cluster at low d_ff indices (reference looped_blockell/opt/column_reorder.py).

Naming follows the reference: ``fc1`` is the weight whose *column indices*
point into d_ff, ``fc2`` the weight with one *block-row* per d_ff tile-column
(R == C_ff).  In the SwiGLU of this package the down projection indexes d_ff
by column and gate/up have d_ff block-rows; ``reorder_swiglu_dff`` applies
one permutation to all three, which leaves the FFN's output unchanged.
"""

from __future__ import annotations

from typing import Any, Tuple

import torch
from torch.utils._pytree import tree_map


def compute_column_importance(fc1_alive_mask: torch.Tensor, fc2_alive_mask: torch.Tensor,
                              fc1_col_indices: torch.Tensor, fc2_col_indices: torch.Tensor,
                              C_ff: int) -> torch.Tensor:
    """[C_ff] f32: alive fc1 tiles whose column is c, plus the alive tiles of
    fc2 block-row c (reference :36-98; fc2 rows beyond C_ff are dropped, missing
    ones count 0; fc1 sentinels (-1) count nothing)."""
    cols = fc1_col_indices.reshape(-1).long()
    alive = fc1_alive_mask.reshape(-1).to(torch.float32)
    valid = (cols >= 0).to(torch.float32)
    imp = torch.zeros(C_ff, dtype=torch.float32, device=cols.device)
    imp.scatter_add_(0, cols.clamp(0, C_ff - 1), alive * valid)
    rows = fc2_alive_mask.to(torch.float32).sum(dim=1)
    n = min(rows.shape[0], C_ff)
    imp[:n] += rows[:n]
    return imp


def compute_permutation(importance: torch.Tensor) -> torch.Tensor:
    """[C_ff] int32, most important d_ff column first (reference :105-120: an
    argsort of -importance; equal importances keep ascending index order)."""
    return torch.argsort(-importance, stable=True).to(torch.int32)


def apply_permutation_to_block_ell(values: torch.Tensor, col_indices: torch.Tensor, alive_mask: torch.Tensor,
                                   perm: torch.Tensor, is_column_dim: bool = True
                                   ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """``perm[new] = old`` (reference :127-176).  Column dim (fc1): remap
    ``col_indices`` through the inverse permutation, sentinels stay -1, tiles
    stay in their slots.  Row dim (fc2): reorder block-rows by ``perm``."""
    p = perm.long()
    if is_column_dim:
        inv = torch.empty_like(p)
        inv[p] = torch.arange(p.numel(), device=p.device)
        safe = col_indices.long().clamp(0, p.numel() - 1)
        new_cols = torch.where(col_indices < 0, torch.full_like(col_indices, -1), inv[safe].to(col_indices.dtype))
        return values, new_cols, alive_mask
    return values[p], col_indices[p], alive_mask[p]


def compute_k_active_macros(alive_mask: torch.Tensor, col_indices: torch.Tensor, tiles_per_macro: int,
                            C_ff: int) -> torch.Tensor:
    """ceil((largest alive column + 1) / tiles_per_macro), 0 when nothing is
    alive (reference :236-268)."""
    safe = torch.where(alive_mask.to(torch.bool), col_indices, torch.full_like(col_indices, -1))
    mx = safe.max().to(torch.float32) if safe.numel() else torch.tensor(-1.0, device=col_indices.device)
    return torch.where(mx < 0, torch.zeros((), dtype=torch.int32, device=mx.device),
                       torch.ceil((mx + 1) / tiles_per_macro).to(torch.int32))


def _permute_opt_leaves(opt_state: Any, perm: torch.Tensor, C_ff: int) -> Any:
    """Moments shaped like fc2 (first dim C_ff) follow its row reorder; fc1's
    tiles do not move, so its moments stay (reference :183-233)."""
    p = perm.long()
    return tree_map(lambda t: t[p] if isinstance(t, torch.Tensor) and t.dim() >= 1 and t.shape[0] == C_ff else t,
                    opt_state)


def full_reorder_step(fc1_values, fc1_col_indices, fc1_alive, fc2_values, fc2_col_indices, fc2_alive,
                      opt_state: Any, C_ff: int, tiles_per_macro: int):
    """Importance -> permutation -> fc1 column remap -> fc2 row reorder ->
    optimizer moments -> active macro count (reference :276-345).  Returns
    ``(fc1_vals, fc1_cols, fc1_alive, fc2_vals, fc2_cols, fc2_alive,
    opt_state, k_active_macros)``."""
    imp = compute_column_importance(fc1_alive, fc2_alive, fc1_col_indices, fc2_col_indices, C_ff)
    perm = compute_permutation(imp)
    v1, c1, a1 = apply_permutation_to_block_ell(fc1_values, fc1_col_indices, fc1_alive, perm, is_column_dim=True)
    v2, c2, a2 = apply_permutation_to_block_ell(fc2_values, fc2_col_indices, fc2_alive, perm, is_column_dim=False)
    opt_state = _permute_opt_leaves(opt_state, perm, C_ff) if opt_state is not None else None
    k_active = compute_k_active_macros(a1, c1, tiles_per_macro, C_ff)
    return v1, c1, a1, v2, c2, a2, opt_state, k_active


def reorder_swiglu_dff(vg, cg, vu, cu, vd, cd, tiles_per_macro: int = 1):
    """One d_ff permutation for a SwiGLU: gate and up block-rows reordered,
    down column indices remapped.  Alive = column index >= 0.  Importance
    counts the down tiles per d_ff column and the gate and up tiles per d_ff
    block-row.  Returns ``(vg, cg, vu, cu, vd, cd, perm, k_active)``; the FFN
    computes the same function afterwards."""
    C_ff = vg.shape[0]
    ag, au, ad = cg >= 0, cu >= 0, cd >= 0
    imp = compute_column_importance(ad, ag, cd, cg, C_ff)
    imp += au.to(torch.float32).sum(dim=1)
    perm = compute_permutation(imp)
    vd2, cd2, _ = apply_permutation_to_block_ell(vd, cd, ad, perm, is_column_dim=True)
    vg2, cg2, _ = apply_permutation_to_block_ell(vg, cg, ag, perm, is_column_dim=False)
    vu2, cu2, _ = apply_permutation_to_block_ell(vu, cu, au, perm, is_column_dim=False)
    k_active = compute_k_active_macros(cd2 >= 0, cd2, tiles_per_macro, C_ff)
    return vg2, cg2, vu2, cu2, vd2, cd2, perm, k_active
