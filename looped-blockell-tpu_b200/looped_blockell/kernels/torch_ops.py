"""The reference's native op names under ``torch.ops.titan``.

The reference extension registers its CUDA ops with ``TORCH_LIBRARY_FRAGMENT
(titan, ...)`` (csrc/block_ell/block_ell_ops.cpp:49-98, csrc/loop/loop_ops.cpp:
36-67) and Meta implementations so traced code sees the output shapes
(block_ell_ops.cpp:179-237).  ``register()`` defines the same schemas here and
routes the CUDA dispatch key to this package's sm_100a kernels, so code
written against ``torch.ops.titan.block_ell_swiglu_fwd(...)`` runs unchanged.

Like the reference's native ops, these take ``[B_out, B_in]`` weight tiles
(the reference CUDA kernels' layout); the Python ops in ``kernels.ops`` default
to the JAX ``[B_in, B_out]`` layout.  The Meta implementation takes d_ff from
``v_gate.size(0) * v_gate.size(2)`` (the reference hard-codes a tile size of
16 there, block_ell_ops.cpp:208).  There is no CPU kernel: CPU tensors fail at
dispatch, as with the reference extension.  ``block_ell_swiglu_bwd`` returns
``(dx, d_v_gate, d_v_up, d_v_down)`` with ``grad_out`` added into ``dx``, as the
reference op does (swiglu_bwd.cu:785-796).
"""

from __future__ import annotations

from typing import List

import torch

from . import backward as _bwd
from . import loop as _loop
from . import ops as _ops

_LIB = None

_SCHEMAS = {
    "block_ell_swiglu_fwd": "block_ell_swiglu_fwd(Tensor x, Tensor v_gate, Tensor ci_gate, Tensor v_up, "
                            "Tensor ci_up, Tensor v_down, Tensor ci_down, bool add_residual) -> Tensor",
    "block_ell_swiglu_fwd_with_intermediate":
        "block_ell_swiglu_fwd_with_intermediate(Tensor x, Tensor v_gate, Tensor ci_gate, Tensor v_up, "
        "Tensor ci_up, Tensor v_down, Tensor ci_down, bool add_residual) -> (Tensor, Tensor, Tensor, Tensor)",
    "block_ell_swiglu_bwd": "block_ell_swiglu_bwd(Tensor grad_out, Tensor x, Tensor gate_pre_act, Tensor up_out, "
                            "Tensor h, Tensor v_gate, Tensor ci_gate, Tensor v_up, Tensor ci_up, Tensor v_down, "
                            "Tensor ci_down) -> (Tensor, Tensor, Tensor, Tensor)",
    "pin_weights_l2": "pin_weights_l2(Tensor[] weights) -> ()",
    "unpin_weights_l2": "unpin_weights_l2() -> ()",
    "persistent_mlp_step": "persistent_mlp_step(Tensor h, Tensor e, Tensor log_A, Tensor log_dt, "
                           "Tensor[] norm_scales, Tensor[] gate_values, Tensor[] gate_col_idx, Tensor[] up_values, "
                           "Tensor[] up_col_idx, Tensor[] down_values, Tensor[] down_col_idx) -> Tensor",
}


def _fwd_cuda(x, v_gate, ci_gate, v_up, ci_up, v_down, ci_down, add_residual):
    return _ops.block_ell_swiglu_fwd(x, v_gate, ci_gate, v_up, ci_up, v_down, ci_down, add_residual=add_residual,
                                     layout=_ops.TILE_OUT_IN)


def _fwd_int_cuda(x, v_gate, ci_gate, v_up, ci_up, v_down, ci_down, add_residual):
    return tuple(_ops.block_ell_swiglu_fwd_with_intermediate(x, v_gate, ci_gate, v_up, ci_up, v_down, ci_down,
                                                             add_residual=add_residual, layout=_ops.TILE_OUT_IN))


def _fwd_meta(x, v_gate, ci_gate, v_up, ci_up, v_down, ci_down, add_residual):
    return torch.empty_like(x)


def _fwd_int_meta(x, v_gate, ci_gate, v_up, ci_up, v_down, ci_down, add_residual):
    d_ff = v_gate.size(0) * v_gate.size(2)
    mid = x.new_empty((x.size(0), d_ff))
    return torch.empty_like(x), mid, torch.empty_like(mid), torch.empty_like(mid)


def _bwd_cuda(grad_out, x, gate_pre_act, up_out, h, v_gate, ci_gate, v_up, ci_up, v_down, ci_down):
    return tuple(_bwd.block_ell_swiglu_bwd(grad_out, x, gate_pre_act, up_out, h, v_gate, ci_gate, v_up, ci_up,
                                           v_down, ci_down, layout=_ops.TILE_OUT_IN))


def _bwd_meta(grad_out, x, gate_pre_act, up_out, h, v_gate, ci_gate, v_up, ci_up, v_down, ci_down):
    return torch.empty_like(x), torch.empty_like(v_gate), torch.empty_like(v_up), torch.empty_like(v_down)


def _pin(weights: List[torch.Tensor]):
    _loop.pin_weights_l2(weights)


def _unpin():
    _loop.unpin_weights_l2()


def _step_cuda(h, e, log_A, log_dt, norm_scales, gate_values, gate_col_idx, up_values, up_col_idx, down_values,
               down_col_idx):
    # the reference op's RMSNorm eps (persistent_core.cu:317)
    return _loop.persistent_mlp_step(h, e, log_A, log_dt, norm_scales, gate_values, gate_col_idx, up_values,
                                     up_col_idx, down_values, down_col_idx, eps=1e-6, layout=_ops.TILE_OUT_IN)


def _step_meta(h, e, log_A, log_dt, norm_scales, gate_values, gate_col_idx, up_values, up_col_idx, down_values,
               down_col_idx):
    return torch.empty_like(h)


def registered() -> bool:
    return _LIB is not None


def register() -> bool:
    """Define the ``titan::`` ops (once).  Returns False, defining nothing,
    when ``torch.ops.titan.block_ell_swiglu_fwd`` already exists (e.g. the
    reference extension is loaded in this process)."""
    global _LIB
    if _LIB is not None:
        return True
    try:
        torch.ops.titan.block_ell_swiglu_fwd  # noqa: B018
        return False
    except (AttributeError, RuntimeError):
        pass
    lib = torch.library.Library("titan", "FRAGMENT")
    for schema in _SCHEMAS.values():
        lib.define(schema)
    lib.impl("block_ell_swiglu_fwd", _fwd_cuda, "CUDA")
    lib.impl("block_ell_swiglu_fwd", _fwd_meta, "Meta")
    lib.impl("block_ell_swiglu_fwd_with_intermediate", _fwd_int_cuda, "CUDA")
    lib.impl("block_ell_swiglu_fwd_with_intermediate", _fwd_int_meta, "Meta")
    lib.impl("block_ell_swiglu_bwd", _bwd_cuda, "CUDA")
    lib.impl("block_ell_swiglu_bwd", _bwd_meta, "Meta")
    lib.impl("pin_weights_l2", _pin, "CompositeExplicitAutograd")
    lib.impl("unpin_weights_l2", _unpin, "CompositeExplicitAutograd")
    lib.impl("persistent_mlp_step", _step_cuda, "CUDA")
    lib.impl("persistent_mlp_step", _step_meta, "Meta")
    _LIB = lib
    return True
