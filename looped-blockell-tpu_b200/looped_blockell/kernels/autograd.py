"""Differentiable Block-ELL ops for training through the layers.

The reference layers are trainable Flax modules: gradients flow into the
tile values of ``block_ell_matmul`` (reference tests/test_block_ell.py:57-72)
and through ``MLPBlock`` (looped_blockell/layers/mlp.py:46-82, 119-145).
These autograd nodes run both directions on this package's kernels:

* ``BlockEllLinearFn`` — ``y = x W^T``: forward ``bell_linear_bf16``; backward
  ``dx = dy W`` as a linear over the transposed Block-ELL (same tile bytes,
  other tile layout) and ``dW`` from the tile-gradient kernel
  (``bell_sddmm_bf16``), summed in fp32.
* ``BlockEllSwiGLUFn`` — the fused SwiGLU forward with intermediates and the
  five-launch backward of ``kernels.backward``.

Both take the trainable ``master`` tensors (any float dtype, typically fp32
``nn.Parameter``s) next to the bf16 ``compute`` copies the kernels read, and
return the weight gradients for the masters in fp32 (cast to the master's
dtype), so optimizers see full-precision sums.  Column indices get no
gradient; dead slots (-1) get zero gradient, as the reference's alive_mask
multiplication gives.
"""

from __future__ import annotations

import torch

from .backward import block_ell_sddmm, block_ell_swiglu_bwd, transpose_ell
from .ops import TILE_IN_OUT, block_ell_linear, block_ell_swiglu_fwd_with_intermediate


class BlockEllLinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, master, compute, cols, layout, residual=None):
        y = block_ell_linear(x, compute, cols, residual=residual, layout=layout)
        ctx.save_for_backward(x, compute, cols)
        ctx.layout = layout
        ctx.master_dtype = master.dtype
        ctx.has_residual = residual is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        x, compute, cols = ctx.saved_tensors
        R, K, B, _ = compute.shape
        dy = dy.to(compute.dtype).contiguous()
        dx = dw = dres = None
        if ctx.needs_input_grad[0]:
            vT, cT, lt = transpose_ell([compute], [cols], x.shape[1] // B, ctx.layout)
            dx = block_ell_linear(dy, vT, cT, layout=lt)
        if ctx.needs_input_grad[1]:
            dw = block_ell_sddmm(x, dy, cols, B, ctx.layout).to(ctx.master_dtype)
        if ctx.has_residual and ctx.needs_input_grad[5]:
            dres = dy
        return dx, dw, None, None, None, dres


def block_ell_linear_ad(x: torch.Tensor, master: torch.Tensor, cols: torch.Tensor, compute: torch.Tensor = None,
                        layout: int = TILE_IN_OUT, residual: torch.Tensor = None) -> torch.Tensor:
    """Differentiable ``y = x W^T (+ residual)``; ``x`` [N, in] bf16,
    ``master`` the trainable tiles, ``compute`` their bf16 copy (``master``
    itself when None)."""
    if compute is None:
        compute = master if master.dtype == torch.bfloat16 else master.detach().to(torch.bfloat16)
    return BlockEllLinearFn.apply(x, master, compute.contiguous(), cols, layout, residual)


class BlockEllLinearF32Fn(torch.autograd.Function):
    """fp32 ``y = x W^T``: forward and ``dx`` on the fp32 Block-ELL kernel
    (the transposed product for ``dx``), ``dW`` from ``bell_sddmm_f32``."""

    @staticmethod
    def forward(ctx, x, master, compute, cols, layout, residual=None):
        y = block_ell_linear(x, compute, cols, residual=residual, layout=layout)
        ctx.save_for_backward(x, compute, cols)
        ctx.layout = layout
        ctx.master_dtype = master.dtype
        ctx.has_residual = residual is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        x, compute, cols = ctx.saved_tensors
        B = compute.shape[2]
        dy = dy.to(torch.float32).contiguous()
        dx = dw = dres = None
        if ctx.needs_input_grad[0]:
            vT, cT, lt = transpose_ell([compute], [cols], x.shape[1] // B, ctx.layout)
            dx = block_ell_linear(dy, vT, cT, layout=lt)
        if ctx.needs_input_grad[1]:
            dw = block_ell_sddmm(x, dy, cols, B, ctx.layout).to(ctx.master_dtype)
        if ctx.has_residual and ctx.needs_input_grad[5]:
            dres = dy
        return dx, dw, None, None, None, dres


def block_ell_linear_f32_ad(x: torch.Tensor, master: torch.Tensor, cols: torch.Tensor, compute: torch.Tensor = None,
                            layout: int = TILE_IN_OUT, residual: torch.Tensor = None) -> torch.Tensor:
    """Differentiable fp32 ``y = x W^T (+ residual)`` (``x`` cast to fp32)."""
    if compute is None:
        compute = master.detach().to(torch.float32)
    return BlockEllLinearF32Fn.apply(x.to(torch.float32).contiguous(), master, compute.contiguous(), cols, layout,
                                     residual)


class BlockEllSwiGLUFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, m_gate, v_gate, ci_gate, m_up, v_up, ci_up, m_down, v_down, ci_down, add_residual, layout,
                shared_topology):
        out, h, g, u = block_ell_swiglu_fwd_with_intermediate(x, v_gate, ci_gate, v_up, ci_up, v_down, ci_down,
                                                              add_residual=add_residual, layout=layout,
                                                              shared_topology=shared_topology)
        ctx.save_for_backward(x, g, u, h, v_gate, ci_gate, v_up, ci_up, v_down, ci_down)
        ctx.add_residual = bool(add_residual)
        ctx.layout = layout
        ctx.dtypes = (m_gate.dtype, m_up.dtype, m_down.dtype)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        x, g, u, h, v_gate, ci_gate, v_up, ci_up, v_down, ci_down = ctx.saved_tensors
        dx, dvg, dvu, dvd = block_ell_swiglu_bwd(grad_out.to(torch.bfloat16).contiguous(), x, g, u, h, v_gate,
                                                 ci_gate, v_up, ci_up, v_down, ci_down, layout=ctx.layout,
                                                 add_residual=ctx.add_residual, fp32_weight_grads=True)
        dg, du, dd = (t.to(dt) for t, dt in zip((dvg, dvu, dvd), ctx.dtypes))
        return dx, dg, None, None, du, None, None, dd, None, None, None, None, None


def block_ell_swiglu_ad(x, m_gate, v_gate, ci_gate, m_up, v_up, ci_up, m_down, v_down, ci_down,
                        add_residual: bool = False, layout: int = TILE_IN_OUT, shared_topology: bool = False):
    """Differentiable fused SwiGLU: ``m_*`` the trainable tiles, ``v_*`` their
    bf16 copies (the kernels' operands)."""
    return BlockEllSwiGLUFn.apply(x, m_gate, v_gate, ci_gate, m_up, v_up, ci_up, m_down, v_down, ci_down,
                                  add_residual, layout, shared_topology)
