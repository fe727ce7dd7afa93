"""Backward of the bf16 Block-ELL SwiGLU — reference titan::block_ell_swiglu_bwd.

The reference op (csrc/block_ell/block_ell_ops.cpp:83-97, host code
csrc/block_ell/swiglu_bwd.cu:640-836) returns ``(dx, d_v_gate, d_v_up,
d_v_down)``, all bf16, with weight gradients accumulated in fp32 and cast on
return, and ``dx`` always including ``grad_out`` (the residual branch,
swiglu_bwd.cu:785-796).  Here the same result comes from five launches of this
package's sm_100a kernels:

1.+2. ``[d_gate | d_up]`` — at tile size 64 the forward linear kernel on the
   transposed down weight computes ``d_h = grad_out @ W_down`` in TMEM and its
   epilogue applies the SiLU*up backward, writing both halves of one
   ``[T, 2 d_ff]`` buffer (``bell_down_silu_bwd_bf16``; d_h never reaches
   memory).  At tile size 128 (or ``fuse_silu=False``) d_h is written in bf16
   and ``bell_silu_mul_bwd_bf16`` runs as its own pass, the reference's order;
3. ``dx = [d_gate | d_up] @ [W_gate ; W_up] + grad_out`` — one linear launch
   over the transposed, stacked gate/up weight with ``grad_out`` as the
   residual of its epilogue;
4. ``d_W_gate``, ``d_W_up``, ``d_W_down`` — ``bell_sddmm_bf16`` (tcgen05 tile
   gradients over the token dimension).

A transposed Block-ELL holds the same tile bytes regrouped by column and read
in the other tile layout, so the transposed products need no kernel of their
own.  Its topology (which tile lands where) depends only on the column
indices; it is built on the device once per column-index tensor (object and
version) and cached, and only the tile gather runs on every call.
"""

from __future__ import annotations

import ctypes as C
import weakref
from collections import OrderedDict
from typing import Optional, Sequence, Tuple

import torch

from . import _lib
from .ops import TILE_IN_OUT, TILE_OUT_IN, _check_cuda, _check_out, _ell, _stream, block_ell_linear, plan_bytes

# (C_blocks, ids of the column-index tensors) -> (weak references, versions, result).
# A hit needs the very same tensor objects (alive) at the same version: a new
# tensor that happens to reuse a freed tensor's memory or id never matches.
_TOPO_CACHE: "OrderedDict[tuple, tuple]" = OrderedDict()
_TOPO_CACHE_MAX = 16


def _topo_lookup(mats: Sequence[torch.Tensor], C_blocks: int):
    key = (C_blocks,) + tuple(id(m) for m in mats)
    hit = _TOPO_CACHE.get(key)
    if hit is None:
        return key, None
    refs, versions, result = hit
    if all(r() is m for r, m in zip(refs, mats)) and versions == tuple(m._version for m in mats):
        _TOPO_CACHE.move_to_end(key)
        return key, result
    del _TOPO_CACHE[key]
    return key, None


def transposed_topology(mats: Sequence[torch.Tensor], C_blocks: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Topology of the transpose of the row-stacked Block-ELL matrices ``mats``.

    ``mats`` are column-index tensors ``[R_i, K_i]`` over the same ``C_blocks``
    column blocks, stacked as block-rows ``0..R_0-1``, ``R_0..R_0+R_1-1``, ...
    Returns ``(cols_t, tile_idx)``, both ``[C_blocks, K_t]``: transposed row c
    lists the stacked block-rows that use column block c (ascending, duplicates
    kept), and ``tile_idx`` the position of that tile in the concatenation of
    the flattened value tensors.  Padding slots hold column -1 and tile 0.
    Dead slots (-1) and indices outside [0, C_blocks) are left out.  One
    device-to-host read (the maximum column count) sizes K_t.
    """
    key, hit = _topo_lookup(mats, C_blocks)
    if hit is not None:
        return hit
    dev = mats[0].device
    cs, rs, ts = [], [], []
    row_off = tile_off = 0
    for m in mats:
        R, K = m.shape
        cs.append(m.reshape(-1).long())
        rs.append(torch.arange(R, device=dev, dtype=torch.long).repeat_interleave(K) + row_off)
        ts.append(torch.arange(R * K, device=dev, dtype=torch.long) + tile_off)
        row_off += R
        tile_off += R * K
    c = torch.cat(cs)
    r = torch.cat(rs)
    t = torch.cat(ts)
    n = c.numel()
    live = (c >= 0) & (c < C_blocks)
    grp = torch.where(live, c, torch.full_like(c, C_blocks))
    # order by column block, then by tile position (which ascends with the
    # stacked block-row and the slot)
    order = torch.argsort(grp * max(n, 1) + t)
    grp_s, r_s, t_s = grp[order], r[order], t[order]
    counts = torch.zeros(C_blocks + 1, dtype=torch.long, device=dev).scatter_add_(0, grp, torch.ones_like(grp))
    K_t = max(1, int(counts[:C_blocks].max().item())) if C_blocks > 0 and n > 0 else 1
    starts = torch.cumsum(counts, 0) - counts
    pos = torch.arange(n, device=dev, dtype=torch.long) - starts[grp_s]
    keep = grp_s < C_blocks
    cols_t = torch.full((C_blocks, K_t), -1, dtype=torch.int32, device=dev)
    tile_idx = torch.zeros((C_blocks, K_t), dtype=torch.long, device=dev)
    cols_t[grp_s[keep], pos[keep]] = r_s[keep].to(torch.int32)
    tile_idx[grp_s[keep], pos[keep]] = t_s[keep]
    _TOPO_CACHE[key] = (tuple(weakref.ref(m) for m in mats), tuple(m._version for m in mats), (cols_t, tile_idx))
    while len(_TOPO_CACHE) > _TOPO_CACHE_MAX:
        _TOPO_CACHE.popitem(last=False)
    return cols_t, tile_idx


# (ids of the value and column tensors, C_blocks) -> (weak refs, versions, values_t):
# the gathered tiles of a transposed weight, reused while the same tensors
# keep the same contents (the optimizer bumps the version of what it updates)
_TILE_CACHE: "OrderedDict[tuple, tuple]" = OrderedDict()
_TILE_CACHE_MAX = 8


def transpose_ell(values: Sequence[torch.Tensor], cols: Sequence[torch.Tensor], C_blocks: int,
                  layout: int = TILE_IN_OUT) -> Tuple[torch.Tensor, torch.Tensor, int]:
    """Transposed Block-ELL of the row-stacked weights ``values[i]``/``cols[i]``.

    Returns ``(values_t [C_blocks, K_t, B, B], cols_t [C_blocks, K_t], layout_t)``.
    The tiles are the same bytes, gathered; ``layout_t`` is the other tile
    layout, which reads each tile as its transpose.  Both the topology and
    the gathered tiles are cached per (tensor, version), so a backward over
    unchanged weights gathers nothing.
    """
    cols_t, tile_idx = transposed_topology(cols, C_blocks)
    lay_t = TILE_OUT_IN if layout == TILE_IN_OUT else TILE_IN_OUT
    mats = list(values) + list(cols)
    key = (C_blocks,) + tuple(id(m) for m in mats)
    hit = _TILE_CACHE.get(key)
    if hit is not None:
        refs, versions, values_t = hit
        if all(r() is m for r, m in zip(refs, mats)) and versions == tuple(m._version for m in mats):
            _TILE_CACHE.move_to_end(key)
            return values_t, cols_t, lay_t
        del _TILE_CACHE[key]
    B = values[0].shape[-1]
    flat = torch.cat([v.reshape(-1, B, B) for v in values]) if len(values) > 1 else values[0].reshape(-1, B, B)
    values_t = flat.index_select(0, tile_idx.reshape(-1)).view(cols_t.shape[0], cols_t.shape[1], B, B)
    _TILE_CACHE[key] = (tuple(weakref.ref(m) for m in mats), tuple(m._version for m in mats), values_t)
    while len(_TILE_CACHE) > _TILE_CACHE_MAX:
        _TILE_CACHE.popitem(last=False)
    return values_t, cols_t, lay_t


def silu_mul_bwd(d_h: torch.Tensor, gate_pre: torch.Tensor, up_out: torch.Tensor,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``[d_gate | d_up]`` as one ``[T, 2 d_ff]`` bf16 tensor:
    d_gate = d_h * up * silu'(gate), d_up = d_h * silu(gate)."""
    for name, t in (("d_h", d_h), ("gate_pre_act", gate_pre), ("up_out", up_out)):
        _check_cuda(name, t)
        if t.dtype != torch.bfloat16:
            raise RuntimeError(f"{name} must be bf16")
    if gate_pre.shape != d_h.shape or up_out.shape != d_h.shape or d_h.dim() != 2:
        raise RuntimeError("d_h, gate_pre_act and up_out must be [N, d_ff] of one shape")
    T, F = d_h.shape
    if out is None:
        out = torch.empty((T, 2 * F), dtype=torch.bfloat16, device=d_h.device)
    else:
        _check_out("out", out, (T, 2 * F), torch.bfloat16, d_h.device)
    d_h, gate_pre, up_out = d_h.contiguous(), gate_pre.contiguous(), up_out.contiguous()
    with torch.cuda.device(d_h.device):
        _lib.check(_lib.load().bell_silu_mul_bwd_bf16(T, F, d_h.data_ptr(), gate_pre.data_ptr(), up_out.data_ptr(),
                                                      out.data_ptr(), out.data_ptr() + 2 * F, 2 * F, _stream()),
                   "silu_mul_bwd")
    return out


def down_silu_bwd(grad_out: torch.Tensor, v_down_t: torch.Tensor, ci_down_t: torch.Tensor, layout_t: int,
                  gate_pre: torch.Tensor, up_out: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``[d_gate | d_up]`` ([T, 2 d_ff] bf16) from ``grad_out`` and the
    transposed down weight in one launch (d_h stays in TMEM)."""
    T, d_model = grad_out.shape
    R, K, B, _ = v_down_t.shape
    F = R * B
    if d_model % B or tuple(gate_pre.shape) != (T, F) or tuple(up_out.shape) != (T, F):
        raise RuntimeError("grad_out must be [N, C*B] and gate_pre/up_out [N, d_ff]")
    if out is None:
        out = torch.empty((T, 2 * F), dtype=torch.bfloat16, device=grad_out.device)
    else:
        _check_out("out", out, (T, 2 * F), torch.bfloat16, grad_out.device)
    if T == 0:
        return out
    gate_pre, up_out = gate_pre.contiguous(), up_out.contiguous()
    plan = torch.empty(plan_bytes(0, 0, 0, R, K), dtype=torch.uint8, device=grad_out.device)
    d = _lib.BellDownBwdDesc()
    d.T = T
    d.grad_out, d.gate_pre, d.up_out = grad_out.data_ptr(), gate_pre.data_ptr(), up_out.data_ptr()
    d.d_gate_up, d.plan = out.data_ptr(), plan.data_ptr()
    d.w_t = _ell(v_down_t, ci_down_t, d_model // B, layout_t)
    d.status = None
    with torch.cuda.device(grad_out.device):
        _lib.check(_lib.load().bell_down_silu_bwd_bf16(C.byref(d), _stream()), "down_silu_bwd")
    return out


def block_ell_sddmm(a: torch.Tensor, b: torch.Tensor, cols: torch.Tensor, B: int, layout: int = TILE_IN_OUT,
                    grad: Optional[torch.Tensor] = None, accumulate: bool = False,
                    out_bf16: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Tile gradients ``grad[r, k] (+)= a[:, c*B:(c+1)*B]^T b[:, r*B:(r+1)*B]``
    (c = cols[r, k]) in fp32, in ``layout``.  ``a``: [T, C*B], ``b``: [T, R*B]
    bf16 (tcgen05 at B = 64, 128; CUDA cores at 16, 32) or fp32 (CUDA cores,
    ``bell_sddmm_f32``, or at B = 64 / 128 six tcgen05 products of the
    operands' bf16 parts, ``kernels.f32x``, as ``BELL_F32_METHOD`` and the
    token count choose); either may be a column slice of a wider row-major
    tensor.  When ``out_bf16`` is given (bf16 operands only) it receives a
    bf16 copy.  Returns ``grad``."""
    for name, t in (("a", a), ("b", b), ("col_indices", cols)):
        _check_cuda(name, t)
    f32 = a.dtype == torch.float32
    if a.dtype != b.dtype or a.dtype not in (torch.bfloat16, torch.float32):
        raise RuntimeError("a and b must both be bf16 or both fp32")
    if f32 and out_bf16 is not None:
        raise RuntimeError("out_bf16 needs bf16 operands")
    if cols.dtype != torch.int32 or cols.dim() != 2:
        raise RuntimeError("col_indices must be int32 [R, K]")
    if a.dim() != 2 or b.dim() != 2 or a.shape[0] != b.shape[0]:
        raise RuntimeError("a and b must be 2-D with the same number of tokens")
    for name, t in (("a", a), ("b", b)):
        if t.stride(1) != 1:
            raise RuntimeError(f"{name} must have unit stride along features")
    R, K = cols.shape
    T = a.shape[0]
    if a.shape[1] % B or b.shape[1] != R * B:
        raise RuntimeError(f"a must be [T, C*{B}] and b [T, {R}*{B}]")
    cols = cols.contiguous()
    if grad is None:
        grad = torch.empty((R, K, B, B), dtype=torch.float32, device=a.device)
        accumulate = False
    elif grad.shape != (R, K, B, B) or grad.dtype != torch.float32 or not grad.is_contiguous():
        raise RuntimeError("grad must be a contiguous fp32 [R, K, B, B] tensor")
    if f32 and T > 0:
        from . import f32x  # fp32 on the tensor cores: six bf16 products of the operands' parts
        if f32x.resolve_sddmm(None, T, B) == "bf16x6":
            return f32x.sddmm_f32x(a, b, cols, B, layout, grad, accumulate)
    d = _lib.BellSddmmDesc()
    d.T = T
    d.a, d.b = a.data_ptr(), b.data_ptr()
    d.lda, d.ldb = max(a.stride(0), a.shape[1]), max(b.stride(0), b.shape[1])
    d.col_indices = cols.data_ptr()
    d.R, d.C, d.K, d.B = R, a.shape[1] // B, K, B
    d.layout = layout
    d.accumulate = 1 if accumulate else 0
    d.grad = grad.data_ptr()
    d.grad_bf16 = out_bf16.data_ptr() if out_bf16 is not None else None
    d.status = None
    fn = _lib.load().bell_sddmm_f32 if f32 else _lib.load().bell_sddmm_bf16
    with torch.cuda.device(a.device):
        _lib.check(fn(C.byref(d), _stream()), "block_ell_sddmm")
    return grad


def block_ell_swiglu_bwd(grad_out, x, gate_pre_act, up_out, h, v_gate, ci_gate, v_up, ci_up, v_down, ci_down,
                         layout: int = TILE_IN_OUT, add_residual: bool = True, fuse_silu: Optional[bool] = None,
                         fp32_weight_grads: bool = False):
    """Returns ``(dx, d_v_gate, d_v_up, d_v_down)`` (bf16) like the reference
    titan::block_ell_swiglu_bwd (block_ell_ops.cpp:83-97).

    ``dx`` includes ``grad_out`` (the reference adds it unconditionally,
    swiglu_bwd.cu:785-796); ``add_residual=False`` leaves it out, for a forward
    run without the residual.  Weight gradients are summed in fp32 over all
    tokens and returned as bf16 in the tile layout of the weights.

    ``fuse_silu`` (default: tile size 64 only) computes d_h in the down
    kernel's TMEM and applies the SiLU*up backward in its epilogue; at tile
    size 128 the separate feature-major d_h launch plus the elementwise pass
    measured faster (config 5: 18.3 ms against 23.1 ms).

    ``fp32_weight_grads`` returns the weight gradients as the fp32 sums
    (for fp32 master weights) instead of their bf16 casts."""
    tensors = (("grad_out", grad_out), ("x", x), ("gate_pre_act", gate_pre_act), ("up_out", up_out), ("h", h),
               ("v_gate", v_gate), ("v_up", v_up), ("v_down", v_down))
    for name, t in tensors:
        _check_cuda(name, t)
        if t.dtype != torch.bfloat16:
            raise RuntimeError(f"{name} must be bf16")
    for name, t in (("ci_gate", ci_gate), ("ci_up", ci_up), ("ci_down", ci_down)):
        _check_cuda(name, t)
        if t.dtype != torch.int32:
            raise RuntimeError("All col_idx tensors must be int32")
    if x.dim() != 2 or grad_out.shape != x.shape:
        raise RuntimeError("x and grad_out must be [N, d_model] of one shape")
    T, d_model = x.shape
    R_ff, K_g, B, _ = v_gate.shape
    F = R_ff * B
    if v_up.shape[0] != R_ff or v_up.shape[2:] != (B, B) or v_down.shape[2:] != (B, B):
        raise RuntimeError("gate/up/down tiles must share the tile size and gate/up the block-rows")
    if v_down.shape[0] * B != d_model or d_model % B:
        raise RuntimeError(f"down weight rows {v_down.shape[0]}*{B} != d_model {d_model}")
    for name, t in (("gate_pre_act", gate_pre_act), ("up_out", up_out), ("h", h)):
        if tuple(t.shape) != (T, F):
            raise RuntimeError(f"{name} must be [N, d_ff] = {(T, F)}")
    C_model = d_model // B
    grad_out = grad_out.contiguous()
    x = x.contiguous()
    h = h.contiguous()
    dev = x.device

    if T > 0:
        # 1.+2. [d_gate | d_up] from d_h = grad_out @ W_down (transposed down: R_ff rows)
        vdT, cdT, lt = transpose_ell([v_down.contiguous()], [ci_down.contiguous()], R_ff, layout)
        if fuse_silu is None:
            fuse_silu = B == 64
        if fuse_silu:
            dgu = down_silu_bwd(grad_out, vdT, cdT, lt, gate_pre_act, up_out)
        else:
            d_h = block_ell_linear(grad_out, vdT, cdT, layout=lt)
            dgu = silu_mul_bwd(d_h, gate_pre_act, up_out)
        # 3. dx = [d_gate | d_up] @ [W_gate ; W_up] (+ grad_out)
        vguT, cguT, lt = transpose_ell([v_gate.contiguous(), v_up.contiguous()],
                                       [ci_gate.contiguous(), ci_up.contiguous()], C_model, layout)
        dx = block_ell_linear(dgu, vguT, cguT, residual=grad_out if add_residual else None, layout=lt)
    else:  # no tokens: empty dx, zero weight gradients (written by the SDDMM entry point)
        dgu = torch.empty((0, 2 * F), dtype=torch.bfloat16, device=dev)
        dx = torch.empty_like(x)
    # 4. tile gradients, one fp32 buffer, one bf16 result buffer
    n_g, n_u, n_d = v_gate.numel(), v_up.numel(), v_down.numel()
    g32 = torch.empty(n_g + n_u + n_d, dtype=torch.float32, device=dev)
    f_vg, f_vu, f_vd = (g32[:n_g].view(v_gate.shape), g32[n_g:n_g + n_u].view(v_up.shape),
                        g32[n_g + n_u:].view(v_down.shape))
    if fp32_weight_grads:
        d_vg = d_vu = d_vd = None
    else:
        g16 = torch.empty(n_g + n_u + n_d, dtype=torch.bfloat16, device=dev)
        d_vg, d_vu, d_vd = (g16[:n_g].view(v_gate.shape), g16[n_g:n_g + n_u].view(v_up.shape),
                            g16[n_g + n_u:].view(v_down.shape))
    block_ell_sddmm(x, dgu[:, :F], ci_gate, B, layout, grad=f_vg, out_bf16=d_vg)
    block_ell_sddmm(x, dgu[:, F:], ci_up, B, layout, grad=f_vu, out_bf16=d_vu)
    block_ell_sddmm(h, grad_out, ci_down, B, layout, grad=f_vd, out_bf16=d_vd)
    if fp32_weight_grads:
        return dx, f_vg, f_vu, f_vd
    return dx, d_vg, d_vu, d_vd


class BlockEllSwiGLU(torch.autograd.Function):
    """Autograd node over the forward with intermediates and the backward above
    (bf16).  Column indices get no gradient."""

    @staticmethod
    def forward(ctx, x, v_gate, ci_gate, v_up, ci_up, v_down, ci_down, add_residual=False, layout=TILE_IN_OUT):
        from .ops import block_ell_swiglu_fwd_with_intermediate
        out, h, g, u = block_ell_swiglu_fwd_with_intermediate(x, v_gate, ci_gate, v_up, ci_up, v_down, ci_down,
                                                              add_residual=add_residual, layout=layout)
        ctx.save_for_backward(x, g, u, h, v_gate, ci_gate, v_up, ci_up, v_down, ci_down)
        ctx.add_residual = bool(add_residual)
        ctx.layout = layout
        return out

    @staticmethod
    def backward(ctx, grad_out):
        x, g, u, h, v_gate, ci_gate, v_up, ci_up, v_down, ci_down = ctx.saved_tensors
        dx, dvg, dvu, dvd = block_ell_swiglu_bwd(grad_out.to(torch.bfloat16), x, g, u, h, v_gate, ci_gate, v_up,
                                                 ci_up, v_down, ci_down, layout=ctx.layout,
                                                 add_residual=ctx.add_residual)
        return dx, dvg, None, dvu, None, dvd, None, None, None


def block_ell_swiglu(x, v_gate, ci_gate, v_up, ci_up, v_down, ci_down, add_residual: bool = False,
                     layout: int = TILE_IN_OUT):
    """Differentiable bf16 Block-ELL SwiGLU (forward and backward on this
    package's kernels)."""
    return BlockEllSwiGLU.apply(x, v_gate, ci_gate, v_up, ci_up, v_down, ci_down, add_residual, layout)
