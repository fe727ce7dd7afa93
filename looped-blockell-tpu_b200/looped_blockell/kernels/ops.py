"""Python op surface over libbell_b200.so (bf16 / fp32 paths).

Mirrors the reference native ops (csrc/block_ell/block_ell_ops.cpp:49-98):
``block_ell_swiglu_fwd(x, v_gate, ci_gate, v_up, ci_up, v_down, ci_down,
add_residual) -> Tensor`` and ``..._with_intermediate -> (result, h,
gate_pre_act, up_output)``, with the reference's argument meaning and its
TORCH_CHECK-style errors (swiglu_fwd.cu:577-613), plus ``block_ell_linear``
(one Block-ELL projection, looped_blockell/layers/block_ell.py:149-182).
All calls are stream-ordered on torch's current stream; nothing runs on the
CPU.  Tiles default to the JAX [B_in, B_out] layout; pass
``layout=TILE_OUT_IN`` for the reference CUDA [B_out, B_in] layout.
"""

from __future__ import annotations

import ctypes as C
from typing import Optional, Sequence

import torch

from . import _lib, f32x

TILE_IN_OUT = _lib.BELL_TILE_IN_OUT
TILE_OUT_IN = _lib.BELL_TILE_OUT_IN


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream() -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _check_cuda(name: str, t: torch.Tensor) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")


def _ell(values: torch.Tensor, cols: torch.Tensor, C_blocks: int, layout: int) -> _lib.BellEll:
    R, K, B, B2 = values.shape
    if B != B2:
        raise RuntimeError(f"tile must be square, got {B}x{B2}")
    if tuple(cols.shape) != (R, K):
        raise RuntimeError(f"col_indices shape {tuple(cols.shape)} != expected {(R, K)}")
    return _lib.BellEll(values.data_ptr(), cols.data_ptr(), R, C_blocks, K, B, layout, 0)


def _prep_ell(name, values, cols, dtype):
    _check_cuda(f"{name} values", values)
    _check_cuda(f"{name} col_indices", cols)
    if values.dim() != 4:
        raise RuntimeError(f"{name} values must be 4-D [R, K, B, B]")
    if values.dtype != dtype:
        raise RuntimeError("All value tensors must be " + ("bf16" if dtype == torch.bfloat16 else "fp32"))
    if cols.dtype != torch.int32:
        raise RuntimeError("All col_idx tensors must be int32")
    return values.contiguous(), cols.contiguous()


def _check_out(name: str, t: torch.Tensor, shape, dtype, device) -> None:
    """A caller-supplied output or workspace must be exactly what the kernel
    writes: the library trusts the pointer, so a smaller or differently typed
    buffer would be written past its end."""
    if tuple(t.shape) != tuple(shape) or t.dtype != dtype or t.device != device or not t.is_contiguous():
        raise RuntimeError(f"{name} must be a contiguous {dtype} tensor of shape {tuple(shape)} on {device}; "
                           f"got {t.dtype} {tuple(t.shape)} on {t.device}")


def plan_bytes(R_gu: int, K_g: int, K_u: int, R_d: int, K_d: int) -> int:
    return int(_lib.load().bell_plan_bytes(R_gu, K_g, K_u, R_d, K_d))


def _swiglu(x, v_gate, ci_gate, v_up, ci_up, v_down, ci_down, add_residual, layout, want_intermediates,
            residual=None, out=None, h=None, shared_topology=False, fp32_method=None):
    """The forward behind every SwiGLU op.  fp32 inputs run the method
    ``f32x.resolve(fp32_method, ...)`` picks: FFMA on the CUDA cores or the
    bf16x6 split on the tensor cores (same results within the fp32 target)."""
    lib = _lib.load()
    _check_cuda("x", x)
    if x.dim() != 2:
        raise RuntimeError("x must be 2D [N, d_model]")
    if x.dtype == torch.bfloat16:
        dtype, code, fn = torch.bfloat16, _lib.BELL_DTYPE_BF16, lib.bell_swiglu_fwd_bf16
    elif x.dtype == torch.float32:
        dtype, code, fn = torch.float32, _lib.BELL_DTYPE_F32, lib.bell_swiglu_fwd_f32
    else:
        raise RuntimeError("x must be bf16 (or fp32 for the accuracy path)")
    x = x.contiguous()
    vg, cg = _prep_ell("gate", v_gate, ci_gate, dtype)
    vu, cu = _prep_ell("up", v_up, ci_up, dtype)
    vd, cd = _prep_ell("down", v_down, ci_down, dtype)
    N, d_model = x.shape
    B = vg.shape[2]
    d_ff = vg.shape[0] * B
    if d_model % B != 0:
        raise RuntimeError(f"d_model={d_model} is not a multiple of the tile size {B}")
    dev = x.device
    split = dtype == torch.float32 and f32x.resolve(fp32_method, N, vg.shape[1], vu.shape[1], vd.shape[1]) == "bf16x6"
    if h is None:
        # the bf16x6 forward keeps h in bf16 parts; an fp32 copy only when asked for
        h = torch.empty((N, d_ff), dtype=dtype, device=dev) if not split or want_intermediates else None
    else:
        _check_out("h", h, (N, d_ff), dtype, dev)
    if out is None:
        out = torch.empty((N, d_model), dtype=dtype, device=dev)
    else:
        _check_out("out", out, (N, d_model), dtype, dev)
    if residual is not None:
        _check_out("residual", residual, (N, d_model), dtype, dev)
    gate_pre = torch.empty((N, d_ff), dtype=dtype, device=dev) if want_intermediates else None
    up_out = torch.empty((N, d_ff), dtype=dtype, device=dev) if want_intermediates else None
    if split:
        f32x.swiglu_fwd_f32x(x, vg, cg, vu, cu, vd, cd, add_residual, layout, out, h, gate_pre, up_out, residual)
        return out, h, gate_pre, up_out
    plan = torch.empty(plan_bytes(vg.shape[0], vg.shape[1], vu.shape[1], vd.shape[0], vd.shape[1]),
                       dtype=torch.uint8, device=dev)
    desc = _lib.BellFFNDesc()
    desc.T, desc.d_model, desc.d_ff, desc.dtype = N, d_model, d_ff, code
    desc.add_residual = 1 if add_residual else 0
    desc.x, desc.residual, desc.h = x.data_ptr(), (residual.data_ptr() if residual is not None else None), h.data_ptr()
    desc.gate_pre = gate_pre.data_ptr() if gate_pre is not None else None
    desc.up_out = up_out.data_ptr() if up_out is not None else None
    desc.out, desc.plan = out.data_ptr(), plan.data_ptr()
    desc.gate = _ell(vg, cg, d_model // B, layout)
    if shared_topology:
        desc.gate.flags = _lib.BELL_ELL_SAME_COLS_AS_UP
    desc.up = _ell(vu, cu, d_model // B, layout)
    desc.down = _ell(vd, cd, d_ff // vd.shape[2], layout)
    desc.status = None
    with torch.cuda.device(dev):
        _lib.check(fn(C.byref(desc), _stream()), "block_ell_swiglu_fwd")
    return out, h, gate_pre, up_out


def block_ell_gate_up(x, v_gate, ci_gate, v_up, ci_up, v_down, ci_down, layout: int = TILE_IN_OUT, h=None,
                      max_ctas: int = 0):
    """First half only: ``h = silu(x Wg) * (x Wu)`` (the down weight is only
    shape-checked).  Used by the d_ff-sharded forward.  ``max_ctas`` caps the
    persistent grid (0 = every SM), leaving SMs to a concurrent collective."""
    lib = _lib.load()
    _check_cuda("x", x)
    if x.dim() != 2 or x.dtype != torch.bfloat16:
        raise RuntimeError("x must be 2D bf16")
    x = x.contiguous()
    vg, cg = _prep_ell("gate", v_gate, ci_gate, torch.bfloat16)
    vu, cu = _prep_ell("up", v_up, ci_up, torch.bfloat16)
    vd, cd = _prep_ell("down", v_down, ci_down, torch.bfloat16)
    N, d_model = x.shape
    B = vg.shape[2]
    d_ff = vg.shape[0] * B
    if h is None:
        h = torch.empty((N, d_ff), dtype=torch.bfloat16, device=x.device)
    else:
        _check_out("h", h, (N, d_ff), torch.bfloat16, x.device)
    plan = torch.empty(plan_bytes(vg.shape[0], vg.shape[1], vu.shape[1], vd.shape[0], vd.shape[1]),
                       dtype=torch.uint8, device=x.device)
    desc = _lib.BellFFNDesc()
    desc.T, desc.d_model, desc.d_ff, desc.dtype = N, d_model, d_ff, _lib.BELL_DTYPE_BF16
    desc.x, desc.h, desc.out, desc.plan = x.data_ptr(), h.data_ptr(), h.data_ptr(), plan.data_ptr()
    desc.gate = _ell(vg, cg, d_model // B, layout)
    desc.up = _ell(vu, cu, d_model // B, layout)
    desc.down = _ell(vd, cd, d_ff // vd.shape[2], layout)
    desc.max_ctas = int(max_ctas)
    with torch.cuda.device(x.device):
        _lib.check(lib.bell_gate_up_bf16(C.byref(desc), _stream()), "block_ell_gate_up")
    return h


def block_ell_swiglu_fwd(x, v_gate, ci_gate, v_up, ci_up, v_down, ci_down, add_residual: bool = False,
                         layout: int = TILE_IN_OUT, shared_topology: bool = False,
                         fp32_method: Optional[str] = None) -> torch.Tensor:
    """``W_down(silu(W_gate x) * W_up x) (+ x)`` — reference titan::block_ell_swiglu_fwd.

    ``shared_topology=True`` tells the kernel that gate and up hold the same
    column lists (the reference MLPBlock's default); results are identical
    either way, only the schedule changes.  ``fp32_method`` (fp32 inputs):
    ``"auto"`` (default), ``"simt"`` or ``"bf16x6"`` (``kernels.f32x``)."""
    return _swiglu(x, v_gate, ci_gate, v_up, ci_up, v_down, ci_down, add_residual, layout, False,
                   shared_topology=shared_topology, fp32_method=fp32_method)[0]


def block_ell_swiglu_fwd_with_intermediate(x, v_gate, ci_gate, v_up, ci_up, v_down, ci_down,
                                           add_residual: bool = False, layout: int = TILE_IN_OUT,
                                           shared_topology: bool = False, fp32_method: Optional[str] = None):
    """Returns (result, h, gate_pre_act, up_output) like the reference op (block_ell_ops.cpp:65-76)."""
    return _swiglu(x, v_gate, ci_gate, v_up, ci_up, v_down, ci_down, add_residual, layout, True,
                   shared_topology=shared_topology, fp32_method=fp32_method)


def block_ell_linear(x: torch.Tensor, values: torch.Tensor, cols: torch.Tensor, residual: Optional[torch.Tensor] = None,
                     out_dtype: Optional[torch.dtype] = None, layout: int = TILE_IN_OUT,
                     out: Optional[torch.Tensor] = None, residual_rows: Optional[Sequence[int]] = None,
                     max_ctas: int = 0, fp32_method: Optional[str] = None) -> torch.Tensor:
    """``y = x @ W^T (+ residual)`` for one Block-ELL weight; x is [N, C*B].

    bf16 only: ``residual_rows=(lo, hi)`` adds the residual to output rows
    [lo, hi) only, and ``max_ctas`` caps the persistent grid (0 = every SM).
    fp32 inputs run ``fp32_method`` (``kernels.f32x``): ``"auto"`` (default),
    ``"simt"`` or ``"bf16x6"``."""
    lib = _lib.load()
    _check_cuda("x", x)
    if x.dim() != 2:
        raise RuntimeError("x must be 2D [N, in_features]")
    dtype = x.dtype
    if dtype not in (torch.bfloat16, torch.float32):
        raise RuntimeError("x must be bf16 or fp32")
    x = x.contiguous()
    v, c = _prep_ell("weight", values, cols, dtype)
    R, K, B, _ = v.shape
    N, in_f = x.shape
    if in_f % B != 0:
        raise RuntimeError(f"in_features={in_f} is not a multiple of the tile size {B}")
    out_dtype = out_dtype or dtype
    if dtype == torch.float32 and out_dtype != torch.float32:
        raise RuntimeError("fp32 inputs produce fp32 output")
    if out is None:
        out = torch.empty((N, R * B), dtype=out_dtype, device=x.device)
    else:
        _check_out("out", out, (N, R * B), out_dtype, x.device)
    if residual is not None:
        _check_cuda("residual", residual)
        if residual.shape != (N, R * B) or residual.dtype != dtype:
            raise RuntimeError("residual must be [N, out_features] with the input dtype")
        residual = residual.contiguous()
    if dtype == torch.float32 and residual_rows is None and max_ctas == 0 and \
            f32x.resolve_linear(fp32_method, N, K, residual is not None) == "bf16x6":
        f32x.linear_f32x(x, v, c, residual, layout, out)
        return out
    plan = torch.empty(plan_bytes(0, 0, 0, R, K), dtype=torch.uint8, device=x.device)
    desc = _lib.BellLinearDesc()
    desc.T = N
    desc.dtype = _lib.BELL_DTYPE_BF16 if dtype == torch.bfloat16 else _lib.BELL_DTYPE_F32
    desc.out_dtype = _lib.BELL_DTYPE_BF16 if out_dtype == torch.bfloat16 else _lib.BELL_DTYPE_F32
    desc.add_residual = 1 if residual is not None else 0
    desc.x, desc.out, desc.plan = x.data_ptr(), out.data_ptr(), plan.data_ptr()
    desc.residual = residual.data_ptr() if residual is not None else None
    desc.w = _ell(v, c, in_f // B, layout)
    desc.status = None
    desc.max_ctas = int(max_ctas)
    if residual_rows is not None:
        if dtype != torch.bfloat16:
            raise RuntimeError("residual_rows needs bf16 inputs")
        lo, hi = (int(v_) for v_ in residual_rows)
        if not 0 <= lo <= hi <= N:
            raise RuntimeError(f"residual_rows {(lo, hi)} outside [0, {N}]")
        if lo == hi:
            desc.add_residual = 0
        else:
            desc.residual_row_lo, desc.residual_row_hi = lo, hi
    fn = lib.bell_linear_bf16 if dtype == torch.bfloat16 else lib.bell_linear_f32
    with torch.cuda.device(x.device):
        _lib.check(fn(C.byref(desc), _stream()), "block_ell_linear")
    return out


def rmsnorm(x: torch.Tensor, gain: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """RMSNorm ``x / sqrt(mean(x^2) + eps) * gain`` (looped_blockell/layers/norms.py:8-15):
    bf16 x and gain (fp32 math, bf16 out), or fp32 x and gain (fp32 throughout)."""
    _check_cuda("x", x)
    if x.dtype == torch.bfloat16 and gain.dtype == torch.bfloat16:
        fn = _lib.load().bell_rmsnorm_bf16
    elif x.dtype == torch.float32 and gain.dtype == torch.float32:
        fn = _lib.load().bell_rmsnorm_f32
    else:
        raise RuntimeError("rmsnorm: x and gain must both be bf16 or both fp32")
    x = x.contiguous()
    out = torch.empty_like(x)
    d = x.shape[-1]
    with torch.cuda.device(x.device):
        _lib.check(fn(x.numel() // d, d, x.data_ptr(), gain.contiguous().data_ptr(), float(eps), out.data_ptr(),
                      _stream()), "rmsnorm")
    return out


def sum_slices(slices: torch.Tensor, out: torch.Tensor, local: Optional[torch.Tensor] = None, local_slot: int = -1,
               residual: Optional[torch.Tensor] = None, max_ctas: int = 0) -> torch.Tensor:
    """``out = bf16(sum_s slices[s] (+ residual))`` in fp32, ascending s, one
    rounding (``bell_sum_slices_bf16``).  ``slices`` is ``[n, rows, d]`` bf16
    (rows contiguous, slices any stride); slice ``local_slot`` is taken from
    ``local`` ``[rows, d]`` instead (``slices[local_slot]`` is not read)."""
    _check_cuda("slices", slices)
    if slices.dim() != 3 or slices.dtype != torch.bfloat16 or slices.stride(2) != 1:
        raise RuntimeError("sum_slices: slices must be [n, rows, d] bf16 with contiguous rows")
    n, rows, d = slices.shape
    for name, t in (("out", out), ("local", local), ("residual", residual)):
        if t is None:
            continue
        if t.dtype != torch.bfloat16 or t.dim() != 2 or tuple(t.shape) != (rows, d) or t.stride(1) != 1:
            raise RuntimeError(f"sum_slices: {name} must be [{rows}, {d}] bf16 with contiguous rows")
        if t.device != slices.device:
            raise RuntimeError(f"sum_slices: {name} is on {t.device}, slices on {slices.device}")
    if (local is None) != (local_slot < 0):
        raise RuntimeError("sum_slices: give local together with local_slot >= 0")
    with torch.cuda.device(slices.device):
        _lib.check(_lib.load().bell_sum_slices_bf16(
            slices.data_ptr(), slices.stride(0), slices.stride(1), n, local_slot, _ptr(local),
            local.stride(0) if local is not None else 0, _ptr(residual),
            residual.stride(0) if residual is not None else 0, out.data_ptr(), out.stride(0), rows, d,
            int(max_ctas), _stream()), "sum_slices")
    return out


def read_status(clear: bool = True) -> int:
    """Read (and clear) the library's device status word (synchronises)."""
    v = C.c_int32(0)
    _lib.check(_lib.load().bell_read_status(C.byref(v), 1 if clear else 0, _stream()), "read_status")
    return int(v.value)
