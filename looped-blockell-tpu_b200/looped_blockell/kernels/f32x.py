"""fp32 Block-ELL SwiGLU on the bf16 tensor cores (the "bf16x6" split).

The reference evaluates ``block_ell_matmul`` / ``MLPBlock`` in fp32
(looped_blockell/layers/block_ell.py:149-182, mlp.py:119-145).  Two GPU
methods reach its rel-L2 <= 1e-5 target:

* ``"simt"``: FFMA on the CUDA cores (``bell_swiglu_fwd_f32``);
* ``"bf16x6"``: every fp32 operand split into three bf16 parts and the six
  leading cross products accumulated in fp32 on tcgen05
  (``bell_swiglu_fwd_f32x``; Henry, Tang & Heinecke, ARITH 2019).

``method="auto"`` takes bf16x6 from ``AUTO_MIN_TOKENS`` tokens up and SIMT
below that (smaller calls were not measured) or when an expanded row would
exceed the forward's 254 slots.  Measured on B200 at config 1's shapes
(d=512, F=2048, B=64, 25 %), SIMT against bf16x6: T=1024 0.214 / 0.096 ms,
T=8192 0.721 / 0.218 ms, T=65536 5.34 / 1.17 ms, T=262144 22.5 / 4.84 ms
(18 against 85 effective fp32 TFLOP/s).  ``BELL_F32_METHOD`` overrides the
default.

The expanded weights (bf16 tiles and column indices, 3x the fp32 bytes) are
made once per weight tensor and version and cached like the backward's
transposed tiles: a hit needs the very same tensor objects at the same
version.
"""

from __future__ import annotations

import ctypes as C
import os
import weakref
from collections import OrderedDict
from typing import Optional

import torch

from . import _lib

AUTO_MIN_TOKENS = 1024
METHODS = ("auto", "simt", "bf16x6")

_CACHE: "OrderedDict[tuple, tuple]" = OrderedDict()
_CACHE_MAX = 16


def default_method() -> str:
    m = os.environ.get("BELL_F32_METHOD", "auto")
    if m not in METHODS:
        raise RuntimeError(f"BELL_F32_METHOD must be one of {METHODS}, got {m!r}")
    return m


def resolve(method: Optional[str], T: int, K_gate: int, K_up: int, K_down: int) -> str:
    """The method a call of T tokens runs: ``"simt"`` or ``"bf16x6"``."""
    m = method or default_method()
    if m not in METHODS:
        raise RuntimeError(f"fp32 method must be one of {METHODS}, got {m!r}")
    fits = 6 * max(K_gate, K_up) <= 254 and 6 * K_down + 3 <= 254
    if m == "bf16x6":
        if not fits:
            raise RuntimeError("bf16x6 needs at most 42 slots per gate/up row and 41 per down row")
        return m
    if m == "simt":
        return m
    return "bf16x6" if fits and T >= AUTO_MIN_TOKENS else "simt"


def resolve_linear(method: Optional[str], T: int, K: int, residual: bool) -> str:
    """The method an fp32 linear of T tokens runs (6K slots per expanded row,
    plus 3 identity slots for a residual)."""
    m = method or default_method()
    if m not in METHODS:
        raise RuntimeError(f"fp32 method must be one of {METHODS}, got {m!r}")
    fits = 6 * K + (3 if residual else 0) <= 254
    if m == "bf16x6":
        if not fits:
            raise RuntimeError("bf16x6 needs at most 42 slots per row (41 with a residual)")
        return m
    if m == "simt":
        return m
    return "bf16x6" if fits and T >= AUTO_MIN_TOKENS else "simt"


def _expand(values: torch.Tensor, cols: torch.Tensor, C_blocks: int, layout: int, col_base: int, part_cols: int,
            ident_base: int, ident_stride: int):
    key = (id(values), id(cols), C_blocks, layout, col_base, part_cols, ident_base, ident_stride)
    hit = _CACHE.get(key)
    if hit is not None:
        refs, versions, result = hit
        if refs[0]() is values and refs[1]() is cols and versions == (values._version, cols._version):
            _CACHE.move_to_end(key)
            return result
        del _CACHE[key]
    lib = _lib.load()
    R, K, B, _ = values.shape
    K6 = int(lib.bell_f32x_slots(K, 1 if ident_base >= 0 else 0))
    v6 = torch.empty((R, K6, B, B), dtype=torch.bfloat16, device=values.device)
    c6 = torch.empty((R, K6), dtype=torch.int32, device=values.device)
    ell = _lib.BellEll(values.data_ptr(), cols.data_ptr(), R, C_blocks, K, B, layout, 0)
    stream = C.c_void_p(torch.cuda.current_stream(values.device).cuda_stream)
    with torch.cuda.device(values.device):
        _lib.check(lib.bell_f32x_expand_ell(C.byref(ell), col_base, part_cols, ident_base, ident_stride,
                                            C.c_void_p(v6.data_ptr()), C.c_void_p(c6.data_ptr()), stream),
                   "bell_f32x_expand_ell")
    result = (v6, c6)
    _CACHE[key] = ((weakref.ref(values), weakref.ref(cols)), (values._version, cols._version), result)
    while len(_CACHE) > _CACHE_MAX:
        _CACHE.popitem(last=False)
    return result


def linear_f32x(x: torch.Tensor, values: torch.Tensor, cols: torch.Tensor, residual: Optional[torch.Tensor],
                layout: int, out: torch.Tensor) -> None:
    """bell_linear_f32x on validated contiguous fp32 tensors: out = x W
    (+ residual), x [T, C*B], tiles [R, K, B, B]."""
    lib = _lib.load()
    T, in_f = x.shape
    R, K, B, _ = values.shape
    Cx = in_f // B
    ident = residual is not None
    w6, c6 = _expand(values, cols, Cx, layout, 0, Cx, 3 * Cx if ident else -1, R if ident else 0)
    CA = 3 * Cx + (3 * R if ident else 0)
    ws = torch.empty(int(lib.bell_f32x_linear_workspace_bytes(T, in_f, R * B, R, w6.shape[1])), dtype=torch.uint8,
                     device=x.device)
    desc = _lib.BellLinearDesc()
    desc.T = T
    desc.dtype = desc.out_dtype = _lib.BELL_DTYPE_F32
    desc.add_residual = 1 if ident else 0
    desc.x, desc.out, desc.plan = x.data_ptr(), out.data_ptr(), None
    desc.residual = residual.data_ptr() if ident else None
    desc.w = _lib.BellEll(w6.data_ptr(), c6.data_ptr(), R, CA, w6.shape[1], B, layout, 0)
    desc.status = None
    desc.max_ctas = 0
    stream = C.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)
    with torch.cuda.device(x.device):
        _lib.check(lib.bell_linear_f32x(C.byref(desc), C.c_void_p(ws.data_ptr()), stream),
                   "block_ell_linear (fp32, bf16x6)")


# the six (a part, b part) products of a split product, leading terms first
PAIRS = ((0, 0), (0, 1), (1, 0), (0, 2), (1, 1), (2, 0))


def split_rows(src: torch.Tensor) -> torch.Tensor:
    """[T, n] fp32 (rows may be strided, unit stride along n) -> [T, 3n] bf16
    holding its three bf16 parts side by side (``bell_f32x_split_rows``)."""
    T, n = src.shape
    dst = torch.empty((T, 3 * n), dtype=torch.bfloat16, device=src.device)
    stream = C.c_void_p(torch.cuda.current_stream(src.device).cuda_stream)
    with torch.cuda.device(src.device):
        _lib.check(_lib.load().bell_f32x_split_rows(T, n, C.c_void_p(src.data_ptr()), max(src.stride(0), n),
                                                    C.c_void_p(dst.data_ptr()), 3 * n, 0, stream),
                   "bell_f32x_split_rows")
    return dst


def resolve_sddmm(method: Optional[str], T: int, B: int) -> str:
    """The method fp32 tile gradients of T tokens run: bf16x6 needs the
    tcgen05 tile-gradient kernel (tile size 64 or 128)."""
    m = method or default_method()
    if m not in METHODS:
        raise RuntimeError(f"fp32 method must be one of {METHODS}, got {m!r}")
    if m == "simt" or B < 64:
        return "simt"
    if m == "bf16x6":
        return m
    return "bf16x6" if T >= AUTO_MIN_TOKENS else "simt"


def sddmm_f32x(a: torch.Tensor, b: torch.Tensor, cols: torch.Tensor, B: int, layout: int, grad: torch.Tensor,
               accumulate: bool) -> torch.Tensor:
    """fp32 tile gradients grad[r, k] (+)= a[:, c*B:(c+1)*B]^T b[:, r*B:(r+1)*B]
    as six bf16 tile-gradient products of the operands' parts, summed into
    the fp32 ``grad``."""
    from .backward import block_ell_sddmm
    na, nb = a.shape[1], b.shape[1]
    ap, bp = split_rows(a), split_rows(b)
    for idx, (i, j) in enumerate(PAIRS):
        block_ell_sddmm(ap[:, i * na:(i + 1) * na], bp[:, j * nb:(j + 1) * nb], cols, B, layout, grad=grad,
                        accumulate=accumulate or idx > 0)
    return grad


def swiglu_fwd_f32x(x, vg, cg, vu, cu, vd, cd, add_residual: bool, layout: int, out: torch.Tensor,
                    h: Optional[torch.Tensor], gate_pre: Optional[torch.Tensor], up_out: Optional[torch.Tensor],
                    residual: Optional[torch.Tensor] = None) -> None:
    """bell_swiglu_fwd_f32x on validated contiguous fp32 tensors (x [T, d],
    tiles [R, K, B, B], int32 columns); writes out (and h / gate_pre / up_out
    when given)."""
    lib = _lib.load()
    T, d = x.shape
    B = vg.shape[2]
    F = vg.shape[0] * B
    Cd, Cf = d // B, F // B
    CA = 3 * Cf + 3 * Cd
    g6, gc6 = _expand(vg, cg, Cd, layout, 3 * Cf, Cd, -1, 0)
    u6, uc6 = _expand(vu, cu, Cd, layout, 3 * Cf, Cd, -1, 0)
    d6, dc6 = _expand(vd, cd, Cf, layout, 0, Cf, 3 * Cf, Cd)
    ws = torch.empty(int(lib.bell_f32x_workspace_bytes(T, d, F, B, g6.shape[1], u6.shape[1], d6.shape[1])),
                     dtype=torch.uint8, device=x.device)
    desc = _lib.BellFFNDesc()
    desc.T, desc.d_model, desc.d_ff, desc.dtype = T, d, F, _lib.BELL_DTYPE_F32
    desc.add_residual = 1 if add_residual else 0
    desc.x = x.data_ptr()
    desc.residual = residual.data_ptr() if residual is not None else None
    desc.h = h.data_ptr() if h is not None else None
    desc.gate_pre = gate_pre.data_ptr() if gate_pre is not None else None
    desc.up_out = up_out.data_ptr() if up_out is not None else None
    desc.out = out.data_ptr()
    desc.plan = None
    desc.gate = _lib.BellEll(g6.data_ptr(), gc6.data_ptr(), g6.shape[0], CA, g6.shape[1], B, layout, 0)
    desc.up = _lib.BellEll(u6.data_ptr(), uc6.data_ptr(), u6.shape[0], CA, u6.shape[1], B, layout, 0)
    desc.down = _lib.BellEll(d6.data_ptr(), dc6.data_ptr(), d6.shape[0], CA, d6.shape[1], B, layout, 0)
    desc.status = None
    stream = C.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)
    with torch.cuda.device(x.device):
        _lib.check(lib.bell_swiglu_fwd_f32x(C.byref(desc), C.c_void_p(ws.data_ptr()), stream),
                   "block_ell_swiglu_fwd (fp32, bf16x6)")
