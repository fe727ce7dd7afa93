"""Ternary Block-ELL: 2-bit packed {-1, 0, +1} tiles with one fp32 scale per
tile, int8 per-token activations, exact int32 tile products on tcgen05.

Weight preparation (offline, once per weight set) follows the AbsMean
ternariser of bonsai-test/bitlinear.py:34-55 with the group = one B x B tile:
``s = mean|w|`` (clamped to 1e-8), ``t = round(w / s).clamp(-1, 1)``.  The
packed format is this library's (the reference has no packed ternary
Block-ELL): tile (r, k) stored output-column major, 16 B_in entries per
little-endian uint32 at 2 bits each, codes 00 = 0, 01 = +1, 11 = -1.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib
from .ops import _check_cuda, _stream, plan_bytes


@dataclass
class TernaryBlockELL:
    packed: torch.Tensor       # uint8 [R, K, B, B // 4]
    scales: torch.Tensor       # fp32 [R, K]
    col_indices: torch.Tensor  # int32 [R, K]
    C: int                     # input column blocks

    @property
    def R(self):
        return self.packed.shape[0]

    @property
    def K(self):
        return self.packed.shape[1]

    @property
    def B(self):
        return self.packed.shape[2]

    def _abi(self) -> _lib.BellTernaryEll:
        return _lib.BellTernaryEll(self.packed.data_ptr(), self.scales.data_ptr(), self.col_indices.data_ptr(),
                                   self.R, self.C, self.K, self.B)


def ternary_quantize_tiles(values: torch.Tensor):
    """Per-tile AbsMean ternarisation; returns (t int8 same shape, s fp32 [R, K])."""
    v = values.float()
    R, K = v.shape[:2]
    flat = v.reshape(R, K, -1)
    s = flat.abs().mean(dim=2).clamp(min=1e-8)
    t = (flat / s[:, :, None]).round().clamp(-1, 1).to(torch.int8)
    return t.reshape(v.shape), s.contiguous()


def pack_ternary(t: torch.Tensor) -> torch.Tensor:
    """int8 tiles [R, K, B_in, B_out] -> uint8 [R, K, B, B // 4] (format above)."""
    R, K, B, _ = t.shape
    kt = t.transpose(-1, -2).to(torch.int32)  # [R, K, B_out, B_in]
    codes = torch.where(kt == 0, 0, torch.where(kt > 0, 1, 3)).to(torch.int64)
    codes = codes.reshape(R, K, B, B // 16, 16)
    shifts = 2 * torch.arange(16, device=t.device, dtype=torch.int64)
    words = (codes << shifts).sum(dim=-1)  # < 2**32
    words = torch.where(words >= 2 ** 31, words - 2 ** 32, words).to(torch.int32)
    return words.contiguous().view(torch.uint8).reshape(R, K, B, B // 4)


def make_ternary(values: torch.Tensor, col_indices: torch.Tensor, C_blocks: int) -> TernaryBlockELL:
    t, s = ternary_quantize_tiles(values)
    return TernaryBlockELL(pack_ternary(t).contiguous(), s.float().contiguous(),
                           col_indices.to(torch.int32).contiguous(), C_blocks)


def ternary_swiglu_fwd(x: torch.Tensor, gate: TernaryBlockELL, up: TernaryBlockELL, down: TernaryBlockELL,
                       add_residual: bool = False, return_intermediates: bool = False):
    """Ternary SwiGLU forward; x [T, d_model] bf16 -> out [T, d_model] fp32."""
    lib = _lib.load()
    _check_cuda("x", x)
    if x.dim() != 2 or x.dtype != torch.bfloat16:
        raise RuntimeError("x must be 2D [N, d_model] bf16")
    x = x.contiguous()
    T, d = x.shape
    F = gate.R * gate.B
    dev = x.device
    ws = dict(q_x=torch.empty((T, d), dtype=torch.int8, device=dev),
              s_x=torch.empty(T, dtype=torch.float32, device=dev),
              h=torch.empty((T, F), dtype=torch.float32, device=dev),
              q_h=torch.empty((T, F), dtype=torch.int8, device=dev),
              s_h=torch.empty(T, dtype=torch.float32, device=dev))
    if return_intermediates:
        ws["gate"] = torch.empty((T, F), dtype=torch.float32, device=dev)
        ws["up"] = torch.empty((T, F), dtype=torch.float32, device=dev)
    out = torch.empty((T, d), dtype=torch.float32, device=dev)
    plan = torch.empty(plan_bytes(gate.R, gate.K, up.K, down.R, down.K), dtype=torch.uint8, device=dev)
    desc = _lib.BellTernaryFFNDesc()
    desc.T, desc.d_model, desc.d_ff, desc.add_residual = T, d, F, 1 if add_residual else 0
    desc.x = x.data_ptr()
    desc.q_x, desc.s_x, desc.h = ws["q_x"].data_ptr(), ws["s_x"].data_ptr(), ws["h"].data_ptr()
    desc.q_h, desc.s_h = ws["q_h"].data_ptr(), ws["s_h"].data_ptr()
    desc.gate_pre = ws["gate"].data_ptr() if return_intermediates else None
    desc.up_out = ws["up"].data_ptr() if return_intermediates else None
    desc.out, desc.plan = out.data_ptr(), plan.data_ptr()
    desc.gate, desc.up, desc.down = gate._abi(), up._abi(), down._abi()
    desc.status = None
    with torch.cuda.device(dev):
        _lib.check(lib.bell_swiglu_fwd_ternary(C.byref(desc), _stream()), "ternary_swiglu_fwd")
    if return_intermediates:
        return out, ws
    return out
