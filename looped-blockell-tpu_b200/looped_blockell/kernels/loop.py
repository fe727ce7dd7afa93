"""Loop ops: the shared-weight L-iteration RMSNorm -> SwiGLU loop, the
reference's per-block ``persistent_mlp_step`` (csrc/loop/loop_ops.cpp:52-66,
persistent_core.cu:273-337) and the L2 pinning pair (l2_policy.cu:48-155)."""

from __future__ import annotations

import ctypes as C
from typing import Sequence

import torch

from . import _lib
from .ops import TILE_IN_OUT, _check_cuda, _ell, _prep_ell, _stream, plan_bytes, rmsnorm


LOOP_AUTO = _lib.BELL_LOOP_AUTO
LOOP_LAUNCHES = _lib.BELL_LOOP_LAUNCHES
LOOP_PERSISTENT = _lib.BELL_LOOP_PERSISTENT


def loop_uses_persistent(mode: int, B: int) -> bool:
    """Whether ``looped_ffn`` with ``mode`` and tile size ``B`` runs the
    single persistent kernel."""
    return mode == LOOP_PERSISTENT or (mode == LOOP_AUTO and B == 64 and AUTO_PERSISTENT)


# LOOP_AUTO's choice at tile size 64 (the library applies the same rule)
AUTO_PERSISTENT = False


def looped_ffn(h: torch.Tensor, norm_gain: torch.Tensor, v_gate, ci_gate, v_up, ci_up, v_down, ci_down, L: int,
               eps: float = 1e-5, layout: int = TILE_IN_OUT, out: torch.Tensor = None,
               mode: int = LOOP_AUTO) -> torch.Tensor:
    """L iterations of ``h = h + FFN(RMSNorm(h))`` with one weight set (bf16).

    ``mode`` picks the implementation: ``LOOP_AUTO`` (the library's fastest),
    ``LOOP_LAUNCHES`` (1 + 3L kernel launches) or ``LOOP_PERSISTENT`` (one
    persistent kernel, tile size 64)."""
    lib = _lib.load()
    _check_cuda("h", h)
    if h.dim() != 2 or h.dtype != torch.bfloat16:
        raise RuntimeError("h must be 2D [N, d_model] bf16")
    h = h.contiguous()
    vg, cg = _prep_ell("gate", v_gate, ci_gate, torch.bfloat16)
    vu, cu = _prep_ell("up", v_up, ci_up, torch.bfloat16)
    vd, cd = _prep_ell("down", v_down, ci_down, torch.bfloat16)
    N, d = h.shape
    B = vg.shape[2]
    F = vg.shape[0] * B
    dev = h.device
    if out is None:
        out = torch.empty_like(h)
    elif out.shape != h.shape or out.dtype != h.dtype or not out.is_contiguous() or out.device != h.device:
        raise RuntimeError("out must be a contiguous tensor like h")
    hn = torch.empty_like(h)
    mid = torch.empty((N, F), dtype=torch.bfloat16, device=dev)
    plan = torch.empty(plan_bytes(vg.shape[0], vg.shape[1], vu.shape[1], vd.shape[0], vd.shape[1]),
                       dtype=torch.uint8, device=dev)
    ws = torch.empty(int(lib.bell_loop_workspace_bytes(N, d, vg.shape[0], vg.shape[1], vu.shape[1], B)),
                     dtype=torch.uint8, device=dev)
    desc = _lib.BellLoopDesc()
    desc.T, desc.d_model, desc.d_ff, desc.L, desc.eps = N, d, F, int(L), float(eps)
    desc.h_in, desc.h_out = h.data_ptr(), out.data_ptr()
    gain_keep = norm_gain.to(torch.bfloat16).contiguous()
    desc.norm_gain = gain_keep.data_ptr()
    desc.hn, desc.h_mid, desc.plan, desc.workspace = hn.data_ptr(), mid.data_ptr(), plan.data_ptr(), ws.data_ptr()
    desc.gate = _ell(vg, cg, d // B, layout)
    desc.up = _ell(vu, cu, d // B, layout)
    desc.down = _ell(vd, cd, F // B, layout)
    desc.status = None
    desc.mode = int(mode)
    with torch.cuda.device(dev):
        _lib.check(lib.bell_loop_fwd_bf16(C.byref(desc), _stream()), "looped_ffn")
    return out


def diagonal_injection(h, e, log_A, log_dt) -> torch.Tensor:
    """``h = exp(-softplus(log_dt) exp(log_A)) h + softplus(log_dt) e`` (persistent_core.cu:53-83)."""
    _check_cuda("h", h)
    h, e = h.contiguous(), e.contiguous()
    la, ld = log_A.float().contiguous(), log_dt.float().contiguous()
    out = torch.empty_like(h)
    d = h.shape[-1]
    with torch.cuda.device(h.device):
        _lib.check(_lib.load().bell_diag_injection_bf16(h.numel() // d, d, h.data_ptr(), e.data_ptr(), la.data_ptr(),
                                                        ld.data_ptr(), out.data_ptr(), _stream()), "injection")
    return out


def inject_rmsnorm(h, e, log_A, log_dt, gain, eps: float = 1e-5):
    """``(h_inj, RMSNorm(h_inj) * gain)`` in one pass, ``h_inj`` the diagonal
    injection of ``h`` (bit-identical to ``diagonal_injection`` then
    ``rmsnorm``)."""
    _check_cuda("h", h)
    if h.dtype != torch.bfloat16 or e.dtype != torch.bfloat16 or gain.dtype != torch.bfloat16:
        raise RuntimeError("inject_rmsnorm: h, e and gain must be bf16")
    h, e, gain = h.contiguous(), e.contiguous(), gain.contiguous()
    la, ld = log_A.float().contiguous(), log_dt.float().contiguous()
    d = h.shape[-1]
    h_out, normed = torch.empty_like(h), torch.empty_like(h)
    with torch.cuda.device(h.device):
        _lib.check(_lib.load().bell_inject_rmsnorm_bf16(h.numel() // d, d, h.data_ptr(), e.data_ptr(), la.data_ptr(),
                                                        ld.data_ptr(), gain.data_ptr(), float(eps), h_out.data_ptr(),
                                                        normed.data_ptr(), _stream()), "inject_rmsnorm")
    return h_out, normed


def persistent_mlp_step(h, e, log_A, log_dt, norm_scales: Sequence[torch.Tensor], gate_values, gate_col_idx,
                        up_values, up_col_idx, down_values, down_col_idx, eps: float = 1e-5,
                        layout: int = TILE_IN_OUT) -> torch.Tensor:
    """Reference ``titan::persistent_mlp_step``: injection, then for each of the
    n_core blocks ``h = h + SwiGLU(RMSNorm(h))`` (persistent_core.cu:273-337),
    the injection fused with the first RMSNorm.  The reference op hard-codes
    eps 1e-6 in CUDA while its JAX/PyTorch models use 1e-5 (config.py:110);
    ``eps`` defaults to the model value and ``torch.ops.titan`` passes 1e-6."""
    from .ops import block_ell_swiglu_fwd
    n = len(norm_scales)
    if n == 0:
        raise RuntimeError("persistent_mlp_step: n_core must be > 0")
    if not (len(gate_values) == len(gate_col_idx) == len(up_values) == len(up_col_idx) == len(down_values)
            == len(down_col_idx) == n):
        raise RuntimeError("persistent_mlp_step: all weight vector sizes must equal n_core")
    if h.dim() != 2:
        raise RuntimeError(f"persistent_mlp_step: h must be 2D [N, d_model], got shape {tuple(h.shape)}")
    if h.dtype != torch.bfloat16:
        raise RuntimeError("persistent_mlp_step: h must be bf16")
    cur, normed = inject_rmsnorm(h, e, log_A, log_dt, norm_scales[0].to(torch.bfloat16), eps)
    for i in range(n):
        if i > 0:
            normed = rmsnorm(cur, norm_scales[i].to(torch.bfloat16), eps)
        from .ops import _swiglu
        cur = _swiglu(normed, gate_values[i], gate_col_idx[i], up_values[i], up_col_idx[i], down_values[i],
                      down_col_idx[i], True, layout, False, residual=cur)[0]
    return cur


def pin_weights_l2(weights: Sequence[torch.Tensor]) -> None:
    """Persisting-L2 window over the address span of ``weights`` on the current stream."""
    if not weights:
        return
    lo = min(t.data_ptr() for t in weights)
    hi = max(t.data_ptr() + t.numel() * t.element_size() for t in weights)
    for t in weights:
        _check_cuda("pin_weights_l2 tensors", t)
        if not t.is_contiguous():
            raise RuntimeError("pin_weights_l2: all tensors must be contiguous")
    _lib.check(_lib.load().bell_pin_l2(C.c_void_p(lo), hi - lo, _stream()), "pin_weights_l2")


def unpin_weights_l2() -> None:
    _lib.check(_lib.load().bell_unpin_l2(_stream()), "unpin_weights_l2")
