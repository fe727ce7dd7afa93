"""Zero-token calls through every forward entry point.

A batch with no tokens gives an empty result of the right shape, as the
reference's PyTorch ops do for an empty input.  An empty torch tensor has a
NULL data pointer; the C entry points accept NULL activation buffers when
T = 0 (weights stay required), launch nothing and leave the status word clear.
"""

import ctypes as C

import pytest
import torch

from gpu_util import make_case, to_dev

pytestmark = pytest.mark.gpu

D, F, B = 256, 512, 64


def _case(dtype):
    return to_dev(make_case(4, D, F, B, 2, 3, 4, seed=7), dtype)


def _weights(c):
    return c["vg"], c["cg"], c["vu"], c["cu"], c["vd"], c["cd"]


def _status_clear():
    from looped_blockell.kernels import read_status
    torch.cuda.synchronize()
    assert read_status() == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("add_residual", [False, True])
def test_swiglu_forward_zero_tokens(dtype, add_residual):
    from looped_blockell.kernels import ops
    c = _case(dtype)
    x = c["x"][:0]
    out = ops.block_ell_swiglu_fwd(x, *_weights(c), add_residual=add_residual)
    assert out.shape == (0, D) and out.dtype == dtype
    res, h, g, u = ops.block_ell_swiglu_fwd_with_intermediate(x, *_weights(c), add_residual=add_residual)
    assert res.shape == (0, D) and h.shape == g.shape == u.shape == (0, F)
    _status_clear()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_linear_zero_tokens(dtype):
    from looped_blockell.kernels import ops
    c = _case(dtype)
    h = torch.empty((0, F), dtype=dtype, device="cuda")
    res = torch.empty((0, D), dtype=dtype, device="cuda")
    assert ops.block_ell_linear(h, c["vd"], c["cd"]).shape == (0, D)
    assert ops.block_ell_linear(h, c["vd"], c["cd"], residual=res).shape == (0, D)
    _status_clear()


def test_loop_norm_and_injection_zero_tokens():
    from looped_blockell.kernels import loop, ops
    c = _case(torch.bfloat16)
    h = c["x"][:0]
    gain = torch.ones(D, dtype=torch.bfloat16, device="cuda")
    la = torch.zeros(D, dtype=torch.float32, device="cuda")
    assert loop.looped_ffn(h, gain, *_weights(c), L=3).shape == (0, D)
    assert loop.looped_ffn(h, gain, *_weights(c), L=0).shape == (0, D)
    assert ops.rmsnorm(h, gain).shape == (0, D)
    assert loop.diagonal_injection(h, h, la, la).shape == (0, D)
    h_out, normed = loop.inject_rmsnorm(h, h, la, la, gain)
    assert h_out.shape == normed.shape == (0, D)
    _status_clear()


def test_ternary_zero_tokens():
    from looped_blockell.kernels.ternary import make_ternary, ternary_swiglu_fwd
    c = _case(torch.float32)
    g = make_ternary(c["vg"], c["cg"], D // B)
    u = make_ternary(c["vu"], c["cu"], D // B)
    w = make_ternary(c["vd"], c["cd"], F // B)
    x = c["x"][:0].to(torch.bfloat16)
    out, ws = ternary_swiglu_fwd(x, g, u, w, add_residual=True, return_intermediates=True)
    assert out.shape == (0, D) and ws["h"].shape == (0, F) and ws["q_x"].shape == (0, D)
    _status_clear()


def test_c_abi_zero_tokens_with_null_buffers():
    """The C ABI itself: NULL activation pointers with T = 0 succeed, the same
    NULL pointers with T = 1 are refused as an argument error."""
    from looped_blockell.kernels import _lib as L
    lib = L.load()
    c = _case(torch.bfloat16)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)

    def desc(T):
        d = L.BellFFNDesc()
        d.T, d.d_model, d.d_ff, d.dtype, d.add_residual = T, D, F, L.BELL_DTYPE_BF16, 1
        d.x = d.residual = d.h = d.plan = d.gate_pre = d.up_out = d.out = d.status = None
        d.gate = L.BellEll(c["vg"].data_ptr(), c["cg"].data_ptr(), F // B, D // B, c["vg"].shape[1], B, 0, 0)
        d.up = L.BellEll(c["vu"].data_ptr(), c["cu"].data_ptr(), F // B, D // B, c["vu"].shape[1], B, 0, 0)
        d.down = L.BellEll(c["vd"].data_ptr(), c["cd"].data_ptr(), D // B, F // B, c["vd"].shape[1], B, 0, 0)
        return d

    assert lib.bell_swiglu_fwd_bf16(C.byref(desc(0)), stream) == L.BELL_OK
    assert lib.bell_swiglu_fwd_bf16_noalloc(C.byref(desc(0)), stream) == L.BELL_OK
    assert L.ERRORS[lib.bell_swiglu_fwd_bf16(C.byref(desc(1)), stream)] == "ARG"
    _status_clear()
