"""GPU tests of the drop-in surfaces: torch.ops.titan.* (reference schemas,
[B_out, B_in] tiles) against the oracle, and the host-buffer pipelined entry
points against the device entry points (identical results)."""

import numpy as np
import pytest
import torch

import oracle as O
from gpu_util import make_case, oracle_ffn, to_dev

pytestmark = pytest.mark.gpu


def _K():
    from looped_blockell import kernels as K
    return K


@pytest.mark.parametrize("add_residual", [False, True])
def test_titan_swiglu_matches_oracle_out_in_tiles(add_residual):
    K = _K()
    c = make_case(200, 256, 512, 64, 2, 3, 4, seed=11)
    d = to_dev(c, torch.bfloat16, O.LAYOUT_OUT_IN)  # tiles stored [B_out, B_in], as the reference CUDA op expects
    out = torch.ops.titan.block_ell_swiglu_fwd(d["x"], d["vg"], d["cg"], d["vu"], d["cu"], d["vd"], d["cd"],
                                               add_residual)
    ref_in = {k: (v.astype(np.float64) if not k.startswith("c") else v) for k, v in c.items()}
    ref_in["x"] = d["x"].float().cpu().numpy().astype(np.float64)
    for k in ("vg", "vu", "vd"):
        ref_in[k] = np.swapaxes(d[k].float().cpu().numpy().astype(np.float64), -1, -2)
    ro = oracle_ffn(ref_in, add_residual=add_residual)[0]
    assert O.rel_l2(out.float().cpu().numpy(), ro) < 1e-2
    res, h, g, u = torch.ops.titan.block_ell_swiglu_fwd_with_intermediate(d["x"], d["vg"], d["cg"], d["vu"], d["cu"],
                                                                          d["vd"], d["cd"], add_residual)
    assert torch.equal(res, out)
    assert h.shape == (200, 512) and g.shape == (200, 512) and u.shape == (200, 512)
    assert K.read_status() == 0


def test_titan_persistent_mlp_step_matches_python_op():
    K = _K()
    c = make_case(130, 256, 512, 64, 2, 2, 4, seed=12)
    d = to_dev(c, torch.bfloat16, O.LAYOUT_OUT_IN)
    g = torch.Generator().manual_seed(3)
    e = torch.randn(130, 256, generator=g).to(torch.bfloat16).cuda()
    la, ld = torch.randn(256, generator=g).cuda(), torch.randn(256, generator=g).cuda()
    gain = torch.ones(256, dtype=torch.bfloat16, device="cuda")
    args = (d["x"], e, la, ld, [gain, gain], [d["vg"]] * 2, [d["cg"]] * 2, [d["vu"]] * 2, [d["cu"]] * 2,
            [d["vd"]] * 2, [d["cd"]] * 2)
    a = torch.ops.titan.persistent_mlp_step(*args)
    b = K.persistent_mlp_step(*args, eps=1e-6, layout=K.TILE_OUT_IN)  # the reference op's eps
    assert torch.equal(a, b)


@pytest.mark.parametrize("T,chunk", [(337, 100), (256, 256), (5, 64)])
def test_host_pipeline_equals_device_op(T, chunk):
    K = _K()
    c = make_case(T, 256, 512, 64, 2, 3, 4, seed=T)
    d = to_dev(c, torch.bfloat16)
    ref = K.block_ell_swiglu_fwd(d["x"], d["vg"], d["cg"], d["vu"], d["cu"], d["vd"], d["cd"], add_residual=True)
    xh = d["x"].cpu().pin_memory()
    out = K.block_ell_swiglu_fwd_host(xh, d["vg"], d["cg"], d["vu"], d["cu"], d["vd"], d["cd"], add_residual=True,
                                      chunk_tokens=chunk)
    torch.cuda.synchronize()
    assert not out.is_cuda
    assert torch.equal(out, ref.cpu())


def test_looped_host_pipeline_equals_device_op():
    K = _K()
    c = make_case(300, 256, 512, 64, 2, 3, 4, seed=21)
    d = to_dev(c, torch.bfloat16)
    gain = torch.ones(256, dtype=torch.bfloat16, device="cuda")
    ref = K.looped_ffn(d["x"], gain, d["vg"], d["cg"], d["vu"], d["cu"], d["vd"], d["cd"], L=3)
    out = K.looped_ffn_host(d["x"].cpu().pin_memory(), gain, d["vg"], d["cg"], d["vu"], d["cu"], d["vd"], d["cd"],
                            L=3, chunk_tokens=128)
    torch.cuda.synchronize()
    assert torch.equal(out, ref.cpu())


def test_gate_up_then_down_equals_fused_entry():
    """bell_gate_up_bf16 followed by bell_down_bf16 on the same descriptor gives
    the fused entry's result exactly."""
    import ctypes as C
    K = _K()
    from looped_blockell.kernels import _lib, ops
    c = make_case(300, 256, 512, 64, 2, 3, 4, seed=31)
    d = to_dev(c, torch.bfloat16)
    ref = K.block_ell_swiglu_fwd(d["x"], d["vg"], d["cg"], d["vu"], d["cu"], d["vd"], d["cd"], add_residual=True)
    lib = _lib.load()
    x = d["x"].contiguous()
    h = torch.empty((300, 512), dtype=torch.bfloat16, device="cuda")
    out = torch.empty_like(x)
    plan = torch.empty(ops.plan_bytes(8, 2, 3, 4, 4), dtype=torch.uint8, device="cuda")
    desc = _lib.BellFFNDesc()
    desc.T, desc.d_model, desc.d_ff, desc.dtype, desc.add_residual = 300, 256, 512, _lib.BELL_DTYPE_BF16, 1
    desc.x, desc.h, desc.out, desc.plan = x.data_ptr(), h.data_ptr(), out.data_ptr(), plan.data_ptr()
    desc.gate = ops._ell(d["vg"], d["cg"], 4, 0)
    desc.up = ops._ell(d["vu"], d["cu"], 4, 0)
    desc.down = ops._ell(d["vd"], d["cd"], 8, 0)
    _lib.check(lib.bell_gate_up_bf16(C.byref(desc), ops._stream()), "gate_up")
    _lib.check(lib.bell_down_bf16(C.byref(desc), ops._stream()), "down")
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
