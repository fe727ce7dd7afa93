"""The reference's native op names (torch.ops.titan.*) are registered with the
reference schemas; Meta shapes; no CPU kernel (fails at dispatch)."""

import pytest
import torch


def _K():
    from looped_blockell import kernels as K
    return K


def test_titan_ops_registered_with_reference_schemas():
    _K()
    for name in ("block_ell_swiglu_fwd", "block_ell_swiglu_fwd_with_intermediate", "pin_weights_l2",
                 "unpin_weights_l2", "persistent_mlp_step"):
        assert hasattr(torch.ops.titan, name), name
    schema = str(torch.ops.titan.block_ell_swiglu_fwd.default._schema)
    assert "Tensor x, Tensor v_gate, Tensor ci_gate, Tensor v_up, Tensor ci_up, Tensor v_down, Tensor ci_down, " \
           "bool add_residual" in schema


def test_titan_meta_shapes_use_the_tile_size():
    _K()
    m = dict(device="meta")
    x = torch.empty(10, 256, dtype=torch.bfloat16, **m)
    vg = torch.empty(8, 2, 64, 64, dtype=torch.bfloat16, **m)
    cg = torch.empty(8, 2, dtype=torch.int32, **m)
    vd = torch.empty(4, 4, 64, 64, dtype=torch.bfloat16, **m)
    cd = torch.empty(4, 4, dtype=torch.int32, **m)
    out = torch.ops.titan.block_ell_swiglu_fwd(x, vg, cg, vg, cg, vd, cd, True)
    assert out.shape == (10, 256)
    res, h, g, u = torch.ops.titan.block_ell_swiglu_fwd_with_intermediate(x, vg, cg, vg, cg, vd, cd, False)
    assert res.shape == (10, 256) and h.shape == g.shape == u.shape == (10, 512)


def test_titan_ops_have_no_cpu_kernel():
    _K()
    z = torch.zeros
    with pytest.raises(NotImplementedError):
        torch.ops.titan.block_ell_swiglu_fwd(z(4, 128, dtype=torch.bfloat16), z(4, 1, 64, 64, dtype=torch.bfloat16),
                                             z(4, 1, dtype=torch.int32), z(4, 1, 64, 64, dtype=torch.bfloat16),
                                             z(4, 1, dtype=torch.int32), z(2, 2, 64, 64, dtype=torch.bfloat16),
                                             z(2, 2, dtype=torch.int32), False)


def test_caller_buffers_are_checked_before_the_library_sees_them():
    """A caller-supplied output or workspace of the wrong size or dtype is
    refused on the host (the library writes through the pointer as given)."""
    import pytest
    import torch
    from looped_blockell.kernels import ops
    good = torch.zeros(4, 8)
    ops._check_out("out", good, (4, 8), torch.float32, good.device)
    with pytest.raises(RuntimeError, match="must be a contiguous"):
        ops._check_out("out", torch.zeros(4, 8, dtype=torch.bfloat16), (4, 8), torch.float32, good.device)
    with pytest.raises(RuntimeError, match="must be a contiguous"):
        ops._check_out("h", torch.zeros(4, 4), (4, 8), torch.float32, good.device)
    with pytest.raises(RuntimeError, match="must be a contiguous"):
        ops._check_out("h", torch.zeros(8, 4).t(), (4, 8), torch.float32, good.device)
