"""Host logic of the backward: the transposed Block-ELL builder (pure torch,
runs on CPU tensors) against the dense transpose, and the titan backward op's
schema and Meta shapes."""

import numpy as np
import pytest
import torch

import oracle as O


def _K():
    from looped_blockell import kernels as K
    return K


def _dense(values, cols, R, C, layout):
    return O.block_ell_to_dense(values.numpy().astype(np.float64), cols.numpy(), R * values.shape[-1],
                                C * values.shape[-1], layout)


@pytest.mark.parametrize("layout", [O.LAYOUT_IN_OUT, O.LAYOUT_OUT_IN])
def test_transpose_ell_is_the_dense_transpose(layout):
    K = _K()
    rng = np.random.default_rng(0)
    R, C, Kk, B = 6, 5, 3, 4
    cols = np.stack([rng.choice(C, size=Kk, replace=False) for _ in range(R)]).astype(np.int32)
    cols[1, 2] = -1          # dead slot
    cols[2, 1] = cols[2, 0]  # duplicate column (both tiles count)
    vals = torch.from_numpy(rng.standard_normal((R, Kk, B, B)))
    ct = torch.from_numpy(cols)
    vt, ctt, lt = K.transpose_ell([vals], [ct], C, layout)
    assert lt != layout and vt.shape[:2] == ctt.shape and ctt.shape[0] == C
    W = _dense(vals, ct, R, C, layout)
    Wt = _dense(vt, ctt, C, R, lt)
    np.testing.assert_allclose(Wt, W.T, rtol=0, atol=0)
    # every live slot appears once; rows list ascending block-rows
    live = int((cols >= 0).sum())
    assert int((ctt >= 0).sum()) == live
    for c in range(C):
        row = ctt[c][ctt[c] >= 0].tolist()
        assert row == sorted(row)


def test_transpose_ell_of_stacked_gate_up():
    K = _K()
    rng = np.random.default_rng(1)
    R, C, Kg, Ku, B = 4, 3, 2, 3, 2
    cg = torch.from_numpy(np.stack([rng.choice(C, size=Kg, replace=False) for _ in range(R)]).astype(np.int32))
    cu = torch.from_numpy(np.stack([rng.choice(C, size=Ku, replace=False) for _ in range(R)]).astype(np.int32))
    cu[3, 0] = -1
    vg = torch.from_numpy(rng.standard_normal((R, Kg, B, B)))
    vu = torch.from_numpy(rng.standard_normal((R, Ku, B, B)))
    vt, ctt, lt = K.transpose_ell([vg, vu], [cg, cu], C, O.LAYOUT_IN_OUT)
    Wg = _dense(vg, cg, R, C, O.LAYOUT_IN_OUT)
    Wu = _dense(vu, cu, R, C, O.LAYOUT_IN_OUT)
    Wt = _dense(vt, ctt, C, 2 * R, lt)
    np.testing.assert_allclose(Wt, np.concatenate([Wg, Wu]).T, rtol=0, atol=0)


def test_transposed_topology_drops_out_of_range_and_is_cached():
    K = _K()
    cols = torch.tensor([[0, 7], [-1, 1], [1, -3]], dtype=torch.int32)  # 7 and -3 are outside [-1, C)
    ct, idx = K.transposed_topology([cols], 2)
    assert ct.tolist() == [[0, -1], [1, 2]]
    assert idx[0, 0].item() == 0 and idx[1].tolist() == [3, 4]
    ct2, _ = K.transposed_topology([cols], 2)
    assert ct2 is ct  # same tensor version -> cached
    cols[0, 0] = 1      # in-place change bumps the version -> rebuilt
    ct3, _ = K.transposed_topology([cols], 2)
    assert ct3 is not ct and ct3.tolist() == [[-1, -1, -1], [0, 1, 2]]


def test_titan_bwd_schema_and_meta_shapes():
    _K()
    schema = str(torch.ops.titan.block_ell_swiglu_bwd.default._schema)
    assert "Tensor grad_out, Tensor x, Tensor gate_pre_act, Tensor up_out, Tensor h, Tensor v_gate" in schema
    m = dict(device="meta")
    x = torch.empty(10, 256, dtype=torch.bfloat16, **m)
    mid = torch.empty(10, 512, dtype=torch.bfloat16, **m)
    vg = torch.empty(8, 2, 64, 64, dtype=torch.bfloat16, **m)
    vu = torch.empty(8, 3, 64, 64, dtype=torch.bfloat16, **m)
    vd = torch.empty(4, 4, 64, 64, dtype=torch.bfloat16, **m)
    ci = torch.empty(1, 1, dtype=torch.int32, **m)
    dx, a, b, c = torch.ops.titan.block_ell_swiglu_bwd(x, x, mid, mid, mid, vg, ci, vu, ci, vd, ci)
    assert dx.shape == x.shape and a.shape == vg.shape and b.shape == vu.shape and c.shape == vd.shape


def test_topology_cache_never_matches_a_different_tensor():
    """A new index tensor with the same shape (even reusing freed memory) is a miss."""
    K = _K()
    a = torch.tensor([[0, 1], [1, 0]], dtype=torch.int32)
    ta, _ = K.transposed_topology([a], 2)
    b = torch.tensor([[1, -1], [0, -1]], dtype=torch.int32)
    tb, _ = K.transposed_topology([b], 2)
    assert ta.tolist() == [[0, 1], [0, 1]] and tb.tolist() == [[1], [0]]
    del a
    c = torch.tensor([[1, 1], [1, 1]], dtype=torch.int32)
    tc, _ = K.transposed_topology([c], 2)
    assert tc.tolist() == [[-1, -1, -1, -1], [0, 0, 1, 1]]


def test_transpose_ell_caches_tiles_per_weight_version():
    """transpose_ell reuses its gathered tiles while the value and column
    tensors keep their contents, and regathers after an in-place update."""
    import torch
    from looped_blockell.kernels.backward import transpose_ell
    g = torch.Generator().manual_seed(0)
    v = torch.randn(4, 2, 16, 16, generator=g)
    c = torch.tensor([[0, 2], [1, 2], [0, 1], [2, -1]], dtype=torch.int32)
    a = transpose_ell([v], [c], 3)
    b = transpose_ell([v], [c], 3)
    assert a[0] is b[0]
    v.mul_(2.0)  # an optimizer-style in-place update bumps the version
    d = transpose_ell([v], [c], 3)
    assert d[0] is not a[0]
    assert torch.equal(d[0], a[0] * 2.0)
