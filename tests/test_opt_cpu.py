"""Topology maintenance (compaction, d_ff column reorder) against the oracle's
restatements of looped_blockell/opt, on CPU tensors; the reorder leaves the
SwiGLU's output unchanged."""

import numpy as np
import pytest
import torch

import oracle as O


def _opt():
    from looped_blockell import opt
    return opt


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_compaction_matches_oracle(seed):
    opt = _opt()
    rng = np.random.default_rng(seed)
    R, K, B = 7, 6, 4
    vals = rng.standard_normal((R, K, B, B)).astype(np.float32)
    cols = rng.integers(0, 9, size=(R, K)).astype(np.int32)
    alive = rng.random((R, K)) < 0.5
    alive[3] = False  # a row with nothing alive
    v, c, a, kn = opt.compact_single_layer(torch.from_numpy(vals), torch.from_numpy(cols), torch.from_numpy(alive))
    ov, oc, oa, okn = O.compact_block_ell(vals, cols, alive)
    assert kn == okn
    np.testing.assert_array_equal(v.numpy(), ov)
    np.testing.assert_array_equal(c.numpy(), oc)
    np.testing.assert_array_equal(a.numpy(), oa)


def test_compaction_all_dead_keeps_one_slot():
    opt = _opt()
    v, c, a, kn = opt.compact_single_layer(torch.zeros(2, 3, 2, 2), torch.zeros(2, 3, dtype=torch.int32),
                                           torch.zeros(2, 3, dtype=torch.bool))
    assert kn == 1 and v.shape == (2, 1, 2, 2) and not a.any()


def test_column_reorder_functions_match_oracle():
    opt = _opt()
    rng = np.random.default_rng(4)
    C_ff, R1, K1, K2 = 10, 5, 4, 3
    fc1_cols = rng.integers(-1, C_ff, size=(R1, K1)).astype(np.int32)
    fc1_alive = rng.random((R1, K1)) < 0.7
    fc2_alive = rng.random((C_ff, K2)) < 0.6
    fc2_cols = rng.integers(0, 6, size=(C_ff, K2)).astype(np.int32)
    imp = opt.compute_column_importance(torch.from_numpy(fc1_alive), torch.from_numpy(fc2_alive),
                                        torch.from_numpy(fc1_cols), torch.from_numpy(fc2_cols), C_ff)
    perm = opt.compute_permutation(imp)
    np.testing.assert_array_equal(perm.numpy(), O.dff_permutation(fc1_alive, fc2_alive, fc1_cols, C_ff))
    v1 = torch.from_numpy(rng.standard_normal((R1, K1, 2, 2)))
    _, c1, _ = opt.apply_permutation_to_block_ell(v1, torch.from_numpy(fc1_cols), torch.from_numpy(fc1_alive), perm,
                                                  is_column_dim=True)
    inv = np.empty(C_ff, np.int64)
    inv[perm.numpy()] = np.arange(C_ff)
    want = np.where(fc1_cols < 0, -1, inv[np.clip(fc1_cols, 0, C_ff - 1)])
    np.testing.assert_array_equal(c1.numpy(), want)
    v2 = torch.from_numpy(rng.standard_normal((C_ff, K2, 2, 2)))
    nv2, nc2, na2 = opt.apply_permutation_to_block_ell(v2, torch.from_numpy(fc2_cols), torch.from_numpy(fc2_alive),
                                                       perm, is_column_dim=False)
    np.testing.assert_array_equal(nv2.numpy(), v2.numpy()[perm.numpy()])
    k = opt.compute_k_active_macros(torch.from_numpy(fc1_alive), c1, 4, C_ff)
    live = np.where(fc1_alive, c1.numpy(), -1).max()
    assert int(k) == (0 if live < 0 else int(np.ceil((live + 1) / 4)))


def test_swiglu_dff_reorder_preserves_the_function():
    opt = _opt()
    rng = np.random.default_rng(5)
    T, d, F, B = 6, 8, 16, 2
    Rf, Cd, Rd, Cf = F // B, d // B, d // B, F // B
    cg = np.stack([rng.choice(Cd, 2, replace=False) for _ in range(Rf)]).astype(np.int32)
    cu = np.stack([rng.choice(Cd, 3, replace=False) for _ in range(Rf)]).astype(np.int32)
    cd = np.stack([rng.choice(Cf, 3, replace=False) for _ in range(Rd)]).astype(np.int32)
    cd[0, 2] = -1
    vg, vu = rng.standard_normal((Rf, 2, B, B)), rng.standard_normal((Rf, 3, B, B))
    vd = rng.standard_normal((Rd, 3, B, B))
    x = rng.standard_normal((T, d))
    ref = O.swiglu_ffn(x, (vg, cg, 0), (vu, cu, 0), (vd, cd, 0))
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a))  # noqa: E731
    vg2, cg2, vu2, cu2, vd2, cd2, perm, k = opt.reorder_swiglu_dff(t(vg), t(cg), t(vu), t(cu), t(vd), t(cd))
    out = O.swiglu_ffn(x, (vg2.numpy(), cg2.numpy(), 0), (vu2.numpy(), cu2.numpy(), 0), (vd2.numpy(), cd2.numpy(), 0))
    np.testing.assert_allclose(out, ref, rtol=1e-12, atol=1e-12)
    # the most used d_ff blocks come first
    imp = np.zeros(Cf)
    for c in cd.reshape(-1):
        if c >= 0:
            imp[c] += 1
    imp += 2 + 3  # every gate/up row is fully alive here
    assert list(np.argsort(-imp, kind="stable")) == perm.tolist()


def test_create_block_ell_from_dense_cpu_matches_oracle():
    from looped_blockell.layers.block_ell import create_block_ell_from_dense
    rng = np.random.default_rng(6)
    dense = rng.standard_normal((32, 48)).astype(np.float32)
    be = create_block_ell_from_dense(torch.from_numpy(dense), tile_size=8, density=0.5)
    ov, oc = O.dense_to_block_ell(dense, 8, 0.5)
    np.testing.assert_array_equal(be.col_indices.numpy(), oc)
    np.testing.assert_array_equal(be.values.numpy(), ov)
