"""Loading the reference PyTorch MLP's weights into the Block-ELL container
(density 1.0, tile masks, top-K), checked on CPU tensors against the oracle."""

import numpy as np
import torch

import oracle as O


def _io():
    from looped_blockell import interop
    return interop


def test_full_conversion_round_trip():
    io = _io()
    rng = np.random.default_rng(0)
    w = torch.from_numpy(rng.standard_normal((24, 40)).astype(np.float32))
    v, c = io.dense_to_block_ell_full(w, 8)
    assert v.shape == (3, 5, 8, 8) and c.tolist() == [[0, 1, 2, 3, 4]] * 3
    np.testing.assert_array_equal(io.block_ell_to_dense_weight(v, c, 24, 40).numpy(), w.numpy())
    np.testing.assert_array_equal(O.block_ell_to_dense(v.numpy(), c.numpy(), 24, 40), w.numpy())


def test_tile_mask_conversion():
    io = _io()
    rng = np.random.default_rng(1)
    w = torch.from_numpy(rng.standard_normal((16, 32)).astype(np.float32))
    mask = torch.tensor([[1, 0, 1, 1], [0, 0, 1, 0]], dtype=torch.bool)
    v, c = io.masked_dense_to_block_ell(w, mask, 8)
    assert c.tolist() == [[0, 2, 3], [2, -1, -1]]
    dense = io.block_ell_to_dense_weight(v, c, 16, 32).numpy()
    want = w.numpy() * np.kron(mask.numpy(), np.ones((8, 8)))
    np.testing.assert_array_equal(dense, want)


def test_swiglu_from_state_dict_matches_dense_mlp():
    io = _io()
    rng = np.random.default_rng(2)
    d, F, B = 16, 32, 8
    sd = {"core.0.mlp.w_gate.weight": torch.from_numpy(rng.standard_normal((F, d))),
          "core.0.mlp.w_up.weight": torch.from_numpy(rng.standard_normal((F, d))),
          "core.0.mlp.w_down.weight": torch.from_numpy(rng.standard_normal((d, F)))}
    sd["core.0.mlp.w_up.tile_mask"] = torch.from_numpy(rng.random((F // B, d // B)) < 0.6)
    w = io.swiglu_from_state_dict(sd, "core.0.mlp.", tile_size=B, dtype=torch.float64)
    x = rng.standard_normal((5, d))
    got = O.swiglu_ffn(x, (w["vg"].numpy(), w["cg"].numpy(), 0), (w["vu"].numpy(), w["cu"].numpy(), 0),
                       (w["vd"].numpy(), w["cd"].numpy(), 0))
    Wg, Wd = sd["core.0.mlp.w_gate.weight"].numpy(), sd["core.0.mlp.w_down.weight"].numpy()
    Wu = sd["core.0.mlp.w_up.weight"].numpy() * np.kron(sd["core.0.mlp.w_up.tile_mask"].numpy(), np.ones((B, B)))
    g = x @ Wg.T
    want = (g / (1 + np.exp(-g)) * (x @ Wu.T)) @ Wd.T  # pt_model.py:896-898
    np.testing.assert_allclose(got, want, rtol=1e-10, atol=1e-10)
