"""GPU dense -> Block-ELL conversion (bell_dense_to_ell) against the oracle's
restatement of create_block_ell_from_dense: the kept columns and the copied
tiles are exact; norms within fp32 rounding."""

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


def _K():
    from looped_blockell import kernels as K
    return K


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("B,layout", [(64, 0), (64, 1), (128, 0), (128, 1)])
def test_dense_to_ell_matches_oracle(B, layout, dtype):
    K = _K()
    rng = np.random.default_rng(B + layout)
    out_f, in_f = 3 * B, 7 * B
    dense = torch.from_numpy(rng.standard_normal((out_f, in_f)).astype(np.float32)).to(dtype)
    v, c, n = K.dense_to_block_ell(dense.cuda(), B, density=0.5, layout=layout)
    torch.cuda.synchronize()
    dn = dense.float().numpy().astype(np.float64)
    ov, oc = O.dense_to_block_ell(dn, B, 0.5)
    np.testing.assert_array_equal(c.cpu().numpy(), oc)
    got = v.float().cpu().numpy().astype(np.float64)
    if layout == 1:
        got = np.swapaxes(got, -1, -2)  # stored [B_out, B_in]
    np.testing.assert_array_equal(got, ov)
    blocks = dn.reshape(out_f // B, B, in_f // B, B)
    want_n = np.sqrt((blocks ** 2).sum(axis=(1, 3)))
    np.testing.assert_allclose(n.cpu().numpy(), want_n, rtol=1e-5)


def test_dense_to_ell_edges_and_ties():
    K = _K()
    B = 64
    # identical tiles: every norm ties, so the first K columns are kept (stable order)
    tile = torch.randn(B, B)
    dense = tile.repeat(2, 5).cuda()
    v, c, _ = K.dense_to_block_ell(dense, B, K=3)
    assert c.tolist() == [[0, 1, 2], [0, 1, 2]]
    # K = C keeps everything in column order; K = 1 keeps the largest tile
    dense = torch.randn(B, 4 * B)
    dense[:, 2 * B:3 * B] *= 10
    v, c, _ = K.dense_to_block_ell(dense.cuda(), B, K=4)
    assert c.tolist() == [[0, 1, 2, 3]]
    v, c, _ = K.dense_to_block_ell(dense.cuda(), B, K=1)
    assert c.tolist() == [[2]]
    torch.testing.assert_close(v[0, 0].cpu(), dense[:, 2 * B:3 * B].t(), rtol=0, atol=0)
    with pytest.raises(ValueError):
        K.dense_to_block_ell(torch.zeros(64, 100, device="cuda"), 64)


def test_layer_create_from_dense_uses_the_kernel_and_runs_forward():
    from looped_blockell.layers.block_ell import block_ell_matmul, create_block_ell_from_dense
    rng = np.random.default_rng(3)
    dense = torch.from_numpy(rng.standard_normal((256, 512)).astype(np.float32) * 0.02).to(torch.bfloat16).cuda()
    be = create_block_ell_from_dense(dense, tile_size=64, density=0.25)
    ov, oc = O.dense_to_block_ell(dense.float().cpu().numpy().astype(np.float64), 64, 0.25)
    np.testing.assert_array_equal(be.col_indices.cpu().numpy(), oc)
    x = torch.from_numpy(rng.standard_normal((100, 512)).astype(np.float32)).to(torch.bfloat16).cuda()
    y = block_ell_matmul(x, be)
    ref = O.block_ell_matmul(x.float().cpu().numpy().astype(np.float64), ov, oc)
    assert O.rel_l2(y.float().cpu().numpy(), ref) < 1e-2


@pytest.mark.parametrize("density", [None, 0.5])
def test_swiglu_from_state_dict_on_gpu_runs_the_forward(density):
    from looped_blockell import interop
    K = _K()
    rng = np.random.default_rng(11)
    d, F, B, T = 256, 512, 64, 130
    sd = {f"mlp.{k}.weight": torch.from_numpy((rng.standard_normal(s) * 0.05).astype(np.float32)).cuda()
          for k, s in (("w_gate", (F, d)), ("w_up", (F, d)), ("w_down", (d, F)))}
    w = interop.swiglu_from_state_dict(sd, "mlp.", tile_size=B, density=density)
    x = torch.from_numpy(rng.standard_normal((T, d)).astype(np.float32)).to(torch.bfloat16).cuda()
    out = K.block_ell_swiglu_fwd(x, w["vg"], w["cg"], w["vu"], w["cu"], w["vd"], w["cd"])
    torch.cuda.synchronize()
    f = lambda t: t.float().cpu().numpy().astype(np.float64)  # noqa: E731
    ref = O.swiglu_ffn(f(x), (f(w["vg"]), w["cg"].cpu().numpy(), 0), (f(w["vu"]), w["cu"].cpu().numpy(), 0),
                       (f(w["vd"]), w["cd"].cpu().numpy(), 0))
    assert O.rel_l2(f(out), ref) < 1e-2
    if density is None:  # every tile kept: the dense MLP of the (bf16) weights
        Wg, Wu, Wd = (f(sd[f"mlp.{k}.weight"].to(torch.bfloat16)) for k in ("w_gate", "w_up", "w_down"))
        g = f(x) @ Wg.T
        dense = (g / (1 + np.exp(-g)) * (f(x) @ Wu.T)) @ Wd.T
        assert O.rel_l2(f(out), dense) < 1e-2
