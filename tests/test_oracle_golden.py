"""Pin the CPU oracle against fixtures produced by the reference's own code.

Fixtures come from tests/golden/make_golden.py, which ran the reference's
interop/pt_model.py MLPBlock/RMSNorm, interop/convert_checkpoint.py and
bonsai-test/bitlinear.py.  These tests run on CPU only.
"""

import os

import numpy as np
import pytest

import oracle as O
from conftest import GOLDEN


def _load(name):
    return np.load(os.path.join(GOLDEN, f"{name}.npz"))


@pytest.mark.parametrize("case", ["swiglu_small", "swiglu_dead"])
def test_swiglu_matches_reference_mlpblock(case):
    z = _load(case)
    out = O.swiglu_ffn(z["x"], (z["vg"], z["cg"], O.LAYOUT_IN_OUT), (z["vu"], z["cu"], O.LAYOUT_IN_OUT),
                       (z["vd"], z["cd"], O.LAYOUT_IN_OUT))
    assert O.rel_l2(out, z["out"]) < 1e-12


def test_swiglu_residual_epilogue():
    z = _load("swiglu_small")
    out = O.swiglu_ffn(z["x"], (z["vg"], z["cg"], 0), (z["vu"], z["cu"], 0), (z["vd"], z["cd"], 0),
                       add_residual=True)
    assert O.rel_l2(out, z["out"] + z["x"]) < 1e-12


def test_tile_layout_is_in_out():
    """values[r, k] is [B_in, B_out] (convert_checkpoint.py:118-131)."""
    z = _load("tile_layout")
    v, c = O.dense_to_block_ell(z["W"], 64, 1.0)
    np.testing.assert_array_equal(c, z["cols"])
    np.testing.assert_array_equal(v, z["values"])
    back = O.block_ell_to_dense(z["values"], z["cols"], 128, 256)
    np.testing.assert_array_equal(back, z["back"])
    x = np.random.default_rng(0).standard_normal((5, 256)).astype(np.float32)
    y = O.block_ell_matmul(x, z["values"], z["cols"])
    np.testing.assert_allclose(y, x.astype(np.float64) @ z["W"].T.astype(np.float64), rtol=1e-10, atol=1e-10)


def test_out_in_layout_equivalent():
    z = _load("tile_layout")
    x = np.random.default_rng(1).standard_normal((7, 256))
    y0 = O.block_ell_matmul(x, z["values"], z["cols"], O.LAYOUT_IN_OUT)
    y1 = O.block_ell_matmul(x, np.swapaxes(z["values"], -1, -2), z["cols"], O.LAYOUT_OUT_IN)
    np.testing.assert_allclose(y0, y1, rtol=0, atol=0)


def test_rmsnorm_matches_reference():
    z = _load("rmsnorm")
    out = O.rmsnorm(z["x"], z["gain"], float(z["eps"]))
    np.testing.assert_allclose(out, z["out"], rtol=1e-13, atol=1e-13)


def test_loop_matches_reference_order():
    z = _load("loop")
    out = O.looped_ffn(z["h0"], z["gain"], (z["vg"], z["cg"], 0), (z["vu"], z["cu"], 0),
                       (z["vd"], z["cd"], 0), L=int(z["L"]), eps=float(z["eps"]))
    assert O.rel_l2(out, z["out"]) < 1e-12


def test_ternary_quantizers_match_bitlinear():
    z = _load("ternary")
    t, s = O.ternary_quantize_tiles(z["vg"])
    np.testing.assert_allclose(s.ravel(), z["s"], rtol=2e-7, atol=0)
    np.testing.assert_array_equal(t, z["t"])
    q, scale = O.activation_quantize_int(z["x"])
    # the reference returns the dequantised activation q / scale
    np.testing.assert_array_equal((q.astype(np.float32) / scale[:, None]).astype(np.float32), z["x_dq"])


def test_ternary_matmul_matches_fake_quant_linear():
    z = _load("ternary")
    t, s = O.ternary_quantize_tiles(z["vg"])
    q, scale = O.activation_quantize_int(z["x"])
    y = O.ternary_block_ell_matmul(q, scale, t, s, z["cg"])
    assert O.rel_l2(y, z["y"]) < 1e-6


def test_pack_roundtrip_and_codes():
    rng = np.random.default_rng(2)
    t = rng.integers(-1, 2, size=(3, 2, 64, 64)).astype(np.int8)
    p = O.pack_ternary(t)
    assert p.shape == (3, 2, 64, 16) and p.dtype == np.uint8
    np.testing.assert_array_equal(O.unpack_ternary(p), t)
    # element (i=B_in 0, j=B_out 0) -> word 0 bits 0-1
    t2 = np.zeros((1, 1, 64, 64), np.int8)
    t2[0, 0, 1, 0] = -1  # B_in 1 of output column 0 -> bits 2-3 of word 0
    w = O.pack_ternary(t2).view(np.uint32)
    assert w[0, 0, 0, 0] == 0b1100


def test_ternary_tile_sums_exact_int():
    rng = np.random.default_rng(4)
    T, B, R, K, C = 9, 64, 2, 2, 3
    q = rng.integers(-128, 128, size=(T, C * B)).astype(np.int8)
    t = rng.integers(-1, 2, size=(R, K, B, B)).astype(np.int8)
    cols = np.array([[0, 2], [1, -1]], np.int32)
    s_w = np.ones((R, K), np.float32)
    y, sums = O.ternary_block_ell_matmul(q, np.ones(T, np.float32), t, s_w, cols, return_tile_sums=True)
    ref = q[:, 0:64].astype(np.int64) @ t[0, 0].astype(np.int64)
    np.testing.assert_array_equal(sums[(0, 0)], ref)
    assert (1, 1) not in sums


def test_random_topology_unique_sorted():
    rng = np.random.default_rng(0)
    c = O.random_topology(16, 32, 8, rng)
    assert c.shape == (16, 8) and c.dtype == np.int32
    for row in c:
        assert len(np.unique(row)) == 8 and np.all(np.diff(row) > 0)


def test_oracle_backward_matches_torch_autograd():
    """The oracle's SwiGLU gradients equal torch autograd through the dense
    restatement (float64), including dead and duplicate slots."""
    import torch
    rng = np.random.default_rng(7)
    T, d, F, B = 9, 128, 256, 64
    cg = np.array([[0, 1], [1, -1], [0, 0], [1, 0]], dtype=np.int32)
    cu = np.array([[1, 0], [0, 1], [-1, 1], [0, 1]], dtype=np.int32)
    cd = np.array([[0, 2, 3], [1, 3, -1]], dtype=np.int32)
    vg = rng.standard_normal((4, 2, B, B)) * 0.05
    vu = rng.standard_normal((4, 2, B, B)) * 0.05
    vd = rng.standard_normal((2, 3, B, B)) * 0.05
    x = rng.standard_normal((T, d))
    dy = rng.standard_normal((T, d))
    dx, dvg, dvu, dvd = O.swiglu_ffn_backward(x, (vg, cg, 0), (vu, cu, 0), (vd, cd, 0), dy, add_residual=True)
    tv = [torch.tensor(a, dtype=torch.float64, requires_grad=True) for a in (x, vg, vu, vd)]

    def ell(v, c, out_f, in_f):
        W = torch.zeros(out_f, in_f, dtype=torch.float64)
        for r in range(c.shape[0]):
            for k in range(c.shape[1]):
                if c[r, k] >= 0:
                    W = W.index_put((torch.arange(r * B, (r + 1) * B)[:, None],
                                     torch.arange(c[r, k] * B, (c[r, k] + 1) * B)[None, :]),
                                    v[r, k].T, accumulate=True)
        return W

    xt, vgt, vut, vdt = tv
    out = (torch.nn.functional.silu(xt @ ell(vgt, cg, F, d).T) * (xt @ ell(vut, cu, F, d).T)) @ ell(vdt, cd, d, F).T + xt
    out.backward(torch.tensor(dy))
    for mine, ref in ((dx, xt.grad), (dvg, vgt.grad), (dvu, vut.grad), (dvd, vdt.grad)):
        np.testing.assert_allclose(mine, ref.numpy(), rtol=1e-10, atol=1e-12)


@pytest.mark.parametrize("layout", [0, 1])
def test_oracle_sparse_backward_matches_dense(layout):
    """The tile-by-tile backward (the CPU timing arm) equals the dense restatement."""
    rng = np.random.default_rng(7)
    T, d, F, B = 9, 8, 12, 4
    Rf, Cd, Rd, Cf = F // B, d // B, d // B, F // B
    cg = np.array([[0, 1], [1, -1], [0, 0]], np.int32)
    cu = np.array([[1, 0], [0, 1], [-1, 1]], np.int32)
    cd = np.array([[0, 2], [1, -1]], np.int32)
    vg, vu = rng.standard_normal((Rf, 2, B, B)), rng.standard_normal((Rf, 2, B, B))
    vd = rng.standard_normal((Rd, 2, B, B))
    x, dy = rng.standard_normal((T, d)), rng.standard_normal((T, d))
    mats = ((vg, cg, layout), (vu, cu, layout), (vd, cd, layout))
    out, h, g, u = O.swiglu_ffn(x, *mats, return_intermediates=True)
    dense = O.swiglu_ffn_backward(x, *mats, dy)
    sparse = O.swiglu_ffn_backward_sparse(x, *mats, dy, g, u, h)
    for a, b in zip(dense, sparse):
        np.testing.assert_allclose(a, b, rtol=1e-10, atol=1e-10)


def test_fma_f32_is_correctly_rounded():
    """The oracle's float32 FMA against exact rational arithmetic, on random
    operands shaped like the ternary combination (scale x integer tile sum +
    accumulator) and on cases built to land on a float32 rounding midpoint."""
    from fractions import Fraction
    rng = np.random.default_rng(7)
    a = (np.abs(rng.standard_normal(4000)) * 0.02 + 1e-4).astype(np.float32)
    b = rng.integers(-8192, 8193, size=4000).astype(np.float32)
    c = (rng.standard_normal(4000) * 50).astype(np.float32)
    # midpoints: c = -a*b rounded, plus half an ulp of a product-sized value
    c[:500] = (-(a[:500].astype(np.float64) * b[:500])).astype(np.float32)
    got = O.fma_f32(a, b, c)

    def exact(ai, bi, ci):
        v = Fraction(float(ai)) * Fraction(float(bi)) + Fraction(float(ci))
        # nearest float32, ties to even, from the exact rational
        f = np.float32(float(v))
        lo, hi = sorted((f, np.nextafter(f, np.float32(np.inf) if Fraction(float(f)) < v else np.float32(-np.inf))))
        dlo, dhi = abs(Fraction(float(lo)) - v), abs(Fraction(float(hi)) - v)
        if dlo != dhi:
            return lo if dlo < dhi else hi
        return lo if (lo.view(np.int32) & 1) == 0 else hi

    want = np.array([exact(x, y, z) for x, y, z in zip(a, b, c)], dtype=np.float32)
    np.testing.assert_array_equal(got.view(np.int32), want.view(np.int32))
