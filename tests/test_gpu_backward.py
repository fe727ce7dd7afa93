"""GPU parity of the SwiGLU backward (d_h, SiLU*up backward, d_x, tile
gradients) against the float64 oracle restatement of the reference backward
(csrc/block_ell/swiglu_bwd.cu).  bf16 inputs and outputs: rel-L2 <= 2e-2 for
the end-to-end gradients (the reference keeps d_h, d_gate, d_up in bf16 too);
the tile-gradient kernel alone is checked in fp32 against exact float64 sums
of the same bf16 inputs (rel-L2 <= 1e-5)."""

import numpy as np
import pytest
import torch

import oracle as O
from gpu_util import make_case, to_dev

pytestmark = pytest.mark.gpu

TOL = 2e-2


def _K():
    from looped_blockell import kernels as K
    return K


def _f64(t):
    return t.float().cpu().numpy().astype(np.float64)


def _bwd_case(T, d, F, B, Kg, Ku, Kd, layout, seed, dead=0, dup=False, fuse_silu=True):
    K = _K()
    c = make_case(T, d, F, B, Kg, Ku, Kd, seed=seed, dead=dead, dup=dup)
    dv = to_dev(c, torch.bfloat16, layout)
    g = torch.Generator().manual_seed(seed + 1)
    dy = torch.randn(T, d, generator=g).to(torch.bfloat16).cuda()
    out, h, gp, up = K.block_ell_swiglu_fwd_with_intermediate(dv["x"], dv["vg"], dv["cg"], dv["vu"], dv["cu"],
                                                              dv["vd"], dv["cd"], add_residual=True, layout=layout)
    res = K.block_ell_swiglu_bwd(dy, dv["x"], gp, up, h, dv["vg"], dv["cg"], dv["vu"], dv["cu"], dv["vd"], dv["cd"],
                                 layout=layout, fuse_silu=fuse_silu)
    torch.cuda.synchronize()
    assert K.read_status() == 0
    mats = [(_f64(dv[v]), dv[ci].cpu().numpy(), layout) for v, ci in (("vg", "cg"), ("vu", "cu"), ("vd", "cd"))]
    ref = O.swiglu_ffn_backward(_f64(dv["x"]), *mats, _f64(dy), add_residual=True)
    return res, ref, dv


@pytest.mark.parametrize("fuse_silu", [True, False])
@pytest.mark.parametrize("B,layout", [(64, O.LAYOUT_IN_OUT), (64, O.LAYOUT_OUT_IN), (128, O.LAYOUT_IN_OUT),
                                      (128, O.LAYOUT_OUT_IN)])
def test_swiglu_backward_matches_oracle(B, layout, fuse_silu):
    F = 4 * B * 2
    d = 2 * B * 2
    res, ref, dv = _bwd_case(333, d, F, B, 2, 3, 3, layout, seed=B + layout, dead=2, dup=True, fuse_silu=fuse_silu)
    for name, a, b in zip(("dx", "d_vg", "d_vu", "d_vd"), res, ref):
        assert tuple(a.shape) == b.shape, name
        assert a.dtype == torch.bfloat16
        assert O.rel_l2(_f64(a), b) < TOL, name
    # dead slots carry zero tiles
    for (vname, cname), grad in zip((("vg", "cg"), ("vu", "cu"), ("vd", "cd")), res[1:]):
        dead = dv[cname].cpu().numpy() < 0
        if dead.any():
            assert float(grad.float().cpu().numpy()[dead].__abs__().max()) == 0.0


def test_swiglu_backward_odd_slot_count_and_ragged_tokens():
    # K odd at B=64 (a unit pairs two slots, the last one alone); T not a multiple of 64
    res, ref, _ = _bwd_case(71, 256, 512, 64, 3, 1, 5, O.LAYOUT_IN_OUT, seed=5)
    for name, a, b in zip(("dx", "d_vg", "d_vu", "d_vd"), res, ref):
        assert O.rel_l2(_f64(a), b) < TOL, name


def test_swiglu_backward_single_token_and_empty():
    K = _K()
    res, ref, _ = _bwd_case(1, 256, 512, 64, 2, 2, 4, O.LAYOUT_IN_OUT, seed=8)
    for name, a, b in zip(("dx", "d_vg", "d_vu", "d_vd"), res, ref):
        assert O.rel_l2(_f64(a), b) < TOL, name
    c = make_case(1, 256, 512, 64, 2, 2, 4, seed=9)
    dv = to_dev(c, torch.bfloat16)
    z = torch.empty(0, 256, dtype=torch.bfloat16, device="cuda")
    zf = torch.empty(0, 512, dtype=torch.bfloat16, device="cuda")
    dx, a, b, cc = K.block_ell_swiglu_bwd(z, z, zf, zf, zf, dv["vg"], dv["cg"], dv["vu"], dv["cu"], dv["vd"], dv["cd"])
    assert dx.shape == (0, 256)
    for t in (a, b, cc):
        assert float(t.float().abs().max()) == 0.0


@pytest.mark.parametrize("B,layout,T", [(64, O.LAYOUT_IN_OUT, 5000), (64, O.LAYOUT_OUT_IN, 129),
                                        (128, O.LAYOUT_IN_OUT, 3001), (128, O.LAYOUT_OUT_IN, 64)])
def test_sddmm_exact_in_fp32(B, layout, T):
    """Tile gradients alone: fp32 sums of bf16 products against float64."""
    K = _K()
    rng = np.random.default_rng(B + T)
    R, C, Kk = 5, 4, 3
    cols = np.stack([rng.choice(C, size=Kk, replace=False) for _ in range(R)]).astype(np.int32)
    cols[2, 1] = -1
    a = torch.from_numpy(rng.standard_normal((T, C * B)).astype(np.float32)).to(torch.bfloat16)
    b = torch.from_numpy(rng.standard_normal((T, R * B)).astype(np.float32)).to(torch.bfloat16)
    grad = K.block_ell_sddmm(a.cuda(), b.cuda(), torch.from_numpy(cols).cuda(), B, layout)
    torch.cuda.synchronize()
    a64, b64 = _f64(a), _f64(b)
    want = np.zeros((R, Kk, B, B))
    for r in range(R):
        for k in range(Kk):
            c = cols[r, k]
            if c >= 0:
                t = a64[:, c * B:(c + 1) * B].T @ b64[:, r * B:(r + 1) * B]  # [B_in, B_out]
                want[r, k] = t if layout == O.LAYOUT_IN_OUT else t.T
    got = grad.cpu().numpy().astype(np.float64)
    assert O.rel_l2(got, want) < 1e-5
    assert np.all(got[cols < 0] == 0)


def test_sddmm_accumulates_and_strided_operand():
    K = _K()
    rng = np.random.default_rng(3)
    T, B, R, C = 700, 64, 3, 2
    cols = torch.tensor([[0, 1], [1, -1], [0, 0]], dtype=torch.int32, device="cuda")
    a = torch.from_numpy(rng.standard_normal((T, C * B)).astype(np.float32)).to(torch.bfloat16).cuda()
    wide = torch.from_numpy(rng.standard_normal((T, 2 * R * B)).astype(np.float32)).to(torch.bfloat16).cuda()
    b = wide[:, R * B:]  # right half of a wider row-major tensor
    g1 = K.block_ell_sddmm(a, b, cols, B)
    g2 = K.block_ell_sddmm(a, b.contiguous(), cols, B)
    torch.cuda.synchronize()
    assert torch.allclose(g1, g2, rtol=1e-6, atol=1e-5)
    K.block_ell_sddmm(a, b, cols, B, grad=g1, accumulate=True)
    torch.cuda.synchronize()
    assert torch.allclose(g1, 2 * g2, rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("B", [64, 128])
def test_fused_down_silu_bwd_matches_formula(B):
    """[d_gate | d_up] of the fused launch against float64 from the same bf16 inputs."""
    K = _K()
    c = make_case(300, 2 * B * 2, 4 * B * 2, B, 2, 2, 3, seed=B, dead=1)
    dv = to_dev(c, torch.bfloat16)
    T, d, F = 300, 4 * B, 8 * B
    g = torch.Generator().manual_seed(6)
    dy = torch.randn(T, d, generator=g).to(torch.bfloat16).cuda()
    gp, up = (torch.randn(T, F, generator=g).to(torch.bfloat16).cuda() for _ in range(2))
    vdT, cdT, lt = K.transpose_ell([dv["vd"]], [dv["cd"]], F // B)
    out = K.down_silu_bwd(dy, vdT, cdT, lt, gp, up)
    torch.cuda.synchronize()
    Wd = O.block_ell_to_dense(_f64(dv["vd"]), dv["cd"].cpu().numpy(), d, F)
    dh = _f64(dy) @ Wd
    gg, uu = _f64(gp), _f64(up)
    s = 1.0 / (1.0 + np.exp(-gg))
    assert O.rel_l2(_f64(out[:, :F]), dh * uu * (s + gg * s * (1 - s))) < 1e-2
    assert O.rel_l2(_f64(out[:, F:]), dh * gg * s) < 1e-2
    assert K.read_status() == 0


def test_silu_mul_bwd_matches_formula():
    K = _K()
    g = torch.Generator().manual_seed(4)
    T, F = 77, 192
    dh, gp, up = (torch.randn(T, F, generator=g).to(torch.bfloat16).cuda() for _ in range(3))
    out = K.silu_mul_bwd(dh, gp, up)
    torch.cuda.synchronize()
    h, gg, u = _f64(dh), _f64(gp), _f64(up)
    s = 1.0 / (1.0 + np.exp(-gg))
    assert O.rel_l2(_f64(out[:, :F]), h * u * (s + gg * s * (1 - s))) < 1e-2
    assert O.rel_l2(_f64(out[:, F:]), h * gg * s) < 1e-2


def test_titan_bwd_and_autograd_match_python_op():
    K = _K()
    c = make_case(150, 256, 512, 64, 2, 2, 4, seed=21)
    dv = to_dev(c, torch.bfloat16, O.LAYOUT_OUT_IN)
    dy = torch.randn(150, 256, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16).cuda()
    out, h, gp, up = torch.ops.titan.block_ell_swiglu_fwd_with_intermediate(dv["x"], dv["vg"], dv["cg"], dv["vu"],
                                                                            dv["cu"], dv["vd"], dv["cd"], True)
    a = torch.ops.titan.block_ell_swiglu_bwd(dy, dv["x"], gp, up, h, dv["vg"], dv["cg"], dv["vu"], dv["cu"],
                                             dv["vd"], dv["cd"])
    b = K.block_ell_swiglu_bwd(dy, dv["x"], gp, up, h, dv["vg"], dv["cg"], dv["vu"], dv["cu"], dv["vd"], dv["cd"],
                               layout=K.TILE_OUT_IN)
    # dx has no atomics (bit-identical); the tile gradients add partial
    # tiles with fp32 atomics in arrival order, so runs agree to rounding
    _same_grads(a, b)
    x = dv["x"].clone().requires_grad_(True)
    vg, vu, vd = (dv[k].clone().requires_grad_(True) for k in ("vg", "vu", "vd"))
    y = K.block_ell_swiglu(x, vg, dv["cg"], vu, dv["cu"], vd, dv["cd"], add_residual=True, layout=K.TILE_OUT_IN)
    assert torch.equal(y.detach(), out)
    y.backward(dy)
    _same_grads((x.grad, vg.grad, vu.grad, vd.grad), b)


def _same_grads(a, b):
    assert torch.equal(a[0], b[0])
    for x, y in zip(a[1:], b[1:]):
        xf, yf = x.float(), y.float()
        assert torch.all((xf - yf).abs() <= yf.abs() * 2.0 ** -7 + 1e-6)


@pytest.mark.parametrize("B", [64, 128])
def test_swiglu_backward_dead_rows_and_unused_columns(B):
    """Block-rows whose gate (or down) slots are all dead, and d_ff columns no
    down slot uses: their gradients are exactly zero, the rest match."""
    K = _K()
    T, d, F = 200, 2 * B * 2, 4 * B * 2
    c = make_case(T, d, F, B, 2, 2, 3, seed=B + 7)
    c["cg"][1, :] = -1          # gate block-row 1 entirely dead
    c["cd"][0, :] = -1          # down block-row 0 entirely dead
    dv = to_dev(c, torch.bfloat16)
    g = torch.Generator().manual_seed(3)
    dy = torch.randn(T, d, generator=g).to(torch.bfloat16).cuda()
    out, h, gp, up = K.block_ell_swiglu_fwd_with_intermediate(dv["x"], dv["vg"], dv["cg"], dv["vu"], dv["cu"],
                                                              dv["vd"], dv["cd"], add_residual=True)
    res = K.block_ell_swiglu_bwd(dy, dv["x"], gp, up, h, dv["vg"], dv["cg"], dv["vu"], dv["cu"], dv["vd"], dv["cd"])
    torch.cuda.synchronize()
    assert K.read_status() == 0
    mats = [(_f64(dv[v]), dv[ci].cpu().numpy(), 0) for v, ci in (("vg", "cg"), ("vu", "cu"), ("vd", "cd"))]
    ref = O.swiglu_ffn_backward(_f64(dv["x"]), *mats, _f64(dy), add_residual=True)
    for name, a, b in zip(("dx", "d_vg", "d_vu", "d_vd"), res, ref):
        assert O.rel_l2(_f64(a), b) < TOL, name
    assert float(res[1][1].float().abs().max()) == 0.0
    assert float(res[3][0].float().abs().max()) == 0.0
