"""The reference's own tile sizes (16 x 16 and 32 x 32) on the B200 against
the CPU oracle.

The reference native op exists only for 16 x 16 tiles in the [B_out, B_in]
layout (csrc/block_ell/swiglu_fwd.cu:84, block_ell_ops.cpp:51-62) and the
reference model's default tile_size is 16 (looped_blockell/config.py:63,
layers/mlp.py:28-44).  These tests run the same argument lists and module
defaults through this package: the fused SwiGLU (bf16 rel-L2 <= 1e-2, fp32
<= 1e-5), the linear, the titan op, and training through BlockELLLinear /
MLPBlock / block_ell_matmul (gradients vs the oracle backward, rel-L2 <= 2e-2
in bf16).  Edge cases: ragged token counts, a single token, dead slots,
duplicate columns, K_g != K_u, shared gate/up columns, output block-rows that
do not fill the kernel's row groups, and units with more than 32 plan steps.
"""

import numpy as np
import pytest
import torch

import oracle as O
from gpu_util import dev_inputs_as_f64, make_case, oracle_ffn, to_dev

pytestmark = pytest.mark.gpu

TOL_BF16 = 1e-2
TOL_F32 = 1e-5
TOL_GRAD = 2e-2


def _K():
    from looped_blockell import kernels as K
    return K


CASES = [
    # T,   d,    F,   B,  Kg, Ku, Kd, extra
    (200, 256, 512, 16, 3, 2, 5, {}),
    (1, 128, 256, 16, 2, 2, 3, {}),                      # a single token
    (333, 128, 80, 16, 2, 3, 2, {"dead": 3}),            # R_ff = 5, R_down = 8: partial groups; dead slots
    (129, 1024, 256, 16, 40, 36, 12, {}),                # > 32 plan steps per unit
    (150, 256, 512, 16, 4, 4, 6, {"shared": True}),      # gate/up share every column
    (96, 256, 512, 16, 3, 3, 4, {"dup": True}),          # a duplicated column
    (257, 256, 512, 32, 2, 3, 4, {}),
    (130, 96, 160, 32, 2, 1, 3, {"dead": 2}),            # R_ff = 5, R_down = 3
]


@pytest.mark.parametrize("layout", [O.LAYOUT_IN_OUT, O.LAYOUT_OUT_IN])
@pytest.mark.parametrize("case", CASES)
def test_small_tile_swiglu_bf16_matches_oracle(case, layout):
    T, d, F, B, Kg, Ku, Kd, extra = case
    K = _K()
    c = make_case(T, d, F, B, Kg, Ku, Kd, seed=T + B + d, **extra)
    dc = to_dev(c, torch.bfloat16, layout)
    ref_in = dev_inputs_as_f64(to_dev(c, torch.bfloat16))
    for add_res in (False, True):
        out, h, g, u = K.block_ell_swiglu_fwd_with_intermediate(dc["x"], dc["vg"], dc["cg"], dc["vu"], dc["cu"],
                                                                 dc["vd"], dc["cd"], add_residual=add_res,
                                                                 layout=layout, shared_topology=extra.get("shared",
                                                                                                          False))
        ro, rh, rg, ru = oracle_ffn(ref_in, add_residual=add_res)
        assert O.rel_l2(out.float().cpu().numpy(), ro) < TOL_BF16
        assert O.rel_l2(h.float().cpu().numpy(), rh) < TOL_BF16
        assert O.rel_l2(g.float().cpu().numpy(), rg) < TOL_BF16
        assert O.rel_l2(u.float().cpu().numpy(), ru) < TOL_BF16
    assert K.read_status() == 0


@pytest.mark.parametrize("B", [16, 32])
@pytest.mark.parametrize("layout", [O.LAYOUT_IN_OUT, O.LAYOUT_OUT_IN])
def test_small_tile_swiglu_fp32_matches_oracle(B, layout):
    K = _K()
    c = make_case(300, 256, 512, B, 3, 2, 5, seed=B, dead=2)
    dc = to_dev(c, torch.float32, layout)
    ref = {k: v.astype(np.float64) if not k.startswith("c") else v for k, v in c.items()}
    out = K.block_ell_swiglu_fwd(dc["x"], dc["vg"], dc["cg"], dc["vu"], dc["cu"], dc["vd"], dc["cd"],
                                 add_residual=True, layout=layout)
    assert O.rel_l2(out.cpu().numpy(), oracle_ffn(ref, add_residual=True)[0]) < TOL_F32


@pytest.mark.parametrize("B,out_dtype", [(16, torch.bfloat16), (16, torch.float32), (32, torch.bfloat16)])
def test_small_tile_linear_matches_oracle(B, out_dtype):
    K = _K()
    rng = np.random.default_rng(B)
    T, C, R, Ks = 333, 12, 11, 5
    cols = np.stack([np.sort(rng.choice(C, Ks, replace=False)) for _ in range(R)]).astype(np.int32)
    cols[3, 1] = -1
    v = (rng.standard_normal((R, Ks, B, B)) * 0.05).astype(np.float32)
    x = rng.standard_normal((T, C * B)).astype(np.float32)
    res = rng.standard_normal((T, R * B)).astype(np.float32)
    vb, xb, rb = (torch.from_numpy(a).to(torch.bfloat16).cuda() for a in (v, x, res))
    y = K.block_ell_linear(xb, vb, torch.from_numpy(cols).cuda(), residual=rb, out_dtype=out_dtype)
    ref = O.block_ell_matmul(xb.float().cpu().numpy(), vb.float().cpu().numpy(), cols) + rb.float().cpu().numpy()
    assert y.dtype == out_dtype
    assert O.rel_l2(y.float().cpu().numpy(), ref) < TOL_BF16
    assert K.read_status() == 0


@pytest.mark.parametrize("add_residual", [False, True])
def test_titan_op_with_reference_16x16_tiles(add_residual):
    """torch.ops.titan.block_ell_swiglu_fwd with the reference op's own
    argument list and tiles: [R, K, 16, 16] in the [B_out, B_in] layout."""
    K = _K()
    c = make_case(256, 512, 2048, 16, 8, 8, 32, seed=16)
    d = to_dev(c, torch.bfloat16, O.LAYOUT_OUT_IN)
    assert d["vg"].shape == (128, 8, 16, 16)
    out = torch.ops.titan.block_ell_swiglu_fwd(d["x"], d["vg"], d["cg"], d["vu"], d["cu"], d["vd"], d["cd"],
                                               add_residual)
    ref_in = dev_inputs_as_f64(to_dev(c, torch.bfloat16))
    assert O.rel_l2(out.float().cpu().numpy(), oracle_ffn(ref_in, add_residual=add_residual)[0]) < TOL_BF16
    res, h, g, u = torch.ops.titan.block_ell_swiglu_fwd_with_intermediate(d["x"], d["vg"], d["cg"], d["vu"], d["cu"],
                                                                          d["vd"], d["cd"], add_residual)
    assert torch.equal(res, out) and h.shape == (256, 2048)
    grads = torch.ops.titan.block_ell_swiglu_bwd(torch.ones_like(out), d["x"], g, u, h, d["vg"], d["cg"], d["vu"],
                                                 d["cu"], d["vd"], d["cd"])
    assert [t.shape for t in grads] == [d["x"].shape, d["vg"].shape, d["vu"].shape, d["vd"].shape]
    assert K.read_status() == 0


@pytest.mark.parametrize("B", [16, 32])
def test_small_tile_sddmm_matches_oracle(B):
    K = _K()
    from looped_blockell.kernels import backward as kb
    rng = np.random.default_rng(B + 1)
    T, C, R, Ks = 4500, 6, 5, 3
    cols = np.stack([np.sort(rng.choice(C, Ks, replace=False)) for _ in range(R)]).astype(np.int32)
    cols[1, 2] = -1
    a = rng.standard_normal((T, C * B)).astype(np.float32)
    b = rng.standard_normal((T, R * B)).astype(np.float32)
    for dt in (torch.bfloat16, torch.float32):
        at, bt = torch.from_numpy(a).to(dt).cuda(), torch.from_numpy(b).to(dt).cuda()
        af, bf = at.double().cpu().numpy(), bt.double().cpu().numpy()
        for layout in (O.LAYOUT_IN_OUT, O.LAYOUT_OUT_IN):
            g = kb.block_ell_sddmm(at, bt, torch.from_numpy(cols).cuda(), B, layout)
            ref = np.zeros((R, Ks, B, B))
            for r in range(R):
                for k in range(Ks):
                    if cols[r, k] >= 0:
                        t = af[:, cols[r, k] * B:(cols[r, k] + 1) * B].T @ bf[:, r * B:(r + 1) * B]
                        ref[r, k] = t if layout == O.LAYOUT_IN_OUT else t.T
            assert O.rel_l2(g.cpu().numpy(), ref) < 1e-5
    assert K.read_status() == 0


def _dense_ref_linear(x, vals, cols, B, out_f, in_f, dy):
    """y, dx, dW (tiles [B_in, B_out]) in float64 from the dense weight."""
    W = O.block_ell_to_dense(vals, cols, out_f, in_f)
    y = x @ W.T
    dx = dy @ W
    dWd = dy.T @ x
    dv = np.zeros_like(vals)
    for r in range(cols.shape[0]):
        for k in range(cols.shape[1]):
            c = cols[r, k]
            if c >= 0:
                dv[r, k] = dWd[r * B:(r + 1) * B, c * B:(c + 1) * B].T
    return y, dx, dv


@pytest.mark.parametrize("B,dtype", [(16, torch.bfloat16), (64, torch.bfloat16), (16, torch.float32)])
def test_block_ell_linear_module_trains(B, dtype):
    """BlockELLLinear forward and backward (x, values, bias) vs the dense
    float64 reference on the same rounded inputs."""
    from looped_blockell.layers import BlockELLLinear
    torch.manual_seed(B)
    m = BlockELLLinear(8 * B, 4 * B, tile_size=B, density=0.5, dtype=dtype, device="cuda")
    m.alive_mask[1, 0] = False  # a dead tile: zero output contribution, zero gradient
    x = torch.randn(3, 37, 4 * B, device="cuda").to(dtype).requires_grad_(True)
    y = m(x)
    dy = torch.randn_like(y)
    y.backward(dy)
    cols = m.effective_col_indices().cpu().numpy()
    vals = m.values.detach().to(dtype).double().cpu().numpy()
    xf = x.detach().double().cpu().numpy().reshape(-1, 4 * B)
    dyf = dy.double().cpu().numpy().reshape(-1, 8 * B)
    ry, rdx, rdv = _dense_ref_linear(xf, vals, cols, B, 8 * B, 4 * B, dyf)
    tol = TOL_BF16 if dtype == torch.bfloat16 else 1e-5
    gtol = TOL_GRAD if dtype == torch.bfloat16 else 1e-5
    assert O.rel_l2(y.detach().double().cpu().numpy().reshape(-1, 8 * B), ry) < tol
    assert O.rel_l2(x.grad.double().cpu().numpy().reshape(-1, 4 * B), rdx) < gtol
    assert O.rel_l2(m.values.grad.double().cpu().numpy(), rdv) < gtol
    assert float(m.values.grad[1, 0].abs().max()) == 0.0
    assert O.rel_l2(m.bias.grad.double().cpu().numpy(), dyf.sum(0)) < tol  # bf16 dy summed by torch
    assert m.values.grad.dtype == m.values.dtype


def test_block_ell_matmul_gradient_flow_like_reference():
    """The reference's tests/test_block_ell.py:57-72 on this package: an fp32
    [32, 64] weight at tile 16, density 0.5; the values' gradient of
    y.sum() is non-zero and equals the dense reference."""
    from looped_blockell.layers import BlockELLTensor, block_ell_matmul, create_block_ell_from_dense
    g = torch.Generator().manual_seed(0)
    W = torch.randn(32, 64, generator=g)
    x = torch.randn(2, 4, 64, generator=g)
    bell = create_block_ell_from_dense(W, tile_size=16, density=0.5)
    values = bell.values.cuda().requires_grad_(True)
    ell = BlockELLTensor(values=values, col_indices=bell.col_indices.cuda(), config=bell.config)
    y = block_ell_matmul(x.cuda(), ell)
    y.sum().backward()
    assert values.grad.shape == values.shape and bool((values.grad != 0).any())
    cols = bell.col_indices.numpy()
    _, _, rdv = _dense_ref_linear(x.double().numpy().reshape(-1, 64), bell.values.double().numpy(), cols, 16, 32, 64,
                                  np.ones((8, 32)))
    assert O.rel_l2(values.grad.double().cpu().numpy(), rdv) < 1e-5


@pytest.mark.parametrize("density", [1.0, 0.5])
def test_mlpblock_default_tile_trains(density):
    """MLPBlock(d_model, d_ff, use_swiglu=True) with the reference defaults
    (tile_size 16, bf16): forward vs the oracle, and loss.backward() gives the
    oracle backward's gradients for x and every values tensor."""
    from looped_blockell.layers import MLPBlock
    torch.manual_seed(int(density * 10))
    m = MLPBlock(256, 512, use_swiglu=True, density=density, device="cuda")
    assert m.w_gate.tile_size == 16
    x = torch.randn(300, 256, device="cuda").to(torch.bfloat16).requires_grad_(True)
    out = m(x, residual=True)
    dy = torch.randn_like(out)
    out.backward(dy)
    f = lambda t: t.detach().double().cpu().numpy()  # noqa: E731
    mats = [(f(w.kernel_values()), w.effective_col_indices().cpu().numpy(), 0) for w in (m.w_gate, m.w_up, m.w_down)]
    ro = O.swiglu_ffn(f(x), *mats, add_residual=True)
    assert O.rel_l2(f(out), ro) < TOL_BF16
    rdx, rdg, rdu, rdd = O.swiglu_ffn_backward(f(x), *mats, f(dy), add_residual=True)
    assert O.rel_l2(f(x.grad), rdx) < TOL_GRAD
    for w, ref in zip((m.w_gate, m.w_up, m.w_down), (rdg, rdu, rdd)):
        assert w.values.grad is not None and w.values.grad.dtype == torch.float32
        assert O.rel_l2(f(w.values.grad), ref) < TOL_GRAD
    assert _K().read_status() == 0


def test_mlpblock_weight_cache_follows_optimizer_steps():
    """The bf16 copy the kernels read is rebuilt after an in-place optimizer
    update (the parameter's version counter), and reused otherwise."""
    from looped_blockell.layers import MLPBlock
    torch.manual_seed(3)
    m = MLPBlock(128, 256, use_swiglu=True, density=0.5, device="cuda")
    x = torch.randn(64, 128, device="cuda").to(torch.bfloat16)
    v0 = m.w_gate.kernel_values()
    assert m.w_gate.kernel_values() is v0  # cached
    opt = torch.optim.SGD(m.parameters(), lr=0.5)
    m(x).float().pow(2).sum().backward()
    opt.step()
    v1 = m.w_gate.kernel_values()
    assert v1 is not v0 and not torch.equal(v1, v0)
    assert torch.equal(v1, m.w_gate.values.detach().to(torch.bfloat16))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_rmsnorm_layer_keeps_precision_and_trains(dtype):
    from looped_blockell.layers import RMSNorm
    torch.manual_seed(4)
    n = RMSNorm(256, device="cuda")
    with torch.no_grad():
        n.scale.mul_(1.0 + 0.1 * torch.randn(256, device="cuda"))
    x = (torch.randn(77, 256, device="cuda") * 3).to(dtype).requires_grad_(True)
    y = n(x)
    assert y.dtype == dtype
    dy = torch.randn_like(y)
    y.backward(dy)
    xr = x.detach().double().requires_grad_(True)
    sr = n.scale.detach().double().requires_grad_(True)
    yr = xr / torch.sqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-5) * sr
    yr.backward(dy.double())
    tol = 1e-6 if dtype == torch.float32 else TOL_BF16
    assert O.rel_l2(y.detach().double().cpu().numpy(), yr.detach().cpu().numpy()) < tol
    assert O.rel_l2(x.grad.double().cpu().numpy(), xr.grad.cpu().numpy()) < max(tol, 1e-5)
    assert O.rel_l2(n.scale.grad.double().cpu().numpy(), sr.grad.cpu().numpy()) < max(tol, 1e-5)
