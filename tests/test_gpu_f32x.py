"""The fp32 forward on the bf16 tensor cores (bf16x6 split) against the fp64
oracle at the fp32 target, rel-L2 <= 1e-5, and against the CUDA-core fp32
path.  Covers BASELINE config 1 at full size (both tile layouts, residual on
and off, the intermediates; the fused tile-64 gate/up kernel that writes h's
bf16 parts itself and the two fp32-output linears), ragged and tiny token
counts, tile sizes 32 and 128, dead and duplicate slots, K_gate != K_up, a
residual other than x, a weight updated in place between calls (the expanded
weights are cached per tensor version), a 65536-token row sample, the C ABI's
argument checks, the single fp32 linear (block_ell_matmul) the same way,
alone and inside a trained BlockELLLinear, and the fp32 tile gradients as six
bf16 tile-gradient products."""

import ctypes as C
import os

import numpy as np
import pytest
import torch

import oracle as O
from gpu_util import make_case, oracle_ffn, to_dev

pytestmark = pytest.mark.gpu

TOL_F32 = 1e-5


def _K():
    from looped_blockell import kernels as K
    return K


def _f64(c):
    return {k: v.astype(np.float64) if not k.startswith("c") else v for k, v in c.items()}


@pytest.mark.parametrize("layout", [O.LAYOUT_IN_OUT, O.LAYOUT_OUT_IN])
def test_config1_bf16x6_matches_oracle(layout):
    """T=1024, d=512, F=2048, B=64, 25 %."""
    K = _K()
    c = make_case(1024, 512, 2048, 64, 2, 2, 8, seed=1)
    dc = to_dev(c, torch.float32, layout)
    for add_res in (False, True):
        out, h, g, u = K.block_ell_swiglu_fwd_with_intermediate(dc["x"], dc["vg"], dc["cg"], dc["vu"], dc["cu"],
                                                                 dc["vd"], dc["cd"], add_residual=add_res,
                                                                 layout=layout, fp32_method="bf16x6")
        ro, rh, rg, ru = oracle_ffn(_f64(c), add_residual=add_res)
        for got, ref in ((out, ro), (h, rh), (g, rg), (u, ru)):
            assert O.rel_l2(got.cpu().numpy(), ref) < TOL_F32
        # without intermediates, tile 64 runs one gate/up kernel that writes the
        # bf16 parts of h itself (the call above ran two fp32-output linears)
        for fused in ("0", "1"):
            os.environ["BELL_F32X_FUSED"] = fused
            try:
                out2 = K.block_ell_swiglu_fwd(dc["x"], dc["vg"], dc["cg"], dc["vu"], dc["cu"], dc["vd"], dc["cd"],
                                              add_residual=add_res, layout=layout, fp32_method="bf16x6")
            finally:
                del os.environ["BELL_F32X_FUSED"]
            assert O.rel_l2(out2.cpu().numpy(), ro) < TOL_F32
            assert O.rel_l2(out2.cpu().numpy(), out.cpu().numpy().astype(np.float64)) < 1e-6
        assert K.read_status() == 0


@pytest.mark.parametrize("shape", [
    # T,   d,   F,    B,  Kg, Ku, Kd, extra
    (77, 256, 1024, 128, 2, 1, 3, {}),
    (77, 256, 1024, 128, 2, 1, 3, {"dead": 3}),
    (300, 256, 512, 64, 2, 2, 3, {"dup": True}),
    (1, 128, 512, 32, 1, 2, 4, {}),
    (1000, 384, 1536, 32, 3, 3, 12, {"dead": 2}),
])
def test_bf16x6_edge_cases(shape):
    K = _K()
    T, d, F, B, Kg, Ku, Kd, extra = shape
    c = make_case(T, d, F, B, Kg, Ku, Kd, seed=T + B, **extra)
    dc = to_dev(c, torch.float32)
    ref = oracle_ffn(_f64(c), add_residual=True)[0]
    out = K.block_ell_swiglu_fwd(dc["x"], dc["vg"], dc["cg"], dc["vu"], dc["cu"], dc["vd"], dc["cd"],
                                 add_residual=True, fp32_method="bf16x6")
    simt = K.block_ell_swiglu_fwd(dc["x"], dc["vg"], dc["cg"], dc["vu"], dc["cu"], dc["vd"], dc["cd"],
                                  add_residual=True, fp32_method="simt")
    assert O.rel_l2(out.cpu().numpy(), ref) < TOL_F32
    assert O.rel_l2(simt.cpu().numpy(), ref) < TOL_F32
    assert K.read_status() == 0


def test_bf16x6_zero_tokens():
    K = _K()
    c = make_case(4, 128, 512, 64, 2, 2, 4, seed=5)
    dc = to_dev(c, torch.float32)
    x0 = dc["x"][:0]
    out = K.block_ell_swiglu_fwd(x0, dc["vg"], dc["cg"], dc["vu"], dc["cu"], dc["vd"], dc["cd"], add_residual=True,
                                 fp32_method="bf16x6")
    assert out.shape == (0, 128)


def test_bf16x6_residual_other_than_x():
    from looped_blockell.kernels import ops
    c = make_case(257, 256, 1024, 64, 2, 2, 4, seed=9)
    dc = to_dev(c, torch.float32)
    res = torch.randn_like(dc["x"])
    out = ops._swiglu(dc["x"], dc["vg"], dc["cg"], dc["vu"], dc["cu"], dc["vd"], dc["cd"], True, O.LAYOUT_IN_OUT,
                      False, residual=res, fp32_method="bf16x6")[0]
    ref = oracle_ffn(_f64(c), add_residual=False)[0] + res.double().cpu().numpy()
    assert O.rel_l2(out.cpu().numpy(), ref) < TOL_F32


def test_bf16x6_weight_update_refreshes_the_expansion():
    """The expanded weights are cached per tensor version: an in-place update
    must be seen by the next call."""
    K = _K()
    c = make_case(512, 256, 1024, 64, 2, 2, 4, seed=11)
    dc = to_dev(c, torch.float32)
    args = (dc["x"], dc["vg"], dc["cg"], dc["vu"], dc["cu"], dc["vd"], dc["cd"])
    first = K.block_ell_swiglu_fwd(*args, add_residual=True, fp32_method="bf16x6")
    again = K.block_ell_swiglu_fwd(*args, add_residual=True, fp32_method="bf16x6")
    assert torch.equal(first, again)
    dc["vd"].mul_(-0.5)
    c["vd"] = c["vd"] * np.float32(-0.5)
    second = K.block_ell_swiglu_fwd(*args, add_residual=True, fp32_method="bf16x6")
    assert O.rel_l2(second.cpu().numpy(), oracle_ffn(_f64(c), add_residual=True)[0]) < TOL_F32


def test_bf16x6_large_token_row_sample():
    """65536 tokens at config 1's shapes (the size where auto picks bf16x6):
    512 rows spread over the whole range, first and last included."""
    K = _K()
    from looped_blockell.kernels import f32x
    T = 65536
    assert f32x.resolve("auto", T, 2, 2, 8) == "bf16x6"
    c = make_case(T, 512, 2048, 64, 2, 2, 8, seed=13)
    dc = to_dev(c, torch.float32)
    out = K.block_ell_swiglu_fwd(dc["x"], dc["vg"], dc["cg"], dc["vu"], dc["cu"], dc["vd"], dc["cd"],
                                 add_residual=True)
    rows = np.unique(np.concatenate([[0, T - 1], np.random.default_rng(0).integers(0, T, 510)]))
    ref = oracle_ffn(_f64(c), add_residual=True, rows=rows)[0]
    assert O.rel_l2(out[torch.from_numpy(rows).cuda()].cpu().numpy(), ref) < TOL_F32
    assert K.read_status() == 0


def test_bf16x6_abi_rejects_bad_descriptors():
    from looped_blockell.kernels import _lib as L
    lib = L.load()
    c = make_case(64, 128, 512, 64, 2, 2, 4, seed=3)
    dc = to_dev(c, torch.float32)
    out = torch.empty_like(dc["x"])
    desc = L.BellFFNDesc()
    desc.T, desc.d_model, desc.d_ff, desc.dtype = 64, 128, 512, L.BELL_DTYPE_F32
    desc.x, desc.out = dc["x"].data_ptr(), out.data_ptr()
    # fp32 tiles where expanded bf16 ones belong: wrong column count
    desc.gate = L.BellEll(dc["vg"].data_ptr(), dc["cg"].data_ptr(), 8, 2, 2, 64, 0, 0)
    desc.up = L.BellEll(dc["vu"].data_ptr(), dc["cu"].data_ptr(), 8, 2, 2, 64, 0, 0)
    desc.down = L.BellEll(dc["vd"].data_ptr(), dc["cd"].data_ptr(), 2, 8, 4, 64, 0, 0)
    ws = torch.empty(1 << 20, dtype=torch.uint8, device="cuda")
    assert lib.bell_swiglu_fwd_f32x(C.byref(desc), C.c_void_p(ws.data_ptr()), None) == -2
    assert "expand" in L.last_error()
    # an expansion that would exceed 254 slots per row is refused
    ell = L.BellEll(dc["vg"].data_ptr(), dc["cg"].data_ptr(), 8, 2, 43, 64, 0, 0)
    v6 = torch.empty(1, dtype=torch.bfloat16, device="cuda")
    c6 = torch.empty(1, dtype=torch.int32, device="cuda")
    assert lib.bell_f32x_expand_ell(C.byref(ell), 0, 2, -1, 0, C.c_void_p(v6.data_ptr()),
                                    C.c_void_p(c6.data_ptr()), None) == -2
    assert lib.bell_f32x_workspace_bytes(-1, 128, 512, 64, 12, 12, 27) == 0


@pytest.mark.parametrize("B", [32, 64, 128])
@pytest.mark.parametrize("layout", [O.LAYOUT_IN_OUT, O.LAYOUT_OUT_IN])
def test_bf16x6_linear_matches_oracle(B, layout):
    """One fp32 Block-ELL linear (block_ell_matmul) on the tensor cores, with
    and without a residual, against the fp64 oracle and the CUDA-core path."""
    from looped_blockell.kernels import block_ell_linear
    rng = np.random.default_rng(B + layout)
    T, C, R, K = 1000, 8, 6, 3
    cols = np.stack([np.sort(rng.choice(C, K, replace=False)) for _ in range(R)]).astype(np.int32)
    cols[2, 1] = -1  # a dead slot
    vals = (rng.standard_normal((R, K, B, B)) * 0.02).astype(np.float32)
    x = rng.standard_normal((T, C * B)).astype(np.float32)
    res = rng.standard_normal((T, R * B)).astype(np.float32)
    dv = torch.from_numpy(vals if layout == O.LAYOUT_IN_OUT else np.swapaxes(vals, -1, -2).copy()).cuda()
    dc, dx, dr = torch.from_numpy(cols).cuda(), torch.from_numpy(x).cuda(), torch.from_numpy(res).cuda()
    ref = O.block_ell_matmul(x.astype(np.float64), vals.astype(np.float64), cols)
    for residual in (None, dr):
        want = ref if residual is None else ref + res.astype(np.float64)
        got = block_ell_linear(dx, dv, dc, residual=residual, layout=layout, fp32_method="bf16x6")
        simt = block_ell_linear(dx, dv, dc, residual=residual, layout=layout, fp32_method="simt")
        assert O.rel_l2(got.cpu().numpy(), want) < TOL_F32
        assert O.rel_l2(simt.cpu().numpy(), want) < TOL_F32


def test_bf16x6_linear_layer_trains(monkeypatch):
    """BlockELLLinear in fp32 with every linear (forward and the backward's
    transposed products) on the bf16x6 path: output and gradients against the
    dense float64 reference at the fp32 tolerance."""
    from looped_blockell.layers import BlockELLLinear
    from test_gpu_small_tiles import _dense_ref_linear
    monkeypatch.setenv("BELL_F32_METHOD", "bf16x6")
    B = 64
    torch.manual_seed(3)
    m = BlockELLLinear(8 * B, 4 * B, tile_size=B, density=0.5, dtype=torch.float32, device="cuda")
    x = torch.randn(4, 300, 4 * B, device="cuda").requires_grad_(True)
    y = m(x)
    dy = torch.randn_like(y)
    y.backward(dy)
    cols = m.effective_col_indices().cpu().numpy()
    vals = m.values.detach().double().cpu().numpy()
    xf = x.detach().double().cpu().numpy().reshape(-1, 4 * B)
    dyf = dy.double().cpu().numpy().reshape(-1, 8 * B)
    ry, rdx, rdv = _dense_ref_linear(xf, vals, cols, B, 8 * B, 4 * B, dyf)
    assert O.rel_l2(y.detach().double().cpu().numpy().reshape(-1, 8 * B), ry) < TOL_F32
    assert O.rel_l2(x.grad.double().cpu().numpy().reshape(-1, 4 * B), rdx) < TOL_F32
    assert O.rel_l2(m.values.grad.double().cpu().numpy(), rdv) < TOL_F32


@pytest.mark.parametrize("B,layout,T", [(64, O.LAYOUT_IN_OUT, 3001), (128, O.LAYOUT_OUT_IN, 2048)])
def test_bf16x6_tile_gradients_match_fp64(B, layout, T, monkeypatch):
    """fp32 tile gradients as six tcgen05 products of the operands' bf16
    parts (what ``auto`` picks from 1024 tokens up at tile 64/128): against
    float64 sums, with a strided operand, a dead slot and accumulation onto
    an existing gradient; and against the CUDA-core kernel."""
    from looped_blockell.kernels import block_ell_sddmm, f32x
    assert f32x.resolve_sddmm(None, T, B) == "bf16x6"
    rng = np.random.default_rng(B + T)
    R, Cc, Kk = 5, 4, 3
    cols = np.stack([rng.choice(Cc, size=Kk, replace=False) for _ in range(R)]).astype(np.int32)
    cols[2, 1] = -1
    a = rng.standard_normal((T, Cc * B)).astype(np.float32)
    bw = rng.standard_normal((T, 2 * R * B)).astype(np.float32)  # b is the right half of a wider row
    base = rng.standard_normal((R, Kk, B, B)).astype(np.float32)
    da, dbw, dcols = torch.from_numpy(a).cuda(), torch.from_numpy(bw).cuda(), torch.from_numpy(cols).cuda()
    db = dbw[:, R * B:]
    grad = torch.from_numpy(base).cuda()
    block_ell_sddmm(da, db, dcols, B, layout, grad=grad, accumulate=True)
    monkeypatch.setenv("BELL_F32_METHOD", "simt")
    simt = block_ell_sddmm(da, db, dcols, B, layout)
    b = bw[:, R * B:].astype(np.float64)
    want = base.astype(np.float64).copy()
    exact = np.zeros((R, Kk, B, B))
    for r in range(R):
        for k in range(Kk):
            c = cols[r, k]
            if c >= 0:
                t = a[:, c * B:(c + 1) * B].astype(np.float64).T @ b[:, r * B:(r + 1) * B]
                exact[r, k] = t if layout == O.LAYOUT_IN_OUT else t.T
    want += exact
    assert O.rel_l2(grad.cpu().numpy().astype(np.float64), want) < TOL_F32
    assert O.rel_l2(simt.cpu().numpy().astype(np.float64), exact) < TOL_F32
    assert np.all(simt.cpu().numpy()[cols < 0] == 0)
