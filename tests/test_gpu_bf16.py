"""bf16 Block-ELL SwiGLU on the B200 vs the CPU oracle (rel-L2 <= 1e-2).

Inputs are rounded to bf16 first; the oracle runs in float64 on exactly the
values the GPU saw.  Edge cases follow the reference's own tests and hazards:
ragged token counts, dead (-1) slots (tests/test_column_reorder.py:99-113),
duplicate columns, different K for gate and up (swiglu_fwd.cu:599-600), both
tile layouts, B = 64 and 128, residual on/off, intermediates.
"""

import numpy as np
import pytest
import torch

import oracle as O
from gpu_util import dev_inputs_as_f64, make_case, oracle_ffn, to_dev

pytestmark = pytest.mark.gpu

TOL_BF16 = 1e-2  # rel-L2 vs the fp32/fp64 reference (north_star tolerance)


def _kernels():
    from looped_blockell import kernels as K
    return K


CASES = [
    # T,   d,   F,    B,  Kg, Ku, Kd, extra
    (128, 256, 512, 64, 2, 2, 4, {}),
    (300, 256, 512, 64, 1, 3, 2, {}),                 # ragged T, K_g != K_u
    (1, 256, 512, 64, 2, 2, 4, {}),                   # a single token
    (257, 512, 1024, 128, 2, 2, 3, {}),               # B = 128
    (200, 512, 1024, 128, 3, 3, 4, {"shared": True}),  # gate/up share every column
    (130, 256, 512, 64, 3, 3, 5, {"dead": 4}),        # dead slots
    (96, 256, 512, 64, 3, 2, 4, {"dup": True}),       # duplicate column in a row
]


@pytest.mark.parametrize("layout", [O.LAYOUT_IN_OUT, O.LAYOUT_OUT_IN])
@pytest.mark.parametrize("case", CASES)
def test_swiglu_bf16_matches_oracle(case, layout):
    T, d, F, B, Kg, Ku, Kd, extra = case
    K = _kernels()
    c = make_case(T, d, F, B, Kg, Ku, Kd, seed=T + B, **extra)
    dc = to_dev(c, torch.bfloat16, layout)
    ref_in = dev_inputs_as_f64(to_dev(c, torch.bfloat16))
    for add_res in (False, True):
        out, h, g, u = K.block_ell_swiglu_fwd_with_intermediate(dc["x"], dc["vg"], dc["cg"], dc["vu"], dc["cu"],
                                                                 dc["vd"], dc["cd"], add_residual=add_res, layout=layout)
        torch.cuda.synchronize()
        ro, rh, rg, ru = oracle_ffn(ref_in, add_residual=add_res)
        assert O.rel_l2(out.float().cpu().numpy(), ro) < TOL_BF16
        assert O.rel_l2(h.float().cpu().numpy(), rh) < TOL_BF16
        assert O.rel_l2(g.float().cpu().numpy(), rg) < TOL_BF16
        assert O.rel_l2(u.float().cpu().numpy(), ru) < TOL_BF16
    assert K.read_status() == 0


def test_swiglu_bf16_golden_fixtures():
    """The reference-generated fixtures, run through the bf16 kernel."""
    import os
    from conftest import GOLDEN
    K = _kernels()
    for name in ("swiglu_small", "swiglu_dead"):
        z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
        c = {k: z[k] for k in ("x", "vg", "cg", "vu", "cu", "vd", "cd")}
        dc = to_dev(c, torch.bfloat16)
        out = K.block_ell_swiglu_fwd(dc["x"], dc["vg"], dc["cg"], dc["vu"], dc["cu"], dc["vd"], dc["cd"])
        assert O.rel_l2(out.float().cpu().numpy(), z["out"]) < TOL_BF16


@pytest.mark.parametrize("B,K_slots,out_dtype", [(64, 3, torch.bfloat16), (128, 2, torch.float32)])
def test_linear_bf16_matches_oracle(B, K_slots, out_dtype):
    K = _kernels()
    rng = np.random.default_rng(B)
    T, C, R = 333, 4, 3
    cols = np.stack([np.sort(rng.choice(C, K_slots, replace=False)) for _ in range(R)]).astype(np.int32)
    v = (rng.standard_normal((R, K_slots, B, B)) * 0.05).astype(np.float32)
    x = rng.standard_normal((T, C * B)).astype(np.float32)
    res = rng.standard_normal((T, R * B)).astype(np.float32)
    vb, xb, rb = (torch.from_numpy(a).to(torch.bfloat16).cuda() for a in (v, x, res))
    y = K.block_ell_linear(xb, vb, torch.from_numpy(cols).cuda(), residual=rb, out_dtype=out_dtype)
    ref = O.block_ell_matmul(xb.float().cpu().numpy(), vb.float().cpu().numpy(), cols) + rb.float().cpu().numpy()
    assert y.dtype == out_dtype
    assert O.rel_l2(y.float().cpu().numpy(), ref) < TOL_BF16


def test_config2_full_size_row_sample():
    """BASELINE config 2 (T=32768, d=2048, F=8192, B=64, 12.5%) on the GPU at
    full size; the oracle checks a 1024-token sample (tokens are independent)."""
    from looped_blockell.synth import CONFIGS, make_ffn
    K = _kernels()
    cfg = CONFIGS[2]
    c = make_ffn(cfg, device="cuda")
    out = K.block_ell_swiglu_fwd(c["x"], c["vg"], c["cg"], c["vu"], c["cu"], c["vd"], c["cd"], add_residual=True)
    rows = np.random.default_rng(0).choice(cfg.T, 1024, replace=False)
    ref_in = {k: (v.float().cpu().numpy().astype(np.float64) if not k.startswith("c") else v.cpu().numpy())
              for k, v in c.items()}
    ro = oracle_ffn(ref_in, add_residual=True, rows=rows)[0]
    assert O.rel_l2(out[torch.from_numpy(rows).cuda()].float().cpu().numpy(), ro) < TOL_BF16
    assert K.read_status() == 0


def test_bad_column_index_sets_status_not_fault():
    """An index outside [-1, C) is dropped by the plan kernel and reported in
    the status word; nothing reads out of bounds."""
    K = _kernels()
    c = make_case(64, 256, 512, 64, 2, 2, 2, seed=9)
    c["cg"][0, 0] = 99
    dc = to_dev(c, torch.bfloat16)
    K.block_ell_swiglu_fwd(dc["x"], dc["vg"], dc["cg"], dc["vu"], dc["cu"], dc["vd"], dc["cd"])
    assert K.read_status() & 1
    assert K.read_status() == 0  # cleared


def test_errors_match_reference_checks():
    K = _kernels()
    c = to_dev(make_case(8, 256, 512, 64, 1, 1, 1), torch.bfloat16)
    with pytest.raises(RuntimeError, match="x must be 2D"):
        K.block_ell_swiglu_fwd(c["x"][None], c["vg"], c["cg"], c["vu"], c["cu"], c["vd"], c["cd"])
    with pytest.raises(RuntimeError, match="must be bf16"):
        K.block_ell_swiglu_fwd(c["x"], c["vg"].float(), c["cg"], c["vu"], c["cu"], c["vd"], c["cd"])
    with pytest.raises(RuntimeError, match="int32"):
        K.block_ell_swiglu_fwd(c["x"], c["vg"], c["cg"].long(), c["vu"], c["cu"], c["vd"], c["cd"])
    with pytest.raises(RuntimeError, match="same R_ff"):
        K.block_ell_swiglu_fwd(c["x"], c["vg"], c["cg"], c["vu"][:4], c["cu"][:4], c["vd"], c["cd"])


@pytest.mark.parametrize("shared,layout", [(False, O.LAYOUT_IN_OUT), (True, O.LAYOUT_IN_OUT),
                                           (False, O.LAYOUT_OUT_IN)])
def test_config5_full_size_row_sample(shared, layout):
    """BASELINE config 5 (T=262144, d=4096, F=16384, B=128, 25 %), the
    benchmark's exact call (bench.py: make_ffn, independent gate/up
    topologies unless --shared-gate-up, [B_in, B_out] tiles unless --layout
    out_in), at full size on one GPU.  This runs the feature-major B = 128
    kernels through every path the benchmark takes: 1024 token tiles x 128
    block-rows of persistent-unit wrap-around, K = 8 gate/up and K = 32 down
    plan rows, 64-bit offsets into the 8.6 GB h.  The oracle checks a
    1024-token sample (tokens are independent), spread over the whole token
    range so early, late and wrapped-around units are all covered."""
    from looped_blockell.synth import CONFIGS, make_ffn
    K = _kernels()
    cfg = CONFIGS[5]
    c = make_ffn(cfg, device="cuda", shared_gate_up=shared)
    ref_in = {k: (v.float().cpu().numpy().astype(np.float64) if k.startswith("v") else v.cpu().numpy())
              for k, v in c.items() if k != "x"}
    if layout == O.LAYOUT_OUT_IN:  # the same weights, stored [B_out, B_in]
        for k in ("vg", "vu", "vd"):
            c[k] = c[k].transpose(-1, -2).contiguous()
    out = K.block_ell_swiglu_fwd(c["x"], c["vg"], c["cg"], c["vu"], c["cu"], c["vd"], c["cd"], add_residual=True,
                                 layout=layout, shared_topology=shared)
    rows = np.sort(np.random.default_rng(5).choice(cfg.T, 1024, replace=False))
    rows[0], rows[-1] = 0, cfg.T - 1
    ridx = torch.from_numpy(rows).cuda()
    ref_in["x"] = c["x"].index_select(0, ridx).float().cpu().numpy().astype(np.float64)
    ro = oracle_ffn(ref_in, add_residual=True)[0]
    got = out.index_select(0, ridx).float().cpu().numpy()
    assert O.rel_l2(got, ro) < TOL_BF16
    x0 = ref_in["x"]
    assert O.rel_l2(got - x0, ro - x0) < 2e-2  # the FFN part alone, without the residual
    assert K.read_status() == 0
