"""Ternary Block-ELL SwiGLU on the B200 vs the CPU oracle.

Integer tile products must be bit-exact.  The kernel combines them as
``acc = fl(acc + fl(s_k * I_k))`` in ascending slot order and divides by the
token scale with IEEE round-to-nearest, exactly as the oracle does, so the
gate and up pre-activations (and the down output given the same int8 h) are
compared bit for bit: any integer difference would show.  silu uses expf,
which is not correctly rounded on either side, so h and the final output
are compared with a tolerance, and h's int8 codes are checked against the
oracle's quantiser applied to the GPU's own h.
"""

import numpy as np
import pytest
import torch

import oracle as O
from gpu_util import make_case

pytestmark = pytest.mark.gpu


def _run(case, add_residual):
    from looped_blockell.kernels.ternary import make_ternary, ternary_swiglu_fwd
    d, F = case["x"].shape[1], case["vg"].shape[0] * 64
    dev = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    g = make_ternary(dev(case["vg"]), dev(case["cg"]), d // 64)
    u = make_ternary(dev(case["vu"]), dev(case["cu"]), d // 64)
    w = make_ternary(dev(case["vd"]), dev(case["cd"]), F // 64)
    xb = torch.from_numpy(case["x"]).to(torch.bfloat16).cuda()
    out, ws = ternary_swiglu_fwd(xb, g, u, w, add_residual=add_residual, return_intermediates=True)
    torch.cuda.synchronize()
    host = lambda t: t.cpu().numpy()  # noqa: E731
    mats = {}
    for name, m in (("g", g), ("u", u), ("d", w)):
        mats[name] = (O.unpack_ternary(host(m.packed)), host(m.scales), host(m.col_indices))
    return host(xb.float()), {k: host(v) for k, v in ws.items()}, host(out), mats


@pytest.mark.parametrize("add_residual", [False, True])
@pytest.mark.parametrize("shape", [(300, 256, 512, 2, 3, 4, 0), (128, 512, 1024, 4, 4, 8, 3), (1, 256, 512, 1, 1, 2, 0)])
def test_ternary_bit_exact_stages(shape, add_residual):
    T, d, F, Kg, Ku, Kd, dead = shape
    case = make_case(T, d, F, 64, Kg, Ku, Kd, seed=T + Kd, dead=dead)
    x, ws, out, m = _run(case, add_residual)
    # weights: the package's quantiser equals the oracle's restatement of bitlinear
    t_ref, s_ref = O.ternary_quantize_tiles(case["vg"])
    np.testing.assert_array_equal(m["g"][0], t_ref)
    # tile means summed in a different order (GPU reduction vs numpy pairwise): a few ulp
    np.testing.assert_allclose(m["g"][1], s_ref, rtol=1e-6, atol=0)
    # 1. int8 activations and their scale: bit-exact
    q_x, s_x = O.activation_quantize_int(x)
    np.testing.assert_array_equal(ws["q_x"], q_x)
    np.testing.assert_array_equal(ws["s_x"], s_x)
    # 2. gate / up pre-activations: bit-exact (integer tile sums + fixed-order fp32)
    np.testing.assert_array_equal(ws["gate"], O.ternary_block_ell_matmul(q_x, s_x, *m["g"]))
    np.testing.assert_array_equal(ws["up"], O.ternary_block_ell_matmul(q_x, s_x, *m["u"]))
    # 3. h = silu(gate) * up in fp32 (expf differs by ulps)
    g, u = ws["gate"], ws["up"]
    h_ref = (g / (np.float32(1) + np.exp(-g)) * u).astype(np.float32)
    np.testing.assert_allclose(ws["h"], h_ref, rtol=1e-5, atol=1e-6)
    # 4. h re-quantised per token over all of d_ff: bit-exact given the GPU's h
    q_h, s_h = O.activation_quantize_int(ws["h"])
    np.testing.assert_array_equal(ws["q_h"], q_h)
    np.testing.assert_array_equal(ws["s_h"], s_h)
    # 5. down output given the same int8 h: bit-exact
    ref = O.ternary_block_ell_matmul(q_h, s_h, *m["d"])
    if add_residual:
        ref = (ref + x).astype(np.float32)
    np.testing.assert_array_equal(out, ref)
    # 6. whole forward vs the independent oracle pipeline
    full = O.ternary_swiglu_ffn(x, m["g"], m["u"], m["d"], add_residual=add_residual)
    assert O.rel_l2(out, full["out"]) < 1e-3


def test_ternary_config3_row_sample():
    """BASELINE config 3 (T=32768, d=2048, F=8192, B=64, 25%) at full size;
    bit-exact checks on a 256-token sample."""
    from looped_blockell.kernels.ternary import make_ternary, ternary_swiglu_fwd
    from looped_blockell.synth import CONFIGS, make_ffn
    cfg = CONFIGS[3]
    c = make_ffn(cfg, device="cuda")
    g = make_ternary(c["vg"], c["cg"], cfg.d_model // 64)
    u = make_ternary(c["vu"], c["cu"], cfg.d_model // 64)
    w = make_ternary(c["vd"], c["cd"], cfg.d_ff // 64)
    xb = c["x"].to(torch.bfloat16)
    out, ws = ternary_swiglu_fwd(xb, g, u, w, add_residual=True, return_intermediates=True)
    rows = torch.from_numpy(np.random.default_rng(3).choice(cfg.T, 256, replace=False)).cuda()
    host = lambda t: t.cpu().numpy()  # noqa: E731
    mg = (O.unpack_ternary(host(g.packed)), host(g.scales), host(g.col_indices))
    md = (O.unpack_ternary(host(w.packed)), host(w.scales), host(w.col_indices))
    x = host(xb[rows].float())
    q_x, s_x = O.activation_quantize_int(x)
    np.testing.assert_array_equal(host(ws["q_x"][rows]), q_x)
    np.testing.assert_array_equal(host(ws["gate"][rows]), O.ternary_block_ell_matmul(q_x, s_x, *mg))
    q_h, s_h = host(ws["q_h"][rows]), host(ws["s_h"][rows])
    ref = (O.ternary_block_ell_matmul(q_h, s_h, *md) + x).astype(np.float32)
    np.testing.assert_array_equal(host(out[rows]), ref)
    from looped_blockell.kernels import read_status
    assert read_status() == 0


@pytest.mark.parametrize("seed", range(6))
def test_ternary_random_shapes_bit_exact(seed):
    """Seeded random shapes, slot counts, dead slots and ragged token counts:
    the gate / up pre-activations stay bit-exact."""
    rng = np.random.default_rng(500 + seed)
    Cd, Rf = int(rng.integers(2, 6)), int(rng.integers(2, 9))
    T = int(rng.integers(1, 600))
    Kg, Ku, Kd = int(rng.integers(1, Cd + 1)), int(rng.integers(1, Cd + 1)), int(rng.integers(1, Rf + 1))
    case = make_case(T, Cd * 64, Rf * 64, 64, Kg, Ku, Kd, seed=seed, dead=int(rng.integers(0, 3)))
    x, ws, out, m = _run(case, bool(seed % 2))
    q_x, s_x = O.activation_quantize_int(x)
    np.testing.assert_array_equal(ws["q_x"], q_x)
    np.testing.assert_array_equal(ws["gate"], O.ternary_block_ell_matmul(q_x, s_x, *m["g"]))
    np.testing.assert_array_equal(ws["up"], O.ternary_block_ell_matmul(q_x, s_x, *m["u"]))
