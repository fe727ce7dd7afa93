"""Randomised parity sweep: seeded random shapes, tile sizes, layouts, slot
counts, dead and duplicate slots, shared or independent gate/up columns and
ragged token counts, for the bf16 forward (rel-L2 <= 1e-2 against the fp64
oracle on the bf16 inputs) and its backward (rel-L2 <= 2e-2)."""

import numpy as np
import pytest
import torch

import oracle as O
from gpu_util import make_case, to_dev

pytestmark = pytest.mark.gpu


def _K():
    from looped_blockell import kernels as K
    return K


def _f64(t):
    return t.float().cpu().numpy().astype(np.float64)


def _draw(seed):
    rng = np.random.default_rng(1000 + seed)
    B = int(rng.choice([64, 128]))
    Cd = int(rng.integers(2, 5))      # d_model blocks
    Rf = int(rng.integers(2, 7))      # d_ff blocks
    T = int(rng.integers(1, 700))
    Kg = int(rng.integers(1, Cd + 1))
    Ku = int(rng.integers(1, Cd + 1))
    Kd = int(rng.integers(1, Rf + 1))
    layout = int(rng.integers(0, 2))
    shared = bool(rng.integers(0, 2)) and Kg == Ku
    dead = int(rng.integers(0, 3))
    dup = bool(rng.integers(0, 2))
    return dict(T=T, d=Cd * B, F=Rf * B, B=B, Kg=Kg, Ku=Ku, Kd=Kd, layout=layout, shared=shared, dead=dead,
                dup=dup)


@pytest.mark.parametrize("seed", range(12))
def test_random_forward_and_backward(seed):
    K = _K()
    p = _draw(seed)
    c = make_case(p["T"], p["d"], p["F"], p["B"], p["Kg"], p["Ku"], p["Kd"], seed=seed, dead=p["dead"],
                  shared=p["shared"], dup=p["dup"])
    dv = to_dev(c, torch.bfloat16, p["layout"])
    out, h, g, u = K.block_ell_swiglu_fwd_with_intermediate(dv["x"], dv["vg"], dv["cg"], dv["vu"], dv["cu"],
                                                            dv["vd"], dv["cd"], add_residual=True,
                                                            layout=p["layout"], shared_topology=p["shared"])
    dy = torch.randn(p["T"], p["d"], generator=torch.Generator().manual_seed(seed)).to(torch.bfloat16).cuda()
    grads = K.block_ell_swiglu_bwd(dy, dv["x"], g, u, h, dv["vg"], dv["cg"], dv["vu"], dv["cu"], dv["vd"],
                                   dv["cd"], layout=p["layout"])
    torch.cuda.synchronize()
    assert K.read_status() == 0, p
    lay = p["layout"]
    mats = [(_f64(dv[v]), dv[ci].cpu().numpy(), lay) for v, ci in (("vg", "cg"), ("vu", "cu"), ("vd", "cd"))]
    x = _f64(dv["x"])
    ref_out = O.swiglu_ffn(x, *mats, add_residual=True)
    assert O.rel_l2(_f64(out), ref_out) < 1e-2, p
    ref = O.swiglu_ffn_backward(x, *mats, _f64(dy), add_residual=True)
    for name, a, b in zip(("dx", "d_vg", "d_vu", "d_vd"), grads, ref):
        if np.abs(b).max() == 0:
            assert float(a.float().abs().max()) == 0.0, (name, p)
        else:
            assert O.rel_l2(_f64(a), b) < 2e-2, (name, p)
