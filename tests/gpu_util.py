"""Helpers shared by the GPU parity tests: random Block-ELL cases and the
oracle comparison (the oracle is the CPU checker, never the thing tested)."""

from __future__ import annotations

import numpy as np
import torch

import oracle as O


def rand_cols(rng, R, C, K, dead=0, dup=False):
    cols = np.stack([np.sort(rng.choice(C, size=K, replace=False)) for _ in range(R)]).astype(np.int32)
    for _ in range(dead):
        cols[rng.integers(R), rng.integers(K)] = -1
    if dup and K >= 2:
        cols[0, 1] = cols[0, 0]
    return cols


def make_case(T, d, F, B, Kg, Ku, Kd, seed=0, dead=0, shared=False, dup=False):
    """numpy float32 case, tiles [B_in, B_out]."""
    rng = np.random.default_rng(seed)
    Rf, Cd, Rd, Cf = F // B, d // B, d // B, F // B
    cg = rand_cols(rng, Rf, Cd, Kg, dead, dup)
    cu = cg.copy() if shared and Ku == Kg else rand_cols(rng, Rf, Cd, Ku, dead)
    cd = rand_cols(rng, Rd, Cf, Kd, dead)
    vg = (rng.standard_normal((Rf, Kg, B, B)) * 0.02).astype(np.float32)
    vu = (rng.standard_normal((Rf, Ku, B, B)) * 0.02).astype(np.float32)
    vd = (rng.standard_normal((Rd, Kd, B, B)) * 0.02).astype(np.float32)
    x = rng.standard_normal((T, d)).astype(np.float32)
    return dict(x=x, vg=vg, cg=cg, vu=vu, cu=cu, vd=vd, cd=cd)


def to_dev(case, dtype, layout=O.LAYOUT_IN_OUT):
    out = {}
    for k, v in case.items():
        if k.startswith("c"):
            out[k] = torch.from_numpy(v).cuda()
        else:
            t = torch.from_numpy(v)
            if k.startswith("v") and layout == O.LAYOUT_OUT_IN:
                t = t.transpose(-1, -2).contiguous()
            out[k] = t.to(dtype).cuda()
    return out


def dev_inputs_as_f64(dev_case):
    """The exact values the GPU saw (after bf16 rounding), tiles [B_in, B_out]."""
    return {k: v.float().cpu().numpy().astype(np.float64) if not k.startswith("c") else v.cpu().numpy()
            for k, v in dev_case.items()}


def oracle_ffn(c, add_residual=False, layout=O.LAYOUT_IN_OUT, rows=None):
    x = c["x"] if rows is None else c["x"][rows]
    return O.swiglu_ffn(x, (c["vg"], c["cg"], layout), (c["vu"], c["cu"], layout), (c["vd"], c["cd"], layout),
                        add_residual=add_residual, return_intermediates=True)
