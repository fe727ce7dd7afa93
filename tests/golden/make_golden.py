"""Generate golden fixtures from the REFERENCE's own runnable code.

Run in a container that has the reference checked out (read-only is fine):

    python tests/golden/make_golden.py --reference /path/to/looped-blockell-tpu

It imports, from the reference tree:
  * interop/pt_model.py            MLPBlock (SwiGLU, bias-free nn.Linear) and RMSNorm
  * interop/convert_checkpoint.py  _block_ell_to_dense / _dense_to_block_ell
  * bonsai-test/bitlinear.py       ternary_quantize / activation_quantize
and writes small ``.npz`` fixtures next to this script.  The fixtures are
committed; tests never read the reference tree at run time.

The reference JAX path (looped_blockell/layers/block_ell.py) cannot run here
(no jax), so the Block-ELL matmul semantics are pinned through the
reference's converter + its PyTorch MLP: dense weights scattered from the
Block-ELL tiles by ``_block_ell_to_dense`` and run through ``MLPBlock``.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _load_reference(root: str):
    sys.path.insert(0, root)
    sys.path.insert(0, os.path.join(root, "bonsai-test"))
    from interop.pt_model import MLPBlock, RMSNorm, InteropConfig  # noqa: E402
    from interop.convert_checkpoint import _block_ell_to_dense, _dense_to_block_ell  # noqa: E402
    import bitlinear  # noqa: E402
    return MLPBlock, RMSNorm, InteropConfig, _block_ell_to_dense, _dense_to_block_ell, bitlinear


def _topology(rng, R, C, K):
    return np.stack([np.sort(rng.choice(C, size=K, replace=False)) for _ in range(R)]).astype(np.int32)


def _dense_alive(to_dense, values, cols, out_f, in_f, B):
    """Reference dense weight with dead (-1) slots zeroed, as alive_mask does
    (looped_blockell/layers/mlp.py:73-77)."""
    v = values.copy()
    c = cols.copy()
    dead = c < 0
    v[dead] = 0.0
    c[dead] = 0  # any valid column: its tile is zero
    # _block_ell_to_dense assigns (not accumulates); zero tiles written over a
    # live tile would erase it, so write dead tiles first by ordering.
    order = np.argsort(~dead, axis=1, kind="stable")
    v = np.take_along_axis(v, order[:, :, None, None], axis=1)
    c = np.take_along_axis(c, order, axis=1)
    return to_dense(v, c, out_f, in_f, tile_size=B)


def make_swiglu_case(ref, name, T, d, F, B, Kg, Ku, Kd, seed, dead_slots=0):
    MLPBlock, _, InteropConfig, to_dense, _, _ = ref
    rng = np.random.default_rng(seed)
    Rf, Cd, Rd, Cf = F // B, d // B, d // B, F // B
    cg, cu, cd = _topology(rng, Rf, Cd, Kg), _topology(rng, Rf, Cd, Ku), _topology(rng, Rd, Cf, Kd)
    for _ in range(dead_slots):
        cg[rng.integers(Rf), rng.integers(Kg)] = -1
        cd[rng.integers(Rd), rng.integers(Kd)] = -1
    vg = (rng.standard_normal((Rf, Kg, B, B)) * 0.02).astype(np.float32)
    vu = (rng.standard_normal((Rf, Ku, B, B)) * 0.02).astype(np.float32)
    vd = (rng.standard_normal((Rd, Kd, B, B)) * 0.02).astype(np.float32)
    x = rng.standard_normal((T, d)).astype(np.float32)

    cfg = InteropConfig(d_model=d, d_ff=F, use_swiglu=True, tile_size=B)
    mlp = MLPBlock(cfg, prunable=False).double()
    with torch.no_grad():
        mlp.w_gate.weight.copy_(torch.from_numpy(_dense_alive(to_dense, vg, cg, F, d, B)).double())
        mlp.w_up.weight.copy_(torch.from_numpy(_dense_alive(to_dense, vu, cu, F, d, B)).double())
        mlp.w_down.weight.copy_(torch.from_numpy(_dense_alive(to_dense, vd, cd, d, F, B)).double())
        out = mlp(torch.from_numpy(x).double()).numpy()
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), x=x, vg=vg, cg=cg, vu=vu, cu=cu,
                        vd=vd, cd=cd, out=out, B=B, d=d, F=F)


def make_layout_case(ref):
    _, _, _, to_dense, from_dense, _ = ref
    rng = np.random.default_rng(7)
    W = rng.standard_normal((128, 256)).astype(np.float32)  # [out, in]
    values, cols = from_dense(W, tile_size=64)
    back = to_dense(values, cols, 128, 256, tile_size=64)
    np.savez_compressed(os.path.join(HERE, "tile_layout.npz"), W=W, values=values, cols=cols, back=back)


def make_rmsnorm_case(ref):
    _, RMSNorm, _, _, _, _ = ref
    rng = np.random.default_rng(11)
    x = rng.standard_normal((16, 256)).astype(np.float32)
    gain = (1.0 + 0.1 * rng.standard_normal(256)).astype(np.float32)
    norm = RMSNorm(256).double()
    with torch.no_grad():
        norm.scale.copy_(torch.from_numpy(gain).double())
        out = norm(torch.from_numpy(x).double()).numpy()
    np.savez_compressed(os.path.join(HERE, "rmsnorm.npz"), x=x, gain=gain, out=out, eps=1e-5)


def make_loop_case(ref):
    """L iterations of h = h + MLP(RMSNorm(h)) with the reference modules, in
    the order of csrc/loop/persistent_core.cu:315-335."""
    MLPBlock, RMSNorm, InteropConfig, to_dense, _, _ = ref
    rng = np.random.default_rng(13)
    T, d, F, B, K, Kd, L = 40, 128, 256, 64, 1, 2, 3
    Rf, Cd, Rd, Cf = F // B, d // B, d // B, F // B
    cg = _topology(rng, Rf, Cd, K)
    cd = _topology(rng, Rd, Cf, Kd)
    vg = (rng.standard_normal((Rf, K, B, B)) * 0.02).astype(np.float32)
    vu = (rng.standard_normal((Rf, K, B, B)) * 0.02).astype(np.float32)
    vd = (rng.standard_normal((Rd, Kd, B, B)) * 0.02).astype(np.float32)
    h0 = rng.standard_normal((T, d)).astype(np.float32)
    gain = np.ones(d, dtype=np.float32)
    cfg = InteropConfig(d_model=d, d_ff=F, use_swiglu=True, tile_size=B)
    mlp = MLPBlock(cfg, prunable=False).double()
    norm = RMSNorm(d, 1e-5).double()
    with torch.no_grad():
        mlp.w_gate.weight.copy_(torch.from_numpy(to_dense(vg, cg, F, d, tile_size=B)).double())
        mlp.w_up.weight.copy_(torch.from_numpy(to_dense(vu, cg, F, d, tile_size=B)).double())
        mlp.w_down.weight.copy_(torch.from_numpy(to_dense(vd, cd, d, F, tile_size=B)).double())
        h = torch.from_numpy(h0).double()
        for _ in range(L):
            h = h + mlp(norm(h))
        out = h.numpy()
    np.savez_compressed(os.path.join(HERE, "loop.npz"), h0=h0, gain=gain, vg=vg, cg=cg, vu=vu,
                        cu=cg, vd=vd, cd=cd, out=out, L=L, B=B, eps=1e-5)


def make_ternary_case(ref):
    """bitlinear quantizers with group = one B x B tile, and the reference's
    fake-quant linear (dequantised activations x dequantised weights)."""
    _, _, _, to_dense, _, bitlinear = ref
    rng = np.random.default_rng(17)
    T, d, F, B, K = 24, 128, 256, 64, 1
    Rf, Cd = F // B, d // B
    cg = _topology(rng, Rf, Cd, K)
    vg = (rng.standard_normal((Rf, K, B, B)) * 0.02).astype(np.float32)
    x = rng.standard_normal((T, d)).astype(np.float32)
    wt = torch.from_numpy(vg).float()
    w_q, scales = bitlinear.ternary_quantize(wt.reshape(-1), group_size=B * B)
    w_q = w_q.reshape(vg.shape)
    x_dq = bitlinear.activation_quantize(torch.from_numpy(x).float(), bits=8)
    deq = (w_q * scales.reshape(Rf, K, 1, 1)).numpy().astype(np.float32)
    dense = torch.from_numpy(to_dense(deq, cg, F, d, tile_size=B)).double()
    y = (x_dq.double() @ dense.T).numpy()
    np.savez_compressed(os.path.join(HERE, "ternary.npz"), x=x, vg=vg, cg=cg,
                        t=w_q.numpy().astype(np.int8), s=scales.numpy().astype(np.float32),
                        x_dq=x_dq.numpy().astype(np.float32), y=y, B=B)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the reference checkout")
    args = ap.parse_args()
    torch.manual_seed(0)
    ref = _load_reference(args.reference)
    make_swiglu_case(ref, "swiglu_small", T=48, d=128, F=256, B=64, Kg=1, Ku=2, Kd=2, seed=3)
    make_swiglu_case(ref, "swiglu_dead", T=70, d=128, F=256, B=64, Kg=2, Ku=2, Kd=3, seed=5, dead_slots=2)
    make_layout_case(ref)
    make_rmsnorm_case(ref)
    make_loop_case(ref)
    make_ternary_case(ref)
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
