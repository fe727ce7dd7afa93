"""CPU-only checks of the C ABI: the in-tree library loads, exports every
entry point include/bell.h declares, and rejects bad descriptors on the host
(no kernel is launched; no GPU is needed)."""

import ctypes as C
import os
import re

import pytest

from conftest import ROOT


def _lib():
    from looped_blockell.kernels import _lib
    if not os.path.exists(_lib.LIB_PATH):
        pytest.skip("library not built")
    return _lib


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "bell.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(bell_[a-z0-9_]+)\s*\(", src)))


def test_every_declared_symbol_is_exported():
    L = _lib()
    lib = L.load()
    syms = declared_symbols()
    assert len(syms) >= 15
    for s in syms:
        assert hasattr(lib, s), f"{s} not exported"
        assert s in L.SIGNATURES, f"{s} has no ctypes signature"


def test_abi_version_and_plan_bytes():
    lib = _lib().load()
    assert lib.bell_abi_version() == 2
    # gate/up: 128 rows x (8+8) entries, counts; down: 32 x 32, counts — 16-byte aligned sections
    assert lib.bell_plan_bytes(128, 8, 8, 32, 32) == 128 * 16 * 4 + 128 * 4 + 32 * 32 * 4 + 32 * 4
    assert lib.bell_plan_bytes(0, 0, 0, 3, 5) % 16 == 0


def test_null_descriptor_is_rejected_on_host():
    L = _lib()
    lib = L.load()
    assert lib.bell_swiglu_fwd_bf16(None, None) == -8
    assert "NULL" in L.last_error()
    assert lib.bell_loop_fwd_bf16(None, None) == -8


def test_bad_shapes_rejected_before_any_launch():
    L = _lib()
    lib = L.load()
    d = L.BellFFNDesc()
    d.T, d.d_model, d.d_ff, d.dtype = 16, 256, 512, L.BELL_DTYPE_BF16
    d.x = d.h = d.out = d.plan = 1024  # never dereferenced: validation fails first
    d.gate = L.BellEll(1024, 1024, 8, 4, 2, 48, 0, 0)  # B = 48 unsupported
    d.up = L.BellEll(1024, 1024, 8, 4, 2, 64, 0, 0)
    d.down = L.BellEll(1024, 1024, 4, 8, 2, 64, 0, 0)
    assert lib.bell_swiglu_fwd_bf16(C.byref(d), None) == -2
    assert "tile size" in L.last_error()
    d.gate = L.BellEll(1024, 1024, 8, 4, 2, 64, 0, 0)
    d.up = L.BellEll(1024, 1024, 4, 4, 2, 64, 0, 0)
    assert lib.bell_swiglu_fwd_bf16(C.byref(d), None) == -2
    assert "same R_ff" in L.last_error()
    d.up = L.BellEll(1024, 1024, 8, 4, 2, 64, 0, 0)
    d.dtype = L.BELL_DTYPE_F32
    assert lib.bell_swiglu_fwd_bf16(C.byref(d), None) == -1
    lin = L.BellLinearDesc()
    lin.dtype, lin.out_dtype = L.BELL_DTYPE_BF16, 7
    lin.w = L.BellEll(1024, 1024, 4, 4, 2, 64, 0, 0)
    assert lib.bell_linear_bf16(C.byref(lin), None) == -1


def test_python_surface_shapes_on_cpu():
    """Format utilities and module construction run without a GPU; the
    kernels themselves refuse CPU tensors."""
    import torch
    from looped_blockell.layers import (BlockELLConfig, BlockELLTensor, MLPBlock, block_ell_matmul,
                                        block_ell_to_dense, create_block_ell_from_dense, create_random_topology)
    cfg = BlockELLConfig(R=4, C=8, K=3, B=16)
    assert (cfg.out_features, cfg.in_features, cfg.density, cfg.total_blocks) == (64, 128, 0.375, 12)
    with pytest.raises(ValueError):
        BlockELLConfig(R=1, C=2, K=3)
    cols = create_random_topology(4, 8, 3, key=0)
    assert cols.dtype == torch.int32 and all(len(set(r.tolist())) == 3 for r in cols)
    W = torch.randn(64, 128)
    e = create_block_ell_from_dense(W, tile_size=16, density=1.0)
    assert torch.allclose(block_ell_to_dense(e), W)
    with pytest.raises(ValueError):
        BlockELLTensor(values=torch.zeros(2, 2, 16, 16), col_indices=torch.zeros(2, 3, dtype=torch.int32), config=BlockELLConfig(2, 4, 2, 16))
    m = MLPBlock(256, 512, use_swiglu=True, tile_size=64, density=0.5)
    assert torch.equal(m.w_gate.col_indices, m.w_up.col_indices)  # reference: same seed for gate and up
    with pytest.raises(RuntimeError, match="CUDA"):
        block_ell_matmul(torch.randn(2, 3, 128), e)


def test_dense_roundtrip_matches_oracle_convention():
    import numpy as np
    import torch
    import oracle as O
    from looped_blockell.layers import block_ell_to_dense, create_block_ell_from_dense
    W = np.random.default_rng(3).standard_normal((128, 256)).astype(np.float32)
    e = create_block_ell_from_dense(torch.from_numpy(W), tile_size=64, density=0.5)
    v, c = O.dense_to_block_ell(W, 64, 0.5)
    np.testing.assert_array_equal(e.col_indices.numpy(), c)
    np.testing.assert_array_equal(e.values.numpy(), v)
    np.testing.assert_array_equal(block_ell_to_dense(e).numpy(), O.block_ell_to_dense(v, c, 128, 256))


def test_noalloc_scratch_bytes_sizes():
    """bell_noalloc_scratch_bytes: plan + h rounded to 256 bytes each, and 0
    for any size no forward accepts (so a caller can ask whether a call fits)."""
    lib = _lib().load()
    plan = lib.bell_plan_bytes(16, 2, 3, 4, 6)
    up = lambda v: (v + 255) & ~255  # noqa: E731
    assert lib.bell_noalloc_scratch_bytes(700, 2048, 16, 2, 3, 4, 6) == up(plan) + up(700 * 2048 * 2)
    assert lib.bell_noalloc_scratch_bytes(-1, 2048, 16, 2, 3, 4, 6) == 0
    assert lib.bell_noalloc_scratch_bytes(700, 2048, -16, 2, 3, 4, 6) == 0
    assert lib.bell_noalloc_scratch_bytes(700, 2048, 16, 0, 3, 4, 6) == 0
    assert lib.bell_noalloc_scratch_bytes(700, 2048, 16, 2, 3, 4, -6) == 0
