"""Host logic of the fp32 tensor-core forward (bf16x6 split), no GPU: which
method a call runs, the expanded slot counts and the workspace size."""

import os

import pytest


def _f32x():
    from looped_blockell.kernels import f32x
    return f32x


def _lib():
    from looped_blockell.kernels import _lib
    if not os.path.exists(_lib.LIB_PATH):
        pytest.skip("library not built")
    return _lib.load()


def test_method_choice():
    f = _f32x()
    assert f.resolve("simt", 1 << 20, 2, 2, 8) == "simt"
    assert f.resolve("bf16x6", 1, 2, 2, 8) == "bf16x6"
    assert f.resolve("auto", f.AUTO_MIN_TOKENS, 2, 2, 8) == "bf16x6"
    assert f.resolve("auto", f.AUTO_MIN_TOKENS - 1, 2, 2, 8) == "simt"
    # 6K slots per gate/up row and 6K + 3 per down row must fit in 254
    assert f.resolve("auto", 1 << 16, 42, 42, 41) == "bf16x6"
    assert f.resolve("auto", 1 << 16, 43, 2, 8) == "simt"
    assert f.resolve("auto", 1 << 16, 2, 2, 42) == "simt"
    with pytest.raises(RuntimeError):
        f.resolve("bf16x6", 1 << 16, 2, 2, 42)
    with pytest.raises(RuntimeError):
        f.resolve("tf32", 1 << 16, 2, 2, 8)


def test_method_env_override(monkeypatch):
    f = _f32x()
    monkeypatch.setenv("BELL_F32_METHOD", "simt")
    assert f.resolve(None, 1 << 20, 2, 2, 8) == "simt"
    monkeypatch.setenv("BELL_F32_METHOD", "bogus")
    with pytest.raises(RuntimeError):
        f.resolve(None, 1 << 20, 2, 2, 8)


def test_slots_and_workspace_bytes():
    lib = _lib()
    assert lib.bell_f32x_slots(8, 0) == 48 and lib.bell_f32x_slots(8, 1) == 51
    T, d, F, B = 1000, 512, 2048, 64
    up = lambda v: (v + 255) // 256 * 256  # noqa: E731
    # one plan buffer, used in turn: the fused gate/up's (gate, up and down
    # lists) or each linear's
    plan = max(lib.bell_plan_bytes(F // B, 12, 12, d // B, 51), lib.bell_plan_bytes(0, 0, 0, F // B, 12),
               lib.bell_plan_bytes(0, 0, 0, d // B, 51))
    want = up(T * (3 * F + 3 * d) * 2) + 2 * up(T * F * 4) + up(plan)
    assert lib.bell_f32x_workspace_bytes(T, d, F, B, 12, 12, 51) == want
    assert lib.bell_f32x_workspace_bytes(-1, d, F, B, 12, 12, 51) == 0
    assert lib.bell_f32x_workspace_bytes(T, d, F, B, 0, 12, 51) == 0


def test_bad_arguments_rejected_before_any_launch():
    """The fp32 tensor-core entry points check their descriptors on the host
    first (no GPU needed): wrong dtypes, weights that are not expansions,
    residual row ranges, split strides."""
    import ctypes as C
    from looped_blockell.kernels import _lib as L
    lib = _lib()
    d = L.BellFFNDesc()
    d.T, d.d_model, d.d_ff, d.dtype = 16, 256, 512, L.BELL_DTYPE_BF16
    d.x = d.out = 1024  # never dereferenced: validation fails first
    assert lib.bell_swiglu_fwd_f32x(C.byref(d), C.c_void_p(1024), None) == -1
    d.dtype = L.BELL_DTYPE_F32
    CA = 3 * 8 + 3 * 4  # [h parts | x parts] at B = 64
    d.gate = L.BellEll(1024, 1024, 8, CA, 12, 64, 0, 0)
    d.up = L.BellEll(1024, 1024, 8, CA, 12, 64, 0, 0)
    d.down = L.BellEll(1024, 1024, 4, CA, 26, 64, 0, 0)  # 26 = 6K + 2: not an expansion
    assert lib.bell_swiglu_fwd_f32x(C.byref(d), C.c_void_p(1024), None) == -2
    d.down = L.BellEll(1024, 1024, 4, CA, 24, 64, 0, 0)  # no identity slots ...
    d.add_residual = 1  # ... but a residual asked for
    assert lib.bell_swiglu_fwd_f32x(C.byref(d), C.c_void_p(1024), None) == -8
    lin = L.BellLinearDesc()
    lin.T, lin.dtype, lin.out_dtype = 16, L.BELL_DTYPE_F32, L.BELL_DTYPE_BF16
    lin.x = lin.out = 1024
    lin.w = L.BellEll(1024, 1024, 4, 3 * 4 + 3 * 4, 15, 64, 0, 0)
    assert lib.bell_linear_f32x(C.byref(lin), C.c_void_p(1024), None) == -1
    lin.out_dtype = L.BELL_DTYPE_F32
    lin.residual_row_hi = 8
    assert lib.bell_linear_f32x(C.byref(lin), C.c_void_p(1024), None) == -8
    lin.residual_row_hi = 0
    lin.w = L.BellEll(1024, 1024, 4, 3 * 4 + 3 * 4, 14, 64, 0, 0)  # 14 slots: not 6K or 6K + 3
    assert lib.bell_linear_f32x(C.byref(lin), C.c_void_p(1024), None) == -2
    # split: n and the strides must be multiples of 4, the parts must fit the row
    assert lib.bell_f32x_split_rows(8, 6, C.c_void_p(1024), 8, C.c_void_p(1024), 64, 0, None) == -2
    assert lib.bell_f32x_split_rows(8, 8, C.c_void_p(1024), 8, C.c_void_p(1024), 16, 0, None) == -2
    assert lib.bell_f32x_linear_workspace_bytes(-1, 256, 256, 4, 15) == 0


def _split3(v):
    """numpy restatement of the device split (bell_ptx.cuh split3_bf16): three
    round-to-nearest bf16 parts, each difference formed exactly in fp32."""
    import numpy as np
    import oracle as O
    v = np.asarray(v, np.float32)
    p0 = O.bf16_round(v)
    r1 = (v - p0).astype(np.float32)
    p1 = O.bf16_round(r1)
    p2 = O.bf16_round((r1 - p1).astype(np.float32))
    return p0, p1, p2


def test_split_residual_bound():
    """|v - p0 - p1 - p2| <= 2^-27 |v| for normal fp32 values of any sign and
    magnitude, and every part is a bf16 value."""
    import numpy as np
    rng = np.random.default_rng(0)
    v = (rng.standard_normal(200000) * np.exp2(rng.integers(-60, 60, 200000))).astype(np.float32)
    p0, p1, p2 = _split3(v)
    for p in (p0, p1, p2):
        assert np.all((p.view(np.uint32) & 0xFFFF) == 0)
    err = np.abs(v.astype(np.float64) - p0.astype(np.float64) - p1.astype(np.float64) - p2.astype(np.float64))
    assert np.all(err <= np.exp2(-27) * np.abs(v.astype(np.float64)))


def test_six_products_meet_the_fp32_target():
    """The six leading cross products of the split operands, summed in
    float64, against the exact products: the dropped terms stay below the
    rel-L2 1e-5 target by orders of magnitude (the kernels then add fp32
    accumulation rounding, which the GPU tests bound)."""
    import numpy as np
    rng = np.random.default_rng(1)
    x = rng.standard_normal((256, 512)).astype(np.float32)
    w = (rng.standard_normal((512, 384)) * 0.02).astype(np.float32)
    xs, ws = _split3(x), _split3(w)
    pairs = ((0, 0), (0, 1), (1, 0), (0, 2), (1, 1), (2, 0))
    got = sum(xs[i].astype(np.float64) @ ws[j].astype(np.float64) for i, j in pairs)
    exact = x.astype(np.float64) @ w.astype(np.float64)
    rel = np.linalg.norm(got - exact) / np.linalg.norm(exact)
    assert rel < 1e-7, rel
