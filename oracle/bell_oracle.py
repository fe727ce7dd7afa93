"""NumPy restatement of the reference Block-ELL SwiGLU path (TEST INFRASTRUCTURE).

Every function cites the reference file:line it follows (paths are relative
to the bigwolfeman/looped-blockell-tpu project root).  Used only by tests/,
``__graft_entry__.smoke()`` and bench.py's CPU-baseline legs.

Conventions
-----------
* Block-ELL weight: ``values [R, K, B, B]`` and ``col_indices [R, K]`` int32.
  Logical weight is ``[out = R*B, in = C*B]``.
* Tile layout ``IN_OUT`` (default): ``values[r, k]`` is ``[B_in, B_out]``, the
  JAX/Flax convention (looped_blockell/layers/block_ell.py:96-99,169-177;
  interop/convert_checkpoint.py:118-131).  ``OUT_IN`` is the reference CUDA
  kernels' ``[B_out, B_in]`` convention (csrc/block_ell/swiglu_fwd.cu:273-284).
* A column index of ``-1`` is a dead slot and contributes nothing.  The
  reference zeroes dead tiles through ``alive_mask`` (looped_blockell/layers/
  mlp.py:73-77) and the column-reorder pass keeps ``-1`` in dead slots
  (looped_blockell/opt/column_reorder.py:131-136).
"""

from __future__ import annotations

import numpy as np

LAYOUT_IN_OUT = 0
LAYOUT_OUT_IN = 1

__all__ = [
    "LAYOUT_IN_OUT", "LAYOUT_OUT_IN",
    "random_topology", "block_ell_to_dense", "dense_to_block_ell",
    "compact_block_ell", "dff_permutation", "block_ell_matmul", "block_ell_matmul_t", "silu", "swiglu_ffn", "swiglu_ffn_backward",
    "swiglu_ffn_backward_sparse", "rmsnorm", "looped_ffn",
    "ternary_quantize_tiles", "activation_quantize_int", "pack_ternary",
    "unpack_ternary", "fma_f32", "ternary_block_ell_matmul", "ternary_swiglu_ffn",
    "bf16_round", "rel_l2", "nnz_flops",
]


# ----------------------------------------------------------------------------
# helpers
# ----------------------------------------------------------------------------

def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), as float32."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    u = (u + 0x7FFF + lsb) & 0xFFFF0000
    out = u.astype(np.uint32).view(np.float32)
    # NaN stays NaN
    return np.where(np.isnan(a), a, out)


def rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    """||a - b||_2 / ||b||_2 in float64."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b.ravel())
    num = np.linalg.norm((a - b).ravel())
    return float(num / den) if den > 0 else float(num)


def nnz_flops(T: int, d_model: int, d_ff: int, density_gu: float, density_d: float) -> float:
    """Nonzero FLOPs of one SwiGLU forward: 2*T*B^2 per live tile."""
    return 2.0 * T * d_model * d_ff * (2.0 * density_gu + density_d)


def random_topology(R: int, C: int, K: int, rng: np.random.Generator, sort: bool = True) -> np.ndarray:
    """K unique column blocks per block-row, uniform without replacement.

    Follows looped_blockell/layers/block_ell.py:69-76 (choice without
    replacement per row); the benchmark configs additionally sort each row,
    as create_block_ell_from_dense does (block_ell.py:104-105).
    """
    cols = np.stack([rng.choice(C, size=K, replace=False) for _ in range(R)]).astype(np.int32)
    if sort:
        cols.sort(axis=1)
    return cols


def _tile_in_out(values: np.ndarray, layout: int) -> np.ndarray:
    """Return tiles as [.., B_in, B_out] whatever the stored layout."""
    if layout == LAYOUT_IN_OUT:
        return values
    return np.swapaxes(values, -1, -2)


# ----------------------------------------------------------------------------
# format conversion
# ----------------------------------------------------------------------------

def block_ell_to_dense(values: np.ndarray, cols: np.ndarray, out_features: int,
                       in_features: int, layout: int = LAYOUT_IN_OUT) -> np.ndarray:
    """Scatter Block-ELL to dense ``[out, in]``.

    Follows interop/convert_checkpoint.py:134-148 and
    looped_blockell/layers/block_ell.py:118-146: ``dense[r-block, c-block] =
    values[r, k].T`` for [B_in, B_out] tiles.  Dead slots (col < 0) are
    skipped; duplicate columns accumulate (the matmul semantics).
    """
    tiles = _tile_in_out(values, layout)
    R, K, B, _ = tiles.shape
    dense = np.zeros((out_features, in_features), dtype=np.float64)
    for r in range(R):
        for k in range(K):
            c = int(cols[r, k])
            if c < 0:
                continue
            dense[r * B:(r + 1) * B, c * B:(c + 1) * B] += tiles[r, k].T
    return dense.astype(values.dtype)


def dense_to_block_ell(dense: np.ndarray, tile_size: int, density: float):
    """Top-K Frobenius-norm blocks per block-row, columns sorted.

    Follows looped_blockell/layers/block_ell.py:79-116: K = max(1, int(C*density)),
    blocks reshaped to [R, C, B_in, B_out], top-K by norm, sorted columns.
    Returns (values [R,K,B_in,B_out], cols [R,K] int32).
    """
    out_f, in_f = dense.shape
    B = tile_size
    R, C = out_f // B, in_f // B
    K = max(1, int(C * density))
    blocks = dense.reshape(R, B, C, B).transpose(0, 2, 3, 1)
    norms = np.sqrt((blocks.astype(np.float64) ** 2).sum(axis=(2, 3)))
    top = np.argsort(-norms, axis=1, kind="stable")[:, :K]
    cols = np.sort(top, axis=1).astype(np.int32)
    values = np.stack([blocks[r, cols[r]] for r in range(R)])
    return values, cols


def compact_block_ell(values: np.ndarray, cols: np.ndarray, alive: np.ndarray):
    """Pack alive slots to the front of each row (stable), cut to
    K_new = max(1, max alive count).  Follows looped_blockell/opt/compaction.py:
    31-61 (argsort of ~alive, truncate; dead survivors keep index and tile).
    Returns (values, cols, alive, K_new)."""
    alive = np.asarray(alive, dtype=bool)
    K_new = max(1, int(alive.sum(axis=1).max()) if alive.shape[0] else 1)
    order = np.argsort(~alive, axis=1, kind="stable")[:, :K_new]
    rows = np.arange(cols.shape[0])[:, None]
    return values[rows, order], cols[rows, order], alive[rows, order], K_new


def dff_permutation(fc1_alive, fc2_alive, fc1_cols, C_ff: int) -> np.ndarray:
    """d_ff order by descending importance: alive fc1 tiles per column plus
    alive fc2 tiles per block-row (looped_blockell/opt/column_reorder.py:36-120).
    Returns perm with perm[new] = old."""
    imp = np.zeros(C_ff, dtype=np.float64)
    for c, a in zip(np.asarray(fc1_cols).reshape(-1), np.asarray(fc1_alive).reshape(-1)):
        if c >= 0 and a:
            imp[min(int(c), C_ff - 1)] += 1.0
    rows = np.asarray(fc2_alive, dtype=np.float64).sum(axis=1)
    n = min(rows.shape[0], C_ff)
    imp[:n] += rows[:n]
    return np.argsort(-imp, kind="stable").astype(np.int32)


# ----------------------------------------------------------------------------
# bf16 / fp32 path
# ----------------------------------------------------------------------------

def block_ell_matmul(x: np.ndarray, values: np.ndarray, cols: np.ndarray,
                     layout: int = LAYOUT_IN_OUT, dtype=np.float64) -> np.ndarray:
    """``y[t, r*B + D] = sum_k sum_d x[t, c(r,k)*B + d] * V[r,k,d,D]``.

    Follows looped_blockell/layers/block_ell.py:149-182 (gather the input
    column tiles named by col_indices, contract with einsum 'bsrkd,rkdD').
    x is [T, C*B] (the reference's [b, s, in] flattened over b, s).  Each
    block-row is one BLAS GEMM over its live tiles.
    """
    tiles = _tile_in_out(values, layout)
    R, K, B, _ = tiles.shape
    x = np.asarray(x, dtype=dtype)
    T = x.shape[0]
    y = np.zeros((T, R * B), dtype=dtype)
    for r in range(R):
        live = [k for k in range(K) if cols[r, k] >= 0]
        if not live:
            continue
        xg = np.concatenate([x[:, int(cols[r, k]) * B:(int(cols[r, k]) + 1) * B] for k in live], axis=1)
        w = tiles[r, live].astype(dtype).reshape(len(live) * B, B)
        y[:, r * B:(r + 1) * B] = xg @ w
    return y


def block_ell_matmul_t(y: np.ndarray, values: np.ndarray, cols: np.ndarray, in_features: int,
                       layout: int = LAYOUT_IN_OUT, dtype=np.float64) -> np.ndarray:
    """``dx = dy @ W`` for the Block-ELL W of ``block_ell_matmul`` (the input
    gradient of y = x W^T): ``dx[:, c(r,k) block] += dy[:, r block] @ V[r,k]^T``
    for [B_in, B_out] tiles.  The reference computes it by scattering per slot
    (csrc/block_ell/swiglu_bwd.cu:7-12, 16-24); restated with one GEMM per slot."""
    tiles = _tile_in_out(values, layout)
    R, K, B, _ = tiles.shape
    y = np.asarray(y, dtype=dtype)
    dx = np.zeros((y.shape[0], in_features), dtype=dtype)
    for r in range(R):
        yr = y[:, r * B:(r + 1) * B]
        for k in range(K):
            c = int(cols[r, k])
            if c >= 0:
                dx[:, c * B:(c + 1) * B] += yr @ tiles[r, k].astype(dtype).T
    return dx


def silu(a: np.ndarray) -> np.ndarray:
    """x * sigmoid(x) (jax.nn.silu / F.silu)."""
    return a / (1.0 + np.exp(-a))


def swiglu_ffn(x, gate, up, down, add_residual=False, residual=None,
               dtype=np.float64, round_h_bf16=False, return_intermediates=False):
    """``out = W_down(silu(W_gate x) * W_up x) (+ residual)``.

    Follows looped_blockell/layers/mlp.py:119-145 (SwiGLU, bias-free per
    interop/pt_model.py:862-867) and the residual epilogue of
    csrc/block_ell/swiglu_fwd.cu:551-553 (``add_residual`` adds x).
    ``gate``/``up``/``down`` are (values, cols, layout) triples.
    ``round_h_bf16`` models the bf16 intermediate the reference CUDA op keeps
    (swiglu_fwd.cu:625).
    """
    g = block_ell_matmul(x, *gate, dtype=dtype)
    u = block_ell_matmul(x, *up, dtype=dtype)
    h = silu(g) * u
    if round_h_bf16:
        h = bf16_round(h.astype(np.float32)).astype(dtype)
    out = block_ell_matmul(h, *down, dtype=dtype)
    if add_residual:
        res = x if residual is None else residual
        out = out + np.asarray(res, dtype=dtype)
    if return_intermediates:
        return out, h, g, u
    return out


def _tile_grads(dense_grad: np.ndarray, cols: np.ndarray, B: int, layout: int) -> np.ndarray:
    """Per-slot tile gradients from a dense ``[out, in]`` gradient: slot (r, k)
    gets block (r, cols[r, k]) as a [B_in, B_out] tile (zeros for dead slots),
    returned in the stored ``layout``."""
    R, K = cols.shape
    out = np.zeros((R, K, B, B), dtype=np.float64)
    for r in range(R):
        for k in range(K):
            c = int(cols[r, k])
            if c >= 0:
                out[r, k] = dense_grad[r * B:(r + 1) * B, c * B:(c + 1) * B].T
    return out if layout == LAYOUT_IN_OUT else np.swapaxes(out, -1, -2)


def swiglu_ffn_backward(x, gate, up, down, dy, add_residual=True):
    """Gradients of ``out = W_down(silu(W_gate x) * W_up x) (+ x)``.

    The reference's backward (csrc/block_ell/swiglu_bwd.cu:7-35) computes
    d_h = dy W_down, d_gate = d_h * up * silu'(gate), d_up = d_h * silu(gate)
    (:305-334), d_x = d_gate W_gate + d_up W_up, plus dy for the residual
    (:785-796, always added there; ``add_residual`` selects it here), and
    d_W[r, k] = a[:, c]^T b[:, r] per live tile (:13-14, :29-30).  Restated
    densely in float64: returns (dx, dv_gate, dv_up, dv_down) with the tile
    gradients in each matrix's stored layout (dead slots get zeros).
    """
    xv = np.asarray(x, dtype=np.float64)
    dyv = np.asarray(dy, dtype=np.float64)
    d = xv.shape[1]
    (vg, cg, lg), (vu, cu, lu), (vd, cd, ld) = gate, up, down
    B = vg.shape[-1]
    F = vg.shape[0] * B
    Wg = block_ell_to_dense(vg, cg, F, d, lg)
    Wu = block_ell_to_dense(vu, cu, F, d, lu)
    Wd = block_ell_to_dense(vd, cd, d, F, ld)
    g, u = xv @ Wg.T, xv @ Wu.T
    sig = 1.0 / (1.0 + np.exp(-g))
    h = g * sig * u
    dh = dyv @ Wd
    dg = dh * u * (sig + g * sig * (1.0 - sig))
    du = dh * g * sig
    dx = dg @ Wg + du @ Wu
    if add_residual:
        dx = dx + dyv
    return (dx, _tile_grads(dg.T @ xv, cg, B, lg), _tile_grads(du.T @ xv, cu, B, lu),
            _tile_grads(dyv.T @ h, cd, B, ld))


def swiglu_ffn_backward_sparse(x, gate, up, down, dy, g, u, h, add_residual=True, dtype=np.float64):
    """The same gradients as ``swiglu_ffn_backward`` from the saved forward
    intermediates (g = gate pre-activation, u = up output, h = silu(g) * u),
    as the reference op takes them (block_ell_ops.cpp:83-97), computed tile by
    tile: transposed Block-ELL products for d_h and d_x and one
    a[:, c]^T b[:, r] product per live slot for the tile gradients
    (swiglu_bwd.cu:13-14, 29-30).  Cost grows with the live tiles, not with
    d_model * d_ff, so it serves as the CPU timing arm too."""
    x, dy, g, u, h = (np.asarray(a, dtype=dtype) for a in (x, dy, g, u, h))
    (vg, cg, lg), (vu, cu, lu), (vd, cd, ld) = gate, up, down
    d = x.shape[1]
    F = g.shape[1]
    dh = block_ell_matmul_t(dy, vd, cd, F, ld, dtype)
    sig = 1.0 / (1.0 + np.exp(-g))
    dg = dh * u * (sig + g * sig * (1.0 - sig))
    du = dh * g * sig
    dx = block_ell_matmul_t(dg, vg, cg, d, lg, dtype) + block_ell_matmul_t(du, vu, cu, d, lu, dtype)
    if add_residual:
        dx = dx + dy

    def tile_grads(a, b, values, cols, layout):
        R, K, B, _ = values.shape
        out = np.zeros((R, K, B, B), dtype=dtype)
        for r in range(R):
            br = b[:, r * B:(r + 1) * B]
            for k in range(K):
                c = int(cols[r, k])
                if c >= 0:
                    t = a[:, c * B:(c + 1) * B].T @ br  # [B_in, B_out]
                    out[r, k] = t if layout == LAYOUT_IN_OUT else t.T
        return out

    return (dx, tile_grads(x, dg, vg, cg, lg), tile_grads(x, du, vu, cu, lu), tile_grads(h, dy, vd, cd, ld))


def rmsnorm(x: np.ndarray, gain: np.ndarray, eps: float = 1e-5, dtype=np.float64) -> np.ndarray:
    """``x / sqrt(mean(x^2) + eps) * scale``.

    Follows looped_blockell/layers/norms.py:8-15 and interop/pt_model.py:147-155
    (eps 1e-5, looped_blockell/config.py:110).
    """
    x = np.asarray(x, dtype=dtype)
    rms = np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)
    return x / rms * np.asarray(gain, dtype=dtype)


def looped_ffn(h, gain, gate, up, down, L: int, eps: float = 1e-5, dtype=np.float64,
               round_bf16=False):
    """L shared-weight iterations of ``h = h + FFN(RMSNorm(h))``.

    Follows the loop order of csrc/loop/persistent_core.cu:315-335 (norm ->
    Block-ELL SwiGLU without fused residual -> add the PRE-norm h) with one
    weight set repeated L times.  ``round_bf16`` rounds the stored state,
    the normed input and the intermediate to bf16 as the bf16 op does.
    """
    h = np.asarray(h, dtype=dtype)
    for _ in range(L):
        hn = rmsnorm(h, gain, eps, dtype=dtype)
        if round_bf16:
            hn = bf16_round(hn.astype(np.float32)).astype(dtype)
        f = swiglu_ffn(hn, gate, up, down, add_residual=False, dtype=dtype, round_h_bf16=round_bf16)
        h = h + f
        if round_bf16:
            h = bf16_round(h.astype(np.float32)).astype(dtype)
    return h


# ----------------------------------------------------------------------------
# ternary path
# ----------------------------------------------------------------------------

def ternary_quantize_tiles(values: np.ndarray):
    """AbsMean ternarisation with one scale per B x B tile.

    Follows bonsai-test/bitlinear.py:34-55 with group = one tile:
    ``s = mean|w|`` clamped to 1e-8, ``t = round(w / s).clamp(-1, 1)``
    (round half to even).  Returns (t int8 same shape, s float32 [R, K]).
    """
    v = np.asarray(values, dtype=np.float32)
    R, K = v.shape[:2]
    flat = v.reshape(R, K, -1)
    s = np.abs(flat).mean(axis=2, dtype=np.float32)
    s = np.maximum(s, np.float32(1e-8)).astype(np.float32)
    t = np.clip(np.rint(flat / s[:, :, None]), -1, 1).astype(np.int8)
    return t.reshape(v.shape), s


def activation_quantize_int(x: np.ndarray):
    """Per-token absmax int8 quantisation (8 bits, Qb = 128).

    Follows bonsai-test/bitlinear.py:58-69: ``absmax = max|x|`` (clamp 1e-8),
    ``scale = 128 / absmax``, ``q = round(x * scale).clamp(-128, 127)``; all
    in IEEE float32 with round-half-even.  Returns the integer codes and the
    float32 scale (the reference returns q / scale, the dequantised value).
    """
    x = np.asarray(x, dtype=np.float32)
    absmax = np.maximum(np.abs(x).max(axis=-1), np.float32(1e-8)).astype(np.float32)
    scale = (np.float32(128.0) / absmax).astype(np.float32)
    q = np.clip(np.rint(x * scale[:, None]), -128, 127).astype(np.int8)
    return q, scale


_CODE = {0: 0b00, 1: 0b01, -1: 0b11}


def pack_ternary(t: np.ndarray, layout: int = LAYOUT_IN_OUT) -> np.ndarray:
    """Pack ternary tiles at 2 bits per weight.

    Packed format (this build's own; the reference has no packed ternary
    Block-ELL): tile (r, k) is stored output-column major, i.e. as
    ``[B_out][B_in]``; each uint32 word holds 16 consecutive B_in entries of
    one output column, entry i at bits 2*(i % 16); codes 0 -> 00, +1 -> 01,
    -1 -> 11.  Result is uint8 ``[R, K, B, B // 4]`` (little-endian words).
    """
    tiles = _tile_in_out(np.asarray(t, dtype=np.int8), layout)
    R, K, B, _ = tiles.shape
    kt = np.swapaxes(tiles, -1, -2).astype(np.int32)  # [R,K,B_out,B_in]
    codes = np.where(kt == 0, 0, np.where(kt > 0, 1, 3)).astype(np.uint32)
    codes = codes.reshape(R, K, B, B // 16, 16)
    shifts = (2 * np.arange(16, dtype=np.uint32))
    words = (codes << shifts).sum(axis=-1, dtype=np.uint64).astype(np.uint32)
    return np.ascontiguousarray(words).view(np.uint8).reshape(R, K, B, B // 4)


def unpack_ternary(packed: np.ndarray) -> np.ndarray:
    """Inverse of pack_ternary; returns int8 tiles in IN_OUT layout [B_in, B_out]."""
    R, K, B, _ = packed.shape
    words = np.ascontiguousarray(packed).view(np.uint32).reshape(R, K, B, B // 16)
    shifts = (2 * np.arange(16, dtype=np.uint32))
    codes = (words[..., None] >> shifts) & 3
    vals = np.where(codes == 3, -1, codes.astype(np.int32)).astype(np.int8)
    kt = vals.reshape(R, K, B, B)  # [B_out, B_in]
    return np.ascontiguousarray(np.swapaxes(kt, -1, -2))


def fma_f32(a, b, c) -> np.ndarray:
    """Correctly rounded float32 fused multiply-add ``fl(a*b + c)`` (what
    ``fma.rn.f32`` computes), for float32 inputs, exactly.

    a*b is exact in float64 (24 + 24 bits <= 53).  The float64 sum s = a*b + c
    is made round-to-odd: when TwoSum shows it inexact and its last bit is
    even, it moves one ulp toward the exact value.  Rounding a round-to-odd
    value of at least 2*24 + 2 bits to float32 (nearest-even) gives the
    correctly rounded result (Boldo & Melquiond, "Emulation of FMA and
    correctly rounded sums: proved algorithms using rounding to odd", 2008).
    """
    a = np.asarray(a, dtype=np.float32).astype(np.float64)
    b = np.asarray(b, dtype=np.float32).astype(np.float64)
    c = np.asarray(c, dtype=np.float32).astype(np.float64)
    p = a * b
    s = p + c
    bb = s - p
    e = (p - (s - bb)) + (c - bb)  # TwoSum: s + e == p + c exactly
    odd = (s.view(np.int64) & 1) == 1
    fix = (e != 0) & ~odd
    s = np.where(fix, np.nextafter(s, s + e), s)
    return s.astype(np.float32)


def ternary_block_ell_matmul(q: np.ndarray, scale: np.ndarray, t: np.ndarray,
                             s_w: np.ndarray, cols: np.ndarray, return_tile_sums=False):
    """Ternary Block-ELL matmul with exact integer tile sums.

    ``I_k[t, j] = sum_i q[t, c*B + i] * t[r, k, i, j]`` in int32 (exact), then
    ``acc = fma(s_w[r,k], float(I_k), acc)`` (float32, one rounding per tile)
    over the live k in ascending order, and ``y = fl(acc / scale[t])``, all
    round-to-nearest.  Dequantisation follows bonsai-test/bitlinear.py:34-69
    (x ~ q / scale, w ~ t * s); the tile-scale grouping is the packed format's.
    """
    R, K, B, _ = t.shape
    T = q.shape[0]
    # integer products via float64 GEMM: every partial sum is an integer
    # below 2^53, so the result is exact (|I| <= 128 * B)
    qf = q.astype(np.float64)
    y = np.zeros((T, R * B), dtype=np.float32)
    sums = {} if return_tile_sums else None
    for r in range(R):
        acc = np.zeros((T, B), dtype=np.float32)
        for k in range(K):
            c = int(cols[r, k])
            if c < 0:
                continue
            I = np.rint(qf[:, c * B:(c + 1) * B] @ t[r, k].astype(np.float64)).astype(np.int32)
            if sums is not None:
                sums[(r, k)] = I
            acc = fma_f32(np.float32(s_w[r, k]), I.astype(np.float32), acc)
        y[:, r * B:(r + 1) * B] = (acc / scale[:, None].astype(np.float32)).astype(np.float32)
    if return_tile_sums:
        return y, sums
    return y


def ternary_swiglu_ffn(x, gate, up, down, add_residual=False):
    """Ternary Block-ELL SwiGLU forward (int8 activations, 2-bit weights).

    ``gate``/``up``/``down`` are (t int8 [R,K,B_in,B_out], s_w [R,K], cols).
    x (float32) is quantised per token (bitlinear.py:58-69), gate/up are the
    ternary matmuls above, ``h = silu(gate) * up`` in float32, h is
    re-quantised per token over all of d_ff, and the down matmul follows;
    ``add_residual`` adds x in float32.  Returns a dict with every stage.
    """
    x = np.asarray(x, dtype=np.float32)
    qx, sx = activation_quantize_int(x)
    g = ternary_block_ell_matmul(qx, sx, *gate)
    u = ternary_block_ell_matmul(qx, sx, *up)
    h = (g / (np.float32(1.0) + np.exp(-g)) * u).astype(np.float32)
    qh, sh = activation_quantize_int(h)
    out = ternary_block_ell_matmul(qh, sh, *down)
    if add_residual:
        out = (out + x).astype(np.float32)
    return dict(q_x=qx, s_x=sx, gate=g, up=u, h=h, q_h=qh, s_h=sh, out=out)
