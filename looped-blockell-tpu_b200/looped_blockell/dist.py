"""d_ff-sharded Block-ELL SwiGLU across GPUs (one process per GPU).

Partitioning: rank g owns gate/up block-rows [lo_g, hi_g) (an even split of
R_ff = d_ff / B) and so the d_ff slice h[:, lo_g*B : hi_g*B].  The down ELL is
repacked per shard: each down block-row keeps the slots whose column block
falls in [lo_g, hi_g), rebased to the shard and padded with -1 to the shard's
max K.  Each rank computes a partial out_g = h_g W_down,g over all tokens;
one NCCL reduce-scatter (sum) over tokens gives every rank its token slice of
the full output, and the residual is added on that slice only.

The token axis is cut into ``chunks``; rank g receives, for every chunk, the
g-th 1/N of that chunk's rows (``owned_rows``).  The reduce-scatter of chunk
i runs on NCCL's stream while the kernels of chunk i+1 run, so the transfer
overlaps compute.  The reference has no multi-GPU code; this follows the
partitioning its scaling plan asks for.
"""

from __future__ import annotations

from typing import List, Tuple

import torch


def shard_ranges(R: int, world: int) -> List[Tuple[int, int]]:
    """Even split of R block-rows over `world` ranks (the first R % world get one more)."""
    base, extra = divmod(R, world)
    out, lo = [], 0
    for g in range(world):
        hi = lo + base + (1 if g < extra else 0)
        out.append((lo, hi))
        lo = hi
    return out


def repack_down(vd: torch.Tensor, cd: torch.Tensor, lo: int, hi: int):
    """Keep the down slots whose column block is in [lo, hi); rebase columns
    to the shard; pad with -1 (zero tiles) to the max kept count (>= 1).
    Slot order within a row is preserved."""
    keep = (cd >= lo) & (cd < hi)
    counts = keep.sum(dim=1)
    k_max = max(1, int(counts.max().item()) if counts.numel() else 1)
    order = torch.argsort((~keep).to(torch.int8), dim=1, stable=True)[:, :k_max]
    kept = torch.gather(keep, 1, order)
    cols = torch.where(kept, torch.gather(cd, 1, order) - lo, torch.full_like(order, -1, dtype=cd.dtype))
    R, _, B, _ = vd.shape
    vals = torch.gather(vd, 1, order[:, :, None, None].expand(R, k_max, B, B))
    vals = torch.where(kept[:, :, None, None], vals, torch.zeros_like(vals))
    return vals.contiguous(), cols.to(torch.int32).contiguous()


def owned_rows(T: int, rank: int, world: int, chunks: int) -> torch.Tensor:
    """Token rows a rank holds after the chunked reduce-scatter."""
    Tc = T // chunks
    per = Tc // world
    idx = [torch.arange(i * Tc + rank * per, i * Tc + (rank + 1) * per) for i in range(chunks)]
    return torch.cat(idx)


def pick_chunks(T: int, world: int, want: int = 4) -> int:
    c = want
    while c > 1 and (T % c or (T // c) % world or (T // c // world) % 128):
        c -= 1
    return max(c, 1)


class ShardedSwiGLU:
    """This rank's share of a d_ff-split SwiGLU forward (bf16)."""

    def __init__(self, vg, cg, vu, cu, vd, cd, rank: int, world: int, chunks: int = 4, group=None):
        R_f = vg.shape[0]
        self.B = vg.shape[2]
        self.rank, self.world, self.group = rank, world, group
        self.lo, self.hi = shard_ranges(R_f, world)[rank]
        self.vg, self.cg = vg[self.lo:self.hi].contiguous(), cg[self.lo:self.hi].contiguous()
        self.vu, self.cu = vu[self.lo:self.hi].contiguous(), cu[self.lo:self.hi].contiguous()
        self.vd, self.cd = repack_down(vd, cd, self.lo, self.hi)
        self.d_model = vd.shape[0] * self.B
        self.want_chunks = chunks
        self._bufs = {}

    def launches_per_step(self, T: int) -> int:
        # per chunk: plan + gate/up, plan + down (NCCL and the residual add are not counted)
        return 4 * pick_chunks(T, self.world, self.want_chunks)

    def alloc_out(self, T: int, x: torch.Tensor) -> torch.Tensor:
        return torch.empty((T // self.world, self.d_model), dtype=torch.bfloat16, device=x.device)

    def _buf(self, name, shape, dtype, dev):
        t = self._bufs.get(name)
        if t is None or t.shape != shape:
            t = torch.empty(shape, dtype=dtype, device=dev)
            self._bufs[name] = t
        return t

    def forward(self, x: torch.Tensor, out: torch.Tensor = None, add_residual: bool = True) -> torch.Tensor:
        """This rank's token slice of the full forward (bf16, CUDA)."""
        from .kernels.ops import block_ell_gate_up, block_ell_linear
        T = x.shape[0]
        Tc = T // pick_chunks(T, self.world, self.want_chunks)
        h = self._buf("h", (Tc, (self.hi - self.lo) * self.B), torch.bfloat16, x.device)

        def partial_fn(xi: torch.Tensor, dst: torch.Tensor) -> None:
            block_ell_gate_up(xi, self.vg, self.cg, self.vu, self.cu, self.vd, self.cd, h=h)
            block_ell_linear(h, self.vd, self.cd, out=dst)

        return self.run_chunks(x, partial_fn, out, add_residual)

    def run_chunks(self, x: torch.Tensor, partial_fn, out: torch.Tensor = None, add_residual: bool = True,
                   dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
        """The chunk pipeline of ``forward`` around any partial computation:
        ``partial_fn(x_chunk, dst)`` writes this rank's partial ``[Tc, d_model]``
        for a token chunk; the reduce-scatter of chunk i runs (async) while
        chunk i+1 computes, two partial buffers alternate, and the residual is
        added on the owned rows at the end."""
        import torch.distributed as dist
        T = x.shape[0]
        n = pick_chunks(T, self.world, self.want_chunks)
        Tc = T // n
        per = Tc // self.world
        if out is None:
            out = torch.empty((T // self.world, self.d_model), dtype=dtype, device=x.device)
        partial = [self._buf(f"p{i % 2}", (Tc, self.d_model), dtype, x.device) for i in range(n)]
        works = []
        for i in range(n):
            xi = x[i * Tc:(i + 1) * Tc]
            if i >= 2:
                works[i - 2].wait()  # partial buffer i%2 is free again
            partial_fn(xi, partial[i])
            works.append(dist.reduce_scatter_tensor(out[i * per:(i + 1) * per], partial[i], op=dist.ReduceOp.SUM,
                                                    group=self.group, async_op=True))
        for w in works:
            w.wait()
        if add_residual:
            rows = owned_rows(T, self.rank, self.world, n).to(x.device)
            out.add_(x.index_select(0, rows).to(out.dtype))
        return out
