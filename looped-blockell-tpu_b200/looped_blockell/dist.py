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
overlaps compute.  Two things make that overlap real on a B200:

* the persistent GEMM grids hold every SM they are given for the whole
  kernel, so a collective queued behind them waits for the next kernel
  boundary.  ``sm_reserve`` SMs are kept out of the GEMM grids (their
  ``max_ctas``), and ``nccl_options`` caps NCCL to that many CTAs on a
  high-priority stream, so the reduce-scatter runs beside the next chunk's
  kernels;
* the residual is added in the down kernel's epilogue, by the owning rank
  only (``residual_rows`` = its rows of the chunk), so the reduce-scatter
  delivers finished rows and no pass over them follows.

The reference has no multi-GPU code; this follows the partitioning its
scaling plan asks for.
"""

from __future__ import annotations

import ctypes as C
import os
from typing import List, Optional, Tuple

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


def nccl_options(max_ctas: Optional[int] = None, high_priority: bool = True):
    """Process-group options for ``init_process_group("nccl", pg_options=...)``
    that let the reduce-scatter run beside the GEMM kernels: NCCL on a
    high-priority stream, and at most ``max_ctas`` CTAs per collective (the SMs
    the sharded forward leaves free; None keeps NCCL's own choice)."""
    import torch.distributed as dist
    opts = dist.ProcessGroupNCCL.Options(is_high_priority_stream=high_priority)
    if max_ctas:
        opts.config.max_ctas = int(max_ctas)
        opts.config.min_ctas = min(int(max_ctas), 4)
    return opts


def default_sm_reserve(world: int = 2, exchange: str = "nccl") -> int:
    """SMs kept out of the GEMM grids while collectives run (BELL_SM_RESERVE
    overrides).  NCCL reduce-scatter, measured at config 5 on B200s: 16 was
    best at 2 ranks (of 0 / 16), 24 at 8 ranks (of 0 / 16 / 24 / 32), where
    each rank sends 7/8 of its partial instead of 1/2.  The copy exchange
    moves data on the copy engines and only needs room for its barrier's
    one-CTA all-reduce."""
    env = os.environ.get("BELL_SM_RESERVE")
    if env is not None:
        return int(env)
    if exchange == "copy":
        return 4
    return 16 if world <= 2 else 24


_IPC_MAPPED = {}  # (device, allocation handle) -> base of its mapping in this process


def _ipc_map(handle: bytes, dev) -> int:
    """Base address in this process of another process's allocation, mapped
    into ``dev``'s context once (a second inbox in the same allocation reuses
    the mapping)."""
    key = (dev.index, handle)
    base = _IPC_MAPPED.get(key)
    if base is None:
        from .kernels import _lib
        p, b = C.c_void_p(), C.c_void_p()
        with torch.cuda.device(dev):
            _lib.check(_lib.load().bell_ipc_open((C.c_uint8 * 64).from_buffer_copy(handle), 0, C.byref(p),
                                                 C.byref(b)), "ShardedSwiGLU inbox")
        base = int(b.value)
        _IPC_MAPPED[key] = base
    return base


def close_ipc_mappings() -> None:
    """Unmap every peer inbox this process mapped for the copy exchange.  Call
    it after the last ``forward`` of every ``ShardedSwiGLU`` that used
    ``exchange="copy"`` (the mappings otherwise live until the process ends)."""
    from .kernels import _lib
    lib = _lib.load() if _IPC_MAPPED else None
    for (dev_index, _), base in list(_IPC_MAPPED.items()):
        with torch.cuda.device(dev_index):
            _lib.check(lib.bell_ipc_close(C.c_void_p(base)), "close_ipc_mappings")
    _IPC_MAPPED.clear()


def default_exchange() -> str:
    """How the sharded forward sums the partials: ``"nccl"`` (reduce-scatter)
    or ``"copy"`` (copy engines + owner-side sum).  BELL_EXCHANGE overrides."""
    return os.environ.get("BELL_EXCHANGE", "nccl")


def pick_chunks(T: int, world: int, want: int = 4) -> int:
    c = want
    while c > 1 and (T % c or (T // c) % world or (T // c // world) % 128):
        c -= 1
    return max(c, 1)


class ShardedSwiGLU:
    """This rank's share of a d_ff-split SwiGLU forward (bf16)."""

    def __init__(self, vg, cg, vu, cu, vd, cd, rank: int, world: int, chunks: int = 8, group=None,
                 sm_reserve: Optional[int] = None, exchange: Optional[str] = None):
        R_f = vg.shape[0]
        self.B = vg.shape[2]
        self.rank, self.world, self.group = rank, world, group
        self.lo, self.hi = shard_ranges(R_f, world)[rank]
        self.vg, self.cg = vg[self.lo:self.hi].contiguous(), cg[self.lo:self.hi].contiguous()
        self.vu, self.cu = vu[self.lo:self.hi].contiguous(), cu[self.lo:self.hi].contiguous()
        self.vd, self.cd = repack_down(vd, cd, self.lo, self.hi)
        self.d_model = vd.shape[0] * self.B
        self.want_chunks = chunks
        self.exchange = default_exchange() if exchange is None else exchange
        if self.exchange not in ("nccl", "copy"):
            raise ValueError(f"ShardedSwiGLU: exchange must be 'nccl' or 'copy', not {self.exchange!r}")
        self.sm_reserve = default_sm_reserve(world, self.exchange) if sm_reserve is None else int(sm_reserve)
        self._bufs = {}

    def grid_cap(self, dev) -> int:
        """``max_ctas`` of this rank's GEMM launches (0 = every SM)."""
        if self.world == 1 or self.sm_reserve <= 0:
            return 0
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        return max(1, sms - self.sm_reserve)

    def _chunking(self, T: int) -> Tuple[int, int, int]:
        """(chunks, tokens per chunk, rows per rank per chunk) for T tokens.
        Every rank must own the same number of rows of every chunk, so T has
        to be a multiple of the world size; anything else would drop rows."""
        n = pick_chunks(T, self.world, self.want_chunks)
        if T % n or (T // n) % self.world:
            raise ValueError(f"ShardedSwiGLU: T={T} tokens cannot be split evenly over {self.world} ranks; "
                             f"pad the batch to a multiple of {self.world}")
        return n, T // n, T // n // self.world

    def launches_per_step(self, T: int) -> int:
        # per chunk: plan + gate/up, plan + down, and with the copy exchange the owner-side sum
        # (NCCL's kernels and the copies are not counted)
        per_chunk = 5 if self.exchange == "copy" and self.world > 1 else 4
        return per_chunk * pick_chunks(T, self.world, self.want_chunks)

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
        if self.exchange == "copy" and self.world > 1:
            return self.forward_copy(x, out, add_residual)
        from .kernels.ops import block_ell_gate_up, block_ell_linear
        T = x.shape[0]
        _, Tc, per = self._chunking(T)
        h = self._buf("h", (Tc, (self.hi - self.lo) * self.B), torch.bfloat16, x.device)
        cap = self.grid_cap(x.device)
        own = (self.rank * per, (self.rank + 1) * per)  # this rank's rows of every chunk
        fold = add_residual and self._can_fold(per)

        def partial_fn(xi: torch.Tensor, dst: torch.Tensor) -> None:
            block_ell_gate_up(xi, self.vg, self.cg, self.vu, self.cu, self.vd, self.cd, h=h, max_ctas=cap)
            # the residual goes into this rank's own rows only, so the sum over ranks adds it once
            block_ell_linear(h, self.vd, self.cd, out=dst, residual=xi if fold else None,
                             residual_rows=own if fold else None, max_ctas=cap)

        return self.run_chunks(x, partial_fn, out, add_residual=add_residual and not fold)

    def _inbox(self, per: int, dev):
        """This rank's inbox ``[2, N, per, d_model]`` bf16 (chunk parity, source
        rank, row, column) and the address of every rank's inbox in this
        process: CUDA IPC handles are exchanged once through the process group
        and mapped into this rank's own device context (``bell_ipc_open``), so
        copies into a peer's inbox run device to device over NVLink."""
        key = ("inbox", per, dev.index)
        got = self._bufs.get(key)
        if got is None:
            import torch.distributed as dist
            from .kernels import _lib
            lib = _lib.load()
            box = torch.empty((2, self.world, per, self.d_model), dtype=torch.bfloat16, device=dev)
            h, off = (C.c_uint8 * 64)(), C.c_uint64(0)
            with torch.cuda.device(dev):
                _lib.check(lib.bell_ipc_handle(C.c_void_p(box.data_ptr()), h, C.byref(off)), "ShardedSwiGLU inbox")
            handles = [None] * self.world
            dist.all_gather_object(handles, (bytes(h), int(off.value)), group=self.group)
            ptrs = []
            for r, (hb, o) in enumerate(handles):
                ptrs.append(box.data_ptr() if r == self.rank else _ipc_map(hb, dev) + o)
            got = (box, ptrs)
            self._bufs[key] = got
        return got

    def forward_copy(self, x: torch.Tensor, out: torch.Tensor = None, add_residual: bool = True) -> torch.Tensor:
        """``forward`` with the exchange on the copy engines instead of an NCCL
        reduce-scatter.  For chunk i (partials and inbox halves alternate):

        * compute stream: gate/up(i), then the owner-side sum of chunk i-2,
          then down(i) into this rank's partial [Tc, d] (all tokens of the
          chunk, this rank's d_ff share);
        * copy stream: one ``cudaMemcpyAsync`` per peer moves the peer's rows
          of partial(i) into the peer's inbox slot for this rank (ranks send in
          rotation, r -> r+1, r+2, ..., so each inbox takes one stream at a
          time); one chunk later a one-element all-reduce (barrier i) marks
          that every rank's copies of chunk i have landed and every rank's sum
          of chunk i-1 is done, so chunk i+1 may refill that inbox half;
        * the sum (``bell_sum_slices_bf16``, every SM) adds the N slices, this
          rank's own from its partial, and the residual, in rank order.

        Lagging the sum two chunks behind lets each chunk's copies run beside
        the next chunk and a half of GEMMs; the GEMMs leave only ``sm_reserve``
        SMs for the barrier's NCCL kernel."""
        import torch.distributed as dist
        from .kernels import _lib
        from .kernels.ops import block_ell_gate_up, block_ell_linear, sum_slices
        T = x.shape[0]
        n, Tc, per = self._chunking(T)
        dev = x.device
        d = self.d_model
        if out is None:
            out = torch.empty((T // self.world, d), dtype=torch.bfloat16, device=dev)
        box, peers = self._inbox(per, dev)
        slot_bytes = per * d * 2  # one (half, source) slot of an inbox
        h = self._buf("h", (Tc, (self.hi - self.lo) * self.B), torch.bfloat16, dev)
        partial = [self._buf(f"p{i}", (Tc, d), torch.bfloat16, dev) for i in range(2)]
        flag = self._buf("flag", (1,), torch.float32, dev)
        cap = self.grid_cap(dev)
        lib = _lib.load()
        cur = torch.cuda.current_stream(dev)
        s_cp = self._stream("copy", dev)
        s_cp.wait_stream(cur)  # the inbox and partials' previous users are done
        ev = {k: [torch.cuda.Event() for _ in range(n)] for k in ("down", "bar", "sum")}
        order = [(self.rank + k) % self.world for k in range(1, self.world)]
        me = slice(self.rank * per, (self.rank + 1) * per)

        def enq_sum(j):  # compute stream
            cur.wait_event(ev["bar"][j])
            xj = x[j * Tc:(j + 1) * Tc]
            sum_slices(box[j % 2], out[j * per:(j + 1) * per], local=partial[j % 2][me], local_slot=self.rank,
                       residual=xj[me] if add_residual else None)
            ev["sum"][j].record(cur)

        def enq_barrier(j):  # copy stream: copies(j) landed everywhere, sum(j-1) done everywhere
            with torch.cuda.stream(s_cp):
                if j >= 1:
                    s_cp.wait_event(ev["sum"][j - 1])
                dist.all_reduce(flag, group=self.group)
                ev["bar"][j].record(s_cp)

        st = C.c_void_p(s_cp.cuda_stream)
        for i in range(n):
            P = partial[i % 2]
            block_ell_gate_up(x[i * Tc:(i + 1) * Tc], self.vg, self.cg, self.vu, self.cu, self.vd, self.cd, h=h,
                              max_ctas=cap)
            if i >= 2:
                enq_sum(i - 2)  # also the last reader of P before down(i) overwrites it
            if i >= 1:
                enq_barrier(i - 1)
            block_ell_linear(h, self.vd, self.cd, out=P, max_ctas=cap)
            ev["down"][i].record(cur)
            s_cp.wait_event(ev["down"][i])
            for o in order:  # after barrier i-1: every rank's sum of chunk i-2 has read this inbox half
                dst = peers[o] + ((i % 2) * self.world + self.rank) * slot_bytes
                _lib.check(lib.bell_memcpy_async(C.c_void_p(dst), C.c_void_p(P[o * per:(o + 1) * per].data_ptr()),
                                                 slot_bytes, st), "forward_copy")
        if n >= 2:
            enq_sum(n - 2)
        enq_barrier(n - 1)
        enq_sum(n - 1)
        with torch.cuda.stream(s_cp):  # every rank's sums are done before any rank refills an inbox
            s_cp.wait_event(ev["sum"][n - 1])
            dist.all_reduce(flag, group=self.group)
        cur.wait_stream(s_cp)
        return out

    def _can_fold(self, per: int) -> bool:
        """Whether the down kernel can add the residual to this rank's rows: at
        tile size 128 its work units are 256-token tiles, so the rows must
        start on such a tile."""
        return self.B != 128 or per % 256 == 0

    def forward_host(self, x_own: torch.Tensor, out_host: torch.Tensor = None, add_residual: bool = True,
                     device=None) -> torch.Tensor:
        """Host-buffer forward with token-sliced input and output.

        ``x_own`` is this rank's token rows of x (``owned_rows`` order, bf16,
        pinned host memory), ``[T / N, d_model]``; the result is the same rows of
        the full forward, written to ``out_host`` (pinned, allocated when None).
        Every rank needs all tokens for its d_ff shard, but only its own 1/N
        crosses its host link: per chunk, the slice is copied in on a copy
        stream, NCCL all-gathers the chunk over NVLink, the partial forward and
        reduce-scatter run as in ``forward``, and a third stream adds the
        residual to the chunk's reduced rows and copies them out once that
        chunk's reduce-scatter is done, while later chunks compute.  The
        all-gather of chunk i+1 is issued from the copy stream before chunk i
        computes, so it overlaps that compute.  Returns after the copies out
        have finished."""
        import torch.distributed as dist
        from .kernels.ops import block_ell_gate_up, block_ell_linear
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        T = x_own.shape[0] * self.world
        n, Tc, per = self._chunking(T)
        d = self.d_model
        if out_host is None:
            out_host = torch.empty((T // self.world, d), dtype=torch.bfloat16).pin_memory()
        xs = self._buf("xs", (T // self.world, d), torch.bfloat16, dev)
        out = self._buf("out_own", (T // self.world, d), torch.bfloat16, dev)
        xfull = [self._buf(f"xf{i}", (Tc, d), torch.bfloat16, dev) for i in range(2)]
        partial = [self._buf(f"p{i}", (Tc, d), torch.bfloat16, dev) for i in range(2)]
        h = self._buf("h", (Tc, (self.hi - self.lo) * self.B), torch.bfloat16, dev)
        cap = self.grid_cap(dev)
        own = (self.rank * per, (self.rank + 1) * per)
        fold = add_residual and self._can_fold(per)
        cur = torch.cuda.current_stream(dev)
        s_in = self._stream("in", dev)
        s_out = self._stream("out", dev)
        s_in.wait_stream(cur)  # the buffers' previous users are done
        s_out.wait_stream(cur)
        done = [None] * n  # compute of chunk i finished with xfull[i % 2]

        def gather(i):
            # issued from s_in, so NCCL waits for the slice's copy in (and for the
            # compute that last read xfull[i % 2]), not for the compute stream
            with torch.cuda.stream(s_in):
                xs[i * per:(i + 1) * per].copy_(x_own[i * per:(i + 1) * per], non_blocking=True)
                if i >= 2:
                    s_in.wait_event(done[i - 2])
                return dist.all_gather_into_tensor(xfull[i % 2], xs[i * per:(i + 1) * per], group=self.group,
                                                   async_op=True)

        works = []
        g_next = gather(0)
        for i in range(n):
            g_cur = g_next
            if i + 1 < n:
                g_next = gather(i + 1)  # overlaps this chunk's compute
            g_cur.wait()
            if i >= 2:
                works[i - 2].wait()  # partial buffer i%2 is free again
            block_ell_gate_up(xfull[i % 2], self.vg, self.cg, self.vu, self.cu, self.vd, self.cd, h=h, max_ctas=cap)
            block_ell_linear(h, self.vd, self.cd, out=partial[i % 2], residual=xfull[i % 2] if fold else None,
                             residual_rows=own if fold else None, max_ctas=cap)
            done[i] = torch.cuda.Event()
            done[i].record(cur)
            works.append(dist.reduce_scatter_tensor(out[i * per:(i + 1) * per], partial[i % 2],
                                                    op=dist.ReduceOp.SUM, group=self.group, async_op=True))
            with torch.cuda.stream(s_out):
                works[i].wait()  # s_out waits for this chunk's reduce-scatter
                if add_residual and not fold:
                    out[i * per:(i + 1) * per].add_(xs[i * per:(i + 1) * per])
                out_host[i * per:(i + 1) * per].copy_(out[i * per:(i + 1) * per], non_blocking=True)
        for w in works:
            w.wait()
        cur.wait_stream(s_out)
        s_out.synchronize()
        return out_host

    def _stream(self, name, dev):
        key = ("stream", name, dev.index)
        st = self._bufs.get(key)
        if st is None:
            st = torch.cuda.Stream(device=dev)
            self._bufs[key] = st
        return st

    def run_chunks(self, x: torch.Tensor, partial_fn, out: torch.Tensor = None, add_residual: bool = False,
                   dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
        """The chunk pipeline of ``forward`` around any partial computation:
        ``partial_fn(x_chunk, dst)`` writes this rank's partial ``[Tc, d_model]``
        for a token chunk; the reduce-scatter of chunk i runs (async) while
        chunk i+1 computes and two partial buffers alternate.  ``add_residual``
        adds x on the owned rows at the end, for a ``partial_fn`` that leaves
        the residual out."""
        import torch.distributed as dist
        T = x.shape[0]
        n, Tc, per = self._chunking(T)
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
