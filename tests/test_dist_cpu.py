"""Host-side logic of the d_ff-sharded forward, on CPU: shard ranges, down-ELL
repacking, token ownership after the chunked reduce-scatter, a world_size-2
gloo run where each rank computes its partial with the oracle and the ranks
sum them (all_reduce + the ownership map), and the chunked reduce-scatter
pipeline itself (``ShardedSwiGLU.run_chunks``) on gloo at world sizes 2 and 4
with oracle partials."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
from looped_blockell.dist import owned_rows, pick_chunks, repack_down, shard_ranges


def test_shard_ranges_cover_rows():
    for R, W in [(128, 8), (130, 8), (7, 2), (3, 4)]:
        rs = shard_ranges(R, W)
        assert rs[0][0] == 0 and rs[-1][1] == R
        assert all(a[1] == b[0] for a, b in zip(rs, rs[1:]))
        assert max(h - l for l, h in rs) - min(h - l for l, h in rs) <= 1


def _case(seed=0, T=40, d=256, F=1024, B=64, K=2, Kd=6):
    rng = np.random.default_rng(seed)
    Rf, Cd, Rd, Cf = F // B, d // B, d // B, F // B
    cols = lambda R, C, K: np.stack([np.sort(rng.choice(C, K, replace=False)) for _ in range(R)]).astype(np.int32)  # noqa: E731
    return dict(x=rng.standard_normal((T, d)), vg=rng.standard_normal((Rf, K, B, B)) * 0.02, cg=cols(Rf, Cd, K),
                vu=rng.standard_normal((Rf, K, B, B)) * 0.02, cu=cols(Rf, Cd, K),
                vd=rng.standard_normal((Rd, Kd, B, B)) * 0.02, cd=cols(Rd, Cf, Kd), B=B)


def _partial(c, lo, hi):
    B = c["B"]
    vd, cd = repack_down(torch.from_numpy(c["vd"]), torch.from_numpy(c["cd"]), lo, hi)
    g = O.block_ell_matmul(c["x"], c["vg"][lo:hi], c["cg"][lo:hi])
    u = O.block_ell_matmul(c["x"], c["vu"][lo:hi], c["cu"][lo:hi])
    h = O.silu(g) * u
    assert h.shape[1] == (hi - lo) * B
    return O.block_ell_matmul(h, vd.numpy(), cd.numpy())


@pytest.mark.parametrize("world", [2, 3, 4])
def test_partials_sum_to_full_output(world):
    c = _case(seed=world)
    full = O.swiglu_ffn(c["x"], (c["vg"], c["cg"], 0), (c["vu"], c["cu"], 0), (c["vd"], c["cd"], 0))
    total = sum(_partial(c, lo, hi) for lo, hi in shard_ranges(c["vg"].shape[0], world))
    assert O.rel_l2(total, full) < 1e-12


def test_repack_down_pads_and_rebases():
    cd = torch.tensor([[0, 5, 9], [1, 2, 3]], dtype=torch.int32)
    vd = torch.arange(2 * 3, dtype=torch.float32).reshape(2, 3, 1, 1).expand(2, 3, 2, 2).contiguous()
    v, c = repack_down(vd, cd, 4, 10)
    assert c.shape == (2, 2) and c[0].tolist() == [1, 5] and c[1].tolist() == [-1, -1]
    assert torch.all(v[1] == 0) and v[0, 0, 0, 0] == vd[0, 1, 0, 0]


def test_owned_rows_partition_tokens():
    T, W = 4096, 4
    n = pick_chunks(T, W, 4)
    allr = torch.cat([owned_rows(T, r, W, n) for r in range(W)])
    assert torch.equal(torch.sort(allr).values, torch.arange(T))


def _worker(rank, world, port, c, full, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    lo, hi = shard_ranges(c["vg"].shape[0], world)[rank]
    part = torch.from_numpy(_partial(c, lo, hi))
    dist.all_reduce(part)
    T = c["x"].shape[0]
    rows = owned_rows(T, rank, world, 1)
    mine = part[rows].numpy() + c["x"][rows.numpy()]
    q.put((rank, O.rel_l2(mine, full[rows.numpy()])))
    dist.destroy_process_group()


def test_gloo_two_ranks_reconstruct_output():
    c = _case(seed=11, T=64)
    full = O.swiglu_ffn(c["x"], (c["vg"], c["cg"], 0), (c["vu"], c["cu"], 0), (c["vd"], c["cd"], 0),
                        add_residual=True)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, c, full, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(err < 1e-12 for _, err in res), res


def _chunk_worker(rank, world, port, c, full, q):
    """The chunked reduce-scatter pipeline of ShardedSwiGLU (run_chunks) on
    gloo, with this rank's partials from the oracle."""
    from looped_blockell.dist import ShardedSwiGLU
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    t = {k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in c.items() if k != "B"}
    model = ShardedSwiGLU(t["vg"], t["cg"], t["vu"], t["cu"], t["vd"], t["cd"], rank, world, chunks=4)
    cl = {k: v for k, v in c.items()}
    lo, hi = model.lo, model.hi

    def partial_fn(xi, dst):
        sub = dict(cl, x=xi.numpy())
        dst.copy_(torch.from_numpy(_partial(sub, lo, hi)))

    x = torch.from_numpy(c["x"])
    n = pick_chunks(x.shape[0], world, 4)
    per = x.shape[0] // n // world

    def partial_fn_own_residual(xi, dst):
        # the down kernel's form: the residual enters this rank's own rows of the chunk only
        partial_fn(xi, dst)
        dst[rank * per:(rank + 1) * per] += xi[rank * per:(rank + 1) * per]

    out = model.run_chunks(x, partial_fn, dtype=torch.float64, add_residual=True)
    out_fold = model.run_chunks(x, partial_fn_own_residual, dtype=torch.float64)
    rows = owned_rows(x.shape[0], rank, world, n)
    err = max(O.rel_l2(out.numpy(), full[rows.numpy()]), O.rel_l2(out_fold.numpy(), full[rows.numpy()]))
    q.put((rank, n, err))
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_gloo_chunked_reduce_scatter_reconstructs_output(world):
    c = _case(seed=21 + world, T=4 * world * 128)
    full = O.swiglu_ffn(c["x"], (c["vg"], c["cg"], 0), (c["vu"], c["cu"], 0), (c["vd"], c["cd"], 0),
                        add_residual=True)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_chunk_worker, args=(r, world, port, c, full, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(n == 4 for _, n, _ in res), res
    assert all(err < 1e-12 for _, _, err in res), res


@pytest.mark.parametrize("T", [10, 4097])
def test_uneven_token_count_is_refused(T):
    """A token count that does not split evenly over the ranks is refused
    before any work (it would otherwise drop the leftover rows)."""
    from looped_blockell.dist import ShardedSwiGLU
    rng = np.random.default_rng(0)
    R, C, K, B = 4, 2, 2, 64
    v = torch.from_numpy(rng.standard_normal((R, K, B, B)).astype(np.float32)).to(torch.bfloat16)
    cols = torch.tensor([[0, 1]] * R, dtype=torch.int32)
    vd = torch.from_numpy(rng.standard_normal((C, K, B, B)).astype(np.float32)).to(torch.bfloat16)
    cd = torch.tensor([[0, 3], [1, 2]], dtype=torch.int32)
    model = ShardedSwiGLU(v, cols, v, cols, vd, cd, rank=0, world=4)
    with pytest.raises(ValueError, match="cannot be split evenly"):
        model.forward(torch.zeros((T, C * B), dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="cannot be split evenly"):
        model._chunking(T)


def _tiny_model(**kw):
    from looped_blockell.dist import ShardedSwiGLU
    rng = np.random.default_rng(1)
    R, C, K, B = 4, 2, 2, 64
    v = torch.from_numpy(rng.standard_normal((R, K, B, B)).astype(np.float32)).to(torch.bfloat16)
    cols = torch.tensor([[0, 1]] * R, dtype=torch.int32)
    vd = torch.from_numpy(rng.standard_normal((C, K, B, B)).astype(np.float32)).to(torch.bfloat16)
    cd = torch.tensor([[0, 3], [1, 2]], dtype=torch.int32)
    return ShardedSwiGLU(v, cols, v, cols, vd, cd, **kw)


def test_exchange_choice_and_defaults(monkeypatch):
    """The exchange is validated; each exchange gets its own SM-reserve
    default (the NCCL one grows with the rank count), and the environment
    overrides both."""
    from looped_blockell.dist import default_exchange, default_sm_reserve
    monkeypatch.delenv("BELL_SM_RESERVE", raising=False)
    monkeypatch.delenv("BELL_EXCHANGE", raising=False)
    assert default_exchange() == "nccl"
    assert default_sm_reserve(2) == 16 and default_sm_reserve(8) == 24
    assert default_sm_reserve(8, "copy") == 4
    assert _tiny_model(rank=0, world=8).sm_reserve == 24
    assert _tiny_model(rank=0, world=8, exchange="copy").sm_reserve == 4
    monkeypatch.setenv("BELL_EXCHANGE", "copy")
    monkeypatch.setenv("BELL_SM_RESERVE", "12")
    m = _tiny_model(rank=1, world=2)
    assert m.exchange == "copy" and m.sm_reserve == 12
    with pytest.raises(ValueError, match="exchange must be"):
        _tiny_model(rank=0, world=2, exchange="ring")


def test_launch_count_per_exchange():
    """Per chunk: plan + gate/up and plan + down, plus the owner-side sum with
    the copy exchange (NCCL's kernels and the copies are not this library's
    launches); one rank runs no exchange at all."""
    from looped_blockell.dist import pick_chunks
    T = 8 * 4 * 256
    n = pick_chunks(T, 4, 8)
    assert _tiny_model(rank=0, world=4).launches_per_step(T) == 4 * n
    assert _tiny_model(rank=0, world=4, exchange="copy").launches_per_step(T) == 5 * n
    assert _tiny_model(rank=0, world=1, exchange="copy").launches_per_step(T) == 4 * pick_chunks(T, 1, 8)
