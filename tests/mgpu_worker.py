"""torchrun worker for tests/test_gpu_multi.py: the d_ff-sharded forward on N
GPUs, with the NCCL reduce-scatter and with the copy-engine exchange.  Every
rank checks a sample of the token rows it owns against the CPU oracle (fp64
on the same bf16 inputs, rel-L2 <= 1e-2) through the device-buffer forward
of each exchange, checks that the token-sliced host-buffer forward gives the
NCCL forward's bits, and that a second copy-exchange call (reused inboxes)
repeats the first bit for bit.  Exit code 0 = pass."""

import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [ROOT, os.path.join(ROOT, "looped-blockell-tpu_b200")]

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
    import numpy as np
    import oracle as O
    from looped_blockell.dist import ShardedSwiGLU, owned_rows, pick_chunks
    from looped_blockell.synth import Config, make_ffn
    ok = True
    T_b128 = 4096 if world <= 4 else 8192  # each rank's share of every chunk stays a multiple of 128 rows
    for cfg in (Config("mg_b128", T=T_b128, d_model=1024, d_ff=4096, B=128, density=0.25, dtype="bf16", seed=7),
                Config("mg_b64", T=2048 * max(1, world // 4), d_model=512, d_ff=2048, B=64, density=0.5,
                       dtype="bf16", seed=8)):
        c = make_ffn(cfg, device="cuda")  # same seed on every rank -> same weights and x
        model = ShardedSwiGLU(c["vg"], c["cg"], c["vu"], c["cu"], c["vd"], c["cd"], rank, world)
        out = model.forward(c["x"])
        torch.cuda.synchronize()
        rows = owned_rows(cfg.T, rank, world, pick_chunks(cfg.T, world, model.want_chunks))
        pick = np.sort(np.random.default_rng(rank).choice(rows.numel(), min(256, rows.numel()), replace=False))
        tok = rows[torch.from_numpy(pick)].cuda()
        f = lambda t: t.float().cpu().numpy().astype(np.float64)  # noqa: E731
        w = [(f(c[v]), c[cc].cpu().numpy(), 0) for v, cc in (("vg", "cg"), ("vu", "cu"), ("vd", "cd"))]
        ref = O.swiglu_ffn(f(c["x"].index_select(0, tok)), *w, add_residual=True)
        got = f(out.index_select(0, torch.from_numpy(pick).cuda()))
        err = O.rel_l2(got, ref)
        print(f"rank {rank}/{world} {cfg.name}: rel-L2 vs oracle on {pick.size} owned rows {err:.3e}", flush=True)
        ok &= err < 1e-2
        # copy-engine exchange: same rows, owner-side sum in rank order
        mc = ShardedSwiGLU(c["vg"], c["cg"], c["vu"], c["cu"], c["vd"], c["cd"], rank, world, exchange="copy")
        outs = [mc.forward(c["x"]) for _ in range(2)]
        torch.cuda.synchronize()
        err_c = O.rel_l2(f(outs[0].index_select(0, torch.from_numpy(pick).cuda())), ref)
        rep = torch.equal(outs[0], outs[1])
        print(f"rank {rank}/{world} {cfg.name}: copy exchange rel-L2 vs oracle {err_c:.3e}, "
              f"second call bit-identical: {rep}", flush=True)
        ok &= err_c < 1e-2 and rep
        # host-buffer entry: this rank's token rows in, the same rows of the result out
        x_own = c["x"].index_select(0, rows.cuda()).cpu().pin_memory()
        for _ in range(2):  # twice: the second call reuses the cached buffers and streams
            out_h = model.forward_host(x_own)
            same = torch.equal(out_h, out.cpu())
            print(f"rank {rank}/{world} {cfg.name}: forward_host bit-identical to forward: {same}", flush=True)
            ok &= same
    t = torch.tensor([0 if ok else 1], device="cuda")
    dist.all_reduce(t)
    dist.barrier()
    from looped_blockell.dist import close_ipc_mappings
    torch.cuda.synchronize()
    close_ipc_mappings()
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(int(t.item() != 0))


if __name__ == "__main__":
    main()
