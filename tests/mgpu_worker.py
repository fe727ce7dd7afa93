"""torchrun worker for tests/test_gpu_multi.py: the d_ff-sharded forward on N
GPUs (NCCL reduce-scatter) against the single-GPU fused forward computed on
each rank; every rank checks the token rows it owns, through the device-buffer
forward and the token-sliced host-buffer forward.  Exit code 0 = pass."""

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
    from looped_blockell.dist import ShardedSwiGLU, owned_rows, pick_chunks
    from looped_blockell.kernels import block_ell_swiglu_fwd
    from looped_blockell.synth import Config, make_ffn
    ok = True
    for cfg in (Config("mg_b128", T=4096, d_model=1024, d_ff=4096, B=128, density=0.25, dtype="bf16", seed=7),
                Config("mg_b64", T=2048, d_model=512, d_ff=2048, B=64, density=0.5, dtype="bf16", seed=8)):
        c = make_ffn(cfg, device="cuda")  # same seed on every rank -> same weights and x
        ref = block_ell_swiglu_fwd(c["x"], c["vg"], c["cg"], c["vu"], c["cu"], c["vd"], c["cd"], add_residual=True)
        model = ShardedSwiGLU(c["vg"], c["cg"], c["vu"], c["cu"], c["vd"], c["cd"], rank, world)
        out = model.forward(c["x"])
        torch.cuda.synchronize()
        rows = owned_rows(cfg.T, rank, world, pick_chunks(cfg.T, world, model.want_chunks)).cuda()
        r = ref.index_select(0, rows).float()
        err = float((out.float() - r).norm() / r.norm())
        print(f"rank {rank} {cfg.name}: rel-L2 vs single GPU {err:.3e}", flush=True)
        ok &= err < 1e-2
        # host-buffer entry: this rank's token rows in, the same rows of the result out
        x_own = c["x"].index_select(0, rows).cpu().pin_memory()
        for _ in range(2):  # twice: the second call reuses the cached buffers and streams
            out_h = model.forward_host(x_own)
            same = torch.equal(out_h, out.cpu())
            err_h = float((out_h.float() - r.cpu()).norm() / r.cpu().norm())
            print(f"rank {rank} {cfg.name}: forward_host rel-L2 vs single GPU {err_h:.3e}, "
                  f"bit-identical to forward: {same}", flush=True)
            ok &= err_h < 1e-2
    t = torch.tensor([0 if ok else 1], device="cuda")
    dist.all_reduce(t)
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(int(t.item() != 0))


if __name__ == "__main__":
    main()
