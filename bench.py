"""Benchmark: Block-ELL SwiGLU forward on B200 (BASELINE config 5 by default).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 5]

One step = one bf16 Block-ELL SwiGLU forward (gate/up + SiLU*up + down +
residual) over the config's T tokens, inputs resident in HBM (x alone is
2 GiB for config 5, larger than the 126 MB L2, so no flush is needed).  N>1
splits the d_ff block-rows across ranks with one NCCL reduce-scatter of the
down-projection partials (strong scaling: the job size is fixed).
Rank 0 prints one JSON line.  ``--impl reference`` times the CPU restatement
of the reference path (oracle/) on the host cores instead.

``--direction bwd`` times the backward of the same FFN instead (one GPU):
one step = titan::block_ell_swiglu_bwd's work — [d_gate | d_up] (at tile
size 64 the down projection fused with the SiLU*up backward, at 128 the two
as separate launches), d_x (+ grad_out), and the three
tile-gradient products — from saved forward intermediates; FLOPs per step are
twice the forward's.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.join(ROOT, "looped-blockell-tpu_b200")
for _p in (ROOT, PKG_ROOT):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "Block-ELL SwiGLU tokens/s & effective TFLOP/s per B200 (1/2/4/8 GPU) vs roofline"


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), float(p["bf16_tflops_sustained"]), "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


class ClockSampler:
    """SM clock and clock-event (throttle) reasons of this rank's GPU, polled
    through NVML (read-only) every 20 ms during the timed region."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4}

    def __init__(self, uuid: str):
        self.uuid, self.samples, self.mask, self.max_mhz, self.err = uuid, [], 0, None, None
        self._stop = threading.Event()

    def _poll(self):
        import pynvml
        try:
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByUUID(self.uuid.encode() if isinstance(self.uuid, str) else self.uuid)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            while not self._stop.is_set():
                self.samples.append(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                self.mask |= pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                time.sleep(0.02)
        except Exception as e:  # sampling is best effort; reported in the JSON
            self.err = repr(e)

    def __enter__(self):
        self.t = threading.Thread(target=self._poll, daemon=True)
        self.t.start()
        time.sleep(0.05)
        return self

    def __exit__(self, *a):
        self._stop.set()
        self.t.join(timeout=5)

    def summary(self):
        out = {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
               "reasons": sorted(n for n, b in self.REASONS.items() if self.mask & b),
               "samples": len(self.samples)}
        if self.err:
            out["error"] = self.err
        return out


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one gate/up launch, from ncu captures
# of the same command on a B200.  Config 5 is captured at T=32768 (x 256 MiB) and scaled by the
# units of a full launch (x8): the kernel walks the same unit order, so traffic grows in proportion.
GU_DRAM_BYTES = {(5, 262144): 8 * (2.390204e9 + 1.065839e9), (2, 32768): 1.42730e8 + 4.82981e8}
GU_DRAM_NOTE = {5: "ncu dram__bytes_{read,write}.sum at T=32768, scaled x8 by units",
                2: "ncu dram__bytes_{read,write}.sum on the full config-2 launch"}


def algorithmic_hbm_bytes(cfg, T: int) -> float:
    """HBM bytes one forward must move (bf16): x read, h written and read
    back, residual read, out written, weights read once; times L for the loop."""
    d, F, B = cfg.d_model, cfg.d_ff, cfg.B
    w = 2.0 * B * B * (2 * (F // B) * cfg.K_gu + (d // B) * cfg.K_d)
    return (2.0 * T * d + 4.0 * T * F + 2.0 * T * d + 2.0 * T * d + w) * cfg.L


def hbm_line(cfg, T, ms, world, hbm_peak, peak_src):
    if cfg.dtype != "bf16":
        return None
    achieved = algorithmic_hbm_bytes(cfg, T) / (ms / 1e3) / 1e9 / world  # per GPU
    return {"achieved": achieved, "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak,
            "peak_source": f"{peak_src} copy bandwidth", "note": "algorithmic bytes of the whole step per GPU"}


def cpu_baseline_sample(cfg, tokens: int, reps: int = 1):
    """Time the oracle (numpy restatement of the reference gather+GEMM path)
    on `tokens` tokens of `cfg` using every host core; returns tokens/s."""
    import numpy as np
    import oracle as O
    from looped_blockell.synth import make_ffn
    c = make_ffn(cfg, device="cpu", T=tokens)
    f = {k: (v.float().numpy() if not k.startswith("c") else v.numpy()) for k, v in c.items()}
    w = ((f["vg"], f["cg"], 0), (f["vu"], f["cu"], 0), (f["vd"], f["cd"], 0))
    O.swiglu_ffn(f["x"][:8], *w, dtype=np.float32)  # warm BLAS
    t0 = time.perf_counter()
    for _ in range(reps):
        if cfg.L > 1:  # the shared-weight loop: L x (RMSNorm -> SwiGLU -> residual)
            O.looped_ffn(f["x"], np.ones(cfg.d_model, np.float32), *w, L=cfg.L, dtype=np.float32)
        else:
            O.swiglu_ffn(f["x"], *w, add_residual=True, dtype=np.float32)
    dt = time.perf_counter() - t0
    return tokens * reps / dt, dt


def cpu_backward_sample(cfg, tokens: int):
    """Time the oracle's tile-by-tile backward (numpy, every host core) on
    `tokens` tokens of `cfg`; returns tokens/s."""
    import numpy as np
    import oracle as O
    from looped_blockell.synth import make_ffn
    c = make_ffn(cfg, device="cpu", T=tokens)
    f = {k: (v.float().numpy() if not k.startswith("c") else v.numpy()) for k, v in c.items()}
    w = ((f["vg"], f["cg"], 0), (f["vu"], f["cu"], 0), (f["vd"], f["cd"], 0))
    _, h, g, u = O.swiglu_ffn(f["x"], *w, dtype=np.float32, return_intermediates=True)
    dy = np.random.default_rng(1).standard_normal(f["x"].shape).astype(np.float32)
    t0 = time.perf_counter()
    O.swiglu_ffn_backward_sparse(f["x"], *w, dy, g, u, h, dtype=np.float32)
    dt = time.perf_counter() - t0
    return tokens / dt, dt


def run_reference(args, cfg, rank, world):
    """CPU arm: the oracle port of the reference path on all host threads."""
    if rank != 0:
        return
    import numpy as np  # noqa: F401
    cores = os.cpu_count()
    sample = args.ref_tokens
    vals = []
    bwd = args.direction == "bwd"
    fn = cpu_backward_sample if bwd else cpu_baseline_sample
    if bwd:
        sample = max(64, sample // 4)  # the backward does twice the work per token
    fn(cfg, max(8, sample // 4))  # warm-up (untimed)
    for _ in range(args.steps):
        v, _ = fn(cfg, sample)
        vals.append(v)
    value = statistics.median(vals)
    ms = cfg.T / value * 1e3
    line = {
        "impl": "reference", "metric": METRIC + (" (backward)" if bwd else ""), "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": cfg.name, "T": cfg.T, "d_model": cfg.d_model, "d_ff": cfg.d_ff, "B": cfg.B,
                   "density": cfg.density, "sample_tokens": sample, "direction": args.direction},
        "tflops_effective": (2 if bwd else 1) * cfg.nnz_flops() / (ms / 1e3) / 1e12,
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{sample} tokens of {cfg.name} per step, numpy "
                                   + ("tile-by-tile restatement of the reference backward "
                                      "(swiglu_ffn_backward_sparse)" if bwd else
                                      "gather+BLAS restatement of block_ell_matmul")
                                   + f" (oracle/bell_oracle.py), scaled linearly to T={cfg.T}"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", type=int, default=5)
    ap.add_argument("--shared-gate-up", action="store_true")
    ap.add_argument("--layout", default="in_out", choices=["in_out", "out_in"], help="weight tile layout")
    ap.add_argument("--tokens", type=int, default=0, help="override T (profiling on a smaller case)")
    ap.add_argument("--tile", type=int, default=0, help="override the tile size B (16, 32, 64, 128)")
    ap.add_argument("--ref-tokens", type=int, default=2048)
    ap.add_argument("--cpu-tokens", type=int, default=2048)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg (profiling runs)")
    ap.add_argument("--no-check", action="store_true",
                    help="skip the parity check of the last step's output against the CPU oracle")
    ap.add_argument("--check-rows", type=int, default=256, help="token rows per rank in the parity check")
    ap.add_argument("--sm-reserve", type=int, default=None,
                    help="N>1: SMs kept out of the GEMM grids for NCCL (default BELL_SM_RESERVE or 16)")
    ap.add_argument("--chunks", type=int, default=8, help="N>1: token chunks of the reduce-scatter pipeline")
    ap.add_argument("--exchange", choices=["nccl", "copy"], default=None,
                    help="N>1: sum the partials with an NCCL reduce-scatter or with copy engines + an owner-side "
                         "sum kernel (default: looped_blockell.dist.default_exchange)")
    ap.add_argument("--loop-mode", default="auto", choices=["auto", "launches", "persistent"],
                    help="config 4: the loop implementation")
    ap.add_argument("--l2-pin", action="store_true",
                    help="keep the gate/up weight tiles in a persisting-L2 window (bell_pin_l2) while timing")
    ap.add_argument("--nccl-max-ctas", type=int, default=None,
                    help="N>1: NCCL CTA cap (default: the SM reserve)")
    ap.add_argument("--f32-method", default=None, choices=["auto", "simt", "bf16x6"],
                    help="config 1 (fp32): FFMA on the CUDA cores or the bf16x6 split on the tensor cores")
    ap.add_argument("--direction", default="fwd", choices=["fwd", "fwd_train", "bwd", "convert"],
                    help="time the forward, the training forward (with the gate/up intermediates the backward "
                         "needs), the backward, or the dense -> Block-ELL conversion of the gate weight")
    args = ap.parse_args()
    from looped_blockell.synth import CONFIGS
    cfg = CONFIGS[args.config]
    if args.tokens:
        import dataclasses
        cfg = dataclasses.replace(cfg, T=args.tokens, name=f"{cfg.name}_T{args.tokens}")
    if args.tile:
        import dataclasses
        cfg = dataclasses.replace(cfg, B=args.tile, name=f"{cfg.name}_B{args.tile}")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        run_reference(args, cfg, rank, world)
        return
    if args.direction == "convert":
        run_convert(args, cfg, rank, world)
        return
    if args.direction == "bwd":
        if cfg.dtype != "bf16" or cfg.L != 1:
            raise SystemExit("--direction bwd: the backward exists for the bf16 SwiGLU configs (2, 5)")
        run_gpu_bwd(args, cfg, rank, world)
        return
    run_gpu(args, cfg, rank, world)


def run_gpu_bwd(args, cfg, rank, world):
    """One backward step per iteration on one GPU (replicas under torchrun:
    each rank times its own copy, max over ranks)."""
    import datetime

    import torch
    import torch.distributed as dist
    from looped_blockell.kernels import backward as kb
    from looped_blockell.kernels import ops
    from looped_blockell.synth import make_ffn

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    hbm_peak, tc_peak, tc_sust, peak_src = load_peaks()
    c = make_ffn(cfg, device="cuda", shared_gate_up=args.shared_gate_up)
    lay = ops.TILE_OUT_IN if args.layout == "out_in" else ops.TILE_IN_OUT
    if lay == ops.TILE_OUT_IN:
        for k in ("vg", "vu", "vd"):
            c[k] = c[k].transpose(-1, -2).contiguous()
    T, d, F, B = cfg.T, cfg.d_model, cfg.d_ff, cfg.B
    x = c["x"]
    _, h, g, u = ops.block_ell_swiglu_fwd_with_intermediate(x, c["vg"], c["cg"], c["vu"], c["cu"], c["vd"], c["cd"],
                                                            add_residual=True, layout=lay)
    dy = torch.randn(T, d, generator=torch.Generator(device="cuda").manual_seed(5), device="cuda").to(torch.bfloat16)
    w = (c["vg"], c["cg"], c["vu"], c["cu"], c["vd"], c["cd"])

    def step():
        return kb.block_ell_swiglu_bwd(dy, x, g, u, h, *w, layout=lay)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    try:
        gpu_id = "GPU-" + str(torch.cuda.get_device_properties(local).uuid)
    except Exception:
        gpu_id = str(local)
    evs = [_events(torch) for _ in range(args.steps)]
    with ClockSampler(gpu_id) as clk:
        for a, b in evs:
            a.record()
            step()
            b.record()
        torch.cuda.synchronize()
    ms = sum(a.elapsed_time(b) for a, b in evs) / args.steps
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    flops = 2.0 * cfg.nnz_flops()
    tflops = flops / (ms / 1e3) / 1e12

    # the kernels of one step, each timed alone with events
    vdT, cdT, lt = kb.transpose_ell([c["vd"]], [c["cd"]], F // B, lay)
    vguT, cguT, lt2 = kb.transpose_ell([c["vg"], c["vu"]], [c["cg"], c["cu"]], d // B, lay)
    dgu = kb.down_silu_bwd(dy, vdT, cdT, lt, g, u)
    dh = torch.empty((T, F), dtype=torch.bfloat16, device="cuda")
    g32 = torch.empty(c["vg"].shape, dtype=torch.float32, device="cuda")
    d32 = torch.empty(c["vd"].shape, dtype=torch.float32, device="cuda")
    parts = {
        "transpose_gather": lambda: (kb.transpose_ell([c["vd"]], [c["cd"]], F // B, lay),
                                     kb.transpose_ell([c["vg"], c["vu"]], [c["cg"], c["cu"]], d // B, lay)),
        "down_silu_bwd": lambda: kb.down_silu_bwd(dy, vdT, cdT, lt, g, u, out=dgu),
        "unfused_d_h_linear": lambda: ops.block_ell_linear(dy, vdT, cdT, layout=lt, out=dh),
        "unfused_silu_mul_bwd": lambda: kb.silu_mul_bwd(dh, g, u, out=dgu),
        "dx_linear": lambda: ops.block_ell_linear(dgu, vguT, cguT, residual=dy, layout=lt2),
        "sddmm_gate": lambda: kb.block_ell_sddmm(x, dgu[:, :F], c["cg"], B, lay, grad=g32),
        "sddmm_down": lambda: kb.block_ell_sddmm(h, dy, c["cd"], B, lay, grad=d32),
    }
    part_ms = {}
    for name, fn in parts.items():
        fn()
        a, b = _events(torch)
        a.record()
        for _ in range(5):
            fn()
        b.record()
        torch.cuda.synchronize()
        part_ms[name] = a.elapsed_time(b) / 5
    R_f, R_d = F // B, d // B
    sd_flops = 2.0 * T * B * B * R_f * cfg.K_gu  # one gate (or up) tile-gradient launch
    sd_tf = sd_flops / (part_ms["sddmm_gate"] / 1e3) / 1e12

    if rank == 0:
        line = {
            "metric": METRIC + " (backward)", "value": T / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak" if world > 1 else "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": cfg.name, "direction": "bwd", "T": T, "d_model": d, "d_ff": F, "B": B,
                       "density": cfg.density, "tile_layout": args.layout,
                       "parallelism": f"replicas{world}" if world > 1 else "single",
                       "l2": "inputs larger than L2 (x, g, u, h, grad_out resident)"},
            "tflops_effective": tflops, "flops_per_step": flops,
            "kernels_ms": part_ms,
            "roofline": {"bound": "tensor", "kernel": "whole backward step", "achieved": tflops, "peak": tc_peak,
                         "unit": "TFLOP/s", "frac": tflops / tc_peak, "peak_source": f"{peak_src} bf16 burst",
                         "traffic": None, "sddmm_gate_tflops": sd_tf, "sddmm_gate_frac": sd_tf / tc_peak},
            "gpu_launches": (10 if B == 64 else 11) * args.steps,
            "clocks": clk.summary(), "e2e": None,
        }
        if world == 1 and not args.no_cpu:
            v, dt = cpu_backward_sample(cfg, max(64, args.cpu_tokens // 4))
            line["cpu_baseline"] = {"value": v, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
                                    "sample": f"{max(64, args.cpu_tokens // 4)} tokens of {cfg.name} ({dt:.1f} s), "
                                              "numpy tile-by-tile restatement of the reference backward"}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_convert(args, cfg, rank, world):
    """Dense -> Block-ELL conversion of one gate-shaped weight [d_ff, d_model]
    (bf16) per step, on one GPU; HBM-bound: the matrix is read once and the
    kept tiles written once."""
    import numpy as np
    import torch
    from looped_blockell.kernels import convert as kc

    if rank != 0:
        return
    torch.cuda.set_device(0)
    hbm_peak, _, _, peak_src = load_peaks()
    d, F, B = cfg.d_model, cfg.d_ff, cfg.B
    g = torch.Generator(device="cuda").manual_seed(0)
    dense = (torch.randn(F, d, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    K = max(1, int((d // B) * cfg.density))
    for _ in range(args.warmup):
        kc.dense_to_block_ell(dense, B, K=K)
    torch.cuda.synchronize()
    try:
        gpu_id = "GPU-" + str(torch.cuda.get_device_properties(0).uuid)
    except Exception:
        gpu_id = "0"
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    evs = [_events(torch) for _ in range(args.steps)]
    with ClockSampler(gpu_id) as clk:
        for a, b in evs:
            flush.fill_(1)
            a.record()
            kc.dense_to_block_ell(dense, B, K=K)
            b.record()
        torch.cuda.synchronize()
    ms = sum(a.elapsed_time(b) for a, b in evs) / args.steps
    R, C = F // B, d // B
    alg = 2.0 * F * d + 2.0 * R * K * B * B + 4.0 * R * C * 2 + 4.0 * R * K  # dense, values, norms w+r, cols
    gbs = alg / (ms / 1e3) / 1e9
    line = {"metric": "dense -> Block-ELL conversion (create_block_ell_from_dense)", "value": 2.0 * F * d / (ms / 1e3) / 1e9,
            "unit": "GB/s of dense input", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"{cfg.name} gate weight", "out_features": F, "in_features": d, "B": B, "K": K,
                       "l2": "L2 flushed between steps (256 MiB write outside the timed events)"},
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak,
                         "peak_source": f"{peak_src} copy bandwidth", "traffic": None,
                         "note": "algorithmic bytes: dense read + kept tiles written + norms + cols"},
            "gpu_launches": 3 * args.steps, "clocks": clk.summary(), "e2e": None}
    if not args.no_cpu:
        import oracle as O
        dn = dense[: min(F, 2048)].float().cpu().numpy()
        t0 = time.perf_counter()
        O.dense_to_block_ell(dn, B, K / C)
        dt = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": dn.nbytes / 2 / dt / 1e9, "unit": "GB/s of dense input (bf16 bytes)",
                                "cores": os.cpu_count(), "kind": "port",
                                "sample": f"{dn.shape[0]} x {dn.shape[1]} rows of the same matrix ({dt:.2f} s), numpy "
                                          "restatement (oracle dense_to_block_ell)"}
    print(json.dumps(line), flush=True)


def parity_check(cfg, c, lay, out, rows, n_rows: int, seed: int = 0):
    """rel-L2 of ``out`` (this rank's result rows; ``rows`` = their token
    indices) against the CPU oracle on a sample of ``n_rows`` of them,
    computed from the same (bf16 or fp32) inputs the GPU saw.  Runs outside
    the timed region."""
    import numpy as np
    import torch
    import oracle as O
    n = min(n_rows, out.shape[0])
    pick = np.sort(np.random.default_rng(seed).choice(out.shape[0], n, replace=False))
    tok = rows[torch.from_numpy(pick)].to(c["x"].device)
    f = lambda t: t.float().cpu().numpy().astype(np.float64)  # noqa: E731
    x = f(c["x"].index_select(0, tok))
    w = [(f(c[v]), c[cc].cpu().numpy(), lay) for v, cc in (("vg", "cg"), ("vu", "cu"), ("vd", "cd"))]
    if cfg.L > 1:
        ref = O.looped_ffn(x, np.ones(cfg.d_model), *w, L=cfg.L)
    else:
        ref = O.swiglu_ffn(x, *w, add_residual=True)
    got = f(out.index_select(0, torch.from_numpy(pick).to(out.device)))
    return O.rel_l2(got, ref), n


def _events(torch):
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def run_gpu(args, cfg, rank, world):
    import datetime

    import torch
    import torch.distributed as dist
    from looped_blockell.kernels import ops
    from looped_blockell.synth import make_ffn

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    sm_reserve = None
    if world > 1:
        from looped_blockell.dist import default_exchange, default_sm_reserve, nccl_options
        exchange = args.exchange or default_exchange()
        sm_reserve = default_sm_reserve(world, exchange) if args.sm_reserve is None else args.sm_reserve
        nmax = args.nccl_max_ctas if args.nccl_max_ctas is not None else sm_reserve
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local),
                                pg_options=nccl_options(max_ctas=nmax or None))
    hbm_peak, tc_peak, tc_sust, peak_src = load_peaks()
    c = make_ffn(cfg, device="cuda", shared_gate_up=args.shared_gate_up)
    lay = ops.TILE_OUT_IN if args.layout == "out_in" else ops.TILE_IN_OUT
    if lay == ops.TILE_OUT_IN:  # same weights, stored [B_out, B_in]
        for k in ("vg", "vu", "vd"):
            c[k] = c[k].transpose(-1, -2).contiguous()
    pinned = None
    if args.l2_pin and cfg.dtype == "bf16":
        # gate and up tiles in one buffer, so one persisting window covers both
        from looped_blockell.kernels import loop as kl
        n_g = c["vg"].numel()
        pinned = torch.cat([c["vg"].reshape(-1), c["vu"].reshape(-1)])
        c["vg"], c["vu"] = pinned[:n_g].view(c["vg"].shape), pinned[n_g:].view(c["vu"].shape)
        kl.pin_weights_l2([pinned])
    T, d, F = cfg.T, cfg.d_model, cfg.d_ff
    launches_per_step = 3
    f32_method = None  # config 1: the fp32 method that runs
    if world > 1:
        from looped_blockell.dist import ShardedSwiGLU
        model = ShardedSwiGLU(c["vg"], c["cg"], c["vu"], c["cu"], c["vd"], c["cd"], rank, world, chunks=args.chunks,
                              sm_reserve=sm_reserve, exchange=exchange)
        step_out = model.alloc_out(T, c["x"])
        launches_per_step = model.launches_per_step(T)

        def step(x):
            return model.forward(x, out=step_out)
    elif cfg.dtype == "ternary":
        # config 3: ternary weights (2-bit packed tiles + per-tile scales), int8 activations
        from looped_blockell.kernels.ternary import make_ternary, ternary_swiglu_fwd
        if world > 1:
            raise SystemExit("the ternary workload runs on one GPU per replica")
        tg = make_ternary(c["vg"], c["cg"], d // cfg.B)
        tu = make_ternary(c["vu"], c["cu"], d // cfg.B)
        td = make_ternary(c["vd"], c["cd"], F // cfg.B)
        c["x"] = c["x"].to(torch.bfloat16)
        launches_per_step = 5  # plan, quantise x, gate/up, quantise h, down

        def step(x):
            return ternary_swiglu_fwd(x, tg, tu, td, add_residual=True)
    elif cfg.L > 1:
        # the shared-weight loop (config 4): L x (RMSNorm, gate/up, down) per step
        from looped_blockell.kernels.loop import looped_ffn
        if world > 1:
            raise SystemExit("the loop workload runs on one GPU per replica")
        out = torch.empty((T, d), dtype=torch.bfloat16, device="cuda")
        h = torch.empty((T, F), dtype=torch.bfloat16, device="cuda")
        gain = torch.ones(d, dtype=torch.bfloat16, device="cuda")
        from looped_blockell.kernels import loop as kl
        mode = {"auto": kl.LOOP_AUTO, "launches": kl.LOOP_LAUNCHES, "persistent": kl.LOOP_PERSISTENT}[args.loop_mode]
        persistent = kl.loop_uses_persistent(mode, cfg.B)
        # copy h_in, plan, then one persistent kernel (+ its counter reset) or RMSNorm + gate/up + down per iteration
        launches_per_step = 2 if persistent else 1 + 3 * cfg.L

        def step(x):
            return looped_ffn(x, gain, c["vg"], c["cg"], c["vu"], c["cu"], c["vd"], c["cd"], L=cfg.L, layout=lay,
                              mode=mode)
    else:
        act = c["x"].dtype  # bf16, or fp32 for the fp32 configuration
        out = torch.empty((T, d), dtype=act, device="cuda")
        train = args.direction == "fwd_train"  # also write gate_pre and up_out, as the training forward does
        if act == torch.float32:
            from looped_blockell.kernels import f32x
            f32_method = f32x.resolve(args.f32_method, T, cfg.K_gu, cfg.K_gu, cfg.K_d)
            launches_per_step = 8 if f32_method == "bf16x6" else 3  # split, 3 x (plan + linear), SiLU split
        # the bf16x6 fp32 forward keeps h in bf16 parts inside its workspace
        h = None if f32_method == "bf16x6" else torch.empty((T, F), dtype=act, device="cuda")

        def step(x):
            return ops._swiglu(x, c["vg"], c["cg"], c["vu"], c["cu"], c["vd"], c["cd"], True, lay, train,
                               out=out, h=h, shared_topology=args.shared_gate_up, fp32_method=f32_method)[0]

    x = c["x"]
    for _ in range(args.warmup):
        step(x)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = _events(torch)
    try:
        gpu_id = "GPU-" + str(torch.cuda.get_device_properties(local).uuid)
    except Exception:
        gpu_id = str(local)
    # working set below 2x L2 (126 MB): flush L2 between timed steps, outside the events
    ws_bytes = 2 * T * (2 * d + F) + 2 * cfg.B * cfg.B * (2 * (F // cfg.B) * cfg.K_gu + (d // cfg.B) * cfg.K_d)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda") if ws_bytes < (252 << 20) else None
    l2_note = ("L2 flushed between steps (256 MiB write outside the timed events)" if flush is not None
               else f"inputs larger than L2 ({ws_bytes / 2**30:.1f} GiB working set)")
    with ClockSampler(gpu_id) as clk:
        if flush is None:
            e0.record()
            for _ in range(args.steps):
                step(x)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / args.steps
        else:
            evs = [_events(torch) for _ in range(args.steps)]
            for a, b in evs:
                flush.fill_(1)
                a.record()
                step(x)
                b.record()
            torch.cuda.synchronize()
            ms = sum(a.elapsed_time(b) for a, b in evs) / args.steps
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = T / (ms / 1e3)
    tflops = cfg.nnz_flops() / (ms / 1e3) / 1e12

    # parity of one more (untimed) step's output against the CPU oracle: every
    # rank checks a sample of the token rows it holds; the worst rank is reported
    parity = None
    if not args.no_check and cfg.dtype in ("bf16", "f32"):
        import torch as _t
        res = step(x)
        _t.cuda.synchronize()
        if world > 1:
            from looped_blockell.dist import owned_rows, pick_chunks
            rows = owned_rows(T, rank, world, pick_chunks(T, world, model.want_chunks))
        else:
            rows = _t.arange(T)
        err, n_chk = parity_check(cfg, c, lay, res, rows, args.check_rows, seed=rank)
        if world > 1:
            t = _t.tensor([err], device="cuda", dtype=_t.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            err = float(t.item())
        parity = {"rel_l2": err, "tolerance": 1e-5 if cfg.dtype == "f32" else 1e-2, "rows_per_rank": n_chk,
                  "ranks": world, "oracle": f"oracle/bell_oracle.py (fp64, on the {cfg.dtype} inputs the GPU saw)"}

    # dominant kernel: the fused gate/up kernel, timed alone with events
    gu = None
    if world == 1 and cfg.L == 1 and cfg.dtype == "bf16":
        from looped_blockell.kernels import _lib
        import ctypes as C
        lib = _lib.load()
        desc = _lib.BellFFNDesc()
        plan = torch.empty(ops.plan_bytes(c["vg"].shape[0], c["vg"].shape[1], c["vu"].shape[1], c["vd"].shape[0],
                                          c["vd"].shape[1]), dtype=torch.uint8, device="cuda")
        desc.T, desc.d_model, desc.d_ff, desc.dtype, desc.add_residual = T, d, F, 0, 1
        desc.x, desc.h, desc.out, desc.plan = x.data_ptr(), h.data_ptr(), out.data_ptr(), plan.data_ptr()
        B = cfg.B
        desc.gate = ops._ell(c["vg"], c["cg"], d // B, lay)
        if args.shared_gate_up:
            desc.gate.flags = _lib.BELL_ELL_SAME_COLS_AS_UP
        desc.up = ops._ell(c["vu"], c["cu"], d // B, lay)
        desc.down = ops._ell(c["vd"], c["cd"], F // B, lay)
        s = ops._stream()
        for _ in range(2):
            _lib.check(lib.bell_gate_up_bf16(C.byref(desc), s), "gate_up")
        g0, g1 = _events(torch)
        n_gu = max(3, min(args.steps, 10))
        g0.record()
        for _ in range(n_gu):
            _lib.check(lib.bell_gate_up_bf16(C.byref(desc), s), "gate_up")
        g1.record()
        torch.cuda.synchronize()
        gu_ms = g0.elapsed_time(g1) / n_gu
        R_f = F // B
        gu_flops = 2.0 * T * B * B * 2 * R_f * cfg.K_gu
        gu = dict(ms=gu_ms, tflops=gu_flops / (gu_ms / 1e3) / 1e12)

    # end to end through the public op with host buffers
    # (one GPU: the public host-buffer op, which pipelines the copies of token
    # chunks with their compute on three streams; several GPUs: the sharded
    # host-buffer op, each rank copying in only its own token rows, all-gathered
    # over NVLink, and copying out its rows of the result)
    e2e = None
    if not args.no_e2e and cfg.dtype == "bf16":
        xh = x.cpu().pin_memory()
        oh = torch.empty((T if world == 1 else step_out.shape[0], d), dtype=torch.bfloat16).pin_memory()
        if world == 1:
            from looped_blockell.kernels import stream as kstream
            if cfg.L > 1:
                def e2e_step():
                    kstream.looped_ffn_host(xh, gain, c["vg"], c["cg"], c["vu"], c["cu"], c["vd"], c["cd"], L=cfg.L,
                                            layout=lay, out_host=oh)
            else:
                def e2e_step():
                    kstream.block_ell_swiglu_fwd_host(xh, c["vg"], c["cg"], c["vu"], c["cu"], c["vd"], c["cd"],
                                                      add_residual=True, layout=lay,
                                                      shared_topology=args.shared_gate_up, out_host=oh)
        else:
            from looped_blockell.dist import owned_rows, pick_chunks
            own = owned_rows(T, rank, world, pick_chunks(T, world, model.want_chunks))
            xh = xh.index_select(0, own).pin_memory()  # this rank's token rows only

            def e2e_step():
                model.forward_host(xh, out_host=oh)
        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        a0, a1 = _events(torch)
        n_e2e = max(3, min(args.steps, 5))
        a0.record()
        for _ in range(n_e2e):
            e2e_step()
        a1.record()
        torch.cuda.synchronize()
        ems = a0.elapsed_time(a1) / n_e2e
        if world > 1:
            t = torch.tensor([ems], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ems = float(t.item())
        # bytes over all ranks' host links (each rank copies its own token rows at N > 1)
        e2e = {"value": T / (ems / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": xh.numel() * 2 * world,
               "d2h_bytes_per_step": oh.numel() * 2 * world, "ms_per_step": ems}

    if rank == 0:
        line = {
            "metric": METRIC + (" (training forward, with gate/up intermediates)" if args.direction == "fwd_train"
                                else ""),
            "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None,
            "dtype": {"ternary": "int8 (ternary weights)", "f32": "f32"}.get(cfg.dtype, "bf16"),
            "data": "synthetic",
            "config": {"workload": cfg.name, "direction": args.direction, "T": T, "d_model": d, "d_ff": F,
                       "B": cfg.B, "density": cfg.density, "gate_up_topology": "shared" if args.shared_gate_up else "independent", "tile_layout": args.layout,
                       "parallelism": f"dff{world}" if world > 1 else "single",
                       "L": cfg.L, "l2": l2_note + ("; gate/up tiles in a persisting-L2 window" if pinned is not None
                                                     else ""),
                       **({"f32_method": f32_method} if f32_method else {}),
                       **({"chunks": args.chunks, "sm_reserve": sm_reserve, "exchange": model.exchange,
                           "nccl_max_ctas": args.nccl_max_ctas if args.nccl_max_ctas is not None else sm_reserve}
                          if world > 1 else {})},
            "tflops_effective": tflops, "tflops_effective_per_gpu": tflops / world,
            "hbm": hbm_line(cfg, T, ms, world, hbm_peak, peak_src),
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk.summary(), "e2e": e2e,
            "parity_rel_l2": None if parity is None else parity["rel_l2"], "parity": parity,
        }
        if gu:
            traffic = GU_DRAM_BYTES.get((args.config, cfg.T))
            line["roofline"] = {"bound": "tensor", "kernel": "gate/up kernel (bell_bf16_fmajor_kernel at B=128, "
                                "bell_bf16_kernel at B=64)", "achieved": gu["tflops"],
                                "peak": tc_peak, "unit": "TFLOP/s", "frac": gu["tflops"] / tc_peak,
                                "frac_of_sustained": gu["tflops"] / tc_sust,
                                "peak_source": f"{peak_src} bf16 burst", "traffic": traffic,
                                "traffic_source": GU_DRAM_NOTE.get(args.config) if traffic else None,
                                "kernel_ms": gu["ms"], "whole_step_frac": tflops / world / tc_peak}
        if cfg.L > 1:  # the whole loop step (gate/up and down kernels dominate)
            line["config"]["loop_mode"] = args.loop_mode + (" (persistent kernel)" if persistent else " (launches)")
            line["roofline"] = {"bound": "tensor", "kernel": "loop step (" + ("loop_kernel, one persistent launch"
                                if persistent else "bell_bf16_kernel gate/up + down launches") + ")", "achieved": tflops,
                                "peak": tc_peak, "unit": "TFLOP/s", "frac": tflops / tc_peak,
                                "peak_source": f"{peak_src} bf16 burst", "traffic": None, "kernel_ms": ms}
        if world == 1 and not args.no_cpu:
            v, dt = cpu_baseline_sample(cfg, args.cpu_tokens)
            line["cpu_baseline"] = {"value": v, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
                                    "sample": f"{args.cpu_tokens} tokens of {cfg.name} ({dt:.1f} s), numpy "
                                              "restatement of the reference path, scaled linearly"}
        print(json.dumps(line), flush=True)
    if pinned is not None:
        from looped_blockell.kernels import loop as kl
        kl.unpin_weights_l2()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
