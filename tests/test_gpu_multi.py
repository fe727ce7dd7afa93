"""d_ff-sharded forward on 2+ GPUs (one process per GPU, NCCL), launched with
torchrun and checked against the CPU oracle on every rank; skipped when
fewer than two GPUs are visible."""

import os
import subprocess
import sys

import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu


def _run(n):
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr=127.0.0.1", "--master-port=29533",
           os.path.join(ROOT, "tests", "mgpu_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env=dict(os.environ))
    print(r.stdout[-4000:], r.stderr[-3000:])
    return r.returncode


def test_sharded_forward_matches_oracle_at_every_rank_count():
    """Every power-of-two rank count from 2 up to the visible GPUs, with NCCL
    configured as the benchmark runs it (NVLS as NCCL chooses)."""
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs >= 2 GPUs")
    k = 2
    while k <= n:
        assert _run(k) == 0, f"{k} ranks"
        k *= 2
