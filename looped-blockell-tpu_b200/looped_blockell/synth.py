"""Seeded synthetic inputs for the five benchmark configurations.

Shapes and distributions follow the benchmark definitions: column indices
per block-row uniform without replacement then sorted, weights N(0, 0.02^2),
activations N(0, 1); bf16 configs cast both to bf16.  Gate and up draw
independent topologies unless ``shared_gate_up`` (the reference MLPBlock's
own behaviour, looped_blockell/layers/mlp.py:84-95).  Generation runs on the
target device with a seeded torch.Generator, so large configs never touch
host memory.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import torch


@dataclass(frozen=True)
class Config:
    name: str
    T: int
    d_model: int
    d_ff: int
    B: int
    density: float
    dtype: str          # "f32" | "bf16" | "ternary"
    L: int = 1
    seed: int = 0

    @property
    def K_gu(self) -> int:
        return max(1, int((self.d_model // self.B) * self.density))

    @property
    def K_d(self) -> int:
        return max(1, int((self.d_ff // self.B) * self.density))

    def nnz_flops(self, T: Optional[int] = None) -> float:
        """2*T*B^2 per live tile, gate+up+down, times L."""
        T = self.T if T is None else T
        R_f, R_d = self.d_ff // self.B, self.d_model // self.B
        tiles = 2 * R_f * self.K_gu + R_d * self.K_d
        return 2.0 * T * self.B * self.B * tiles * self.L


CONFIGS = {
    1: Config("cfg1_fp32_cpu", T=4 * 256, d_model=512, d_ff=2048, B=64, density=0.25, dtype="f32", seed=1),
    2: Config("cfg2_bf16", T=16 * 2048, d_model=2048, d_ff=8192, B=64, density=0.125, dtype="bf16", seed=2),
    3: Config("cfg3_ternary", T=16 * 2048, d_model=2048, d_ff=8192, B=64, density=0.25, dtype="ternary", seed=3),
    4: Config("cfg4_loop_L8", T=8 * 1024, d_model=1024, d_ff=4096, B=64, density=0.25, dtype="bf16", L=8, seed=4),
    5: Config("cfg5_large_bf16", T=64 * 4096, d_model=4096, d_ff=16384, B=128, density=0.25, dtype="bf16", seed=5),
}


def topology(R: int, C: int, K: int, g: torch.Generator, device) -> torch.Tensor:
    """K distinct column blocks per row, uniform without replacement, sorted."""
    keys = torch.rand(R, C, generator=g, device=device)
    cols = torch.topk(keys, K, dim=1).indices
    return torch.sort(cols, dim=1).values.to(torch.int32).contiguous()


def make_ffn(cfg: Config, device="cuda", T: Optional[int] = None, shared_gate_up: bool = False,
             dtype: Optional[torch.dtype] = None, seed: Optional[int] = None):
    """Returns dict(x, vg, cg, vu, cu, vd, cd) for one SwiGLU FFN (tiles [B_in, B_out])."""
    T = cfg.T if T is None else T
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(cfg.seed if seed is None else seed)
    B, d, F = cfg.B, cfg.d_model, cfg.d_ff
    R_f, C_d, R_d, C_f = F // B, d // B, d // B, F // B
    if dtype is None:
        dtype = torch.float32 if cfg.dtype in ("f32", "ternary") else torch.bfloat16
    cg = topology(R_f, C_d, cfg.K_gu, g, dev)
    cu = cg.clone() if shared_gate_up else topology(R_f, C_d, cfg.K_gu, g, dev)
    cd = topology(R_d, C_f, cfg.K_d, g, dev)

    def w(shape):
        return (torch.randn(shape, generator=g, device=dev, dtype=torch.float32) * 0.02).to(dtype)

    vg, vu, vd = w((R_f, cfg.K_gu, B, B)), w((R_f, cfg.K_gu, B, B)), w((R_d, cfg.K_d, B, B))
    x = torch.randn((T, d), generator=g, device=dev, dtype=torch.float32).to(dtype)
    return dict(x=x, vg=vg, cg=cg, vu=vu, cu=cu, vd=vd, cd=cd)
