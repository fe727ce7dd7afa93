"""persistent_mlp_step (injection, then n_core x (RMSNorm -> SwiGLU -> +h))
against the oracle, and the fused injection + RMSNorm kernel against the two
separate kernels (bit-identical)."""

import numpy as np
import pytest
import torch

import oracle as O
from gpu_util import make_case, to_dev

pytestmark = pytest.mark.gpu


def _K():
    from looped_blockell import kernels as K
    return K


def _f64(t):
    return t.float().cpu().numpy().astype(np.float64)


@pytest.mark.parametrize("T,d", [(37, 256), (8, 1024), (1, 64)])
def test_inject_rmsnorm_equals_separate_kernels(T, d):
    K = _K()
    g = torch.Generator().manual_seed(T)
    h = torch.randn(T, d, generator=g).to(torch.bfloat16).cuda()
    e = torch.randn(T, d, generator=g).to(torch.bfloat16).cuda()
    la, ld = torch.randn(d, generator=g).cuda(), (torch.randn(d, generator=g) * 3).cuda()
    gain = (1 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16).cuda()
    hi, nm = K.inject_rmsnorm(h, e, la, ld, gain, 1e-6)
    h2 = K.diagonal_injection(h, e, la, ld)
    n2 = K.rmsnorm(h2, gain, 1e-6)
    assert torch.equal(hi, h2) and torch.equal(nm, n2)


def test_persistent_mlp_step_matches_oracle():
    K = _K()
    n_core, T, d, F, B = 2, 150, 256, 512, 64
    cases = [to_dev(make_case(T, d, F, B, 2, 3, 4, seed=40 + i), torch.bfloat16) for i in range(n_core)]
    g = torch.Generator().manual_seed(9)
    h = torch.randn(T, d, generator=g).to(torch.bfloat16).cuda()
    e = torch.randn(T, d, generator=g).to(torch.bfloat16).cuda()
    la, ld = (0.3 * torch.randn(d, generator=g)).cuda(), torch.randn(d, generator=g).cuda()
    gains = [(1 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16).cuda() for _ in range(n_core)]
    out = K.persistent_mlp_step(h, e, la, ld, gains, [c["vg"] for c in cases], [c["cg"] for c in cases],
                                [c["vu"] for c in cases], [c["cu"] for c in cases], [c["vd"] for c in cases],
                                [c["cd"] for c in cases], eps=1e-6)
    torch.cuda.synchronize()
    # oracle: persistent_core.cu:273-337 in float64
    dt = np.log1p(np.exp(_f64(ld)))
    cur = np.exp(-dt * np.exp(_f64(la))) * _f64(h) + dt * _f64(e)
    for i, c in enumerate(cases):
        normed = O.rmsnorm(cur, _f64(gains[i]), eps=1e-6)
        w = [(_f64(c[v]), c[ci].cpu().numpy(), 0) for v, ci in (("vg", "cg"), ("vu", "cu"), ("vd", "cd"))]
        cur = cur + O.swiglu_ffn(normed, *w)
    assert O.rel_l2(_f64(out), cur) < 1e-2
    assert K.read_status() == 0
