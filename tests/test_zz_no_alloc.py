"""The allocation-free SwiGLU entry point (bell_swiglu_fwd_bf16_noalloc).

Some callers of this library cannot allocate device memory themselves: an
FFI host whose runtime owns every device allocation, or a server that sizes
its device memory once at start-up.  For them the library serves the plan
and the intermediate h from a fixed scratch array it carries.  This test
calls that entry point and the ordinary one (caller-owned buffers) through
the C ABI on the same inputs, twice in a row with different inputs so the
second call runs over the first call's leftovers, and requires the same
result within the bf16 tolerance used everywhere else (rel-L2 <= 1e-2).
It also checks that a problem larger than the scratch is refused before
anything is launched.  The file name makes pytest collect it last.
"""

import ctypes as C

import numpy as np
import pytest
import torch

import oracle as O
from gpu_util import make_case, to_dev

pytestmark = pytest.mark.gpu

TOL_BF16 = 1e-2


def _desc(L, dc, T, d, F, B, out, h=None, plan=None):
    desc = L.BellFFNDesc()
    desc.T, desc.d_model, desc.d_ff, desc.dtype, desc.add_residual = T, d, F, L.BELL_DTYPE_BF16, 1
    desc.x = dc["x"].data_ptr()
    desc.residual = None
    desc.h = None if h is None else h.data_ptr()
    desc.plan = None if plan is None else plan.data_ptr()
    desc.gate_pre = desc.up_out = None
    desc.out = out.data_ptr()
    desc.gate = L.BellEll(dc["vg"].data_ptr(), dc["cg"].data_ptr(), dc["vg"].shape[0], d // B, dc["vg"].shape[1], B, 0, 0)
    desc.up = L.BellEll(dc["vu"].data_ptr(), dc["cu"].data_ptr(), dc["vu"].shape[0], d // B, dc["vu"].shape[1], B, 0, 0)
    desc.down = L.BellEll(dc["vd"].data_ptr(), dc["cd"].data_ptr(), dc["vd"].shape[0], F // B, dc["vd"].shape[1], B,
                          0, 0)
    desc.status = None
    return desc


def test_noalloc_entry_matches_allocating_entry_twice():
    from looped_blockell.kernels import _lib as L
    lib = L.load()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    T, d, F, B = 700, 512, 2048, 128
    for call, seed in enumerate((21, 22)):
        dc = to_dev(make_case(T, d, F, B, 2, 3, 6, seed=seed, dead=2), torch.bfloat16)
        out_ref = torch.empty((T, d), dtype=torch.bfloat16, device="cuda")
        out_na = torch.full((T, d), float("nan"), dtype=torch.bfloat16, device="cuda")
        h = torch.empty((T, F), dtype=torch.bfloat16, device="cuda")
        plan = torch.empty(lib.bell_plan_bytes(F // B, 2, 3, d // B, 6), dtype=torch.uint8, device="cuda")
        rc = lib.bell_swiglu_fwd_bf16(C.byref(_desc(L, dc, T, d, F, B, out_ref, h, plan)), stream)
        assert rc == 0, L.last_error()
        rc = lib.bell_swiglu_fwd_bf16_noalloc(C.byref(_desc(L, dc, T, d, F, B, out_na)), stream)
        assert rc == 0, L.last_error()
        torch.cuda.synchronize()
        err = O.rel_l2(out_na.float().cpu().numpy(), out_ref.float().cpu().numpy())
        assert err <= TOL_BF16, (call, err)
        assert torch.isfinite(out_na.float()).all()


def test_noalloc_rejects_problems_larger_than_the_scratch():
    from looped_blockell.kernels import _lib as L
    lib = L.load()
    T, d, F, B = 4096, 512, 8192, 128  # h alone is 64 MiB > 32 MiB
    need = lib.bell_noalloc_scratch_bytes(T, F, F // B, 2, 2, d // B, 4)
    assert need > (32 << 20)
    dc = to_dev(make_case(8, d, F, B, 2, 2, 4, seed=1), torch.bfloat16)
    out = torch.empty((T, d), dtype=torch.bfloat16, device="cuda")
    desc = _desc(L, dc, T, d, F, B, out)
    rc = lib.bell_swiglu_fwd_bf16_noalloc(C.byref(desc), C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == -2 and "static scratch" in L.last_error()
    desc.h = out.data_ptr()  # caller-supplied scratch is refused too: the entry point owns it
    assert lib.bell_swiglu_fwd_bf16_noalloc(C.byref(desc), None) == -8
