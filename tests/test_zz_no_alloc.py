"""The allocation-free SwiGLU entry point (bell_swiglu_fwd_bf16_noalloc).

Some callers of this library cannot allocate device memory themselves: an
FFI host whose runtime owns every device allocation, or a server that sizes
its device memory once at start-up.  For them the library serves the plan
and the intermediate h from a fixed scratch array it carries.  These tests
call that entry point and the ordinary one (caller-owned buffers) through
the C ABI on the same inputs, twice in a row with different inputs so the
second call runs over the first call's leftovers, and require
  * the same bits as the ordinary entry point (the same kernels run on the
    same plan), and
  * the CPU oracle's result within the bf16 tolerance used everywhere else
    (rel-L2 <= 1e-2).
The cases cover both tile sizes, a caller-supplied status word, the residual
off, and a problem that fills the scratch to within 1 MiB of its end.  A
problem larger than the scratch is refused before anything is launched.  The
file name makes pytest collect it last.
"""

import ctypes as C

import numpy as np
import pytest
import torch

import oracle as O
from gpu_util import dev_inputs_as_f64, make_case, oracle_ffn, to_dev

pytestmark = pytest.mark.gpu

TOL_BF16 = 1e-2
SCRATCH = 32 << 20


def _desc(L, dc, T, d, F, B, out, h=None, plan=None, add_residual=1, status=None):
    desc = L.BellFFNDesc()
    desc.T, desc.d_model, desc.d_ff, desc.dtype, desc.add_residual = T, d, F, L.BELL_DTYPE_BF16, add_residual
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
    desc.status = None if status is None else status.data_ptr()
    return desc


CASES = [
    # T,    d,   F,    B,  Kg, Ku, Kd, add_residual, own status word
    (700, 512, 2048, 128, 2, 3, 6, 1, False),
    (300, 256, 1024, 64, 2, 1, 5, 0, True),
    (2000, 512, 8192, 128, 2, 3, 6, 1, False),  # h is 31.25 MiB: the plan and h end near the scratch's end
]


@pytest.mark.parametrize("case", CASES)
def test_noalloc_entry_matches_allocating_entry_and_oracle_twice(case):
    from looped_blockell.kernels import _lib as L
    T, d, F, B, Kg, Ku, Kd, add_res, own_status = case
    lib = L.load()
    need = lib.bell_noalloc_scratch_bytes(T, F, F // B, Kg, Ku, d // B, Kd)
    assert 0 < need <= SCRATCH
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    status = torch.zeros(1, dtype=torch.int32, device="cuda") if own_status else None
    for call, seed in enumerate((21, 22)):
        c = make_case(T, d, F, B, Kg, Ku, Kd, seed=seed + T, dead=2)
        dc = to_dev(c, torch.bfloat16)
        out_ref = torch.empty((T, d), dtype=torch.bfloat16, device="cuda")
        out_na = torch.full((T, d), float("nan"), dtype=torch.bfloat16, device="cuda")
        h = torch.empty((T, F), dtype=torch.bfloat16, device="cuda")
        plan = torch.empty(lib.bell_plan_bytes(F // B, Kg, Ku, d // B, Kd), dtype=torch.uint8, device="cuda")
        rc = lib.bell_swiglu_fwd_bf16(C.byref(_desc(L, dc, T, d, F, B, out_ref, h, plan, add_res, status)), stream)
        assert rc == 0, L.last_error()
        rc = lib.bell_swiglu_fwd_bf16_noalloc(C.byref(_desc(L, dc, T, d, F, B, out_na, None, None, add_res, status)),
                                              stream)
        assert rc == 0, L.last_error()
        torch.cuda.synchronize()
        assert torch.isfinite(out_na.float()).all()
        assert torch.equal(out_na, out_ref), f"call {call}: not bit-identical to the allocating entry"
        ro = oracle_ffn(dev_inputs_as_f64(dc), add_residual=bool(add_res))[0]
        err = O.rel_l2(out_na.float().cpu().numpy(), ro)
        assert err <= TOL_BF16, (call, err)
    if own_status:
        assert int(status.item()) == 0
    else:
        from looped_blockell.kernels import read_status
        assert read_status() == 0


def test_noalloc_rejects_problems_larger_than_the_scratch():
    from looped_blockell.kernels import _lib as L
    lib = L.load()
    T, d, F, B = 4096, 512, 8192, 128  # h alone is 64 MiB > 32 MiB
    need = lib.bell_noalloc_scratch_bytes(T, F, F // B, 2, 2, d // B, 4)
    assert need > SCRATCH
    dc = to_dev(make_case(8, d, F, B, 2, 2, 4, seed=1), torch.bfloat16)
    out = torch.empty((T, d), dtype=torch.bfloat16, device="cuda")
    desc = _desc(L, dc, T, d, F, B, out)
    rc = lib.bell_swiglu_fwd_bf16_noalloc(C.byref(desc), C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == -2 and "static scratch" in L.last_error()
    desc.h = out.data_ptr()  # caller-supplied scratch is refused too: the entry point owns it
    assert lib.bell_swiglu_fwd_bf16_noalloc(C.byref(desc), None) == -8
    # a wrong shape is reported as such, not as a scratch-size problem
    desc.h = None
    desc.down.K = 300
    assert lib.bell_swiglu_fwd_bf16_noalloc(C.byref(desc), None) == -2
    assert "K must be <= 254" in L.last_error()
