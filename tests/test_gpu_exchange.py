"""The owner-side sum of the copy-engine exchange (``bell_sum_slices_bf16``)
and the stream-ordered copy (``bell_memcpy_async``) on one GPU.

The sum is defined as fp32 additions in ascending slice order starting from
slice 0's value, the residual last, one round to bf16; numpy float32
additions are IEEE round-to-nearest too, so the comparison is bit for bit."""

import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _expected(vals, residual):
    acc = vals[0].astype(np.float32)
    for v in vals[1:]:
        acc = (acc + v.astype(np.float32)).astype(np.float32)
    if residual is not None:
        acc = (acc + residual.astype(np.float32)).astype(np.float32)
    return torch.from_numpy(acc).to(torch.bfloat16)


@pytest.mark.parametrize("n,rows,d,local_slot,with_res", [(8, 4096, 1024, 3, True), (2, 300, 64, 0, False),
                                                          (4, 1, 8, -1, True), (1, 77, 136, 0, True),
                                                          (5, 129, 264, 4, False)])
def test_sum_slices_bit_exact(n, rows, d, local_slot, with_res):
    from looped_blockell.kernels.ops import sum_slices
    g = torch.Generator().manual_seed(n * 1000 + rows)
    # slices inside a wider buffer: row stride d + 16, slice stride rows * (d + 16) + 64
    ld = d + 16
    flat = (torch.randn(n * (rows * ld + 64), generator=g) * 3).to(torch.bfloat16).cuda()
    slices = flat.as_strided((n, rows, d), (rows * ld + 64, ld, 1))
    local = (torch.randn(rows, d, generator=g) * 3).to(torch.bfloat16).cuda() if local_slot >= 0 else None
    res = torch.randn(rows, d, generator=g).to(torch.bfloat16).cuda() if with_res else None
    out = torch.empty(rows, d, dtype=torch.bfloat16, device="cuda")
    sum_slices(slices, out, local=local, local_slot=local_slot, residual=res, max_ctas=16)
    torch.cuda.synchronize()
    vals = [(local if s == local_slot else slices[s]).float().cpu().numpy() for s in range(n)]
    exp = _expected(vals, None if res is None else res.float().cpu().numpy())
    assert torch.equal(out.cpu().view(torch.int16), exp.view(torch.int16))


def test_sum_slices_keeps_negative_zero():
    from looped_blockell.kernels.ops import sum_slices
    z = torch.full((1, 2, 8), -0.0, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(2, 8, dtype=torch.bfloat16, device="cuda")
    sum_slices(z, out)
    torch.cuda.synchronize()
    assert torch.all(torch.signbit(out.float()))


def test_sum_slices_rejects_bad_arguments():
    from looped_blockell.kernels.ops import sum_slices
    s = torch.zeros(2, 4, 12, dtype=torch.bfloat16, device="cuda")  # d not a multiple of 8
    with pytest.raises(RuntimeError):
        sum_slices(s, torch.empty(4, 12, dtype=torch.bfloat16, device="cuda"))
    s = torch.zeros(2, 4, 16, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError):  # local without a slot
        sum_slices(s, torch.empty(4, 16, dtype=torch.bfloat16, device="cuda"), local=s[0])


def test_memcpy_async_stream_ordered():
    from looped_blockell.kernels import _lib
    lib = _lib.load()
    a = torch.arange(1 << 20, dtype=torch.int32, device="cuda")
    b = torch.zeros_like(a)
    st = torch.cuda.current_stream()
    a.add_(1)  # queued before the copy on the same stream
    assert lib.bell_memcpy_async(C.c_void_p(b.data_ptr()), C.c_void_p(a.data_ptr()), a.numel() * 4,
                                 C.c_void_p(st.cuda_stream)) == 0
    torch.cuda.synchronize()
    assert torch.equal(a, b)
