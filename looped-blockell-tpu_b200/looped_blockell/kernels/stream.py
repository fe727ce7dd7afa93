"""Host-buffer entry points: the forward of a token batch that lives in
(pinned) host memory, with the copies overlapped with the compute.

Tokens are independent in every op of this path, so the batch is cut into
chunks and three CUDA streams run a software pipeline: the host->device copy
of chunk i+1, the kernels of chunk i and the device->host copy of chunk i-1
proceed together (PCIe is full duplex).  Device buffers are double-buffered
per chunk; events order each buffer's reuse.  The result is the same as one
call on the whole batch, since no op mixes tokens.
"""

from __future__ import annotations

from typing import Callable, Optional

import torch

from .loop import looped_ffn
from .ops import TILE_IN_OUT, _swiglu

_STREAMS = {}  # device index -> (copy-in, compute, copy-out) streams, created once


def _streams(device: torch.device):
    idx = torch.device(device).index
    idx = torch.cuda.current_device() if idx is None else idx
    if idx not in _STREAMS:
        _STREAMS[idx] = tuple(torch.cuda.Stream(idx) for _ in range(3))
    return _STREAMS[idx]


def auto_chunk(T: int) -> int:
    """About 32 chunks per batch, 4096..16384 tokens each (a multiple of 256):
    the copies of the first and last chunk are not overlapped, and chunks
    below ~4096 tokens lose kernel efficiency.  Measured through this module
    on one B200 (PCIe host copies ~45 GB/s per direction): config 5 (T=262144)
    52.1 / 48.2 / 47.5 / 48.5 ms at 32768 / 16384 / 8192 / 4096 tokens per
    chunk; config 2 (T=32768) 3.44 / 3.69 / 4.29 ms at 4096 / 2048 / 1024."""
    c = -(-T // 32)
    c = -(-c // 256) * 256
    return max(4096, min(16384, c))


def pipeline_tokens(x_host: torch.Tensor, out_features: int, fn: Callable[[torch.Tensor, torch.Tensor], None],
                    device: torch.device, chunk_tokens: Optional[int] = None, out_host: Optional[torch.Tensor] = None,
                    out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """Run ``fn(x_dev_chunk, out_dev_chunk)`` over token chunks of ``x_host``.

    ``fn`` launches its kernels on the current stream and writes the whole
    ``out_dev_chunk``.  Returns ``out_host`` (pinned, allocated if not given);
    on return the caller's current stream is ordered after the last copy, so a
    ``torch.cuda.synchronize()`` (or an event on that stream) makes it readable.
    """
    if x_host.is_cuda:
        raise RuntimeError("x_host must be a host tensor")
    if x_host.dim() != 2:
        raise RuntimeError("x_host must be 2D [tokens, features]")
    T, d_in = x_host.shape
    out_dtype = out_dtype or x_host.dtype
    if out_host is None:
        out_host = torch.empty((T, out_features), dtype=out_dtype, pin_memory=True)
    if T == 0:
        return out_host
    chunk = max(1, min(int(chunk_tokens or auto_chunk(T)), T))
    nbuf = 2
    xs = [torch.empty((chunk, d_in), dtype=x_host.dtype, device=device) for _ in range(nbuf)]
    ys = [torch.empty((chunk, out_features), dtype=out_dtype, device=device) for _ in range(nbuf)]
    caller = torch.cuda.current_stream(device)
    s_in, s_comp, s_out = _streams(device)
    for s in (s_in, s_comp, s_out):
        s.wait_stream(caller)
    ev_in = [torch.cuda.Event() for _ in range(nbuf)]
    ev_comp = [torch.cuda.Event() for _ in range(nbuf)]
    ev_out = [torch.cuda.Event() for _ in range(nbuf)]
    for i, t0 in enumerate(range(0, T, chunk)):
        n = min(chunk, T - t0)
        b = i % nbuf
        with torch.cuda.stream(s_in):
            if i >= nbuf:
                s_in.wait_event(ev_comp[b])  # x buffer b is read by compute of chunk i - nbuf
            xs[b][:n].copy_(x_host[t0:t0 + n], non_blocking=True)
            ev_in[b].record(s_in)
        with torch.cuda.stream(s_comp):
            s_comp.wait_event(ev_in[b])
            if i >= nbuf:
                s_comp.wait_event(ev_out[b])  # out buffer b is read by the copy of chunk i - nbuf
            fn(xs[b][:n], ys[b][:n])
            ev_comp[b].record(s_comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_comp[b])
            out_host[t0:t0 + n].copy_(ys[b][:n], non_blocking=True)
            ev_out[b].record(s_out)
    # the caller's stream (where every buffer here was allocated) is ordered
    # after the last copy, so the buffers are not reused before the pipeline drains
    caller.wait_stream(s_out)
    return out_host


def block_ell_swiglu_fwd_host(x_host: torch.Tensor, v_gate, ci_gate, v_up, ci_up, v_down, ci_down,
                              add_residual: bool = False, layout: int = TILE_IN_OUT, shared_topology: bool = False,
                              chunk_tokens: Optional[int] = None, out_host: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``block_ell_swiglu_fwd`` for a host (pinned) activation batch; returns a
    pinned host output.  The weights and column indices are device tensors."""
    dev = v_gate.device
    d_model = x_host.shape[1]
    F = v_gate.shape[0] * v_gate.shape[2]
    chunk = max(1, min(int(chunk_tokens or auto_chunk(x_host.shape[0])), x_host.shape[0]))
    h = torch.empty((chunk, F), dtype=x_host.dtype, device=dev)

    def fn(xc: torch.Tensor, yc: torch.Tensor) -> None:
        _swiglu(xc, v_gate, ci_gate, v_up, ci_up, v_down, ci_down, add_residual, layout, False, out=yc,
                h=h[:xc.shape[0]], shared_topology=shared_topology)

    return pipeline_tokens(x_host, d_model, fn, dev, chunk, out_host)


def looped_ffn_host(h_host: torch.Tensor, norm_gain, v_gate, ci_gate, v_up, ci_up, v_down, ci_down, L: int,
                    eps: float = 1e-5, layout: int = TILE_IN_OUT, chunk_tokens: Optional[int] = None,
                    out_host: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``looped_ffn`` for a host (pinned) state batch; returns a pinned host output.
    The loop does L times the work of one forward per copied byte, so the
    default cuts the batch into 2 chunks at least 4096 tokens long."""
    dev = v_gate.device
    if chunk_tokens is None:
        chunk_tokens = max(4096, -(-h_host.shape[0] // 2))

    def fn(xc: torch.Tensor, yc: torch.Tensor) -> None:
        looped_ffn(xc, norm_gain, v_gate, ci_gate, v_up, ci_up, v_down, ci_down, L, eps=eps, layout=layout, out=yc)

    return pipeline_tokens(h_host, h_host.shape[1], fn, dev, chunk_tokens, out_host)
