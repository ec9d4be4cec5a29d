"""Host-memory batches through the GPU with copies overlapping compute.

Used by ``CPUMamba.forward_host`` and ``MambaStack.forward_host``: the batch
is cut into slices along its first dimension; each slice is copied to the
device on one stream, computed on one of two compute streams and copied back
on a third.  Rows of a batch are independent in a Mamba block (and in a
residual stack of them), so the result is that of one call on the whole batch
(bit for bit where the slices and the whole batch take the same projection
kernels; the GEMM kernel is chosen by row count).
"""
from __future__ import annotations

from typing import Callable

import torch


def slice_bounds(B: int, n: int, edge: float) -> list:
    """n contiguous [a, b) ranges covering 0..B, the first and last weighted
    ``edge`` against 1 for the others (every range non-empty).  The first
    slice's upload and the last slice's download overlap no compute, so small
    end slices shorten the pipeline's fill and drain."""
    if n <= 2:
        return [(B * i // n, B * (i + 1) // n) for i in range(n)]
    w = [edge] + [1.0] * (n - 2) + [edge]
    tot = sum(w)
    cuts, acc = [0], 0.0
    for i in range(n - 1):
        acc += w[i]
        cuts.append(min(B - (n - 1 - i), max(cuts[-1] + 1, round(B * acc / tot))))
    cuts.append(B)
    return [(cuts[i], cuts[i + 1]) for i in range(n)]


_STREAMS = {}


def _helper_streams(dev: torch.device):
    """Upload, download and second compute stream of a device, created once:
    the caching allocator reuses a freed block only on the stream that
    allocated it, so per-call streams would defeat the cache."""
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    if key not in _STREAMS:
        _STREAMS[key] = tuple(torch.cuda.Stream(dev) for _ in range(3))
    return _STREAMS[key]


def run_streamed(x: torch.Tensor, out: torch.Tensor, dev: torch.device,
                 run: Callable[[torch.Tensor, torch.Tensor], None], chunks: int,
                 slots: int = 3, edge: float = 0.5) -> torch.Tensor:
    """For each slice x[a:b] (host): copy to a device slot, ``run(xd, yd)``
    (writes the slice's result into the device tensor yd, on the current
    stream), copy yd back into out[a:b] (host).  Returns once ``out`` holds
    the whole result."""
    B = x.shape[0]
    if B == 0:
        return out
    n = max(1, min(B, chunks))
    bounds = slice_bounds(B, n, edge)
    rows = max(b - a for a, b in bounds)
    tail = tuple(x.shape[1:])
    cur = torch.cuda.current_stream(dev)
    s_in, s_out, s_c2 = _helper_streams(dev)
    # slices are independent: alternate two compute streams so one slice's
    # kernels fill the tail of the previous one's
    comp = [cur] if n == 1 else [cur, s_c2]
    nslot = min(slots, n)
    xin = [torch.empty((rows,) + tail, device=dev, dtype=x.dtype) for _ in range(nslot)]
    yout = [torch.empty((rows,) + tuple(out.shape[1:]), device=dev, dtype=out.dtype)
            for _ in range(nslot)]
    ev_in = [torch.cuda.Event() for _ in range(n)]
    ev_c = [torch.cuda.Event() for _ in range(n)]
    ev_out = [torch.cuda.Event() for _ in range(n)]
    for s in (s_in, s_out, *comp[1:]):
        s.wait_stream(cur)
    for i, (a, b) in enumerate(bounds):
        k = i % nslot
        c = comp[i % len(comp)]
        with torch.cuda.stream(s_in):
            if i >= nslot:
                s_in.wait_event(ev_c[i - nslot])          # slot's input consumed
            xin[k][: b - a].copy_(x[a:b], non_blocking=True)
            ev_in[i].record(s_in)
        with torch.cuda.stream(c):
            c.wait_event(ev_in[i])
            if i >= nslot:
                c.wait_event(ev_out[i - nslot])           # slot's output copied out
            run(xin[k][: b - a], yout[k][: b - a])
            ev_c[i].record(c)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_c[i])
            out[a:b].copy_(yout[k][: b - a], non_blocking=True)
            ev_out[i].record(s_out)
    for s in (s_in, s_out, *comp[1:]):
        cur.wait_stream(s)
    ev_out[-1].synchronize()
    return out
