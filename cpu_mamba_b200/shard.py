"""A Mamba block with its d_inner channels split over the ranks of a process
group (one process per GPU).

Batch sharding (``dist.shard``) needs no collective, but every rank runs the
whole block and reads all of its weights.  When the batch is smaller than the
number of GPUs, or a decode step's latency is bound by reading the weights,
the channels are split instead.  Rank r owns channels [lo, hi):

* in_proj: the rows of those channels in the x half and in the z half;
* conv1d, dt_proj, A_log, D: the channels' rows (everything between in_proj
  and out_proj is per channel);
* x_proj and out_proj: the channels' columns.  Both contract over d_inner, so
  each rank produces a partial sum and the ranks all-reduce it: x_dbl
  (N, dt_rank + 2 d_state) after x_proj and the output (N, d_model) after
  out_proj.  These are the only collectives;
* out_proj's bias (if any) on rank 0 only, so the sum adds it once.

The compute runs in the library's two shard phases (``mb2_block_forward_shard``
and ``mb2_block_step_shard``); the all-reduces are NCCL's, on the current
stream, through ``torch.distributed`` (or any ``reduce(tensor)`` callable that
sums a tensor over the ranks in place).  The result equals the unsharded
block's to within the reordered sums' rounding.  Recurrent state (h,
conv_state) stays sharded: each rank keeps its channels.
"""
from __future__ import annotations

import ctypes
from typing import Callable, Optional

import torch
import torch.nn as nn

from . import _lib
from . import dist as _dist
from ._lib import check, dtype_code, lib, stream_of
from .module import CPUMamba
from .quant import QuantizedLinear


def channel_range(d_inner: int, world: int, rank: int) -> tuple:
    """[lo, hi) of rank's channels: contiguous, sizes differ by at most one."""
    return _dist.shard(d_inner, world, rank)


def shard_state_dict(sd: dict, d_inner: int, world: int, rank: int) -> dict:
    """Rank's shard of a CPUMamba state_dict (mamba_ssm key layout)."""
    lo, hi = channel_range(d_inner, world, rank)
    out = {}
    for k, v in sd.items():
        if k in ("in_proj.weight", "in_proj.bias"):
            out[k] = torch.cat([v[lo:hi], v[d_inner + lo:d_inner + hi]]).contiguous()
        elif k in ("conv1d.weight", "conv1d.bias", "dt_proj.weight", "dt_proj.bias", "A_log", "D"):
            out[k] = v[lo:hi].contiguous()
        elif k in ("x_proj.weight", "out_proj.weight"):
            out[k] = v[:, lo:hi].contiguous()
        elif k == "out_proj.bias":
            out[k] = v.clone() if rank == 0 else torch.zeros_like(v)
        else:
            raise KeyError(f"shard_state_dict: unexpected key {k!r}")
    return out


def _allreduce(group):
    import torch.distributed as td

    def reduce(t: torch.Tensor) -> None:
        td.all_reduce(t, group=group)
    return reduce


class PeerReducer:
    """Sum over the ranks of ``group`` (one GPU each, one node) through peer
    memory: mb2_peer_allreduce, one kernel per call that pushes this rank's
    tensor into every rank's buffer over NVLink and sums all contributions in
    rank order.  For the small, latency-bound reductions of a decode step;
    tensors above ``max_elems`` elements go to NCCL's all-reduce (its
    bandwidth-optimal ring) instead.  Every rank must make the same calls in
    the same order, each on its current stream; they may be captured in a
    CUDA graph.  A wait longer than ``timeout_s`` is recorded (``status()``)
    instead of hanging the GPU.  ``close()`` releases the buffers (all ranks)."""

    def __init__(self, group=None, max_elems: int = 1 << 20, timeout_s: float = 5.0):
        import torch.distributed as td
        self.group = group
        self.max_elems = int(max_elems)
        on = td.is_initialized()
        world = td.get_world_size(group) if on else 1
        rank = td.get_rank(group) if on else 0
        L = lib()
        nbytes = L.mb2_peer_buffer_bytes(world, self.max_elems)
        if nbytes == 0:
            raise ValueError(f"PeerReducer: world {world} outside 1..8")
        own = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        check(L.mb2_peer_alloc(nbytes, ctypes.byref(own), handle), "peer alloc")
        handles = [handle.raw] * world
        if world > 1:
            handles = [None] * world
            td.all_gather_object(handles, handle.raw, group=group)
        g = _lib.PeerGroup()
        g.world, g.rank, g.slot_elems = world, rank, self.max_elems
        g.timeout_ns = int(timeout_s * 1e9)
        self._opened = []
        for r in range(world):
            if r == rank:
                g.bufs[r] = own.value
                continue
            p = ctypes.c_void_p()
            check(L.mb2_peer_open(handles[r], ctypes.byref(p)), "peer open")
            g.bufs[r] = p.value
            self._opened.append(p.value)
        self._own, self._g = own.value, g
        if world > 1:
            td.barrier(group=group)

    @property
    def world(self) -> int:
        return self._g.world

    def __call__(self, t: torch.Tensor) -> None:
        if self._g is None:
            raise RuntimeError("PeerReducer: closed")
        if not t.is_contiguous():
            raise RuntimeError("PeerReducer: tensor must be contiguous")
        if t.numel() > self.max_elems:
            if self._g.world == 1:
                return                   # the sum over one rank is the tensor itself
            import torch.distributed as td
            td.all_reduce(t, group=self.group)
            return
        check(lib().mb2_peer_allreduce(dtype_code(t.dtype), t.data_ptr(), t.numel(),
                                       ctypes.byref(self._g), stream_of(t)), "peer all-reduce")

    def status(self, clear: bool = True) -> int:
        """0, or MB2_PEER_TIMEOUT if a wait on this rank expired (synchronous)."""
        code = ctypes.c_int()
        check(lib().mb2_peer_status(ctypes.byref(self._g), ctypes.byref(code), int(clear)),
              "peer status")
        return code.value

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (collective: every
        rank calls it, after its last use)."""
        if self._g is None:
            return
        import torch.distributed as td
        torch.cuda.synchronize()
        if td.is_initialized() and self._g.world > 1:
            td.barrier(group=self.group)
        for p in self._opened:
            check(lib().mb2_peer_close(p), "peer close")
        if td.is_initialized() and self._g.world > 1:
            td.barrier(group=self.group)
        check(lib().mb2_peer_free(self._own), "peer free")
        self._g = None


class ChannelShardedMamba(nn.Module):
    """This rank's channel shard of ``block`` (a CPUMamba with dense
    projections).  ``world`` / ``rank`` default to the launcher's environment
    and ``reduce`` to NCCL's all-reduce over ``group``; ``reduce`` may also be
    a PeerReducer (the library's peer-memory all-reduce) or any callable that
    sums a tensor over the ranks in place.  With one rank the shard is the
    whole block and nothing is reduced."""

    def __init__(self, block: CPUMamba, world: Optional[int] = None, rank: Optional[int] = None,
                 group=None, device=None,
                 reduce: Optional[Callable[[torch.Tensor], None]] = None):
        super().__init__()
        for name in ("in_proj", "x_proj", "dt_proj", "out_proj"):
            if isinstance(getattr(block, name), QuantizedLinear):
                raise NotImplementedError("ChannelShardedMamba: quantised projections are not "
                                          "channel-sharded; shard the batch instead")
        ws_env, rank_env, _ = _dist.env()
        self.world = ws_env if world is None else int(world)
        self.rank = rank_env if rank is None else int(rank)
        self.lo, self.hi = channel_range(block.d_inner, self.world, self.rank)
        p = block.conv1d.weight
        device = p.device if device is None else torch.device(device)
        self.d_model, self.d_state, self.d_conv = block.d_model, block.d_state, block.d_conv
        self.d_inner_full = block.d_inner
        self.local = CPUMamba(block.d_model, block.d_state, block.d_conv, block.expand,
                              block.dt_rank, conv_bias=block.conv1d.bias is not None,
                              bias=block.in_proj.bias is not None, device=device, dtype=p.dtype,
                              d_inner=self.hi - self.lo)
        sd = shard_state_dict(block.state_dict(), block.d_inner, self.world, self.rank)
        self.local.load_state_dict(sd, strict=True)
        if reduce is None and self.world > 1:
            reduce = _allreduce(group)
        self._reduce = reduce

    @property
    def d_inner(self) -> int:
        return self.local.d_inner

    def _sum(self, t: torch.Tensor) -> None:
        if self._reduce is not None:
            self._reduce(t)

    def _xdbl_view(self, blk, ws: torch.Tensor, rows: int, step: bool,
                   dtype: torch.dtype) -> torch.Tensor:
        off, ld = ctypes.c_size_t(), ctypes.c_int64()
        check(lib().mb2_block_shard_xdbl(ctypes.byref(blk), rows, int(step), ctypes.byref(off),
                                         ctypes.byref(ld)), "shard x_dbl")
        es = torch.empty((), dtype=dtype).element_size()
        return ws[off.value: off.value + rows * ld.value * es].view(dtype).view(rows, ld.value)

    # ------------------------------------------------------------- forward
    # A forward (or step) is head(), the all-reduce of ctx["x_dbl"] in place,
    # tail(), and the all-reduce of ctx["out"]; forward() / forward_step() do
    # all four, head / tail let a caller drive the reductions itself.
    def head(self, x: torch.Tensor, want_state: bool = False) -> dict:
        m = self.local
        B, T, D = x.shape
        if D != self.d_model:
            raise RuntimeError(f"expected d_model={self.d_model}, got {tuple(x.shape)}")
        m._check_io(x, "forward")
        x = x.contiguous()
        keep = []
        blk = m._descriptor(keep)
        ws_bytes = lib().mb2_block_workspace_bytes(ctypes.byref(blk), B, T)
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x.device)
        ctx = dict(step=False, blk=blk, keep=keep, ws=ws, ws_bytes=ws_bytes, B=B, T=T,
                   out=torch.empty_like(x), h=None, conv_state=None, x=x)
        if want_state:
            ctx["h"] = torch.empty(B, m.d_inner, m.d_state, device=x.device, dtype=torch.float32)
            ctx["conv_state"] = torch.empty(B, m.d_inner, m.d_conv - 1, device=x.device,
                                            dtype=x.dtype)
        cp = None if ctx["conv_state"] is None else ctx["conv_state"].data_ptr()
        check(lib().mb2_block_forward_shard(ctypes.byref(blk), 1, x.data_ptr(), None, B, T,
                                            None, cp, ws.data_ptr(), ws_bytes, stream_of(x)),
              "forward shard head")
        ctx["x_dbl"] = self._xdbl_view(blk, ws, B * T, False, x.dtype)
        return ctx

    def tail(self, ctx: dict) -> torch.Tensor:
        blk, ws = ctx["blk"], ctx["ws"]
        out = ctx["out"]
        if ctx["step"]:
            check(lib().mb2_block_step_shard(ctypes.byref(blk), 2, None, out.data_ptr(),
                                             ctx["h"].data_ptr(), None, ctx["B"], ws.data_ptr(),
                                             ctx["ws_bytes"], stream_of(out)), "step shard tail")
        else:
            hp = None if ctx["h"] is None else ctx["h"].data_ptr()
            check(lib().mb2_block_forward_shard(ctypes.byref(blk), 2, None, out.data_ptr(),
                                                ctx["B"], ctx["T"], hp, None, ws.data_ptr(),
                                                ctx["ws_bytes"], stream_of(out)),
                  "forward shard tail")
        return out

    def _run(self, ctx: dict) -> torch.Tensor:
        if ctx["x_dbl"].numel():
            self._sum(ctx["x_dbl"])
        out = self.tail(ctx)
        if out.numel():
            self._sum(out)
        return out

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        """(B, T, d_model) -> (B, T, d_model): the whole block's output, on
        every rank."""
        return self._run(self.head(hidden_states))

    def forward_with_final_state(self, hidden_states: torch.Tensor) -> tuple:
        """(y, {"h": (B, d_inner_local, d_state), "conv_state": (B,
        d_inner_local, d_conv-1)}): y whole, the state this rank's channels."""
        ctx = self.head(hidden_states, True)
        y = self._run(ctx)
        return y, {"h": ctx["h"], "conv_state": ctx["conv_state"]}

    # ---------------------------------------------------------------- step
    def init_state(self, batch_size: int, device=None, dtype=None) -> dict:
        """Zero decode state of this rank's channels."""
        return self.local.init_state(batch_size, device, dtype)

    def step_head(self, x_step: torch.Tensor, state: dict) -> dict:
        m = self.local
        if x_step.dim() == 3:
            x_step = x_step.squeeze(1)
        B, D = x_step.shape
        if D != self.d_model:
            raise RuntimeError(f"expected d_model={self.d_model}, got {tuple(x_step.shape)}")
        m._check_io(x_step, "forward_step")
        x_step = x_step.contiguous()
        h, conv = state["h"], state["conv_state"]
        if (h.shape != (B, m.d_inner, m.d_state) or h.dtype != torch.float32
                or not h.is_contiguous() or conv.shape != (B, m.d_inner, m.d_conv - 1)
                or conv.dtype != x_step.dtype or not conv.is_contiguous()):
            raise RuntimeError("forward_step: state must be this shard's init_state layout")
        keep = []
        blk = m._descriptor(keep)
        ws_bytes = lib().mb2_step_workspace_bytes(ctypes.byref(blk), B)
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x_step.device)
        ctx = dict(step=True, blk=blk, keep=keep, ws=ws, ws_bytes=ws_bytes, B=B,
                   out=torch.empty_like(x_step), h=h, conv_state=conv, x=x_step)
        check(lib().mb2_block_step_shard(ctypes.byref(blk), 1, x_step.data_ptr(), None, None,
                                         conv.data_ptr(), B, ws.data_ptr(), ws_bytes,
                                         stream_of(x_step)), "step shard head")
        ctx["x_dbl"] = self._xdbl_view(blk, ws, B, True, x_step.dtype)
        return ctx

    def forward_step(self, x_step: torch.Tensor, state: dict) -> tuple:
        """One token for all ranks' channels: (B, d_model) or (B, 1, d_model)
        -> (B, d_model); this rank's state is advanced in place."""
        return self._run(self.step_head(x_step, state)), state
