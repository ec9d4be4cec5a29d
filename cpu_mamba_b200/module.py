"""CPUMamba -- the Mamba S6 block with the API and state_dict of
src/cpu_mamba/_mamba.py:49-279, computed by the B200 CUDA library.

forward / forward_with_final_state / forward_step / init_state keep the
reference's signatures and semantics; parameters keep the mamba_ssm names,
shapes and dtypes, so ``load_state_dict`` of a mamba_ssm or cpu-mamba
checkpoint works unchanged.  The whole block runs as one C-ABI call
(mb2_block_forward / mb2_block_step); there is no CPU path.

Differences from the reference, all on purpose:
  * forward_with_final_state derives h_T and the conv tail in the same pass as
    the output (the reference re-runs the projections and a Python time loop,
    _mamba.py:172-199);
  * forward_step updates state["h"] and state["conv_state"] in place in the
    existing tensors (the reference rebinds the dict entries, :138 and :158);
  * for prompts shorter than d_conv-1 the conv tail is zero-left-padded, which
    forward_step can consume (the reference returns a narrower tensor there);
  * the constructor's device/dtype factory kwargs (from mamba_ssm) are honoured.
The backend attributes ``_scan_backend``, ``_assoc_chunk_T`` and
``_force_time_loop`` (_mamba.py:231-237) are accepted and ignored: every
backend of the reference computes the same recurrence, which here is one kernel.
"""
from __future__ import annotations

import ctypes
import math

import torch
import torch.nn as nn

from . import _lib, ops
from ._lib import Block, LinearW, check, dtype_code, lib, stream_of
from .quant import QuantizedLinear
from .streaming import run_streamed


class CPUMamba(nn.Module):
    """Mamba S6 block, state_dict-compatible with mamba_ssm.Mamba 2.3.x."""

    # device buffers (input + output slice) forward_host keeps in flight
    _host_slots = 3
    # relative size of forward_host's first and last slices: the first slice's
    # upload and the last one's download overlap no compute, so they are small
    _host_edge = 0.5

    def __init__(self, d_model: int, d_state: int = 16, d_conv: int = 4,
                 expand: int = 2, dt_rank="auto",
                 dt_min: float = 0.001, dt_max: float = 0.1, dt_init: str = "random",
                 dt_scale: float = 1.0, dt_init_floor: float = 1e-4,
                 conv_bias: bool = True, bias: bool = False, device=None, dtype=None,
                 *, d_inner: int | None = None, **_unused):
        """d_inner (keyword only, not a reference argument) overrides expand *
        d_model: the channel count of one shard of a channel-sharded block."""
        super().__init__()
        self.d_model = d_model
        self.d_state = d_state
        self.d_conv = d_conv
        self.expand = expand
        self.d_inner = int(d_inner) if d_inner is not None else expand * d_model
        self.dt_rank = math.ceil(d_model / 16) if dt_rank == "auto" else int(dt_rank)
        fk = {"device": device, "dtype": dtype}
        self.in_proj = nn.Linear(d_model, self.d_inner * 2, bias=bias, **fk)
        self.conv1d = nn.Conv1d(self.d_inner, self.d_inner, kernel_size=d_conv,
                                groups=self.d_inner, padding=d_conv - 1, bias=conv_bias, **fk)
        self.act = nn.SiLU()
        self.x_proj = nn.Linear(self.d_inner, self.dt_rank + 2 * d_state, bias=False, **fk)
        self.dt_proj = nn.Linear(self.dt_rank, self.d_inner, bias=True, **fk)
        A = torch.arange(1, d_state + 1, dtype=torch.float32, device=device).repeat(self.d_inner, 1)
        self.A_log = nn.Parameter(torch.log(A).to(dtype or torch.float32))
        self.A_log._no_weight_decay = True
        self.D = nn.Parameter(torch.ones(self.d_inner, device=device, dtype=dtype))
        self.D._no_weight_decay = True
        self.out_proj = nn.Linear(self.d_inner, d_model, bias=bias, **fk)
        self._split_cache = {}

    # ------------------------------------------------------------------ state
    def init_state(self, batch_size: int, device=None, dtype=None) -> dict:
        """Zero state for forward_step: h (B, d_inner, d_state) float32 and
        conv_state (B, d_inner, d_conv-1) in the parameter dtype (_mamba.py:87-101)."""
        p = next(self.parameters())
        device = p.device if device is None else device
        dtype = p.dtype if dtype is None else dtype
        return {
            "h": torch.zeros(batch_size, self.d_inner, self.d_state, device=device,
                             dtype=torch.float32),
            "conv_state": torch.zeros(batch_size, self.d_inner, self.d_conv - 1,
                                      device=device, dtype=dtype),
        }

    # ------------------------------------------------------------ descriptor
    def _param_dtype(self) -> torch.dtype:
        return self.conv1d.weight.dtype

    def _check_io(self, x: torch.Tensor, what: str):
        if not x.is_cuda or not self.conv1d.weight.is_cuda:
            raise RuntimeError(f"{what}: cpu_mamba_b200 runs on CUDA devices only; move the "
                               "module and its inputs to the GPU (.cuda())")
        if x.dtype != self._param_dtype():
            raise RuntimeError(f"{what}: input dtype {x.dtype} does not match the parameter "
                               f"dtype {self._param_dtype()}")
        dtype_code(x.dtype)

    def _tf32_split(self, name: str, w: torch.Tensor):
        """TF32 hi/lo halves of an fp32 weight (derived cache, not module state)."""
        key = (w.data_ptr(), w._version, tuple(w.shape))
        ent = self._split_cache.get(name)
        if ent is None or ent[0] != key:
            ent = (key, ops.split_tf32(w))
            self._split_cache[name] = ent
        return ent[1]

    def _f16_split(self, name: str, w: torch.Tensor):
        """Scaled fp16 halves of an fp32 weight for the F16X3 tensor-core GEMM
        (derived cache, not module state)."""
        key = (w.data_ptr(), w._version, tuple(w.shape))
        ent = self._split_cache.get("f16:" + name)
        if ent is None or ent[0] != key:
            ent = (key, ops.split_f16(w))
            self._split_cache["f16:" + name] = ent
        return ent[1]

    def _linear_desc(self, name: str, keep: list) -> LinearW:
        mod = getattr(self, name)
        d = LinearW()
        if isinstance(mod, QuantizedLinear):
            d.weight_q = mod.weight_q.data_ptr()
            scale = mod.scale if mod.scale.dtype == torch.float32 else mod.scale.float()
            keep.append(scale)
            d.scale = scale.data_ptr()
            d.scheme = _lib.SCHEMES[mod.scheme]
            d.group_size = mod.group_size or 0
            if name == "dt_proj":
                # dt_proj runs densely (the tensor-core dt GEMM, or W_dt's rows
                # in the fused scan): pass deq(W) and, in fp32, its TF32 halves
                dense = mod.dense_weight(self._param_dtype())
                keep.append(dense)
                d.weight = dense.data_ptr()
                if dense.dtype == torch.float32:
                    d.weight_split = self._tf32_split("dt_proj_deq", dense).data_ptr()
                    if dense.shape[1] % 8 == 0:
                        d.weight_f16 = self._f16_split("dt_proj_deq", dense).data_ptr()
        elif isinstance(mod, nn.Linear):
            w = mod.weight
            if not w.is_contiguous():
                w = w.contiguous()
                keep.append(w)
            d.weight = w.data_ptr()
            d.scheme = 0
            if w.dtype == torch.float32:
                d.weight_split = self._tf32_split(name, w).data_ptr()
                if w.shape[1] % 8 == 0:
                    # prefill projections (>= 256 rows) on the fp16 tensor cores
                    d.weight_f16 = self._f16_split(name, w).data_ptr()
        else:
            raise TypeError(f"{name} must be nn.Linear or QuantizedLinear, got {type(mod)}")
        d.bias = mod.bias.data_ptr() if mod.bias is not None else None
        return d

    def _descriptor(self, keep: list) -> Block:
        b = Block()
        b.d_model, b.d_inner, b.d_state = self.d_model, self.d_inner, self.d_state
        b.d_conv, b.dt_rank = self.d_conv, self.dt_rank
        b.dtype = dtype_code(self._param_dtype())
        for name in ("in_proj", "x_proj", "dt_proj", "out_proj"):
            setattr(b, name, self._linear_desc(name, keep))
        for name, t in (("conv_w", self.conv1d.weight), ("A_log", self.A_log), ("D", self.D)):
            if not t.is_contiguous():
                t = t.contiguous()
                keep.append(t)
            setattr(b, name, t.data_ptr())
        b.conv_b = self.conv1d.bias.data_ptr() if self.conv1d.bias is not None else None
        for t in (self.A_log, self.D, self.conv1d.bias):
            if t is not None and t.dtype != self._param_dtype():
                raise RuntimeError("A_log, D and conv1d.bias must share the parameter dtype")
        return b

    # ---------------------------------------------------------------- forward
    def _run(self, x: torch.Tensor, want_state: bool, out: torch.Tensor | None = None,
             blk: Block | None = None):
        B, T, D = x.shape
        if D != self.d_model:
            raise RuntimeError(f"expected d_model={self.d_model}, got input of shape {tuple(x.shape)}")
        self._check_io(x, "forward")
        x = x.contiguous()
        keep = []
        if blk is None:
            blk = self._descriptor(keep)
        ws_bytes = lib().mb2_block_workspace_bytes(ctypes.byref(blk), B, T)
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x.device)
        if out is None:
            out = torch.empty_like(x)
        h = conv = None
        if want_state:
            h = torch.empty(B, self.d_inner, self.d_state, device=x.device, dtype=torch.float32)
            conv = torch.empty(B, self.d_inner, self.d_conv - 1, device=x.device, dtype=x.dtype)
        check(lib().mb2_block_forward(ctypes.byref(blk), x.data_ptr(), out.data_ptr(), B, T,
                                      None if h is None else h.data_ptr(),
                                      None if conv is None else conv.data_ptr(),
                                      ws.data_ptr(), ws_bytes, stream_of(x)), "forward")
        return out, h, conv

    def profile_stages(self, hidden_states: torch.Tensor) -> dict:
        """One forward with CUDA events between its six stages (the launches
        forward() makes, on the current stream); returns each stage's ms."""
        x = hidden_states.contiguous()
        B, T, _ = x.shape
        self._check_io(x, "forward")
        keep = []
        blk = self._descriptor(keep)
        ws_bytes = lib().mb2_block_workspace_bytes(ctypes.byref(blk), B, T)
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x.device)
        out = torch.empty_like(x)
        ms = (ctypes.c_float * 6)()
        check(lib().mb2_block_forward_profile(ctypes.byref(blk), x.data_ptr(), out.data_ptr(), B, T,
                                              ws.data_ptr(), ws_bytes, ms, stream_of(x)),
              "profile_stages")
        names = ("in_proj", "conv1d_silu", "x_proj", "dt_proj", "scan", "out_proj")
        return dict(zip(names, (float(v) for v in ms)))

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        """hidden_states: (B, T, d_model) -> (B, T, d_model) (_mamba.py:204-265)."""
        return self._run(hidden_states, False)[0]

    def forward_host(self, hidden_states: torch.Tensor, out: torch.Tensor | None = None,
                     chunks: int | None = None) -> torch.Tensor:
        """forward() for a batch held in host memory; returns a host tensor.

        The batch is cut into ``chunks`` slices along B.  Each slice is copied
        to the GPU on one stream, run through the block on one of two compute
        streams and copied back on another, so PCIe transfers in both
        directions overlap the block's kernels (pinned host memory is needed for the
        copies to be asynchronous).  Batch rows are independent, so the result
        is ``forward`` on the whole batch: bit for bit when the slices and the
        whole batch use the same projection kernel (the tensor-core GEMM takes
        256 rows and more, the CUDA-core GEMM fewer), else to within the two
        kernels' rounding.  ``out`` (host, same shape and
        dtype) receives the result if given.  Returns once the result is in
        host memory."""
        x = hidden_states
        if x.is_cuda:
            raise RuntimeError("forward_host: hidden_states must be a host tensor; use forward()")
        B, T, D = x.shape
        dev = self.conv1d.weight.device
        if out is None:
            out = torch.empty(x.shape, dtype=x.dtype, pin_memory=x.is_pinned())
        if out.shape != x.shape or out.dtype != x.dtype or out.is_cuda:
            raise RuntimeError("forward_host: out must be a host tensor shaped like the input")
        x = x.contiguous()
        n = chunks if chunks is not None else max(1, min(8, B * T // 4096))
        keep = []
        blk = self._descriptor(keep)
        return run_streamed(x, out, dev,
                            lambda xd, yd: self._run(xd, False, out=yd, blk=blk),
                            n, self._host_slots, self._host_edge)

    def capture_step(self, state: dict, example: torch.Tensor) -> "StepGraph":
        """A CUDA graph of forward_step for this state dict and batch size
        (see StepGraph): call it with each token's (B, d_model) input."""
        return StepGraph(self, state, example)

    def forward_with_final_state(self, hidden_states: torch.Tensor) -> tuple:
        """(y, {"h": (B, d_inner, d_state) f32, "conv_state": (B, d_inner, d_conv-1)})
        from one pass (_mamba.py:165-202)."""
        y, h, conv = self._run(hidden_states, True)
        return y, {"h": h, "conv_state": conv}

    def forward_step(self, x_step: torch.Tensor, state: dict) -> tuple:
        """One autoregressive step (_mamba.py:103-163).

        x_step: (B, d_model) or (B, 1, d_model).  Returns (y (B, d_model), state);
        state["h"] and state["conv_state"] are updated in place."""
        if x_step.dim() == 3:
            assert x_step.shape[1] == 1, "forward_step expects T=1"
            x_step = x_step.squeeze(1)
        elif x_step.dim() != 2:
            raise ValueError(f"x_step must be (B, D) or (B, 1, D), got {x_step.shape}")
        B, D = x_step.shape
        assert D == self.d_model
        self._check_io(x_step, "forward_step")
        x_step = x_step.contiguous()
        h, conv = state["h"], state["conv_state"]
        if (h.shape != (B, self.d_inner, self.d_state) or
                conv.shape != (B, self.d_inner, self.d_conv - 1)):
            raise RuntimeError("state shapes do not match the block / batch")
        if h.dtype != torch.float32 or not h.is_contiguous() or h.device != x_step.device:
            h = h.to(device=x_step.device, dtype=torch.float32).contiguous()
            state["h"] = h
        if conv.dtype != x_step.dtype or not conv.is_contiguous() or conv.device != x_step.device:
            conv = conv.to(device=x_step.device, dtype=x_step.dtype).contiguous()
            state["conv_state"] = conv
        keep = []
        blk = self._descriptor(keep)
        ws_bytes = lib().mb2_step_workspace_bytes(ctypes.byref(blk), B)
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x_step.device)
        out = torch.empty_like(x_step)
        check(lib().mb2_block_step(ctypes.byref(blk), x_step.data_ptr(), out.data_ptr(),
                                   h.data_ptr(), conv.data_ptr(), B, ws.data_ptr(), ws_bytes,
                                   stream_of(x_step)), "forward_step")
        return out, state


class StepGraph:
    """``forward_step`` captured once as a CUDA graph for a fixed batch size and
    a fixed state dict, then replayed per token: one graph launch instead of
    the step's host work and kernel launches.

    ``state["h"]`` and ``state["conv_state"]`` are advanced in place by every
    call, exactly as ``forward_step`` does.  The returned output tensor is a
    buffer owned by the graph, overwritten by the next call.  Capture runs one
    warm-up step on a copy of the state first (library set-up happens outside
    the capture); the captured state is not modified by the capture itself.
    Rebuild the graph after changing the module's parameters."""

    def __init__(self, block: "CPUMamba", state: dict, example: torch.Tensor):
        if example.dim() == 3:
            example = example.squeeze(1)
        h, conv = state["h"], state["conv_state"]
        if (h.dtype != torch.float32 or not h.is_contiguous() or not conv.is_contiguous()
                or conv.dtype != example.dtype or h.device != example.device):
            raise RuntimeError("StepGraph: state must be contiguous on the input's device, "
                               "h float32 and conv_state in the input dtype (init_state)")
        self.block, self.state = block, state
        self.x = example.detach().clone().contiguous()
        dev = self.x.device
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side), torch.no_grad():
            block.forward_step(self.x, {k: v.clone() for k, v in state.items()})
        torch.cuda.current_stream(dev).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.no_grad(), torch.cuda.graph(self.graph):
            self.y, _ = block.forward_step(self.x, state)

    def __call__(self, x_step: torch.Tensor) -> torch.Tensor:
        self.x.copy_(x_step.reshape(self.x.shape), non_blocking=True)
        self.graph.replay()
        return self.y


def assert_state_dict_compatible(cpu_mamba: CPUMamba, sd: dict):
    """Raise ValueError when ``sd`` cannot be loaded into ``cpu_mamba``: keys it
    has and the module lacks, keys it lacks, or the first tensor whose shape
    differs (the messages of _mamba.py:268-279)."""
    own = cpu_mamba.state_dict()
    for label, keys in (("unexpected keys in source state_dict", set(sd) - set(own)),
                        ("missing keys in source state_dict", set(own) - set(sd))):
        if keys:
            raise ValueError(f"{label}: {sorted(keys)}")
    mismatched = [k for k in own if own[k].shape != sd[k].shape]
    if mismatched:
        k = mismatched[0]
        raise ValueError(f"shape mismatch on {k}: own {own[k].shape} vs src {sd[k].shape}")
