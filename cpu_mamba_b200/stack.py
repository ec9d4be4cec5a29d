"""MambaStack -- a residual stack of pre-norm Mamba blocks on the B200 library.

x <- x + CPUMamba(RMSNorm(x)) for each layer: the composition a
Mamba-130M-style model makes around the block (24 layers of d_model 768).  The
reference has no stack; it would be composed from its CPUMamba
(src/cpu_mamba/_mamba.py:49-279) and torch.nn.RMSNorm.  Parameter names follow
mamba_ssm's MixerModel layout: ``layers.{i}.norm.weight`` and
``layers.{i}.mixer.<CPUMamba parameters>``.

The whole stack is one C-ABI call (mb2_stack_forward): per layer a row-RMS
pass and the block's five kernels, the norm weight folded into in_proj's
columns (a derived cache, like the TF32 split of fp32 weights), 1/rms applied
in in_proj's epilogue and the residual added in out_proj's epilogue in place.
"""
from __future__ import annotations

import ctypes

import torch
import torch.nn as nn

from . import ops
from ._lib import Block, check, lib, stream_of
from .module import CPUMamba
from .quant import QuantizedLinear
from .streaming import run_streamed


class MambaLayer(nn.Module):
    """RMSNorm pre-norm + CPUMamba mixer (one residual layer)."""

    def __init__(self, d_model: int, eps: float = 1e-5, device=None, dtype=None, **block_kw):
        super().__init__()
        self.norm = nn.RMSNorm(d_model, eps=eps, device=device, dtype=dtype)
        self.mixer = CPUMamba(d_model, device=device, dtype=dtype, **block_kw)


class MambaStack(nn.Module):
    """n_layers residual pre-norm Mamba blocks; forward((B, T, d_model)) ->
    the residual stream after the last layer (no final norm)."""

    # see CPUMamba: device slices in flight and end-slice weight of forward_host
    _host_slots = 3
    _host_edge = 0.5

    def __init__(self, n_layers: int, d_model: int, d_state: int = 16, d_conv: int = 4,
                 expand: int = 2, dt_rank="auto", eps: float = 1e-5, device=None, dtype=None,
                 **block_kw):
        super().__init__()
        if n_layers < 1:
            raise ValueError("n_layers must be >= 1")
        self.d_model = d_model
        self.eps = float(eps)
        self.layers = nn.ModuleList([
            MambaLayer(d_model, eps=eps, device=device, dtype=dtype, d_state=d_state,
                       d_conv=d_conv, expand=expand, dt_rank=dt_rank, **block_kw)
            for _ in range(n_layers)])
        self._fold_cache = {}

    def _folded_in_proj(self, i: int, layer: MambaLayer):
        """W_in * g (and its TF32 halves for fp32): derived, not module state."""
        w, g = layer.mixer.in_proj.weight, layer.norm.weight
        key = (w.data_ptr(), w._version, g.data_ptr(), g._version, w.dtype)
        ent = self._fold_cache.get(i)
        if ent is None or ent[0] != key:
            folded = ops.fold_norm(w, g)
            fp32 = folded.dtype == torch.float32
            split = ops.split_tf32(folded) if fp32 else None
            split16 = ops.split_f16(folded) if fp32 and folded.shape[1] % 8 == 0 else None
            ent = (key, folded, split, split16)
            self._fold_cache[i] = ent
        return ent[1], ent[2], ent[3]

    def _descriptors(self, keep: list):
        n = len(self.layers)
        arr = (Block * n)()
        for i, layer in enumerate(self.layers):
            if isinstance(layer.mixer.in_proj, QuantizedLinear):
                raise NotImplementedError(
                    "MambaStack: a quantised in_proj cannot absorb the RMSNorm weight; "
                    "quantise x_proj / dt_proj / out_proj only, or run the layers one by one")
            if layer.norm.eps != self.eps:
                raise RuntimeError("MambaStack: all layers must share the stack's RMSNorm eps")
            b = layer.mixer._descriptor(keep)
            folded, split, split16 = self._folded_in_proj(i, layer)
            keep.extend([folded, split, split16])
            b.in_proj.weight = folded.data_ptr()
            b.in_proj.weight_split = split.data_ptr() if split is not None else None
            b.in_proj.weight_f16 = split16.data_ptr() if split16 is not None else None
            arr[i] = b
        return arr

    def _run_inplace(self, x: torch.Tensor, arr) -> None:
        B, T, D = x.shape
        n = len(self.layers)
        ws_bytes = lib().mb2_stack_workspace_bytes(arr, n, B, T)
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x.device)
        check(lib().mb2_stack_forward(arr, n, ctypes.c_float(self.eps), x.data_ptr(), B, T,
                                      ws.data_ptr(), ws_bytes, stream_of(x)), "stack_forward")

    def _check(self, x: torch.Tensor):
        if x.dim() != 3 or x.shape[-1] != self.d_model:
            raise RuntimeError(f"expected (B, T, {self.d_model}), got {tuple(x.shape)}")
        self.layers[0].mixer._check_io(x, "MambaStack")

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        """(B, T, d_model) -> (B, T, d_model); the input is not modified."""
        self._check(hidden_states)
        x = hidden_states.contiguous().clone()
        keep = []
        self._run_inplace(x, self._descriptors(keep))
        return x

    def forward_(self, hidden_states: torch.Tensor) -> torch.Tensor:
        """forward() overwriting the (contiguous) input with the result."""
        self._check(hidden_states)
        if not hidden_states.is_contiguous():
            raise RuntimeError("forward_: the residual stream must be contiguous")
        keep = []
        self._run_inplace(hidden_states, self._descriptors(keep))
        return hidden_states

    # ------------------------------------------------------------ decode
    def init_state(self, batch_size: int, device=None, dtype=None) -> list:
        """Zero decode state, one CPUMamba.init_state dict per layer."""
        return [layer.mixer.init_state(batch_size, device, dtype) for layer in self.layers]

    def _state_ptrs(self, states: list, B: int, x: torch.Tensor):
        n = len(self.layers)
        if len(states) != n:
            raise RuntimeError(f"expected {n} layer states, got {len(states)}")
        hs, cs = (ctypes.c_void_p * n)(), (ctypes.c_void_p * n)()
        for i, (layer, st) in enumerate(zip(self.layers, states)):
            m, h, c = layer.mixer, st["h"], st["conv_state"]
            if (h.shape != (B, m.d_inner, m.d_state) or h.dtype != torch.float32
                    or not h.is_contiguous() or h.device != x.device
                    or c.shape != (B, m.d_inner, m.d_conv - 1) or c.dtype != x.dtype
                    or not c.is_contiguous() or c.device != x.device):
                raise RuntimeError(f"layer {i}: state must be init_state's layout on the "
                                   "input's device")
            hs[i], cs[i] = h.data_ptr(), c.data_ptr()
        return hs, cs

    def forward_with_final_state(self, hidden_states: torch.Tensor) -> tuple:
        """(y, [per-layer {"h", "conv_state"}]): forward() plus every layer's
        final state (CPUMamba.forward_with_final_state per layer)."""
        self._check(hidden_states)
        x = hidden_states.contiguous().clone()
        B, T, _ = x.shape
        states = self.init_state(B, x.device, x.dtype)
        hs, cs = self._state_ptrs(states, B, x)
        keep = []
        arr = self._descriptors(keep)
        n = len(self.layers)
        ws_bytes = lib().mb2_stack_workspace_bytes(arr, n, B, T)
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x.device)
        check(lib().mb2_stack_forward_state(arr, n, ctypes.c_float(self.eps), x.data_ptr(), B, T,
                                            hs, cs, ws.data_ptr(), ws_bytes, stream_of(x)),
              "stack_forward_state")
        return x, states

    def forward_step(self, x_step: torch.Tensor, states: list) -> tuple:
        """One token through every layer: (B, d_model) or (B, 1, d_model) ->
        the residual stream after the last layer (B, d_model); each layer's
        state is advanced in place (CPUMamba.forward_step per layer)."""
        if x_step.dim() == 3:
            x_step = x_step.squeeze(1)
        if x_step.dim() != 2 or x_step.shape[-1] != self.d_model:
            raise RuntimeError(f"expected (B, {self.d_model}), got {tuple(x_step.shape)}")
        self.layers[0].mixer._check_io(x_step, "MambaStack.forward_step")
        x = x_step.contiguous().clone()
        B = x.shape[0]
        hs, cs = self._state_ptrs(states, B, x)
        keep = []
        arr = self._descriptors(keep)
        n = len(self.layers)
        ws_bytes = lib().mb2_stack_step_workspace_bytes(arr, n, B)
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x.device)
        check(lib().mb2_stack_step(arr, n, ctypes.c_float(self.eps), x.data_ptr(), hs, cs, B,
                                   ws.data_ptr(), ws_bytes, stream_of(x)), "stack_step")
        return x, states

    def forward_host(self, hidden_states: torch.Tensor, out: torch.Tensor | None = None,
                     chunks: int | None = None) -> torch.Tensor:
        """forward() for a batch in host memory, streamed through the GPU in
        batch slices with the copies overlapping the layers' kernels (see
        CPUMamba.forward_host).  Returns the host result once it is there."""
        x = hidden_states
        if x.is_cuda:
            raise RuntimeError("forward_host: hidden_states must be a host tensor; use forward()")
        B, T, D = x.shape
        dev = self.layers[0].mixer.conv1d.weight.device
        if out is None:
            out = torch.empty(x.shape, dtype=x.dtype, pin_memory=x.is_pinned())
        if out.shape != x.shape or out.dtype != x.dtype or out.is_cuda:
            raise RuntimeError("forward_host: out must be a host tensor shaped like the input")
        keep = []
        arr = self._descriptors(keep)

        def run(xd, yd):
            yd.copy_(xd)
            self._run_inplace(yd, arr)

        n = chunks if chunks is not None else max(1, min(8, B * T // 4096))
        return run_streamed(x.contiguous(), out, dev, run, n, self._host_slots, self._host_edge)
