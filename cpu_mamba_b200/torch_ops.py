"""The library's ops registered with torch, namespace ``mamba_b200``.

The reference loads its native op as a torch extension
(src/cpu_mamba/_mamba.py:37-43) and calls ``selective_scan_cpu(x, dt, A, B,
C, D)``; here the same op, and the quantisation ops and the decode step, are
torch custom ops, callable as ``torch.ops.mamba_b200.<name>`` and traceable
(each has a fake implementation that only computes output shapes):

  selective_scan(x, dt, A, B, C, D) -> y                 (the drop-in's signature)
  selective_scan_state(x, dt, A, B, C, D, h0?) -> (y, h_last)
  quant_pack(w, scheme, group_size=0) -> (weight_q, scale)
  dequant(weight_q, scale, scheme, in_dim, group_size=0) -> w (float32)
  qlinear(x, weight_q, scale, bias?, scheme, in_dim, group_size=0) -> y
  mamba_step(x, h, conv_state, in_proj_w, conv_w, conv_b?, x_proj_w, dt_proj_w,
             dt_proj_b?, A_log, D, out_proj_w) -> y   (h, conv_state updated in place)

Each runs the C-ABI kernels on the inputs' CUDA device and current stream
(no CPU implementation: CPU tensors raise, as the rest of the package does).
``mamba_step`` takes dense weights; its fp32 projections run on the CUDA-core
GEMM (a module's forward_step, which caches the weights' TF32 halves, uses
the tensor cores).
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import ops
from ._lib import Block, LinearW, check, dtype_code, lib, stream_of

NS = "mamba_b200"


@torch.library.custom_op(f"{NS}::selective_scan", mutates_args=())
def selective_scan(x: torch.Tensor, dt: torch.Tensor, A: torch.Tensor, B: torch.Tensor,
                   C: torch.Tensor, D: torch.Tensor) -> torch.Tensor:
    return ops.selective_scan(x, dt, A, B, C, D)


@selective_scan.register_fake
def _(x, dt, A, B, C, D):
    return torch.empty_like(x)


@torch.library.custom_op(f"{NS}::selective_scan_state", mutates_args=())
def selective_scan_state(x: torch.Tensor, dt: torch.Tensor, A: torch.Tensor, B: torch.Tensor,
                         C: torch.Tensor, D: torch.Tensor,
                         h0: Optional[torch.Tensor] = None) -> tuple[torch.Tensor, torch.Tensor]:
    return ops.selective_scan(x, dt, A, B, C, D, h0=h0, return_last_state=True)


@selective_scan_state.register_fake
def _(x, dt, A, B, C, D, h0=None):
    return torch.empty_like(x), x.new_empty(x.shape[0], x.shape[2], A.shape[1])


@torch.library.custom_op(f"{NS}::quant_pack", mutates_args=())
def quant_pack(w: torch.Tensor, scheme: str, group_size: int = 0) -> tuple[torch.Tensor,
                                                                            torch.Tensor]:
    q, s, _ = ops.quantize(scheme, w, group_size or None)
    return q, s


@quant_pack.register_fake
def _(w, scheme, group_size=0):
    rows, cols = w.shape
    q = (w.new_empty(rows, cols, dtype=torch.int8) if scheme == "int8"
         else w.new_empty(rows, (cols + 1) // 2, dtype=torch.uint8))
    s = (w.new_empty(rows, -(-cols // group_size), dtype=torch.float32) if group_size
         else w.new_empty(rows, dtype=torch.float32))
    return q, s


@torch.library.custom_op(f"{NS}::dequant", mutates_args=())
def dequant(weight_q: torch.Tensor, scale: torch.Tensor, scheme: str, in_dim: int,
            group_size: int = 0) -> torch.Tensor:
    return ops.dequantize(scheme, weight_q, scale, in_dim, group_size or None)


@dequant.register_fake
def _(weight_q, scale, scheme, in_dim, group_size=0):
    return weight_q.new_empty(weight_q.shape[0], in_dim, dtype=torch.float32)


@torch.library.custom_op(f"{NS}::qlinear", mutates_args=())
def qlinear(x: torch.Tensor, weight_q: torch.Tensor, scale: torch.Tensor,
            bias: Optional[torch.Tensor], scheme: str, in_dim: int,
            group_size: int = 0) -> torch.Tensor:
    return ops.qlinear(x, scheme, weight_q, scale, bias, in_dim, group_size=group_size or None)


@qlinear.register_fake
def _(x, weight_q, scale, bias, scheme, in_dim, group_size=0):
    return x.new_empty(*x.shape[:-1], weight_q.shape[0])


def _dense(w: torch.Tensor, bias: Optional[torch.Tensor], keep: list) -> LinearW:
    d = LinearW()
    w = w.contiguous()
    keep.append(w)
    d.weight = w.data_ptr()
    if bias is not None:
        bias = bias.contiguous()
        keep.append(bias)
        d.bias = bias.data_ptr()
    return d


@torch.library.custom_op(f"{NS}::mamba_step", mutates_args=("h", "conv_state"))
def mamba_step(x: torch.Tensor, h: torch.Tensor, conv_state: torch.Tensor,
               in_proj_w: torch.Tensor, conv_w: torch.Tensor, conv_b: Optional[torch.Tensor],
               x_proj_w: torch.Tensor, dt_proj_w: torch.Tensor,
               dt_proj_b: Optional[torch.Tensor], A_log: torch.Tensor, D: torch.Tensor,
               out_proj_w: torch.Tensor) -> torch.Tensor:
    """forward_step (_mamba.py:103-163) of a block given as its tensors."""
    B, dm = x.shape
    di, S = A_log.shape
    K = conv_w.shape[-1]
    R = dt_proj_w.shape[1]
    if (h.shape != (B, di, S) or h.dtype != torch.float32 or not h.is_contiguous()
            or conv_state.shape != (B, di, K - 1) or conv_state.dtype != x.dtype
            or not conv_state.is_contiguous()):
        raise RuntimeError("mamba_step: h (B, d_inner, d_state) fp32 and conv_state "
                           "(B, d_inner, d_conv-1) in x's dtype, both contiguous")
    keep = []
    b = Block()
    b.d_model, b.d_inner, b.d_state, b.d_conv, b.dt_rank = dm, di, S, K, R
    b.dtype = dtype_code(x.dtype)
    b.in_proj = _dense(in_proj_w, None, keep)
    b.x_proj = _dense(x_proj_w, None, keep)
    b.dt_proj = _dense(dt_proj_w, dt_proj_b, keep)
    b.out_proj = _dense(out_proj_w, None, keep)
    for name, t in (("conv_w", conv_w), ("conv_b", conv_b), ("A_log", A_log), ("D", D)):
        if t is not None:
            t = t.contiguous()
            keep.append(t)
            setattr(b, name, t.data_ptr())
    x = x.contiguous()
    ws_bytes = lib().mb2_step_workspace_bytes(ctypes.byref(b), B)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x.device)
    out = torch.empty_like(x)
    check(lib().mb2_block_step(ctypes.byref(b), x.data_ptr(), out.data_ptr(), h.data_ptr(),
                               conv_state.data_ptr(), B, ws.data_ptr(), ws_bytes, stream_of(x)),
          "mamba_step")
    return out


@mamba_step.register_fake
def _(x, h, conv_state, in_proj_w, conv_w, conv_b, x_proj_w, dt_proj_w, dt_proj_b, A_log, D,
      out_proj_w):
    return torch.empty_like(x)
