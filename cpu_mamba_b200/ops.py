"""Tensor-level ops over the C ABI (CUDA tensors in, CUDA tensors out).

selective_scan mirrors the reference's native op selective_scan_cpu
(src/cpu_mamba/selective_scan_cpu.cpp:19-41): same arguments, same checks and
RuntimeError messages, newly allocated output.  The other ops expose the fused
stages of the block for tests and for callers composing their own pipeline.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _lib
from ._lib import check, dtype_code, lib, ptr, require_cuda, stream_of


def selective_scan(x, dt, A, B, C, D, h0: Optional[torch.Tensor] = None,
                   return_last_state: bool = False):
    """GPU drop-in for selective_scan_cpu(x, dt, A, B, C, D) -> y.

    x, dt: (batch, T, d_inner); A: (d_inner, d_state); B, C: (batch, T, d_state);
    D: (d_inner).  All contiguous float32 (the reference's contract, cpp:27-32).
    Optional h0 / return_last_state carry the recurrence state across calls.
    """
    tensors = (x, dt, A, B, C, D)
    if not all(t.is_contiguous() for t in tensors):
        raise RuntimeError("all inputs must be contiguous")
    if x.dtype != torch.float32:
        raise RuntimeError("fp32 only in this build")
    if not (x.dim() == 3 and dt.dim() == 3 and A.dim() == 2 and B.dim() == 3
            and C.dim() == 3 and D.dim() == 1):
        raise RuntimeError("shape mismatch")
    require_cuda(*tensors, h0, what="selective_scan")
    bsz, T, di = x.shape
    S = A.shape[1]
    if S > 256:
        raise RuntimeError("d_state > 256 not supported (stack limit)")
    if (dt.shape != x.shape or A.shape[0] != di or B.shape != (bsz, T, S)
            or C.shape != (bsz, T, S) or D.shape[0] != di):
        raise RuntimeError("shape mismatch")
    if any(t.dtype != torch.float32 for t in tensors):
        raise RuntimeError("fp32 only in this build")
    if h0 is not None:
        h0 = h0.contiguous()
        if h0.shape != (bsz, di, S) or h0.dtype != torch.float32:
            raise RuntimeError("h0 must be float32 (batch, d_inner, d_state)")
    y = torch.empty_like(x)
    h_last = torch.empty(bsz, di, S, device=x.device, dtype=torch.float32) if return_last_state else None
    check(lib().mb2_selective_scan(ptr(x), ptr(dt), ptr(A), ptr(B), ptr(C), ptr(D), ptr(y),
                                   bsz, T, di, S, ptr(h0), ptr(h_last), stream_of(x)),
          "selective_scan")
    return (y, h_last) if return_last_state else y


def conv1d_silu(x_in: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor],
                batch: int, seqlen: int, d_inner: int, return_tail: bool = False,
                out: Optional[torch.Tensor] = None):
    """silu(causal depthwise conv1d(x) + bias) over rows of x_in (token-major,
    first d_inner columns; row stride = x_in.stride(0)).  weight: (d_inner, 1, K)
    or (d_inner, K)."""
    require_cuda(x_in, weight, bias, what="conv1d_silu")
    if x_in.stride(-1) != 1:
        raise RuntimeError("conv1d_silu: rows must be contiguous")
    K = weight.shape[-1]
    w = weight.reshape(d_inner, K).contiguous()
    xc = out if out is not None else torch.empty(batch * seqlen, d_inner, device=x_in.device,
                                                 dtype=x_in.dtype)
    tail = (torch.empty(batch, d_inner, K - 1, device=x_in.device, dtype=x_in.dtype)
            if return_tail else None)
    check(lib().mb2_conv1d_silu(dtype_code(x_in.dtype), ptr(x_in), x_in.stride(0), ptr(w),
                                ptr(bias), ptr(xc), xc.stride(0), ptr(tail), batch, seqlen,
                                d_inner, K, stream_of(x_in)), "conv1d_silu")
    return (xc, tail) if return_tail else xc


def scan_fused(xc, dt_low, Bm, Cm, z, w_dt, b_dt, A_log, D, batch, seqlen, h0=None,
               return_last_state=False, out=None):
    """The block's scan stage in one kernel: dt = softplus(dt_low W_dt^T + b_dt),
    A = -exp(A_log), selective scan, D skip, cast and SiLU(z) gate.

    xc, z: (N, d_inner) row views (N = batch*seqlen, any row stride);
    dt_low, Bm, Cm: (N, dt_rank) / (N, d_state) row views (e.g. the column
    slices of x_proj's output); w_dt: (d_inner, dt_rank).  Returns y (N, d_inner)."""
    require_cuda(xc, dt_low, Bm, Cm, z, w_dt, A_log, what="scan_fused")
    di, S = A_log.shape
    R = w_dt.shape[1]
    y = out if out is not None else torch.empty(batch * seqlen, di, device=xc.device, dtype=xc.dtype)
    h_last = (torch.empty(batch, di, S, device=xc.device, dtype=torch.float32)
              if return_last_state else None)
    A_log, w_dt = A_log.contiguous(), w_dt.contiguous()   # keep alive across the call
    h0 = None if h0 is None else h0.contiguous()
    check(lib().mb2_scan_fused(dtype_code(xc.dtype), ptr(xc), xc.stride(0), ptr(dt_low),
                               dt_low.stride(0), ptr(Bm), Bm.stride(0), ptr(Cm), Cm.stride(0),
                               ptr(z), z.stride(0), ptr(w_dt), ptr(b_dt), ptr(A_log), ptr(D),
                               ptr(h0), ptr(h_last), ptr(y), y.stride(0), batch, seqlen, di, S, R,
                               stream_of(xc)), "scan_fused")
    return (y, h_last) if return_last_state else y


def scan_gated(xc, dt, Bm, Cm, z, A_log, D, batch, seqlen, h0=None, return_last_state=False,
               out=None):
    """scan_fused given dt_proj's output dt = linear(dt_low, W_dt, b_dt) (before
    the softplus, which this kernel applies): A = -exp(A_log), selective scan,
    D skip, cast and SiLU(z) gate.
    xc, dt, z: (N, d_inner) row views; Bm, Cm: (N, d_state) row views."""
    require_cuda(xc, dt, Bm, Cm, z, A_log, what="scan_gated")
    di, S = A_log.shape
    y = out if out is not None else torch.empty(batch * seqlen, di, device=xc.device, dtype=xc.dtype)
    h_last = (torch.empty(batch, di, S, device=xc.device, dtype=torch.float32)
              if return_last_state else None)
    A_log = A_log.contiguous()
    h0 = None if h0 is None else h0.contiguous()
    # T-segment scratch for long sequences over few chains (0 bytes otherwise)
    ws_bytes = lib().mb2_scan_workspace_bytes(batch, seqlen, di, S)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=xc.device) if ws_bytes else None
    check(lib().mb2_scan_gated_ws(dtype_code(xc.dtype), ptr(xc), xc.stride(0), ptr(dt),
                                  dt.stride(0), ptr(Bm), Bm.stride(0), ptr(Cm), Cm.stride(0),
                                  ptr(z), z.stride(0), ptr(A_log), ptr(D), ptr(h0), ptr(h_last),
                                  ptr(y), y.stride(0), batch, seqlen, di, S, ptr(ws), ws_bytes,
                                  stream_of(xc)), "scan_gated")
    return (y, h_last) if return_last_state else y


def linear_recurrence(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """h[t] = a[t] * h[t-1] + b[t] (h[-1] = 0) along dim 1 of (B, T, ...)
    tensors: the reference's _associative_prefix_scan (scan_assoc.py:24-55)."""
    require_cuda(a, b, what="linear_recurrence")
    if a.shape != b.shape or a.dim() < 2:
        raise RuntimeError("linear_recurrence: a and b must have the same (B, T, ...) shape")
    if a.dtype != b.dtype:
        raise RuntimeError("linear_recurrence: a and b must share a dtype")
    a, b = a.contiguous(), b.contiguous()
    h = torch.empty_like(a)
    Bt, T = a.shape[0], a.shape[1]
    inner = a.numel() // max(Bt * T, 1) if a.numel() else 0
    check(lib().mb2_linear_recurrence(dtype_code(a.dtype), ptr(a), ptr(b), ptr(h), Bt, T, inner,
                                      stream_of(a)), "linear_recurrence")
    return h


def split_tf32(w: torch.Tensor) -> torch.Tensor:
    """(2, *w.shape) float32: TF32 hi and lo halves of w (a derived cache)."""
    require_cuda(w, what="split_tf32")
    w = w.detach().contiguous()
    if w.dtype != torch.float32:
        raise TypeError("split_tf32 needs float32")
    out = torch.empty((2,) + tuple(w.shape), device=w.device, dtype=torch.float32)
    check(lib().mb2_split_tf32(ptr(w), ptr(out), w.numel(), stream_of(w)), "split_tf32")
    return out


def split_f16(w: torch.Tensor) -> torch.Tensor:
    """The scaled fp16 halves of a float32 (N, K) weight for the F16X3 GEMM
    (mb2_split_f16's layout, a derived cache): a uint8 device buffer."""
    require_cuda(w, what="split_f16")
    w = w.detach().contiguous()
    if w.dtype != torch.float32 or w.dim() != 2:
        raise TypeError("split_f16 needs a float32 matrix")
    n = lib().mb2_split_f16_bytes(w.shape[0], w.shape[1])
    out = torch.empty(n, device=w.device, dtype=torch.uint8)   # 256-byte aligned by torch
    check(lib().mb2_split_f16(ptr(w), w.shape[0], w.shape[1], ptr(out), stream_of(w)),
          "split_f16")
    return out


def fold_norm(weight: torch.Tensor, norm_weight: torch.Tensor) -> torch.Tensor:
    """weight * norm_weight[None, :] rounded to weight's dtype: an RMSNorm
    weight folded into the columns of the projection that follows it."""
    require_cuda(weight, norm_weight, what="fold_norm")
    w = weight.detach().contiguous()
    g = norm_weight.detach().to(w.dtype).contiguous()
    if g.shape != (w.shape[-1],):
        raise RuntimeError(f"fold_norm: norm weight {tuple(g.shape)} vs weight {tuple(w.shape)}")
    out = torch.empty_like(w)
    check(lib().mb2_fold_norm(dtype_code(w.dtype), ptr(w), ptr(g), ptr(out), w.shape[0],
                              w.shape[-1], stream_of(w)), "fold_norm")
    return out


def linear(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
           weight_split: Optional[torch.Tensor] = None, softplus: bool = False,
           out: Optional[torch.Tensor] = None,
           weight_f16: Optional[torch.Tensor] = None, sm_pair: int = -1) -> torch.Tensor:
    """y = x W^T + b over the last dim of x (nn.Linear semantics); softplus=True
    applies F.softplus to the result in the same kernel (dt_proj's epilogue).
    float32 with weight_f16 (split_f16(weight)): the F16X3 tensor-core GEMM
    (sm_pair: 1 pairs of SMs, 0 or -1 single SMs); with
    weight_split (split_tf32(weight)): the 3xTF32 one."""
    require_cuda(x, weight, bias, what="linear")
    N, K = weight.shape
    lead = x.shape[:-1]
    x2 = x.reshape(-1, K)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    y = out if out is not None else torch.empty(x2.shape[0], N, device=x.device, dtype=x.dtype)
    if weight_f16 is not None and x.dtype == torch.float32:
        scratch = torch.empty(lib().mb2_linear_f16_scratch_bytes(), device=x.device,
                              dtype=torch.uint8)
        check(lib().mb2_linear_f16(ptr(x2), x2.stride(0), ptr(weight_f16), ptr(bias), ptr(y),
                                   y.stride(0), x2.shape[0], N, K,
                                   _lib.EPI_SOFTPLUS if softplus else _lib.EPI_NONE,
                                   sm_pair, ptr(scratch), stream_of(x)), "linear_f16")
        return y if out is not None else y.reshape(*lead, N)
    weight = weight.contiguous()
    check(lib().mb2_linear(dtype_code(x.dtype), ptr(x2), x2.stride(0), ptr(weight),
                           ptr(weight_split), ptr(bias), ptr(y), y.stride(0), x2.shape[0], N, K,
                           _lib.EPI_SOFTPLUS if softplus else _lib.EPI_NONE, stream_of(x)), "linear")
    return y if out is not None else y.reshape(*lead, N)


def quantize(scheme: str, w: torch.Tensor, group_size: Optional[int] = None
             ) -> Tuple[torch.Tensor, torch.Tensor, int]:
    """(weight_q, scale, in_dim) with quant.py's exact codes, on the GPU.
    group_size: None for quant.py's one scale per row, or the number of input
    columns per scale (blockwise; scale is then (rows, ceil(cols / group)))."""
    require_cuda(w, what="quantize")
    w = w.detach().to(torch.float32).contiguous()
    rows, cols = w.shape
    if scheme == "int8":
        q = torch.empty(rows, cols, device=w.device, dtype=torch.int8)
    else:
        q = torch.empty(rows, (cols + 1) // 2, device=w.device, dtype=torch.uint8)
    if group_size:
        s = torch.empty(rows, -(-cols // group_size), device=w.device, dtype=torch.float32)
        check(lib().mb2_quantize_grouped(_lib.SCHEMES[scheme], ptr(w), rows, cols, group_size,
                                         ptr(q), ptr(s), stream_of(w)), f"quantize_{scheme}")
    else:
        s = torch.empty(rows, device=w.device, dtype=torch.float32)
        check(lib().mb2_quantize(_lib.SCHEMES[scheme], ptr(w), rows, cols, ptr(q), ptr(s),
                                 stream_of(w)), f"quantize_{scheme}")
    return q, s, cols


def dequantize(scheme: str, weight_q: torch.Tensor, scale: torch.Tensor, in_dim: int,
               group_size: Optional[int] = None) -> torch.Tensor:
    require_cuda(weight_q, scale, what="dequantize")
    weight_q = weight_q.contiguous()
    scale = scale.to(torch.float32).contiguous()
    out = torch.empty(weight_q.shape[0], in_dim, device=weight_q.device, dtype=torch.float32)
    check(lib().mb2_dequantize_grouped(_lib.SCHEMES[scheme], ptr(weight_q), ptr(scale),
                                       weight_q.shape[0], in_dim, group_size or 0, ptr(out),
                                       stream_of(weight_q)), f"dequantize_{scheme}")
    return out


def qlinear(x: torch.Tensor, scheme: str, weight_q: torch.Tensor, scale: torch.Tensor,
            bias: Optional[torch.Tensor], in_features: int, softplus: bool = False,
            group_size: Optional[int] = None) -> torch.Tensor:
    """QuantizedLinear.forward: y = x deq(W)^T + b with W dequantised in-kernel."""
    require_cuda(x, weight_q, scale, bias, what="qlinear")
    N = weight_q.shape[0]
    lead = x.shape[:-1]
    x2 = x.reshape(-1, in_features)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    y = torch.empty(x2.shape[0], N, device=x.device, dtype=x.dtype)
    weight_q, scale = weight_q.contiguous(), scale.to(torch.float32).contiguous()
    check(lib().mb2_qlinear_grouped(_lib.SCHEMES[scheme], group_size or 0, dtype_code(x.dtype),
                                    ptr(x2), x2.stride(0), ptr(weight_q), ptr(scale), ptr(bias),
                                    ptr(y), N, x2.shape[0], N, in_features,
                            _lib.EPI_SOFTPLUS if softplus else _lib.EPI_NONE, stream_of(x)),
          f"qlinear_{scheme}")
    return y.reshape(*lead, N)
