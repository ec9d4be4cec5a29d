"""Weight-only int8 / int4 / nf4 quantisation with the API of
src/cpu_mamba/quant.py: QuantConfig, quantize_/dequantize_{int8,int4,nf4},
QuantizedLinear (buffers ``weight_q`` and ``scale``), quantize_block and
memory_footprint.

Codes, packed bytes, scales and dequantised weights are bit-exact with the
reference (quant.py:60-134); the arithmetic runs in CUDA kernels
(csrc/quant.cu).  QuantizedLinear.forward never materialises the dequantised
weight: the GEMM's weight loader dequantises tiles on the fly (csrc/gemm_simt.cu).

Tensors on the CPU are quantised on the current CUDA device and the results
returned to the input's device, so a module can be quantised before or after
``.cuda()``.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Iterable, Optional

import torch
import torch.nn as nn

from . import ops

_NF4_LUT_VALUES = (
    -1.0, -0.6961928, -0.5250730, -0.39491748,
    -0.28444138, -0.18477343, -0.09105602, 0.0,
    0.07958029, 0.16093020, 0.24611230, 0.33791524,
    0.44070983, 0.56261897, 0.72295684, 1.0,
)  # QLoRA NormalFloat-4 code book, as in quant.py:35-40


@dataclass
class QuantConfig:
    """quant.py:47-53, plus ``group_size``: None keeps the reference's one scale
    per output channel; an integer (e.g. 64) quantises blockwise, one scale per
    run of that many input columns (the reference's roadmap item "blockwise
    NF4 (group_size=64)", README.md:115, :201)."""
    scheme: str = "int8"  # "int8" | "int4" | "nf4"
    group_size: Optional[int] = None

    def __post_init__(self):
        if self.scheme not in ("int8", "int4", "nf4"):
            raise ValueError(f"unknown scheme {self.scheme!r}")
        _check_group(self.scheme, self.group_size)


def _check_group(scheme, group_size):
    if group_size is None:
        return
    if not isinstance(group_size, int) or group_size < 1:
        raise ValueError(f"group_size must be a positive int or None, got {group_size!r}")
    if scheme != "int8" and group_size % 2:
        raise ValueError("4-bit schemes pack column pairs: group_size must be even")


def _on_gpu(t: torch.Tensor) -> torch.Tensor:
    if t.is_cuda:
        return t
    if not torch.cuda.is_available():
        raise RuntimeError("cpu_mamba_b200 quantisation runs on a CUDA device; none is available")
    return t.to("cuda")


def _quant(scheme, weight, group_size=None):
    w = _on_gpu(weight.detach())
    q, s, in_dim = ops.quantize(scheme, w, group_size)
    return q.to(weight.device), s.to(weight.device), in_dim


def _dequant(scheme, wq, scale, in_dim, group_size=None):
    out = ops.dequantize(scheme, _on_gpu(wq), _on_gpu(scale), in_dim, group_size)
    return out.to(wq.device)


def quantize_int8(weight: torch.Tensor):
    """Per-channel symmetric int8 -> (w_q int8 (out, in), scale (out,))."""
    q, s, _ = _quant("int8", weight)
    return q, s


def dequantize_int8(w_q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    return _dequant("int8", w_q, scale, w_q.shape[1])


def quantize_int4(weight: torch.Tensor):
    """Per-channel symmetric int4, two codes per byte -> (packed, scale, in_dim)."""
    return _quant("int4", weight)


def dequantize_int4(packed: torch.Tensor, scale: torch.Tensor, in_dim: int) -> torch.Tensor:
    return _dequant("int4", packed, scale, in_dim)


def quantize_nf4(weight: torch.Tensor):
    """Per-channel NF4 codes, two per byte -> (packed, scale, in_dim)."""
    return _quant("nf4", weight)


def dequantize_nf4(packed: torch.Tensor, scale: torch.Tensor, in_dim: int) -> torch.Tensor:
    return _dequant("nf4", packed, scale, in_dim)


class QuantizedLinear(nn.Module):
    """Drop-in for nn.Linear with weight-only quantisation (quant.py:141-194).

    Buffers: ``weight_q`` (int8, or uint8 packed pairs) and ``scale`` (out,)
    float32 -- or (out, ceil(in / group_size)) when quantised blockwise;
    optional ``bias`` parameter.  ``scheme``, ``group_size`` and
    ``_packed_in_dim`` are plain attributes, as in the reference.
    """

    def __init__(self, weight: torch.Tensor, bias: Optional[torch.Tensor], scheme: str,
                 group_size: Optional[int] = None):
        super().__init__()
        if scheme not in ("int8", "int4", "nf4"):
            raise ValueError(f"unknown scheme {scheme!r}")
        _check_group(scheme, group_size)
        self.scheme = scheme
        self.group_size = group_size
        self.in_features = weight.shape[1]
        self.out_features = weight.shape[0]
        q, s, in_dim = _quant(scheme, weight, group_size)
        self.register_buffer("weight_q", q)
        self.register_buffer("scale", s)
        self._packed_in_dim = in_dim
        if bias is not None:
            self.bias = nn.Parameter(bias.detach().clone())
        else:
            self.register_parameter("bias", None)

    @classmethod
    def from_packed(cls, weight_q: torch.Tensor, scale: torch.Tensor,
                    bias: Optional[torch.Tensor], scheme: str, in_features: int,
                    group_size: Optional[int] = None) -> "QuantizedLinear":
        """A QuantizedLinear around already-quantised buffers (a loaded file),
        without quantising anything."""
        if scheme not in ("int8", "int4", "nf4"):
            raise ValueError(f"unknown scheme {scheme!r}")
        _check_group(scheme, group_size)
        self = cls.__new__(cls)
        nn.Module.__init__(self)
        self.scheme, self.group_size = scheme, group_size
        self.in_features, self.out_features = int(in_features), weight_q.shape[0]
        self.register_buffer("weight_q", weight_q)
        self.register_buffer("scale", scale)
        self._packed_in_dim = int(in_features)
        if bias is not None:
            self.bias = nn.Parameter(bias.detach().clone())
        else:
            self.register_parameter("bias", None)
        return self

    def dequantize_weight(self) -> torch.Tensor:
        return _dequant(self.scheme, self.weight_q, self.scale, self._packed_in_dim,
                        self.group_size)

    def dense_weight(self, dtype: torch.dtype) -> torch.Tensor:
        """deq(W).to(dtype), cached while the buffers are unchanged.  The block's
        fused scan keeps dt_proj's rows in registers and reads this (a derived
        cache of d_inner x dt_rank values, not module state)."""
        key = (self.weight_q.data_ptr(), self.weight_q._version, self.scale.data_ptr(),
               self.scale._version, dtype)
        cache = getattr(self, "_dense_cache", None)
        if cache is None or cache[0] != key:
            cache = (key, self.dequantize_weight().to(dtype).contiguous())
            self._dense_cache = cache
        return cache[1]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.qlinear(x, self.scheme, self.weight_q, self.scale, self.bias, self.in_features,
                           group_size=self.group_size)

    def extra_repr(self) -> str:
        g = f", group_size={self.group_size}" if self.group_size else ""
        return f"in={self.in_features}, out={self.out_features}, scheme={self.scheme!r}{g}"


_QUANTIZABLE_LINEARS = ("in_proj", "x_proj", "dt_proj", "out_proj")


def _linear_sites(module: nn.Module, names: Iterable[str]):
    """Every (parent, attribute, nn.Linear) whose attribute name is one of
    ``names``, found by a depth-first walk that visits each module once and
    does not descend into the linears it returns."""
    wanted = frozenset(names)
    sites, visited, pending = [], set(), [module]
    while pending:
        parent = pending.pop()
        if id(parent) in visited:
            continue
        visited.add(id(parent))
        for attr, child in parent._modules.items():
            if child is None:
                continue
            if attr in wanted and isinstance(child, nn.Linear):
                sites.append((parent, attr, child))
            else:
                pending.append(child)
    return sites


def quantize_block(module: nn.Module, config: QuantConfig,
                   target_names: Iterable[str] = _QUANTIZABLE_LINEARS) -> int:
    """Swap, in place, every nn.Linear held under one of ``target_names``
    (at any depth of ``module``) for a QuantizedLinear of ``config``'s scheme on
    the linear's device, and return how many were swapped -- four per block
    (the interface of quant.py:205-226).  Sites are collected before any swap,
    so the new modules are never revisited."""
    sites = _linear_sites(module, target_names)
    for parent, attr, lin in sites:
        bias = None if lin.bias is None else lin.bias.detach()
        q = QuantizedLinear(lin.weight.detach(), bias, config.scheme, group_size=config.group_size)
        setattr(parent, attr, q.to(device=lin.weight.device))
    return len(sites)


def memory_footprint(module: nn.Module) -> dict:
    """Bytes held by ``module``: quantised buffers (names ending in
    ``.weight_q`` / ``.scale``) apart from everything else (parameters and the
    other buffers), with the keys of quant.py:229-245."""
    def nbytes(t):
        return t.numel() * t.element_size()

    quantised = {".weight_q", ".scale"}
    split = {True: 0, False: 0}
    for name, buf in module.named_buffers():
        split[any(name.endswith(sfx) for sfx in quantised)] += nbytes(buf)
    dense = sum(nbytes(p) for p in module.parameters()) + split[False]
    return {"param_bytes": dense, "quant_buffer_bytes": split[True],
            "total_bytes": dense + split[True]}
