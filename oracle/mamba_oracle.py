"""ORACLE -- test infrastructure only (see oracle/__init__.py).

CPU restatement of the cpu-mamba block.  Linear / conv / softplus / SiLU use
torch CPU (ATen) ops, which is what the reference itself runs
(src/cpu_mamba/_mamba.py:204-265); the scan and the quantisers are the C
restatements in scan_oracle.c / quant_oracle.c, loaded through ctypes.

Parameters are passed as a plain dict keyed like the mamba_ssm state_dict
("in_proj.weight", "conv1d.weight", ..., "A_log", "D").  A quantised linear is
given as "<name>.weight_q" + "<name>.scale" plus an entry in ``quant`` mapping
the linear's name to (scheme, in_dim).
"""
from __future__ import annotations

import ctypes
import math
import os
import pathlib
import subprocess
import threading
from typing import Dict, Optional, Tuple

import torch
import torch.nn.functional as F

__all__ = [
    "load_oracle_lib", "selective_scan", "block_forward",
    "block_forward_with_final_state", "block_step", "init_state",
    "quant_int8", "quant_int4", "quant_nf4", "dequant_int8", "dequant_int4",
    "dequant_nf4", "nf4_lut", "linear", "dequant", "load_ref_scan_op",
    "make_block_params", "stack_forward", "quant_grouped", "dequant_grouped",
    "associative_prefix_scan", "block_forward_f64",
]

_HERE = pathlib.Path(__file__).resolve().parent
_LIB = None
_LOCK = threading.Lock()
_f32p = ctypes.POINTER(ctypes.c_float)
_i64 = ctypes.c_int64


def load_oracle_lib() -> ctypes.CDLL:
    """Load oracle/_build/liboracle.so, building it with make when absent."""
    global _LIB
    with _LOCK:
        if _LIB is not None:
            return _LIB
        so = _HERE / "_build" / "liboracle.so"
        if not so.exists():
            subprocess.run(["make", "-C", str(_HERE), "-s"], check=True)
        lib = ctypes.CDLL(str(so))
        lib.oracle_selective_scan_f32.restype = ctypes.c_int
        lib.oracle_selective_scan_f32.argtypes = [
            ctypes.c_void_p] * 7 + [_i64] * 4 + [ctypes.c_void_p] * 2
        for name in ("oracle_quant_int8", "oracle_quant_int4", "oracle_quant_nf4"):
            fn = getattr(lib, name)
            fn.restype = None
            fn.argtypes = [ctypes.c_void_p, _i64, _i64, ctypes.c_void_p, ctypes.c_void_p]
        for name in ("oracle_dequant_int8", "oracle_dequant_int4", "oracle_dequant_nf4"):
            fn = getattr(lib, name)
            fn.restype = None
            fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, _i64, _i64, ctypes.c_void_p]
        lib.oracle_nf4_lut.restype = None
        lib.oracle_nf4_lut.argtypes = [ctypes.c_void_p]
        _LIB = lib
        return lib


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _cpu_f32(t: torch.Tensor) -> torch.Tensor:
    return t.detach().to("cpu", torch.float32).contiguous()


# ---------------------------------------------------------------------------
# selective scan (selective_scan_cpu.cpp:19-87; time loop _mamba.py:191-199)
# ---------------------------------------------------------------------------
def selective_scan(x, dt, A, B, C, D, h0=None, return_last_state=False):
    """y = scan(x, dt, A, B, C) + D*x on the CPU; optionally the final h too."""
    x, dt, A, B = (_cpu_f32(t) for t in (x, dt, A, B))
    C = None if C is None else _cpu_f32(C)
    D = None if D is None else _cpu_f32(D)
    bsz, T, di = x.shape
    S = A.shape[1]
    y = torch.empty(bsz, T, di, dtype=torch.float32)
    h_last = torch.empty(bsz, di, S, dtype=torch.float32) if return_last_state else None
    h0c = None if h0 is None else _cpu_f32(h0)
    rc = load_oracle_lib().oracle_selective_scan_f32(
        _ptr(x), _ptr(dt), _ptr(A), _ptr(B), _ptr(C), _ptr(D), _ptr(y),
        bsz, T, di, S, _ptr(h0c), _ptr(h_last))
    if rc != 0:
        raise RuntimeError("d_state > 256 not supported (stack limit)")
    return (y, h_last) if return_last_state else y


def associative_prefix_scan(a, b):
    """Recursive-doubling prefix scan over dim 1 (scan_assoc.py:24-55):
    h[t] = a[t] h[t-1] + b[t], h[-1] = 0.  Step stride s combines each
    position with the one s earlier, (a_l, b_l) then (a_r, b_r) ->
    (a_r a_l, a_r b_l + b_r), out of place, s doubling until it covers T."""
    a_p, b_p = _cpu_f32(a), _cpu_f32(b)
    T = a_p.shape[1]
    s = 1
    while s < T:
        a_new = torch.cat([a_p[:, :s], a_p[:, s:] * a_p[:, :-s]], dim=1)
        b_new = torch.cat([b_p[:, :s], a_p[:, s:] * b_p[:, :-s] + b_p[:, s:]], dim=1)
        a_p, b_p = a_new, b_new
        s *= 2
    return b_p


def load_ref_scan_op():
    """The reference's own compiled op from oracle/_ref, or None when not built."""
    import importlib.util
    so = _HERE / "_ref" / "selective_scan_cpu.so"
    if not so.exists():
        return None
    spec = importlib.util.spec_from_file_location("selective_scan_cpu", str(so))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


# ---------------------------------------------------------------------------
# quantisers (quant.py:35-134), bit-exact restatement in C
# ---------------------------------------------------------------------------
def nf4_lut() -> torch.Tensor:
    out = torch.empty(16, dtype=torch.float32)
    load_oracle_lib().oracle_nf4_lut(_ptr(out))
    return out


def quant_int8(w: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    w = _cpu_f32(w)
    rows, cols = w.shape
    q = torch.empty(rows, cols, dtype=torch.int8)
    s = torch.empty(rows, dtype=torch.float32)
    load_oracle_lib().oracle_quant_int8(_ptr(w), rows, cols, _ptr(q), _ptr(s))
    return q, s


def _quant4(fn_name, w):
    w = _cpu_f32(w)
    rows, cols = w.shape
    packed = torch.empty(rows, (cols + 1) // 2, dtype=torch.uint8)
    s = torch.empty(rows, dtype=torch.float32)
    getattr(load_oracle_lib(), fn_name)(_ptr(w), rows, cols, _ptr(packed), _ptr(s))
    return packed, s, cols


def quant_int4(w):
    return _quant4("oracle_quant_int4", w)


def quant_nf4(w):
    return _quant4("oracle_quant_nf4", w)


def dequant_int8(q, scale):
    q = q.detach().cpu().contiguous()
    scale = _cpu_f32(scale)
    out = torch.empty(q.shape, dtype=torch.float32)
    load_oracle_lib().oracle_dequant_int8(_ptr(q), _ptr(scale), q.shape[0], q.shape[1], _ptr(out))
    return out


def _dequant4(fn_name, packed, scale, in_dim):
    packed = packed.detach().cpu().contiguous()
    scale = _cpu_f32(scale)
    out = torch.empty(packed.shape[0], in_dim, dtype=torch.float32)
    getattr(load_oracle_lib(), fn_name)(_ptr(packed), _ptr(scale), packed.shape[0], in_dim, _ptr(out))
    return out


def dequant_int4(packed, scale, in_dim):
    return _dequant4("oracle_dequant_int4", packed, scale, in_dim)


def dequant_nf4(packed, scale, in_dim):
    return _dequant4("oracle_dequant_nf4", packed, scale, in_dim)


def quant_grouped(scheme: str, w: torch.Tensor, group: int):
    """Blockwise quantisation -- the reference's roadmap item "blockwise NF4
    (group_size=64)" (README.md:115, :201), which its code does not implement:
    quant.py's per-row formulas (:60-65 int8, :72-87 int4, :104-121 nf4)
    applied to each run of ``group`` consecutive columns of a row, in the same
    float32 torch ops.  Returns (codes, scale (rows, ceil(cols / group))); 4-bit
    codes are packed as quant.py packs them (even column in the high nibble,
    odd widths padded with code 0 / nibble 7)."""
    w = _cpu_f32(w)
    rows, cols = w.shape
    ng = -(-cols // group)
    g = F.pad(w, (0, ng * group - cols)).view(rows, ng, group)
    amax = g.abs().amax(dim=2).clamp(min=1e-8)
    if scheme == "int8":
        s = amax / 127.0
        q = torch.round(g / s[..., None]).clamp(-127, 127).reshape(rows, -1)[:, :cols]
        return q.to(torch.int8).contiguous(), s
    if scheme == "int4":
        s = amax / 7.0
        q = torch.round(g / s[..., None]).clamp(-7, 7).reshape(rows, -1)[:, :cols]
        codes, pad = (q + 7).to(torch.uint8), 7
    elif scheme == "nf4":
        s = amax
        wn = (g / s[..., None]).clamp(-1.0, 1.0).reshape(rows, -1)[:, :cols]
        codes, pad = (wn[..., None] - nf4_lut()).abs().argmin(-1).to(torch.uint8), 0
    else:
        raise ValueError(scheme)
    if cols % 2:
        codes = torch.cat([codes, torch.full((rows, 1), pad, dtype=torch.uint8)], 1)
    return ((codes[:, 0::2] << 4) | codes[:, 1::2]).contiguous(), s


def dequant_grouped(scheme: str, weight_q: torch.Tensor, scale: torch.Tensor, in_dim: int,
                    group: int) -> torch.Tensor:
    """Inverse of quant_grouped: code value x its group's scale (float32)."""
    scale = _cpu_f32(scale)
    rows = weight_q.shape[0]
    if scheme == "int8":
        v = weight_q.to(torch.float32)
    else:
        b = weight_q.to(torch.int64)
        nib = torch.stack([b >> 4, b & 0xF], -1).reshape(rows, -1)[:, :in_dim]
        v = (nib - 7).to(torch.float32) if scheme == "int4" else nf4_lut()[nib]
    col_scale = scale.repeat_interleave(group, dim=1)[:, :in_dim]
    return v * col_scale


def dequant(scheme: str, weight_q, scale, in_dim: int) -> torch.Tensor:
    if scheme == "int8":
        return dequant_int8(weight_q, scale)
    if scheme == "int4":
        return dequant_int4(weight_q, scale, in_dim)
    if scheme == "nf4":
        return dequant_nf4(weight_q, scale, in_dim)
    raise ValueError(f"unknown scheme {scheme!r}")


# ---------------------------------------------------------------------------
# block composition (_mamba.py:103-265)
# ---------------------------------------------------------------------------
def linear(p: Dict[str, torch.Tensor], name: str, x: torch.Tensor,
           quant: Optional[Dict[str, Tuple[str, int]]] = None) -> torch.Tensor:
    """nn.Linear, or QuantizedLinear.forward (quant.py:188-190) when quantised;
    quant[name] = (scheme, in_dim) or (scheme, in_dim, group_size)."""
    bias = p.get(f"{name}.bias")
    if quant and name in quant:
        scheme, in_dim = quant[name][:2]
        group = quant[name][2] if len(quant[name]) > 2 else None
        if group:
            w = dequant_grouped(scheme, p[f"{name}.weight_q"], p[f"{name}.scale"], in_dim, group)
        else:
            w = dequant(scheme, p[f"{name}.weight_q"], p[f"{name}.scale"], in_dim)
        return F.linear(x, w.to(x.dtype), bias)
    return F.linear(x, p[f"{name}.weight"], bias)


def _dims(p):
    di, S = p["A_log"].shape
    K = p["conv1d.weight"].shape[-1]
    R = p["dt_proj.weight"].shape[1] if "dt_proj.weight" in p else None
    if R is None:
        R = p["x_proj.weight_q"].shape[0] - 2 * S if "x_proj.weight_q" in p else p["x_proj.weight"].shape[0] - 2 * S
    return di, S, K, R


def _front(p, x, quant):
    """in_proj -> causal depthwise conv1d -> SiLU -> x_proj -> dt_proj -> softplus."""
    bsz, T, _ = x.shape
    di, S, K, R = _dims(p)
    xz = linear(p, "in_proj", x, quant)                        # _mamba.py:208
    x_pre, z = xz.chunk(2, dim=-1)                             # :209
    xc = F.conv1d(x_pre.transpose(1, 2), p["conv1d.weight"], p.get("conv1d.bias"),
                  padding=K - 1, groups=di)[..., :T]           # :212-213
    xc = F.silu(xc.transpose(1, 2))                            # :214-215
    x_dbl = linear(p, "x_proj", xc, quant)                     # :217
    dt_low, Bm, Cm = torch.split(x_dbl, [R, S, S], dim=-1)     # :218
    dt = F.softplus(linear(p, "dt_proj", dt_low, quant))       # :219-220
    A = -torch.exp(p["A_log"].float())                         # :222
    return x_pre, z, xc, dt, A, Bm, Cm


def block_forward(p, x, quant=None, scan_op=None):
    """CPUMamba.forward (_mamba.py:204-265) with the C-restated scan, or with
    ``scan_op`` = the reference's own compiled op (load_ref_scan_op())."""
    with torch.no_grad():
        _, z, xc, dt, A, Bm, Cm = _front(p, x, quant)
        args = (xc.float().contiguous(), dt.float().contiguous(), A.contiguous(),
                Bm.float().contiguous(), Cm.float().contiguous(), p["D"].float().contiguous())
        y = scan_op.selective_scan_cpu(*args) if scan_op is not None else selective_scan(*args)
        y = y.to(xc.dtype) * F.silu(z)                         # :263-264
        return linear(p, "out_proj", y, quant)                 # :265


def block_forward_f64(p, x, quant=None):
    """CPUMamba.forward (_mamba.py:204-265) evaluated in float64 throughout,
    with a float64 time-loop scan (_mamba.py:245-261): the yardstick for how
    far a float32 evaluation (the reference's own, or the GPU's) sits from the
    exact result.  Quantised linears use their dequantised float32 weights
    (quant.py:188-190), widened."""
    with torch.no_grad():
        d = {k: v.double() for k, v in p.items() if v.is_floating_point()}
        for name in (quant or {}):
            scheme, in_dim = quant[name][:2]
            d[f"{name}.weight"] = dequant(scheme, p[f"{name}.weight_q"], p[f"{name}.scale"],
                                          in_dim).double()
        x = _cpu_f32(x).double()
        bsz, T, _ = x.shape
        di, S = d["A_log"].shape
        K = d["conv1d.weight"].shape[-1]
        R = d["dt_proj.weight"].shape[1]
        xz = F.linear(x, d["in_proj.weight"], d.get("in_proj.bias"))
        x_pre, z = xz.chunk(2, dim=-1)
        xc = F.conv1d(x_pre.transpose(1, 2), d["conv1d.weight"], d.get("conv1d.bias"),
                      padding=K - 1, groups=di)[..., :T]
        xc = F.silu(xc.transpose(1, 2))
        dt_low, Bm, Cm = torch.split(F.linear(xc, d["x_proj.weight"]), [R, S, S], dim=-1)
        dt = F.softplus(F.linear(dt_low, d["dt_proj.weight"], d.get("dt_proj.bias")))
        A = -torch.exp(d["A_log"])
        h = torch.zeros(bsz, di, S, dtype=torch.float64)
        ys = []
        for t in range(T):
            h = torch.exp(dt[:, t, :, None] * A) * h + \
                (dt[:, t, :, None] * Bm[:, t, None, :]) * xc[:, t, :, None]
            ys.append((h * Cm[:, t, None, :]).sum(-1))
        y = (torch.stack(ys, 1) + d["D"] * xc) * F.silu(z)
        return F.linear(y, d["out_proj.weight"], d.get("out_proj.bias"))


def stack_forward(layers, x, eps=1e-5, scan_op=None):
    """A residual pre-norm stack, x <- x + block(RMSNorm(x)) per layer, in
    float32: torch.nn.RMSNorm (F.rms_norm, weight g, ``eps``) composed with
    CPUMamba.forward (_mamba.py:204-265).  The reference has no stack; this is
    how a model built on it composes the block.  layers: [(block params, g)]."""
    with torch.no_grad():
        x = _cpu_f32(x)
        for p, g in layers:
            pf = {k: v.float() for k, v in p.items()}
            xn = F.rms_norm(x, (x.shape[-1],), g.float(), eps)
            x = x + block_forward(pf, xn, scan_op=scan_op)
        return x


def block_forward_with_final_state(p, x, quant=None):
    """forward_with_final_state (_mamba.py:165-202): y, {h (fp32), conv_state}.

    The conv tail is the last d_conv-1 pre-conv inputs (:180); for prompts
    shorter than that it is left-padded with zeros (the reference would return a
    narrower tensor there, which its own forward_step cannot consume).
    """
    with torch.no_grad():
        x_pre, z, xc, dt, A, Bm, Cm = _front(p, x, quant)
        y, h = selective_scan(xc.float(), dt.float(), A, Bm.float(), Cm.float(),
                              p["D"].float(), return_last_state=True)
        y = linear(p, "out_proj", y.to(xc.dtype) * F.silu(z), quant)
        K = p["conv1d.weight"].shape[-1]
        tail = x_pre.transpose(1, 2)[..., -(K - 1):]
        if tail.shape[-1] < K - 1:
            tail = F.pad(tail, (K - 1 - tail.shape[-1], 0))
        return y, {"h": h, "conv_state": tail.clone()}


def init_state(p, batch_size, dtype=None):
    """init_state (_mamba.py:87-101)."""
    di, S, K, _ = _dims(p)
    dtype = dtype or p["conv1d.weight"].dtype
    return {"h": torch.zeros(batch_size, di, S, dtype=torch.float32),
            "conv_state": torch.zeros(batch_size, di, K - 1, dtype=dtype)}


def block_step(p, x_step, state, quant=None):
    """forward_step (_mamba.py:103-163); returns (y, new_state) without mutating state."""
    with torch.no_grad():
        if x_step.dim() == 3:
            x_step = x_step.squeeze(1)
        di, S, K, R = _dims(p)
        xz = linear(p, "in_proj", x_step, quant)
        xs, z = xz.chunk(2, dim=-1)
        window = torch.cat([state["conv_state"], xs.unsqueeze(-1)], dim=-1)   # :128-130
        xc = (window * p["conv1d.weight"].squeeze(1).unsqueeze(0)).sum(dim=-1)  # :133-134
        if p.get("conv1d.bias") is not None:
            xc = xc + p["conv1d.bias"]
        xc = F.silu(xc)
        x_dbl = linear(p, "x_proj", xc, quant)
        dt_low, Bm, Cm = torch.split(x_dbl, [R, S, S], dim=-1)
        dt = F.softplus(linear(p, "dt_proj", dt_low, quant)).float()
        A = -torch.exp(p["A_log"].float())
        xf = xc.float()
        dA = torch.exp(dt.unsqueeze(-1) * A.unsqueeze(0))                        # :155
        dBx = (dt.unsqueeze(-1) * Bm.float().unsqueeze(1)) * xf.unsqueeze(-1)    # :156
        h = dA * state["h"] + dBx                                               # :157
        y = (h * Cm.float().unsqueeze(1)).sum(dim=-1) + p["D"].float() * xf      # :159
        y = y.to(xc.dtype) * F.silu(z)
        out = linear(p, "out_proj", y, quant)
        return out, {"h": h, "conv_state": window[..., 1:].clone()}


def make_block_params(d_model, d_state=16, d_conv=4, expand=2, dt_rank="auto",
                      seed=0, dtype=torch.float32, dt_min=1e-3, dt_max=0.1,
                      weight_std=None, outlier_frac=0.0):
    """Seeded synthetic parameters with the mamba_ssm state_dict layout.

    Linear weights: nn.Linear's default Kaiming-uniform (bound 1/sqrt(fan_in)),
    or N(0, weight_std) with an optional fraction of +-0.5 outliers.  conv1d
    weight and bias ~ U(-0.5, 0.5).  A_log = log(1..S) per channel, D = 1.
    dt_proj.bias = softplus^-1(dt), dt log-uniform in [dt_min, dt_max].
    """
    g = torch.Generator().manual_seed(seed)
    di = expand * d_model
    R = math.ceil(d_model / 16) if dt_rank == "auto" else int(dt_rank)

    def lin(out_f, in_f):
        if weight_std is None:
            bound = 1.0 / math.sqrt(in_f)
            return (torch.rand(out_f, in_f, generator=g) * 2 - 1) * bound
        w = torch.randn(out_f, in_f, generator=g) * weight_std
        if outlier_frac > 0:
            mask = torch.rand(out_f, in_f, generator=g) < outlier_frac
            sign = torch.where(torch.rand(out_f, in_f, generator=g) < 0.5, -0.5, 0.5)
            w = torch.where(mask, sign, w)
        return w

    p = {
        "in_proj.weight": lin(2 * di, d_model),
        "conv1d.weight": torch.rand(di, 1, d_conv, generator=g) - 0.5,
        "conv1d.bias": torch.rand(di, generator=g) - 0.5,
        "x_proj.weight": lin(R + 2 * d_state, di),
        "dt_proj.weight": lin(di, R),
        "out_proj.weight": lin(d_model, di),
        "A_log": torch.log(torch.arange(1, d_state + 1, dtype=torch.float32).repeat(di, 1)),
        "D": torch.ones(di),
    }
    u = torch.rand(di, generator=g)
    dt = torch.exp(u * (math.log(dt_max) - math.log(dt_min)) + math.log(dt_min))
    p["dt_proj.bias"] = dt + torch.log(-torch.expm1(-dt))      # softplus^-1(dt)
    return {k: v.to(dtype) for k, v in p.items()}
