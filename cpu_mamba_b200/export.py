"""A flat weight file for a block or a stack ("MB2W"): the "ggml/ONNX-style
export" on the reference's roadmap (README.md:203), in a layout a C program
can read with fixed-size records and map without parsing.

Layout, little endian, every offset from the start of the file:

    header   32 B   magic "MB2W", u32 version (1), u32 n_meta, u32 n_tensors,
                    u64 data_offset, u64 file_bytes
    meta     n_meta x 48 B      char key[40] (NUL padded), i64 value
    tensors  n_tensors x 144 B  char name[64] (state_dict key), u32 dtype,
                    u32 ndim, i64 shape[4], u64 offset, u64 nbytes, i32 scheme,
                    i32 group_size, i64 in_dim, 8 B reserved
    data     each tensor's bytes, row-major, at a 64-byte aligned offset

dtype codes: 0 float32, 1 bfloat16, 2 int8, 3 uint8, 4 float16.  scheme (the
C ABI's codes): 0 dense, 1 int8, 2 int4, 3 nf4, set on a quantised
projection's ``weight_q`` record together with its group_size (0 = one scale
per row) and unpacked in_dim; its ``scale`` follows as an ordinary float32
tensor.  Meta keys: kind (0 block, 1 stack), n_layers, d_model, d_inner,
d_state, d_conv, dt_rank, conv_bias, bias, eps_1e12 (the stack's RMSNorm eps
x 1e12), dtype.  Tensor names and shapes are the module's state_dict
(mamba_ssm layout), so a file round-trips through ``save`` / ``load``
bit for bit.
"""
from __future__ import annotations

import struct
from typing import Union

import torch
import torch.nn as nn

from .module import CPUMamba
from .quant import QuantizedLinear
from .stack import MambaStack

MAGIC = b"MB2W"
VERSION = 1
ALIGN = 64
HEADER = struct.Struct("<4sIIIQQ")
META = struct.Struct("<40sq")
TENSOR = struct.Struct("<64sII4qQQiiq8x")
DTYPES = {torch.float32: 0, torch.bfloat16: 1, torch.int8: 2, torch.uint8: 3, torch.float16: 4}
_DTYPE_OF = {v: k for k, v in DTYPES.items()}
SCHEMES = {"none": 0, "int8": 1, "int4": 2, "nf4": 3}
_SCHEME_OF = {v: k for k, v in SCHEMES.items()}


def _align(n: int) -> int:
    return (n + ALIGN - 1) // ALIGN * ALIGN


def _first_block(module) -> CPUMamba:
    return module.layers[0].mixer if isinstance(module, MambaStack) else module


def _meta(module) -> dict:
    blk = _first_block(module)
    stack = isinstance(module, MambaStack)
    return {"kind": int(stack), "n_layers": len(module.layers) if stack else 1,
            "d_model": blk.d_model, "d_inner": blk.d_inner, "d_state": blk.d_state,
            "d_conv": blk.d_conv, "dt_rank": blk.dt_rank,
            "conv_bias": int(blk.conv1d.bias is not None),
            "bias": int(blk.in_proj.bias is not None),
            "eps_1e12": round(module.eps * 1e12) if stack else 0,
            "dtype": DTYPES[blk.conv1d.weight.dtype]}


def save(module: Union[CPUMamba, MambaStack], path: str) -> int:
    """Write ``module`` (a CPUMamba or MambaStack, dense or quantised) to
    ``path``; returns the file size in bytes."""
    if not isinstance(module, (CPUMamba, MambaStack)):
        raise TypeError("save: expected a CPUMamba or a MambaStack")
    quant = {f"{n}.weight_q": m for n, m in module.named_modules()
             if isinstance(m, QuantizedLinear)}
    meta = _meta(module)
    tensors = [(k, v.detach().contiguous().cpu()) for k, v in module.state_dict().items()]
    off = _align(HEADER.size + META.size * len(meta) + TENSOR.size * len(tensors))
    data_offset = off
    records = []
    for name, t in tensors:
        if t.dtype not in DTYPES:
            raise TypeError(f"save: {name} has unsupported dtype {t.dtype}")
        if t.dim() > 4 or len(name.encode()) >= 64:
            raise ValueError(f"save: {name} cannot be recorded (rank > 4 or name too long)")
        nbytes = t.numel() * t.element_size()
        q = quant.get(name)
        scheme = SCHEMES[q.scheme] if q is not None else 0
        group = (q.group_size or 0) if q is not None else 0
        in_dim = q.in_features if q is not None else 0
        shape = list(t.shape) + [0] * (4 - t.dim())
        records.append(TENSOR.pack(name.encode(), DTYPES[t.dtype], t.dim(), *shape, off, nbytes,
                                   scheme, group, in_dim))
        off = _align(off + nbytes)
    with open(path, "wb") as f:
        f.write(HEADER.pack(MAGIC, VERSION, len(meta), len(tensors), data_offset, off))
        for k, v in meta.items():
            f.write(META.pack(k.encode(), int(v)))
        for r in records:
            f.write(r)
        for (name, t), r in zip(tensors, records):
            at = TENSOR.unpack(r)[7]
            f.seek(at)
            f.write(t.view(torch.uint8).reshape(-1).numpy().tobytes() if t.numel() else b"")
        f.truncate(off)
    return off


def read_header(path: str) -> tuple:
    """(meta dict, [tensor record dicts]) of an MB2W file."""
    with open(path, "rb") as f:
        head = f.read(HEADER.size)
        magic, version, n_meta, n_tensors, data_offset, file_bytes = HEADER.unpack(head)
        if magic != MAGIC:
            raise ValueError(f"{path}: not an MB2W file")
        if version != VERSION:
            raise ValueError(f"{path}: MB2W version {version}, this reader knows {VERSION}")
        meta = {}
        for _ in range(n_meta):
            k, v = META.unpack(f.read(META.size))
            meta[k.rstrip(b"\0").decode()] = v
        recs = []
        for _ in range(n_tensors):
            name, dt, ndim, s0, s1, s2, s3, off, nbytes, scheme, group, in_dim = \
                TENSOR.unpack(f.read(TENSOR.size))
            recs.append({"name": name.rstrip(b"\0").decode(), "dtype": _DTYPE_OF[dt],
                         "shape": tuple([s0, s1, s2, s3][:ndim]), "offset": off,
                         "nbytes": nbytes, "scheme": _SCHEME_OF[scheme],
                         "group_size": group or None, "in_dim": in_dim})
    meta["data_offset"], meta["file_bytes"] = data_offset, file_bytes
    return meta, recs


def load(path: str, device=None) -> Union[CPUMamba, MambaStack]:
    """Rebuild the module an MB2W file holds (quantised projections as
    QuantizedLinear around the stored buffers), on ``device``."""
    meta, recs = read_header(path)
    with open(path, "rb") as f:
        raw = f.read()
    if len(raw) < meta["file_bytes"]:
        raise ValueError(f"{path}: truncated ({len(raw)} < {meta['file_bytes']} bytes)")
    sd = {}
    for r in recs:
        buf = bytearray(raw[r["offset"]: r["offset"] + r["nbytes"]])
        t = torch.frombuffer(buf, dtype=torch.uint8) if buf else torch.empty(0, dtype=torch.uint8)
        sd[r["name"]] = t.view(r["dtype"]).reshape(r["shape"])
    dtype = _DTYPE_OF[meta["dtype"]]
    kw = dict(d_state=meta["d_state"], d_conv=meta["d_conv"], dt_rank=meta["dt_rank"],
              conv_bias=bool(meta["conv_bias"]), bias=bool(meta["bias"]), dtype=dtype)
    dm, di = meta["d_model"], meta["d_inner"]
    if meta["kind"] == 1:
        module = MambaStack(meta["n_layers"], dm, eps=meta["eps_1e12"] / 1e12, **kw)
        for layer in module.layers:
            _set_inner(layer.mixer, di)
    else:
        module = CPUMamba(dm, d_inner=di, **kw)
    for r in recs:
        if r["scheme"] == "none":
            continue
        prefix = r["name"][: -len(".weight_q")]
        parent_name, _, child = prefix.rpartition(".")
        parent = module.get_submodule(parent_name) if parent_name else module
        bias = sd.get(f"{prefix}.bias")
        q = QuantizedLinear.from_packed(sd[r["name"]], sd[f"{prefix}.scale"], bias, r["scheme"],
                                        r["in_dim"], r["group_size"])
        setattr(parent, child, q)
    module.load_state_dict(sd, strict=True)
    return module.to(device) if device is not None else module


def _set_inner(blk: CPUMamba, d_inner: int) -> None:
    if blk.d_inner != d_inner:
        raise ValueError(f"stack file: d_inner {d_inner} != expand x d_model ({blk.d_inner})")
