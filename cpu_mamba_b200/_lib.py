"""ctypes binding of the C ABI in include/mamba_b200.h.

The CUDA library is the only compute path: if libmamba_b200.so is missing or
fails to load, every op raises (there is no CPU fallback).
"""
from __future__ import annotations

import ctypes
import pathlib
import threading

import torch

_PKG = pathlib.Path(__file__).resolve().parent
LIB_PATH = _PKG / "_lib" / "libmamba_b200.so"

MB2_OK = 0
MB2_F32, MB2_BF16 = 0, 1
EPI_NONE, EPI_SOFTPLUS = 0, 1
SCHEMES = {"none": 0, "int8": 1, "int4": 2, "nf4": 3}
_ERR_NAMES = {1: "bad argument", 2: "bad shape", 3: "misaligned", 4: "unsupported",
              5: "CUDA error", 6: "workspace too small"}

_c_i64 = ctypes.c_int64
_vp = ctypes.c_void_p


class MambaB200Error(RuntimeError):
    """A failed call into libmamba_b200 (status code in .code)."""

    def __init__(self, what: str, code: int, msg: str):
        super().__init__(f"{what}: {msg} [{_ERR_NAMES.get(code, code)}]")
        self.code = code


class LinearW(ctypes.Structure):
    _fields_ = [("weight", _vp), ("weight_split", _vp), ("weight_q", _vp),
                ("scale", _vp), ("bias", _vp), ("scheme", ctypes.c_int),
                ("group_size", _c_i64), ("weight_f16", _vp)]


class PeerGroup(ctypes.Structure):
    _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32),
                ("slot_elems", ctypes.c_int64), ("timeout_ns", ctypes.c_int64),
                ("bufs", ctypes.c_void_p * 8)]


class Block(ctypes.Structure):
    _fields_ = [("d_model", _c_i64), ("d_inner", _c_i64), ("d_state", _c_i64),
                ("d_conv", _c_i64), ("dt_rank", _c_i64), ("dtype", ctypes.c_int),
                ("in_proj", LinearW), ("x_proj", LinearW), ("dt_proj", LinearW),
                ("out_proj", LinearW), ("conv_w", _vp), ("conv_b", _vp),
                ("A_log", _vp), ("D", _vp)]


# name -> (restype, argtypes)
_SIGS = {
    "mb2_version": (ctypes.c_int, []),
    "mb2_last_error": (ctypes.c_char_p, []),
    "mb2_device_status": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int), ctypes.c_int]),
    "mb2_selective_scan": (ctypes.c_int, [_vp] * 7 + [_c_i64] * 4 + [_vp, _vp, _vp]),
    "mb2_conv1d_silu": (ctypes.c_int, [ctypes.c_int, _vp, _c_i64, _vp, _vp, _vp, _c_i64, _vp,
                                       _c_i64, _c_i64, _c_i64, _c_i64, _vp]),
    "mb2_scan_fused": (ctypes.c_int, [ctypes.c_int, _vp, _c_i64, _vp, _c_i64, _vp, _c_i64,
                                      _vp, _c_i64, _vp, _c_i64, _vp, _vp, _vp, _vp, _vp, _vp,
                                      _vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _vp]),
    "mb2_scan_gated": (ctypes.c_int, [ctypes.c_int, _vp, _c_i64, _vp, _c_i64, _vp, _c_i64,
                                      _vp, _c_i64, _vp, _c_i64, _vp, _vp, _vp, _vp, _vp,
                                      _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _vp]),
    "mb2_scan_workspace_bytes": (ctypes.c_size_t, [_c_i64] * 4),
    "mb2_scan_gated_ws": (ctypes.c_int, [ctypes.c_int, _vp, _c_i64, _vp, _c_i64, _vp, _c_i64,
                                         _vp, _c_i64, _vp, _c_i64, _vp, _vp, _vp, _vp, _vp,
                                         _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _vp,
                                         ctypes.c_size_t, _vp]),
    "mb2_linear_recurrence": (ctypes.c_int, [ctypes.c_int, _vp, _vp, _vp, _c_i64, _c_i64,
                                             _c_i64, _vp]),
    "mb2_linear": (ctypes.c_int, [ctypes.c_int, _vp, _c_i64, _vp, _vp, _vp, _vp, _c_i64,
                                  _c_i64, _c_i64, _c_i64, ctypes.c_int, _vp]),
    "mb2_split_tf32": (ctypes.c_int, [_vp, _vp, _c_i64, _vp]),
    "mb2_split_f16_bytes": (ctypes.c_size_t, [_c_i64, _c_i64]),
    "mb2_split_f16": (ctypes.c_int, [_vp, _c_i64, _c_i64, _vp, _vp]),
    "mb2_linear_f16_scratch_bytes": (ctypes.c_size_t, []),
    "mb2_linear_f16": (ctypes.c_int, [_vp, _c_i64, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64,
                                      _c_i64, ctypes.c_int, ctypes.c_int, _vp, _vp]),
    "mb2_quantize": (ctypes.c_int, [ctypes.c_int, _vp, _c_i64, _c_i64, _vp, _vp, _vp]),
    "mb2_dequantize": (ctypes.c_int, [ctypes.c_int, _vp, _vp, _c_i64, _c_i64, _vp, _vp]),
    "mb2_qlinear": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, _vp, _c_i64, _vp, _vp, _vp,
                                   _vp, _c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_int, _vp]),
    "mb2_quantize_grouped": (ctypes.c_int, [ctypes.c_int, _vp, _c_i64, _c_i64, _c_i64, _vp, _vp,
                                            _vp]),
    "mb2_dequantize_grouped": (ctypes.c_int, [ctypes.c_int, _vp, _vp, _c_i64, _c_i64, _c_i64,
                                              _vp, _vp]),
    "mb2_qlinear_grouped": (ctypes.c_int, [ctypes.c_int, _c_i64, ctypes.c_int, _vp, _c_i64, _vp,
                                           _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_i64,
                                           ctypes.c_int, _vp]),
    "mb2_block_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(Block), _c_i64, _c_i64]),
    "mb2_block_forward": (ctypes.c_int, [ctypes.POINTER(Block), _vp, _vp, _c_i64, _c_i64,
                                         _vp, _vp, _vp, ctypes.c_size_t, _vp]),
    "mb2_block_forward_profile": (ctypes.c_int, [ctypes.POINTER(Block), _vp, _vp, _c_i64, _c_i64,
                                                 _vp, ctypes.c_size_t, _vp, _vp]),
    "mb2_step_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(Block), _c_i64]),
    "mb2_block_step": (ctypes.c_int, [ctypes.POINTER(Block), _vp, _vp, _vp, _vp, _c_i64,
                                      _vp, ctypes.c_size_t, _vp]),
    "mb2_block_step_static": (ctypes.c_int, [ctypes.POINTER(Block), _vp, _vp, _vp, _vp, _c_i64,
                                             _vp]),
    "mb2_stack_forward_state": (ctypes.c_int, [ctypes.POINTER(Block), _c_i64, ctypes.c_float,
                                               _vp, _c_i64, _c_i64, ctypes.POINTER(_vp),
                                               ctypes.POINTER(_vp), _vp, ctypes.c_size_t, _vp]),
    "mb2_stack_step_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(Block), _c_i64, _c_i64]),
    "mb2_stack_step": (ctypes.c_int, [ctypes.POINTER(Block), _c_i64, ctypes.c_float, _vp,
                                      ctypes.POINTER(_vp), ctypes.POINTER(_vp), _c_i64, _vp,
                                      ctypes.c_size_t, _vp]),
    "mb2_block_shard_xdbl": (ctypes.c_int, [ctypes.POINTER(Block), _c_i64, ctypes.c_int,
                                            ctypes.POINTER(ctypes.c_size_t),
                                            ctypes.POINTER(_c_i64)]),
    "mb2_block_forward_shard": (ctypes.c_int, [ctypes.POINTER(Block), ctypes.c_int, _vp, _vp,
                                               _c_i64, _c_i64, _vp, _vp, _vp, ctypes.c_size_t,
                                               _vp]),
    "mb2_block_step_shard": (ctypes.c_int, [ctypes.POINTER(Block), ctypes.c_int, _vp, _vp, _vp,
                                            _vp, _c_i64, _vp, ctypes.c_size_t, _vp]),
    "mb2_peer_buffer_bytes": (ctypes.c_size_t, [ctypes.c_int, _c_i64]),
    "mb2_peer_alloc": (ctypes.c_int, [ctypes.c_size_t, ctypes.POINTER(_vp), ctypes.c_char_p]),
    "mb2_peer_open": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(_vp)]),
    "mb2_peer_close": (ctypes.c_int, [_vp]),
    "mb2_peer_free": (ctypes.c_int, [_vp]),
    "mb2_peer_allreduce": (ctypes.c_int, [ctypes.c_int, _vp, _c_i64, ctypes.POINTER(PeerGroup),
                                          _vp]),
    "mb2_peer_status": (ctypes.c_int, [ctypes.POINTER(PeerGroup), ctypes.POINTER(ctypes.c_int),
                                       ctypes.c_int]),
    "mb2_fold_norm": (ctypes.c_int, [ctypes.c_int, _vp, _vp, _vp, _c_i64, _c_i64, _vp]),
    "mb2_stack_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(Block), _c_i64, _c_i64,
                                                    _c_i64]),
    "mb2_stack_forward": (ctypes.c_int, [ctypes.POINTER(Block), _c_i64, ctypes.c_float, _vp,
                                         _c_i64, _c_i64, _vp, ctypes.c_size_t, _vp]),
}

_LIB = None
_LOCK = threading.Lock()


def lib() -> ctypes.CDLL:
    """Load libmamba_b200.so once; raise if it is absent (no fallback)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH} is not built; run `python -m cpu_mamba_b200.build`. "
                    "cpu_mamba_b200 has no CPU fallback.")
            L = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in _SIGS.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _LIB = L
    return _LIB


def device_status(clear: bool = True) -> int:
    """0, or the code of a kernel-side wait that expired since the last clear."""
    code = ctypes.c_int(0)
    check(lib().mb2_device_status(ctypes.byref(code), int(clear)), "device_status")
    return code.value


def exported_symbols():
    return sorted(_SIGS)


def check(rc: int, what: str) -> None:
    if rc != MB2_OK:
        msg = lib().mb2_last_error()
        raise MambaB200Error(what, rc, msg.decode() if msg else "")


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return MB2_F32
    if dt == torch.bfloat16:
        return MB2_BF16
    raise TypeError(f"unsupported dtype {dt}: cpu_mamba_b200 computes in float32 or bfloat16")


def require_cuda(*tensors, what="op"):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(f"{what}: tensors must be on a CUDA device (cpu_mamba_b200 runs "
                               "on B200 GPUs only; move the module and inputs with .cuda())")
