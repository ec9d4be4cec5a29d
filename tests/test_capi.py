"""The C-ABI library loads without a GPU and exports every entry point that
include/mamba_b200.h declares; argument validation that precedes any CUDA call
reports the documented status codes and messages."""
import ctypes
import pathlib
import re

import pytest

from cpu_mamba_b200 import _lib

HEADER = pathlib.Path(__file__).resolve().parent.parent / "include" / "mamba_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mb2_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    names = declared_functions()
    assert len(names) >= 14
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # the ctypes signature table covers the whole header
    assert set(names) <= set(_lib.exported_symbols())


def test_version_and_error_string():
    lib = _lib.lib()
    assert lib.mb2_version() >= 1
    assert isinstance(lib.mb2_last_error(), bytes)


def test_scan_rejects_large_state_without_gpu():
    lib = _lib.lib()
    rc = lib.mb2_selective_scan(None, None, None, None, None, None, None, 1, 4, 8, 300,
                                None, None, None)
    assert rc == 2
    assert b"d_state > 256" in lib.mb2_last_error()


def test_quantize_rejects_unknown_scheme():
    lib = _lib.lib()
    assert lib.mb2_quantize(9, None, 4, 4, None, None, None) == 1
    assert b"unknown scheme" in lib.mb2_last_error()


def test_block_descriptor_validation():
    lib = _lib.lib()
    blk = _lib.Block()
    blk.d_model, blk.d_inner, blk.d_state, blk.d_conv, blk.dt_rank = 64, 128, 16, 4, 4
    blk.dtype = 0
    # missing conv weight / A_log
    rc = lib.mb2_block_forward(ctypes.byref(blk), None, None, 1, 1, None, None, None, 0, None)
    assert rc == 1
    need = lib.mb2_block_workspace_bytes(ctypes.byref(blk), 2, 16)
    assert need >= 2 * 16 * (2 * 128 + 128) * 4      # xz + xc (y overwrites xc)
    blk.conv_w = blk.A_log = 1  # non-null sentinels; validation stops before any use
    blk.dt_proj.weight = 1
    rc = lib.mb2_block_forward(ctypes.byref(blk), None, None, 2, 16, None, None, None, 0, None)
    assert rc == 6 and b"workspace" in lib.mb2_last_error()


def test_status_raises_runtime_error():
    with pytest.raises(RuntimeError, match="d_state > 256"):
        _lib.check(_lib.lib().mb2_selective_scan(None, None, None, None, None, None, None,
                                                 1, 1, 1, 512, None, None, None), "selective_scan")


def _sentinel_block():
    blk = _lib.Block()
    blk.d_model, blk.d_inner, blk.d_state, blk.d_conv, blk.dt_rank = 64, 128, 16, 4, 4
    blk.dtype = 0
    blk.conv_w = blk.A_log = 1   # non-null sentinels; validation stops before any use
    blk.dt_proj.weight = 1
    return blk


def test_shard_phases_validate_before_any_launch():
    lib = _lib.lib()
    blk = _sentinel_block()
    for phase in (0, 3):
        assert lib.mb2_block_forward_shard(ctypes.byref(blk), phase, None, None, 1, 1, None,
                                           None, None, 0, None) == 1
        assert b"phase" in lib.mb2_last_error()
        assert lib.mb2_block_step_shard(ctypes.byref(blk), phase, None, None, None, None, 1,
                                        None, 0, None) == 1
    # too small a workspace is reported before anything runs
    assert lib.mb2_block_forward_shard(ctypes.byref(blk), 1, None, None, 2, 16, None, None,
                                       None, 0, None) == 6
    off, ld = ctypes.c_size_t(), ctypes.c_int64()
    assert lib.mb2_block_shard_xdbl(ctypes.byref(blk), 32, 0, ctypes.byref(off),
                                    ctypes.byref(ld)) == 0
    # x_dbl rows: dt_rank, B and C segments each rounded up to 8 elements
    assert ld.value == 8 + 16 + 16 and off.value % 256 == 0
    assert off.value + 32 * ld.value * 4 <= lib.mb2_block_workspace_bytes(ctypes.byref(blk),
                                                                           2, 16)


def test_peer_allreduce_validates_group():
    lib = _lib.lib()
    assert lib.mb2_peer_buffer_bytes(0, 16) == 0 and lib.mb2_peer_buffer_bytes(9, 16) == 0
    small, big = lib.mb2_peer_buffer_bytes(2, 1024), lib.mb2_peer_buffer_bytes(2, 2048)
    assert big - small == 2 * 2 * 1024 * 4          # two parities x two ranks x fp32
    g = _lib.PeerGroup()
    g.world, g.rank, g.slot_elems, g.timeout_ns = 2, 2, 16, 1
    assert lib.mb2_peer_allreduce(0, None, 4, ctypes.byref(g), None) == 1       # rank >= world
    g.rank = 0
    assert lib.mb2_peer_allreduce(0, None, 17, ctypes.byref(g), None) == 2      # count > slot
    assert lib.mb2_peer_allreduce(5, None, 4, ctypes.byref(g), None) == 1       # dtype
    g.timeout_ns = 0
    assert lib.mb2_peer_allreduce(0, None, 4, ctypes.byref(g), None) == 1       # no bound
    g.timeout_ns = 1
    assert lib.mb2_peer_allreduce(0, None, 0, ctypes.byref(g), None) == 0       # nothing to do


def test_stack_step_validates_before_any_launch():
    lib = _lib.lib()
    arr = (_lib.Block * 2)(_sentinel_block(), _sentinel_block())
    assert lib.mb2_stack_step(arr, 2, ctypes.c_float(-1.0), None, None, None, 1, None, 0,
                              None) == 1                                        # eps < 0
    need = lib.mb2_stack_step_workspace_bytes(arr, 2, 8)
    assert need > 0
    assert lib.mb2_stack_step(arr, 2, ctypes.c_float(1e-5), None, None, None, 8, None, 0,
                              None) == 6                                        # workspace
    arr[1].d_model = 32
    assert lib.mb2_stack_step(arr, 2, ctypes.c_float(1e-5), None, None, None, 8, None, need,
                              None) == 2                                        # mismatched
