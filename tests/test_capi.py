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
