"""ORACLE -- test infrastructure only: where the reference's project tree is.

The reference is found from the environment variable MB2_REFERENCE_DIR (the
root of a cpu-mamba checkout, the directory holding src/cpu_mamba/), or else
in a directory named ``reference`` beside this repository's own directory.
There is no other default: where neither exists, the reference is absent and
the recipes that need it (build_ref.py, tests/golden/make_golden.py) do
nothing or stop with a message.
"""
from __future__ import annotations

import os
import pathlib

REPO = pathlib.Path(__file__).resolve().parent.parent
SCAN_SRC = pathlib.Path("src") / "cpu_mamba" / "selective_scan_cpu.cpp"


def reference_root() -> pathlib.Path | None:
    env = os.environ.get("MB2_REFERENCE_DIR")
    cands = [pathlib.Path(env)] if env else [REPO.parent / "reference"]
    for c in cands:
        if (c / "src" / "cpu_mamba").is_dir():
            return c
    return None


def scan_source() -> pathlib.Path | None:
    root = reference_root()
    return None if root is None else root / SCAN_SRC
