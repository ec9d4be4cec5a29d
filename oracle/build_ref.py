"""ORACLE build recipe -- test infrastructure only.

Compiles the reference's own C++ selective-scan op
(src/cpu_mamba/selective_scan_cpu.cpp) from its source where it lies, with the
reference's flags (src/cpu_mamba/_mamba.py:37-43) except -march=native, which is
replaced by -march=x86-64-v3 so the module also runs on another host CPU.
Output goes only to oracle/_ref/ (git-ignored); nothing is copied from the
reference tree.

The system g++ is used because the toolchain under /opt/gcc lacks libgomp.spec.

    python oracle/build_ref.py [--src <path to selective_scan_cpu.cpp>] [--out oracle/_ref]

Without --src the source is looked up in the reference tree that
oracle/refpath.py locates (MB2_REFERENCE_DIR, or a ``reference`` directory
beside this repository).
"""
from __future__ import annotations

import argparse
import os
import pathlib
import sys

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
from refpath import scan_source  # noqa: E402


def build(src: str | os.PathLike | None = None, out: str | os.PathLike = HERE / "_ref",
          verbose: bool = False) -> pathlib.Path | None:
    """Build the reference op; returns the .so path, or None when the source is absent."""
    src = src if src is not None else scan_source()
    if src is None:
        return None
    src_p = pathlib.Path(src)
    if not src_p.exists():
        return None
    out_p = pathlib.Path(out)
    out_p.mkdir(parents=True, exist_ok=True)
    if os.path.exists("/usr/bin/g++"):
        os.environ["CXX"] = "/usr/bin/g++"
    from torch.utils.cpp_extension import load
    load(
        name="selective_scan_cpu",
        sources=[str(src_p)],
        extra_cflags=["-O3", "-fopenmp", "-march=x86-64-v3", "-ffast-math"],
        extra_ldflags=["-fopenmp"],
        build_directory=str(out_p),
        verbose=verbose,
    )
    so = out_p / "selective_scan_cpu.so"
    return so if so.exists() else None


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--src", default=None)
    ap.add_argument("--out", default=str(HERE / "_ref"))
    args = ap.parse_args()
    so = build(args.src, args.out, verbose=True)
    if so is None:
        print(f"reference source not found: {args.src or 'set MB2_REFERENCE_DIR'}",
              file=sys.stderr)
        return 1
    print(so)
    return 0


if __name__ == "__main__":
    sys.exit(main())
