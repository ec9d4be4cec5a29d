"""ORACLE -- test infrastructure only.

A CPU restatement of cpu-mamba's hot path (the Mamba S6 block forward, the
stateful step and the int8/int4/nf4 weight quantisers), used as the checker
for the CUDA path.  Only tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline / reference legs may import it; the product package never does.

Pieces:
  scan_oracle.c   -- selective scan (src/cpu_mamba/selective_scan_cpu.cpp:19-87)
  quant_oracle.c  -- quantise / dequantise (src/cpu_mamba/quant.py:35-134)
  mamba_oracle.py -- block composition (src/cpu_mamba/_mamba.py:103-265) in
                     torch CPU ops, the same ATen arithmetic the reference uses
  build_ref.py    -- compiles the reference's own C++ op into oracle/_ref/

Parity of this oracle is pinned against golden vectors that the reference
itself produced (tests/golden/, written by tests/golden/make_golden.py).
"""
from .mamba_oracle import *  # noqa: F401,F403
