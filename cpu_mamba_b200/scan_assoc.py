"""The reference's associative-scan entry points (src/cpu_mamba/scan_assoc.py:58-132).

The reference offers recursive-doubling scans as alternative backends that
compute the same recurrence h_t = exp(dt_t A) h_{t-1} + dt_t B_t x_t as its C++
op (within fp32 reordering).  On the GPU one sequential-in-time kernel keeps h
in registers and is bound by the exponentials, not by the time dependence, so
both names map to it; chunk_T is accepted for API compatibility.
"""
from __future__ import annotations

from .ops import linear_recurrence, selective_scan


def _associative_prefix_scan(a, b):
    """h[t] = a[t] * h[t-1] + b[t], h[-1] = 0, along dim 1 of (B, T, ...)
    tensors (scan_assoc.py:24-55): one sequential-in-time GPU kernel
    (mb2_linear_recurrence) instead of recursive doubling; equal to within
    fp32 reassociation."""
    return linear_recurrence(a, b)


def selective_scan_assoc(x, dt, A, Bp, Cp, D):
    """y = scan(x, dt, A, B, C) + D*x, (B, T, d_inner) float32 CUDA tensors."""
    return selective_scan(x.contiguous(), dt.contiguous(), A.contiguous(), Bp.contiguous(),
                          Cp.contiguous(), D.contiguous())


def selective_scan_assoc_chunked(x, dt, A, Bp, Cp, D, chunk_T: int = 32):
    """Chunked variant of the reference (scan_assoc.py:81-132); same result.

    The reference cuts T into chunks of chunk_T to bound the intermediates of
    its recursive doubling (O(chunk_T) extra tensors per chunk, h carried
    across chunks).  The GPU kernel walks T with h in registers and needs no
    intermediates at any T, so there is nothing for chunk_T to bound; it is
    checked and otherwise has no effect."""
    if chunk_T <= 0:
        raise ValueError("chunk_T must be positive")
    return selective_scan_assoc(x, dt, A, Bp, Cp, D)
