"""The associative-scan primitive h[t] = a[t] h[t-1] + b[t]
(scan_assoc.py:24-55, _associative_prefix_scan).

CPU: the oracle's recursive-doubling restatement equals the sequential
definition, and the C entry point validates its arguments.  GPU: the
sequential-in-time kernel (mb2_linear_recurrence, through
scan_assoc._associative_prefix_scan) matches the oracle on ragged lengths,
extra trailing dims and bf16, and the full selective scan rebuilt from it
(a = exp(dt A), b = dt B x, y = sum(h C) + D x, as scan_assoc.py:58-78 does)
matches the library's fused scan."""
import pytest
import torch

import oracle
from cpu_mamba_b200 import _lib, ops, scan_assoc


def _seq(a, b):
    h = torch.zeros_like(a[:, 0])
    out = []
    for t in range(a.shape[1]):
        h = a[:, t] * h + b[:, t]
        out.append(h)
    return torch.stack(out, 1)


@pytest.mark.parametrize("T", [1, 2, 7, 33])
def test_oracle_doubling_equals_sequential(T):
    g = torch.Generator().manual_seed(T)
    a = torch.rand(2, T, 3, 4, generator=g)
    b = torch.randn(2, T, 3, 4, generator=g)
    assert (oracle.associative_prefix_scan(a, b) - _seq(a, b)).abs().max().item() <= 1e-6


def test_c_entry_validates():
    lib = _lib.lib()
    assert lib.mb2_linear_recurrence(7, None, None, None, 1, 1, 1, None) == 1
    assert lib.mb2_linear_recurrence(0, None, None, None, -1, 1, 1, None) == 2
    assert lib.mb2_linear_recurrence(0, None, None, None, 1, 1, 1, None) == 1
    assert lib.mb2_linear_recurrence(0, None, None, None, 0, 5, 5, None) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(3, 1, 5), (2, 37, 64), (4, 130, 24, 16), (1, 1000, 3)])
def test_kernel_matches_oracle(shape):
    g = torch.Generator().manual_seed(len(shape) + shape[1])
    a = torch.rand(*shape, generator=g)
    b = torch.randn(*shape, generator=g)
    h = scan_assoc._associative_prefix_scan(a.cuda(), b.cuda()).cpu()
    assert (h - oracle.associative_prefix_scan(a, b)).abs().max().item() <= 1e-5


@pytest.mark.gpu
def test_kernel_bf16():
    g = torch.Generator().manual_seed(5)
    a = torch.rand(2, 50, 32, generator=g).bfloat16()
    b = torch.randn(2, 50, 32, generator=g).bfloat16()
    h = ops.linear_recurrence(a.cuda(), b.cuda()).float().cpu()
    ref = oracle.associative_prefix_scan(a.float(), b.float())
    rel = (h - ref).abs() / (ref.abs().clamp(min=1e-3) + 1e-6)
    assert rel.mean().item() <= 2e-2


@pytest.mark.gpu
def test_selective_scan_rebuilt_from_the_primitive():
    g = torch.Generator().manual_seed(8)
    B, T, di, S = 2, 45, 32, 8
    x = torch.randn(B, T, di, generator=g).cuda()
    dt = (torch.rand(B, T, di, generator=g) * 0.1).cuda()
    A = -torch.rand(di, S, generator=g).cuda() * 2
    Bm, Cm = torch.randn(B, T, S, generator=g).cuda(), torch.randn(B, T, S, generator=g).cuda()
    D = torch.randn(di, generator=g).cuda()
    a = torch.exp(dt.unsqueeze(-1) * A)                              # (B, T, di, S)
    b = (dt.unsqueeze(-1) * Bm.unsqueeze(2)) * x.unsqueeze(-1)
    h = scan_assoc._associative_prefix_scan(a, b)
    y = (h * Cm.unsqueeze(2)).sum(-1) + D * x
    assert (y - ops.selective_scan(x, dt, A, Bm, Cm, D)).abs().max().item() <= 1e-5
