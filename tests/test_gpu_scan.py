"""GPU parity of the selective scan (drop-in for selective_scan_cpu) and of the
fused scan stage, against the reference's golden outputs and the pinned oracle.

Bar (fp32): max abs diff <= 1e-5 against the reference's C++ op."""
import pytest
import torch

import oracle
from cpu_mamba_b200 import _lib, ops, selective_scan, selective_scan_assoc_chunked

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _cuda(*ts):
    return [t.cuda() for t in ts]


def test_scan_matches_reference_goldens(golden):
    for case in golden("scan.pt"):
        x, dt, A, B, C, D = _cuda(case["x"], case["dt"], case["A"], case["B"], case["C"], case["D"])
        y = selective_scan(x, dt, A, B, C, D)
        assert y.shape == case["y"].shape and y.dtype == torch.float32
        if y.numel():
            err = (y.cpu() - case["y"]).abs().max().item()
            assert err <= TOL, (tuple(x.shape), A.shape[1], err)


@pytest.mark.parametrize("shape", [(3, 50, 200, 16), (2, 181, 96, 24), (1, 7, 33, 5),
                                   (2, 40, 64, 128), (1, 300, 32, 48)])
def test_scan_state_round_trip_matches_oracle(shape):
    b, T, di, S = shape
    g = torch.Generator().manual_seed(sum(shape))
    x = torch.randn(b, T, di, generator=g)
    dt = torch.nn.functional.softplus(torch.randn(b, T, di, generator=g) - 2)
    A = -torch.rand(di, S, generator=g) * 8 - 0.1
    # B, C scaled so y stays O(1) for any d_state (the 1e-5 bar is absolute)
    sc = min(1.0, (16.0 / S) ** 0.5)
    Bm, Cm = torch.randn(b, T, S, generator=g) * sc, torch.randn(b, T, S, generator=g) * sc
    D = torch.randn(di, generator=g)
    h0 = torch.randn(b, di, S, generator=g)
    y_ref, h_ref = oracle.selective_scan(x, dt, A, Bm, Cm, D, h0=h0, return_last_state=True)
    y, h = selective_scan(*_cuda(x, dt, A, Bm, Cm, D), h0=h0.cuda(), return_last_state=True)
    assert (y.cpu() - y_ref).abs().max().item() <= TOL
    assert (h.cpu() - h_ref).abs().max().item() <= TOL
    # split the sequence: scan(t0) then scan(t1 | h(t0)) == scan(all)
    t0 = T // 3
    xs = [t.cuda() for t in (x, dt, Bm, Cm)]
    y1, h1 = selective_scan(xs[0][:, :t0].contiguous(), xs[1][:, :t0].contiguous(), A.cuda(),
                            xs[2][:, :t0].contiguous(), xs[3][:, :t0].contiguous(), D.cuda(),
                            h0=h0.cuda(), return_last_state=True)
    y2, h2 = selective_scan(xs[0][:, t0:].contiguous(), xs[1][:, t0:].contiguous(), A.cuda(),
                            xs[2][:, t0:].contiguous(), xs[3][:, t0:].contiguous(), D.cuda(),
                            h0=h1, return_last_state=True)
    assert torch.equal(torch.cat([y1, y2], 1), y)
    assert torch.equal(h2, h)


def test_scan_is_deterministic_and_batch_independent():
    g = torch.Generator().manual_seed(3)
    b, T, di, S = 6, 64, 256, 24
    x = torch.randn(b, T, di, generator=g).cuda()
    dt = torch.rand(b, T, di, generator=g).cuda() * 0.1
    A = (-torch.rand(di, S, generator=g) * 10).cuda()
    Bm, Cm = torch.randn(b, T, S, generator=g).cuda(), torch.randn(b, T, S, generator=g).cuda()
    D = torch.ones(di).cuda()
    y = selective_scan(x, dt, A, Bm, Cm, D)
    assert torch.equal(y, selective_scan(x, dt, A, Bm, Cm, D))
    y_half = selective_scan(x[3:].contiguous(), dt[3:].contiguous(), A, Bm[3:].contiguous(),
                            Cm[3:].contiguous(), D)
    assert torch.equal(y[3:], y_half)
    assert torch.equal(selective_scan_assoc_chunked(x, dt, A, Bm, Cm, D, chunk_T=16), y)


def test_scan_empty_sequence():
    x = torch.zeros(2, 0, 8, device="cuda")
    A = -torch.ones(8, 4, device="cuda")
    Bm = torch.zeros(2, 0, 4, device="cuda")
    h0 = torch.randn(2, 8, 4, device="cuda")
    y, h = selective_scan(x, x, A, Bm, Bm, torch.ones(8, device="cuda"), h0=h0,
                          return_last_state=True)
    assert y.shape == (2, 0, 8)
    assert torch.equal(h, h0)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_gated_scan_matches_composition(dtype):
    """dt_proj + softplus, A = -exp(A_log), scan, D skip, cast and SiLU(z) gate in
    one kernel, reading dt_low, B and C as column slices of x_proj's output ==
    the reference's composition."""
    p = oracle.make_block_params(96, 16, seed=11, dtype=dtype)
    di, S = p["A_log"].shape
    R = p["dt_proj.weight"].shape[1]
    b, T = 3, 45
    g = torch.Generator().manual_seed(12)
    xc = torch.nn.functional.silu(torch.randn(b * T, di, generator=g)).to(dtype)
    xdbl = (torch.randn(b * T, R + 2 * S, generator=g) * 0.5).to(dtype)
    z = torch.randn(b * T, di, generator=g).to(dtype)
    dt = torch.nn.functional.softplus(
        torch.nn.functional.linear(xdbl[:, :R], p["dt_proj.weight"], p["dt_proj.bias"]))
    A = -torch.exp(p["A_log"].float())
    y_scan, h_ref = oracle.selective_scan(
        xc.float().view(b, T, di), dt.float().view(b, T, di), A,
        xdbl[:, R:R + S].float().view(b, T, S), xdbl[:, R + S:].float().view(b, T, S),
        p["D"].float(), return_last_state=True)
    y_ref = y_scan.view(b * T, di).to(dtype) * torch.nn.functional.silu(z)
    xd = xdbl.cuda()
    y, h = ops.scan_fused(xc.cuda(), xd[:, :R], xd[:, R:R + S], xd[:, R + S:], z.cuda(),
                          p["dt_proj.weight"].cuda(), p["dt_proj.bias"].cuda(),
                          p["A_log"].cuda(), p["D"].cuda(), b, T, return_last_state=True)
    assert (h.cpu() - h_ref).abs().max().item() <= TOL
    if dtype == torch.float32:
        assert (y.cpu() - y_ref).abs().max().item() <= TOL
    else:
        rel = (y.cpu().float() - y_ref.float()).abs() / (y_ref.float().abs().clamp(min=1e-3) + 1e-6)
        assert rel.mean().item() <= 2e-2


def test_gated_scan_rejects_misaligned_bf16_rows():
    di, S, R = 64, 16, 3
    xc = torch.zeros(4, di, device="cuda", dtype=torch.bfloat16)
    xdbl = torch.zeros(4, 2 * S + R, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="4-byte"):
        ops.scan_fused(xc, xdbl[:, :R], xdbl[:, R:R + S], xdbl[:, R + S:], xc,
                       torch.zeros(di, R, device="cuda", dtype=torch.bfloat16), None,
                       torch.zeros(di, S, device="cuda", dtype=torch.bfloat16),
                       torch.ones(di, device="cuda", dtype=torch.bfloat16), 1, 4)


@pytest.mark.parametrize("T", [1, 2, 3, 5, 17, 33])
def test_gated_scan_ragged_lengths_state(T):
    """Final state after sequence lengths that end inside a chunk / step group."""
    p = oracle.make_block_params(64, 24, seed=T)
    di, S = p["A_log"].shape
    R = p["dt_proj.weight"].shape[1]
    b = 3
    g = torch.Generator().manual_seed(100 + T)
    xc = torch.randn(b * T, di, generator=g)
    xdbl = torch.randn(b * T, R + 2 * S, generator=g) * 0.5
    z = torch.randn(b * T, di, generator=g)
    dt = torch.nn.functional.softplus(
        torch.nn.functional.linear(xdbl[:, :R], p["dt_proj.weight"], p["dt_proj.bias"]))
    _, h_ref = oracle.selective_scan(xc.view(b, T, di), dt.view(b, T, di),
                                     -torch.exp(p["A_log"]), xdbl[:, R:R + S].reshape(b, T, S),
                                     xdbl[:, R + S:].reshape(b, T, S), p["D"],
                                     return_last_state=True)
    xd = xdbl.cuda()
    _, h = ops.scan_fused(xc.cuda(), xd[:, :R], xd[:, R:R + S], xd[:, R + S:], z.cuda(),
                          p["dt_proj.weight"].cuda(), p["dt_proj.bias"].cuda(), p["A_log"].cuda(),
                          p["D"].cuda(), b, T, return_last_state=True)
    assert (h.cpu() - h_ref).abs().max().item() <= TOL


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("b,T,S", [(3, 45, 16), (4, 100, 24), (2, 17, 8), (2, 33, 32),
                                   (1, 20, 12)])
def test_scan_with_given_dt_matches_composition(dtype, b, T, S):
    """The block forward's split form: dt_proj from the projection kernel
    (tensor cores from 256 rows, with the TF32 halves in fp32), then the scan
    applying the softplus to it == the reference composition."""
    p = oracle.make_block_params(96, S, seed=21 + T, dtype=dtype)
    di = p["A_log"].shape[0]
    R = p["dt_proj.weight"].shape[1]
    g = torch.Generator().manual_seed(22 + b)
    xc = torch.nn.functional.silu(torch.randn(b * T, di, generator=g)).to(dtype)
    xdbl = (torch.randn(b * T, R + 2 * S, generator=g) * 0.5).to(dtype)
    z = torch.randn(b * T, di, generator=g).to(dtype)
    dt_ref = torch.nn.functional.softplus(
        torch.nn.functional.linear(xdbl[:, :R], p["dt_proj.weight"], p["dt_proj.bias"]))
    A = -torch.exp(p["A_log"].float())
    y_scan, h_ref = oracle.selective_scan(
        xc.float().view(b, T, di), dt_ref.float().view(b, T, di), A,
        xdbl[:, R:R + S].float().view(b, T, S), xdbl[:, R + S:].float().view(b, T, S),
        p["D"].float(), return_last_state=True)
    y_ref = y_scan.view(b * T, di).to(dtype) * torch.nn.functional.silu(z)
    xd = xdbl.cuda()
    w_dt = p["dt_proj.weight"].cuda()
    split = ops.split_tf32(w_dt) if dtype == torch.float32 else None
    dt = ops.linear(xd[:, :R], w_dt, p["dt_proj.bias"].cuda(), split)
    y, h = ops.scan_gated(xc.cuda(), dt, xd[:, R:R + S], xd[:, R + S:], z.cuda(),
                          p["A_log"].cuda(), p["D"].cuda(), b, T, return_last_state=True)
    assert (h.cpu() - h_ref).abs().max().item() <= TOL
    if dtype == torch.float32:
        assert (y.cpu() - y_ref).abs().max().item() <= TOL
    else:
        rel = (y.cpu().float() - y_ref.float()).abs() / (y_ref.float().abs().clamp(min=1e-3) + 1e-6)
        assert rel.mean().item() <= 2e-2


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("with_h0", [False, True])
def test_scan_op_long_sequence_runs_in_segments(dtype, with_h0):
    """ops.scan_gated on one long sequence over few chains takes the T-segment
    path (its workspace is non-empty) and matches the composition, with and
    without an initial state."""
    b, T, S = 1, 3000, 16
    p = oracle.make_block_params(96, S, seed=31, dtype=dtype)
    di = p["A_log"].shape[0]
    assert _lib.lib().mb2_scan_workspace_bytes(b, T, di, S) > 0
    g = torch.Generator().manual_seed(32)
    xc = torch.nn.functional.silu(torch.randn(b * T, di, generator=g)).to(dtype)
    dt_pre = (torch.randn(b * T, di, generator=g) * 0.5 - 3).to(dtype)
    bc = (torch.randn(b * T, 2 * S, generator=g) * 0.5).to(dtype)
    z = torch.randn(b * T, di, generator=g).to(dtype)
    h0 = torch.randn(b, di, S, generator=g) * 0.1 if with_h0 else None
    A = -torch.exp(p["A_log"].float())
    dt = torch.nn.functional.softplus(dt_pre.float()).to(dtype).float()
    y_scan, h_ref = oracle.selective_scan(
        xc.float().view(b, T, di), dt.view(b, T, di), A, bc[:, :S].float().view(b, T, S),
        bc[:, S:].float().view(b, T, S), p["D"].float(), h0=h0, return_last_state=True)
    y_ref = y_scan.view(b * T, di).to(dtype) * torch.nn.functional.silu(z)
    bcd = bc.cuda()
    y, h = ops.scan_gated(xc.cuda(), dt_pre.cuda(), bcd[:, :S], bcd[:, S:], z.cuda(),
                          p["A_log"].cuda(), p["D"].cuda(), b, T,
                          h0=None if h0 is None else h0.cuda(), return_last_state=True)
    assert (h.cpu() - h_ref).abs().max().item() <= 2e-5
    if dtype == torch.float32:
        assert (y.cpu() - y_ref).abs().max().item() <= TOL
    else:
        rel = (y.cpu().float() - y_ref.float()).abs() / (y_ref.float().abs().clamp(min=1e-3) + 1e-6)
        assert rel.mean().item() <= 2e-2
