"""The ops registered with torch (torch.ops.mamba_b200.*, cpu_mamba_b200.torch_ops).

CPU: every op is registered, its fake implementation gives the right output
shapes and dtypes under FakeTensorMode (so the ops trace), and real CPU
tensors raise (there is no CPU path).  GPU: each op returns what the package's
own functions return (bit for bit; the decode step within 1e-5 of the block's
forward_step, which multiplies on the tensor cores), mamba_step advances h and
conv_state in place, and torch.library.opcheck accepts the registrations."""
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import oracle
from cpu_mamba_b200 import CPUMamba, ops
from cpu_mamba_b200 import torch_ops  # noqa: F401  (registers the ops)

OPS = ("selective_scan", "selective_scan_state", "quant_pack", "dequant", "qlinear",
       "mamba_step")


def test_ops_are_registered():
    for name in OPS:
        assert hasattr(torch.ops.mamba_b200, name), name


def test_fake_shapes():
    with FakeTensorMode():
        x = torch.empty(2, 5, 8)
        A = torch.empty(8, 4)
        Bm = torch.empty(2, 5, 4)
        D = torch.empty(8)
        y = torch.ops.mamba_b200.selective_scan(x, x, A, Bm, Bm, D)
        assert y.shape == (2, 5, 8)
        y, h = torch.ops.mamba_b200.selective_scan_state(x, x, A, Bm, Bm, D, None)
        assert h.shape == (2, 8, 4) and h.dtype == torch.float32
        w = torch.empty(6, 9)
        q, s = torch.ops.mamba_b200.quant_pack(w, "int4", 0)
        assert q.shape == (6, 5) and q.dtype == torch.uint8 and s.shape == (6,)
        q, s = torch.ops.mamba_b200.quant_pack(w, "int8", 4)
        assert q.shape == (6, 9) and q.dtype == torch.int8 and s.shape == (6, 3)
        assert torch.ops.mamba_b200.dequant(q, s, "int8", 9, 4).shape == (6, 9)
        xq = torch.empty(3, 7, 9)
        assert torch.ops.mamba_b200.qlinear(xq, q, s, None, "int8", 9, 4).shape == (3, 7, 6)


def test_cpu_tensors_raise():
    x = torch.zeros(1, 2, 4)
    with pytest.raises(RuntimeError):
        torch.ops.mamba_b200.selective_scan(x, x, torch.zeros(4, 2), torch.zeros(1, 2, 2),
                                            torch.zeros(1, 2, 2), torch.zeros(4))


@pytest.mark.gpu
def test_scan_and_quant_ops_match_the_functions():
    g = torch.Generator().manual_seed(0)
    b, T, di, S = 2, 33, 64, 16
    x = torch.randn(b, T, di, generator=g).cuda()
    dt = (torch.rand(b, T, di, generator=g) * 0.1).cuda()
    A = -torch.rand(di, S, generator=g).cuda()
    Bm, Cm = torch.randn(b, T, S, generator=g).cuda(), torch.randn(b, T, S, generator=g).cuda()
    D = torch.randn(di, generator=g).cuda()
    assert torch.equal(torch.ops.mamba_b200.selective_scan(x, dt, A, Bm, Cm, D),
                       ops.selective_scan(x, dt, A, Bm, Cm, D))
    h0 = torch.randn(b, di, S, generator=g).cuda()
    y, h = torch.ops.mamba_b200.selective_scan_state(x, dt, A, Bm, Cm, D, h0)
    y2, h2 = ops.selective_scan(x, dt, A, Bm, Cm, D, h0=h0, return_last_state=True)
    assert torch.equal(y, y2) and torch.equal(h, h2)
    w = torch.randn(48, 64, generator=g).cuda()
    for scheme, group in (("int8", 0), ("int4", 0), ("nf4", 16)):
        q, s = torch.ops.mamba_b200.quant_pack(w, scheme, group)
        q2, s2, _ = ops.quantize(scheme, w, group or None)
        assert torch.equal(q, q2) and torch.equal(s, s2)
        wd = torch.ops.mamba_b200.dequant(q, s, scheme, 64, group)
        assert torch.equal(wd, ops.dequantize(scheme, q, s, 64, group or None))
        xq = torch.randn(5, 64, generator=g).cuda()
        assert torch.equal(torch.ops.mamba_b200.qlinear(xq, q, s, None, scheme, 64, group),
                           ops.qlinear(xq, scheme, q, s, None, 64, group_size=group or None))
    torch.library.opcheck(torch.ops.mamba_b200.selective_scan.default, (x, dt, A, Bm, Cm, D))
    torch.library.opcheck(torch.ops.mamba_b200.qlinear.default, (xq, q, s, None, "nf4", 64, 16))


@pytest.mark.gpu
def test_mamba_step_op_matches_forward_step():
    dm, S, B = 64, 16, 3
    m = CPUMamba(dm, S)
    m.load_state_dict(oracle.make_block_params(dm, S, seed=9))
    m = m.cuda()
    st = m.init_state(B)
    st2 = {k: v.clone() for k, v in st.items()}
    g = torch.Generator().manual_seed(1)
    for _ in range(4):
        x = torch.randn(B, dm, generator=g).cuda()
        y_ref, _ = m.forward_step(x, st)
        y = torch.ops.mamba_b200.mamba_step(
            x, st2["h"], st2["conv_state"], m.in_proj.weight, m.conv1d.weight, m.conv1d.bias,
            m.x_proj.weight, m.dt_proj.weight, m.dt_proj.bias, m.A_log, m.D, m.out_proj.weight)
        assert (y - y_ref).abs().max().item() <= 1e-5
        assert (st2["h"] - st["h"]).abs().max().item() <= 1e-5
        assert (st2["conv_state"] - st["conv_state"]).abs().max().item() <= 1e-5
