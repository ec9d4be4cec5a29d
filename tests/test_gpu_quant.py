"""GPU quantisation: codes, packed bytes, scales and dequantised weights are
bit-exact with the reference (golden fixtures written by quant.py itself);
QuantizedLinear and quantised blocks match the reference within fp32 noise."""
import pytest
import torch

import oracle
from cpu_mamba_b200 import CPUMamba, QuantConfig, QuantizedLinear, memory_footprint, quantize_block
from cpu_mamba_b200 import quant as q

pytestmark = pytest.mark.gpu
TOL = 1e-5


@pytest.mark.parametrize("name", ["normal", "outlier_odd", "ties"])
def test_quant_primitives_bit_exact(golden, name):
    g = golden("quant.pt")["prims"][name]
    w = g["w"].cuda()
    q8, s8 = q.quantize_int8(w)
    assert torch.equal(q8.cpu(), g["int8"][0]) and torch.equal(s8.cpu(), g["int8"][1])
    assert torch.equal(q.dequantize_int8(q8, s8).cpu(), g["int8"][2])
    p4, s4, d4 = q.quantize_int4(w)
    assert d4 == g["int4"][2]
    assert torch.equal(p4.cpu(), g["int4"][0]) and torch.equal(s4.cpu(), g["int4"][1])
    assert torch.equal(q.dequantize_int4(p4, s4, d4).cpu(), g["int4"][3])
    pn, sn, dn = q.quantize_nf4(w)
    assert torch.equal(pn.cpu(), g["nf4"][0]) and torch.equal(sn.cpu(), g["nf4"][1])
    assert torch.equal(q.dequantize_nf4(pn, sn, dn).cpu(), g["nf4"][3])


def test_quant_large_random_bit_exact():
    g = torch.Generator().manual_seed(21)
    w = torch.randn(3072, 1537, generator=g) * 0.02
    mask = torch.rand(w.shape, generator=g) < 0.01
    w = torch.where(mask, torch.where(torch.rand(w.shape, generator=g) < 0.5, -0.5, 0.5), w)
    for scheme, qf, dqf in (("int8", oracle.quant_int8, oracle.dequant_int8),
                            ("int4", oracle.quant_int4, oracle.dequant_int4),
                            ("nf4", oracle.quant_nf4, oracle.dequant_nf4)):
        ref = qf(w)
        got = getattr(q, f"quantize_{scheme}")(w.cuda())
        assert torch.equal(got[0].cpu(), ref[0]) and torch.equal(got[1].cpu(), ref[1]), scheme
        deq = getattr(q, f"dequantize_{scheme}")(*got) if scheme != "int8" else q.dequantize_int8(*got)
        ref_deq = dqf(*ref) if scheme != "int8" else dqf(ref[0], ref[1])
        assert torch.equal(deq.cpu(), ref_deq), scheme


def test_quantized_linear_matches_reference(golden):
    c = golden("quant.pt")
    for scheme in ("int8", "int4", "nf4"):
        ql = QuantizedLinear(c["lin_weight"].cuda(), c["lin_bias"].cuda(), scheme)
        assert set(dict(ql.named_buffers())) == {"weight_q", "scale"}
        with torch.no_grad():
            y = ql(c["lin_x"].cuda()).cpu()
        assert (y - c["qlin"][scheme]).abs().max().item() <= TOL, scheme


def test_quantized_block_matches_reference(golden):
    c = golden("quant.pt")
    for scheme in ("int8", "int4", "nf4"):
        m = CPUMamba(64, 16).eval()
        m.load_state_dict(c["block_params"], strict=True)
        m = m.cuda()
        assert quantize_block(m, QuantConfig(scheme=scheme)) == 4
        ref = c["qblock"][scheme]
        sd = m.state_dict()
        for k, v in ref["buffers"].items():
            assert torch.equal(sd[k].cpu(), v), (scheme, k)
        assert memory_footprint(m) == ref["footprint"]
        with torch.no_grad():
            y = m(c["block_x"].cuda()).cpu()
        assert (y - ref["y"]).abs().max().item() <= TOL, scheme


def test_quantize_on_cpu_module_then_cuda(golden):
    c = golden("quant.pt")
    m = CPUMamba(64, 16).eval()
    m.load_state_dict(c["block_params"], strict=True)
    quantize_block(m, QuantConfig("int4"))          # buffers come back to the CPU
    assert m.in_proj.weight_q.device.type == "cpu"
    m = m.cuda()
    with torch.no_grad():
        y = m(c["block_x"].cuda()).cpu()
    assert (y - c["qblock"]["int4"]["y"]).abs().max().item() <= TOL


def test_quantized_step_matches_oracle():
    p = oracle.make_block_params(96, 16, seed=31, weight_std=0.02, outlier_frac=0.01)
    for scheme in ("int8", "nf4"):
        m = CPUMamba(96, 16).eval()
        m.load_state_dict(p, strict=True)
        m = m.cuda()
        quantize_block(m, QuantConfig(scheme))
        pq = {k: v.cpu() for k, v in m.state_dict().items()}
        quant = {n: (scheme, getattr(m, n).in_features) for n in ("in_proj", "x_proj", "dt_proj", "out_proj")}
        x = torch.randn(3, 96)
        st = m.init_state(3)
        st_ref = oracle.init_state(pq, 3)
        for _ in range(3):
            with torch.no_grad():
                y, st = m.forward_step(x.cuda(), st)
            y_ref, st_ref = oracle.block_step(pq, x, st_ref, quant)
            assert (y.cpu() - y_ref).abs().max().item() <= TOL
        assert (st["h"].cpu() - st_ref["h"]).abs().max().item() <= TOL


@pytest.mark.parametrize("scheme", ["int8", "int4", "nf4"])
def test_quantized_block_many_rows_on_tensor_cores(scheme):
    """400 rows: each quantised projection is dequantised into the workspace
    (bit-exact values) and run on the tensor cores; matches the oracle's
    QuantizedLinear composition within the fp32 bar."""
    p = oracle.make_block_params(64, 16, seed=41, weight_std=0.02, outlier_frac=0.01)
    m = CPUMamba(64, 16).eval()
    m.load_state_dict(p, strict=True)
    m = m.cuda()
    quantize_block(m, QuantConfig(scheme))
    pq = {k: v.cpu() for k, v in m.state_dict().items()}
    quant = {n: (scheme, getattr(m, n).in_features) for n in ("in_proj", "x_proj", "dt_proj", "out_proj")}
    x = torch.randn(2, 200, 64, generator=torch.Generator().manual_seed(42))
    y_ref = oracle.block_forward(pq, x, quant=quant)
    with torch.no_grad():
        y = m(x.cuda()).cpu()
    assert (y - y_ref).abs().max().item() <= TOL


def test_quantized_block_many_rows_bf16():
    p = oracle.make_block_params(64, 16, seed=43, weight_std=0.02, outlier_frac=0.01)
    m = CPUMamba(64, 16).eval()
    m.load_state_dict(p, strict=True)
    m = m.cuda().to(torch.bfloat16)
    quantize_block(m, QuantConfig("int8"))
    pq = {k: v.cpu().float() if v.is_floating_point() else v.cpu() for k, v in m.state_dict().items()}
    quant = {n: ("int8", getattr(m, n).in_features) for n in ("in_proj", "x_proj", "dt_proj", "out_proj")}
    x = torch.randn(2, 200, 64, generator=torch.Generator().manual_seed(44))
    y_ref = oracle.block_forward(pq, x, quant=quant)
    with torch.no_grad():
        y = m(x.cuda().to(torch.bfloat16)).float().cpu()
    rel = ((y - y_ref).abs() / (y_ref.abs().clamp(min=1e-3) + 1e-6)).mean().item()
    assert rel <= 2e-2


@pytest.mark.parametrize("scheme", ["int8", "int4", "nf4"])
@pytest.mark.parametrize("rows,cols,group", [(48, 256, 64), (17, 100, 64), (5, 33, 16),
                                             (9, 70, 2)])
def test_grouped_quant_kernels_bit_exact(scheme, rows, cols, group):
    """Blockwise codes, scales and dequantised weights == the oracle's
    restatement (last group partial, odd widths padded)."""
    g = torch.Generator().manual_seed(rows * cols + group)
    w = torch.randn(rows, cols, generator=g) * 0.05
    w[torch.rand(rows, cols, generator=g) < 0.02] = 0.7
    w[0, :group] = 0.0                                 # an all-zero group: scale eps
    q_ref, s_ref = oracle.quant_grouped(scheme, w, group)
    from cpu_mamba_b200 import ops
    q, s, in_dim = ops.quantize(scheme, w.cuda(), group)
    assert torch.equal(q.cpu(), q_ref) and torch.equal(s.cpu(), s_ref)
    dq = ops.dequantize(scheme, q, s, in_dim, group).cpu()
    assert torch.equal(dq, oracle.dequant_grouped(scheme, q_ref, s_ref, cols, group))


def test_grouped_with_one_group_per_row_equals_per_row_kernels():
    from cpu_mamba_b200 import ops
    w = torch.randn(24, 96, device="cuda")
    for scheme in ("int8", "int4", "nf4"):
        qg, sg, _ = ops.quantize(scheme, w, 96)
        qr, sr, _ = ops.quantize(scheme, w)
        assert torch.equal(qg, qr) and torch.equal(sg[:, 0], sr)


@pytest.mark.parametrize("scheme", ["int4", "nf4", "int8"])
@pytest.mark.parametrize("T", [100, 200])
def test_grouped_quantized_block_matches_oracle(scheme, T):
    """A block quantised blockwise (group 64): 200 rows take the CUDA-core
    dequantising GEMM, 400 rows the dequantised-operand tensor-core GEMM."""
    p = oracle.make_block_params(64, 16, seed=51, weight_std=0.02, outlier_frac=0.01)
    m = CPUMamba(64, 16).eval()
    m.load_state_dict(p, strict=True)
    m = m.cuda()
    quantize_block(m, QuantConfig(scheme, group_size=64))
    assert m.in_proj.scale.shape == (256, 1) and m.out_proj.scale.shape == (64, 2)
    pq = {k: v.cpu() for k, v in m.state_dict().items()}
    quant = {n: (scheme, getattr(m, n).in_features, 64)
             for n in ("in_proj", "x_proj", "dt_proj", "out_proj")}
    x = torch.randn(2, T, 64, generator=torch.Generator().manual_seed(T))
    y_ref = oracle.block_forward(pq, x, quant=quant)
    with torch.no_grad():
        y = m(x.cuda()).cpu()
    assert (y - y_ref).abs().max().item() <= TOL
