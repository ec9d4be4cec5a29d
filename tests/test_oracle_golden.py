"""Pin the oracle: the CPU restatement must reproduce the reference's own outputs.

The golden fixtures were written by the reference itself (tests/golden/make_golden.py,
with the reference's compiled C++ scan op verified loaded).  Bars:
  * scan / block fp32: max abs diff <= 2e-6 (the reference was built with
    -ffast-math, so the last bits of exp differ from the oracle's expf);
  * quantisers: bit-exact (torch.equal) for codes, packed bytes, scales and
    dequantised weights.
"""
import pytest
import torch

import oracle


def test_scan_matches_reference_op(golden):
    for case in golden("scan.pt"):
        y = oracle.selective_scan(case["x"], case["dt"], case["A"], case["B"], case["C"], case["D"])
        assert y.shape == case["y"].shape
        if y.numel():
            assert (y - case["y"]).abs().max().item() <= 2e-6, case["x"].shape


def test_scan_rejects_large_state():
    x = torch.zeros(1, 2, 3)
    with pytest.raises(RuntimeError, match="d_state > 256"):
        oracle.selective_scan(x, x, torch.zeros(3, 257), torch.zeros(1, 2, 257),
                              torch.zeros(1, 2, 257), torch.zeros(3))


def test_block_fp32_matches_reference(golden):
    for case in golden("block.pt")["fp32"]:
        y = oracle.block_forward(case["params"], case["x"])
        assert (y - case["y"]).abs().max().item() <= 2e-6
        assert (y - case["y_loop"]).abs().max().item() <= 2e-6


def test_block_bf16_matches_reference(golden):
    case = golden("block.pt")["bf16"]
    p16 = {k: v.to(torch.bfloat16) for k, v in case["params"].items()}
    y16 = oracle.block_forward(p16, case["x"].to(torch.bfloat16))
    assert y16.dtype == torch.bfloat16
    # same ATen bf16 ops; only the fp32 scan's last bits differ
    diff = (y16.float() - case["y_bf16"].float()).abs()
    assert diff.max().item() <= 1e-2
    assert (diff > 0).float().mean().item() < 0.05
    y32 = oracle.block_forward(case["params"], case["x"])
    assert (y32 - case["y_fp32"]).abs().max().item() <= 2e-6


def test_stateful_matches_reference(golden):
    c = golden("stateful.pt")
    p, x, Tp = c["params"], c["x"], c["T_pref"]
    y_pref, st = oracle.block_forward_with_final_state(p, x[:, :Tp])
    assert (y_pref - c["y_pref"]).abs().max().item() <= 2e-6
    assert (st["h"] - c["pref_state"]["h"]).abs().max().item() <= 2e-6
    assert torch.equal(st["conv_state"], c["pref_state"]["conv_state"])
    ys = []
    for t in range(Tp, x.shape[1]):
        y, st = oracle.block_step(p, x[:, t], st)
        ys.append(y)
    assert (torch.stack(ys, 1) - c["y_steps"]).abs().max().item() <= 2e-6
    assert (st["h"] - c["final_state"]["h"]).abs().max().item() <= 2e-6
    assert torch.equal(st["conv_state"], c["final_state"]["conv_state"])
    st0 = oracle.init_state(p, x.shape[0])
    ys = []
    for t in range(4):
        y, st0 = oracle.block_step(p, x[:, t].unsqueeze(1), st0)
        ys.append(y)
    assert (torch.stack(ys, 1) - c["y_init_steps"]).abs().max().item() <= 2e-6


@pytest.mark.parametrize("name", ["normal", "outlier_odd", "ties"])
def test_quant_primitives_bit_exact(golden, name):
    c = golden("quant.pt")
    assert torch.equal(oracle.nf4_lut(), c["lut"])
    g = c["prims"][name]
    w = g["w"]
    q8, s8 = oracle.quant_int8(w)
    assert torch.equal(q8, g["int8"][0]) and torch.equal(s8, g["int8"][1])
    assert torch.equal(oracle.dequant_int8(q8, s8), g["int8"][2])
    p4, s4, d4 = oracle.quant_int4(w)
    assert d4 == g["int4"][2]
    assert torch.equal(p4, g["int4"][0]) and torch.equal(s4, g["int4"][1])
    assert torch.equal(oracle.dequant_int4(p4, s4, d4), g["int4"][3])
    pn, sn, dn = oracle.quant_nf4(w)
    assert torch.equal(pn, g["nf4"][0]) and torch.equal(sn, g["nf4"][1])
    assert torch.equal(oracle.dequant_nf4(pn, sn, dn), g["nf4"][3])


def test_quantized_linear_and_block_match_reference(golden):
    c = golden("quant.pt")
    w, b, x = c["lin_weight"], c["lin_bias"], c["lin_x"]
    for scheme in ("int8", "int4", "nf4"):
        wq = {"int8": oracle.quant_int8, "int4": oracle.quant_int4, "nf4": oracle.quant_nf4}[scheme](w)
        p = {"l.weight_q": wq[0], "l.scale": wq[1], "l.bias": b}
        y = oracle.linear(p, "l", x, {"l": (scheme, w.shape[1])})
        assert torch.equal(y, c["qlin"][scheme]), scheme
    p = c["block_params"]
    for scheme in ("int8", "int4", "nf4"):
        bufs = c["qblock"][scheme]["buffers"]
        pq = dict(bufs)
        quant = {}
        for name in ("in_proj", "x_proj", "dt_proj", "out_proj"):
            wq = {"int8": oracle.quant_int8, "int4": oracle.quant_int4, "nf4": oracle.quant_nf4}[scheme](
                p[f"{name}.weight"])
            assert torch.equal(wq[0], bufs[f"{name}.weight_q"]), (scheme, name)
            assert torch.equal(wq[1], bufs[f"{name}.scale"]), (scheme, name)
            quant[name] = (scheme, p[f"{name}.weight"].shape[1])
        y = oracle.block_forward(pq, c["block_x"], quant)
        assert (y - c["qblock"][scheme]["y"]).abs().max().item() <= 2e-6, scheme


def test_grouped_oracle_reduces_to_per_row_when_one_group_spans_the_row():
    """Blockwise quantisation with one group per row is quant.py's per-channel
    scheme: bit-exact with the oracle pinned to the reference."""
    import oracle
    g = torch.Generator().manual_seed(5)
    for cols in (64, 33):
        w = torch.randn(7, cols, generator=g)
        w[0, 3] = 4.0
        for scheme, per_row in (("int8", oracle.quant_int8), ("int4", oracle.quant_int4),
                                ("nf4", oracle.quant_nf4)):
            qg, sg = oracle.quant_grouped(scheme, w, 2 * cols)
            ref = per_row(w)
            assert torch.equal(qg, ref[0]), scheme
            assert torch.equal(sg[:, 0], ref[1].reshape(-1)), scheme
            dq = oracle.dequant_grouped(scheme, qg, sg, cols, 2 * cols)
            dr = oracle.dequant(scheme, ref[0], ref[1], cols)
            assert torch.equal(dq, dr), scheme


def test_grouped_nf4_is_tighter_than_per_row_on_outlier_rows():
    """The roadmap's reason for blockwise NF4: an outlier only coarsens its own
    group's scale."""
    import oracle
    g = torch.Generator().manual_seed(6)
    w = torch.randn(32, 256, generator=g) * 0.02
    w[torch.rand(32, 256, generator=g) < 0.01] = 0.5
    q, s = oracle.quant_grouped("nf4", w, 64)
    err_g = (oracle.dequant_grouped("nf4", q, s, 256, 64) - w).abs().mean()
    qr, sr, _ = oracle.quant_nf4(w)
    err_r = (oracle.dequant("nf4", qr, sr, 256) - w).abs().mean()
    assert err_g < 0.7 * err_r
