"""GPU parity at the benchmark configurations' real dimensions.

The CUDA path runs each configuration's whole batch -- the launch shapes the
benchmark times (tile counts, T segments, split-K) -- and the oracle checks a
slice of the batch rows.  Batch rows are independent through the block and
through the residual stack, so every row of the GPU's output must match the
oracle's output for that row.

Bars (the contract's):
  * fp32: max abs diff <= 1e-5 against the oracle (configurations 0 and 2,
    whose outputs are O(1)).  At configuration 3 the outputs reach |y| ~ 1e3,
    where one fp32 ulp is ~1e-4 and the oracle itself sits ~1e-3 from the
    float64 result (asserted below), so there the 1e-5 bar applies to the
    output relative to its scale: max|y - y_oracle| / max(1, max|y_oracle|).
  * bf16: mean relative error <= 2e-2 against the fp32 oracle, with the
    formula of the reference's tests/test_bf16.py:53.
  * quantisation: packed codes, scales and dequantised weights bit-exact.
Reference tests mirrored: tests/test_parity.py:52-68 (block vs the C++ op),
tests/test_stateful.py:18-49 (prefill + steps vs full forward),
tests/test_bf16.py:36-62, tests/test_quant.py:110-145.
"""
import pytest
import torch

import oracle
from cpu_mamba_b200 import CPUMamba, MambaStack, QuantConfig, quantize_block

pytestmark = pytest.mark.gpu
TOL = 1e-5


def bf16_rel(y_fp, y_bf):
    y_fp, y_bf = y_fp.float().cpu(), y_bf.float().cpu()
    return ((y_fp - y_bf).abs() / (y_fp.abs().clamp(min=1e-3) + 1e-6)).mean().item()


def make_block(p, d_model, d_state, dt_rank, dtype=torch.float32):
    m = CPUMamba(d_model=d_model, d_state=d_state, dt_rank=dt_rank).eval()
    m.load_state_dict({k: v.float() for k, v in p.items()}, strict=True)
    return m.to(device="cuda", dtype=dtype)


def f64_report(p, x, y_gpu, y_ref, quant=None):
    """Where a bar fails: the GPU's and the oracle's distance to float64."""
    y64 = oracle.block_forward_f64(p, x, quant)
    return (f"gpu-oracle {(y_gpu.double() - y_ref.double()).abs().max().item():.3e}, "
            f"gpu-f64 {(y_gpu.double() - y64).abs().max().item():.3e}, "
            f"oracle-f64 {(y_ref.double() - y64).abs().max().item():.3e}")


def test_config0_fp32_block_b151_t180():
    """d_model 768, d_state 24, dt_rank 48, B=151, T=180, fp32, seed 0: every
    row against the oracle (the reference's composition around the C scan)."""
    p = oracle.make_block_params(768, 24, seed=0)
    x = torch.randn(151, 180, 768, generator=torch.Generator().manual_seed(0))
    m = make_block(p, 768, 24, 48)
    with torch.no_grad():
        y = m(x.cuda()).cpu()
    ref = oracle.block_forward(p, x)
    err = (y - ref).abs().max().item()
    if err > TOL:
        pytest.fail(f"config 0: max abs {err:.3e} > {TOL}; rows 0-1: "
                    + f64_report(p, x[:2], y[:2], ref[:2]))
    # the reference's own compiled op, where it was built, gives the same answer
    op = oracle.load_ref_scan_op()
    if op is not None:
        ref_op = oracle.block_forward(p, x[:8], scan_op=op)
        assert (y[:8] - ref_op).abs().max().item() <= TOL


def test_config1_bf16_block_b8_t8192():
    """d_model 768, d_state 16, B=8, T=8192 in bf16 (few chains over a long
    sequence: the scan's few-chain layout): rows 0 and 7 against the fp32
    oracle."""
    p = oracle.make_block_params(768, 16, seed=1)
    x = torch.randn(8, 8192, 768, generator=torch.Generator().manual_seed(1))
    m = make_block(p, 768, 16, 48, torch.bfloat16)
    with torch.no_grad():
        y = m(x.to(device="cuda", dtype=torch.bfloat16)).float().cpu()
    assert torch.isfinite(y).all()
    rows = [0, 7]
    ref = oracle.block_forward(p, x[rows])
    rel = bf16_rel(ref, y[rows])
    assert rel <= 2e-2, rel


def test_config2_prefill_512_then_256_steps_b64():
    """d_model 1024, d_state 16, dt_rank 64, B=64, fp32, seed 1:
    forward_with_final_state on 512 tokens, then 256 forward_step calls on
    fresh tokens; every output and the final h and conv ring buffer of rows 0
    and 63 against the oracle, and prefill + steps against one forward over
    all 768 tokens (the reference's tests/test_stateful.py:18-49 property)."""
    p = oracle.make_block_params(1024, 16, dt_rank=64, seed=1)
    g = torch.Generator().manual_seed(1)
    prompt = torch.randn(64, 512, 1024, generator=g)
    steps = torch.randn(256, 64, 1024, generator=g)
    m = make_block(p, 1024, 16, 64)
    ys = []
    with torch.no_grad():
        y_pref, st = m.forward_with_final_state(prompt.cuda())
        for t in range(256):
            y, st = m.forward_step(steps[t].cuda(), st)
            ys.append(y.cpu())
    y_steps = torch.stack(ys, 1)
    assert st["h"].shape == (64, 2048, 16) and st["conv_state"].shape == (64, 2048, 3)
    rows = [0, 63]
    ref_pref, ref_st = oracle.block_forward_with_final_state(p, prompt[rows])
    assert (y_pref.cpu()[rows] - ref_pref).abs().max().item() <= TOL
    ref_ys = []
    for t in range(256):
        y_r, ref_st = oracle.block_step(p, steps[t][rows], ref_st)
        ref_ys.append(y_r)
    err_y = (y_steps[rows] - torch.stack(ref_ys, 1)).abs().max().item()
    err_h = (st["h"].cpu()[rows] - ref_st["h"]).abs().max().item()
    err_c = (st["conv_state"].cpu()[rows] - ref_st["conv_state"]).abs().max().item()
    assert max(err_y, err_h, err_c) <= TOL, (err_y, err_h, err_c)
    # prefill + steps == one forward over the whole sequence (GPU only)
    with torch.no_grad():
        y_full = m(torch.cat([prompt, steps.transpose(0, 1)], 1).cuda()).cpu()
    both = torch.cat([y_pref.cpu(), y_steps], 1)
    assert (both - y_full).abs().max().item() <= 1e-4


@pytest.mark.parametrize("scheme", ["int8", "int4", "nf4"])
def test_config3_quantised_block_b32_t2048(scheme):
    """d_model 1536, d_state 16, dt_rank 96, B=32, T=2048, weights N(0, 0.02)
    with 1 % +-0.5 outliers, the four projections quantised per channel:
    codes / scales / dequantised weights bit-exact with the oracle, and rows 0
    and 31 of the output against the oracle's quantised block."""
    p = oracle.make_block_params(1536, 16, dt_rank=96, seed=3, weight_std=0.02,
                                 outlier_frac=0.01)
    x = torch.randn(32, 2048, 1536, generator=torch.Generator().manual_seed(3))
    m = make_block(p, 1536, 16, 96)
    assert quantize_block(m, QuantConfig(scheme)) == 4
    pq, quant = dict(p), {}
    for name in ("in_proj", "x_proj", "dt_proj", "out_proj"):
        w = p[f"{name}.weight"]
        if scheme == "int8":
            q, s = oracle.quant_int8(w)
            in_dim = w.shape[1]
        else:
            q, s, in_dim = getattr(oracle, f"quant_{scheme}")(w)
        lin = getattr(m, name)
        assert torch.equal(lin.weight_q.cpu(), q) and torch.equal(lin.scale.cpu(), s), name
        assert torch.equal(lin.dequantize_weight().cpu(), oracle.dequant(scheme, q, s, in_dim)), name
        pq[f"{name}.weight_q"], pq[f"{name}.scale"] = q, s
        quant[name] = (scheme, in_dim)
    with torch.no_grad():
        y = m(x.cuda()).cpu()
    rows = [0, 31]
    ref = oracle.block_forward(pq, x[rows], quant)
    scale = max(1.0, ref.abs().max().item())
    err = (y[rows] - ref).abs().max().item()
    if err / scale > TOL:
        pytest.fail(f"config 3 {scheme}: max abs {err:.3e} at output scale {scale:.1f}; row 0: "
                    + f64_report(pq, x[:1], y[:1], ref[:1], quant))
    # why the bar is relative here: the oracle itself is > 1e-5 from float64
    y64 = oracle.block_forward_f64(pq, x[:1], quant)
    assert (ref[:1].double() - y64).abs().max().item() > TOL


def test_config4_stack24_bf16_b1024_t2048():
    """24 RMSNorm pre-norm residual blocks, d_model 768, d_state 16, bf16,
    B=1024, T=2048 (the whole batch on one GPU): rows 0 and 1023 against the
    fp32 oracle stack (torch RMSNorm around the block)."""
    n, dm = 24, 768
    layers, sd = [], {}
    for i in range(n):
        p = oracle.make_block_params(dm, 16, seed=i)
        layers.append((p, torch.ones(dm)))
        sd[f"layers.{i}.norm.weight"] = torch.ones(dm)
        sd.update({f"layers.{i}.mixer.{k}": v for k, v in p.items()})
    m = MambaStack(n, dm, d_state=16, eps=1e-5).eval()
    m.load_state_dict(sd, strict=True)
    m = m.to(device="cuda", dtype=torch.bfloat16)
    rows = [0, 1023]
    g = torch.Generator(device="cuda").manual_seed(4)
    x = torch.randn(1024, 2048, dm, device="cuda", generator=g).to(torch.bfloat16)
    x_rows = x[rows].float().cpu()
    with torch.no_grad():
        m.forward_(x)                       # in place: 3.2 GB of activations
    y_rows = x[rows].float().cpu()
    del x
    assert torch.isfinite(y_rows).all()
    ref = oracle.stack_forward(layers, x_rows, 1e-5)
    rel = bf16_rel(ref, y_rows)
    assert rel <= 2e-2, rel
