"""GPU parity of the residual pre-norm stack (MambaStack / mb2_stack_forward)
against the oracle's composition of torch RMSNorm and the pinned block.

Bars: fp32 max abs diff <= 1e-5 per layer of depth (each layer adds one
block's rounding to the residual stream); bf16 mean relative error <= 2e-2
against the fp32 oracle (the reference's tests/test_bf16.py:53 formula)."""
import pytest
import torch

import oracle
from cpu_mamba_b200 import MambaStack

pytestmark = pytest.mark.gpu
EPS = 1e-5


def make_stack(n_layers, d_model, d_state, dtype=torch.float32, seed=0):
    layers = []
    g = torch.Generator().manual_seed(seed)
    for i in range(n_layers):
        p = oracle.make_block_params(d_model, d_state, seed=seed * 100 + i)
        norm_w = 1.0 + 0.2 * torch.randn(d_model, generator=g)
        layers.append((p, norm_w))
    m = MambaStack(n_layers, d_model, d_state=d_state, eps=EPS).eval()
    sd = {}
    for i, (p, norm_w) in enumerate(layers):
        sd[f"layers.{i}.norm.weight"] = norm_w
        for k, v in p.items():
            sd[f"layers.{i}.mixer.{k}"] = v.float()
    m.load_state_dict(sd, strict=True)
    return m.to(device="cuda", dtype=dtype), layers


def bf16_rel(y_fp, y_bf):
    y_fp, y_bf = y_fp.float().cpu(), y_bf.float().cpu()
    return ((y_fp - y_bf).abs() / (y_fp.abs().clamp(min=1e-3) + 1e-6)).mean().item()


@pytest.mark.parametrize("n_layers,B,T", [(3, 2, 37), (2, 3, 100), (1, 1, 5)])
def test_stack_fp32_matches_oracle(n_layers, B, T):
    """74 rows run the CUDA-core projections; 300 rows the tensor-core ones
    (row scale and residual in the TMA-store epilogue)."""
    m, layers = make_stack(n_layers, 64, 16, seed=n_layers)
    x = torch.randn(B, T, 64, generator=torch.Generator().manual_seed(B * T))
    ref = oracle.stack_forward(layers, x, EPS)
    with torch.no_grad():
        y = m(x.cuda()).cpu()
    err = (y - ref).abs().max().item()
    assert err <= 1e-5 * n_layers, err


def test_stack_bf16_slice_of_24_layer_config():
    """The 24-layer d_model 768 / d_state 16 stack in bf16 on a batch slice
    (batch rows are independent, so a slice checks what every shard runs)."""
    m, layers = make_stack(24, 768, 16, dtype=torch.bfloat16, seed=7)
    x = torch.randn(2, 256, 768, generator=torch.Generator().manual_seed(0))
    ref = oracle.stack_forward(layers, x.to(torch.bfloat16).float(), EPS)
    with torch.no_grad():
        y = m(x.to(device="cuda", dtype=torch.bfloat16))
    assert torch.isfinite(y.float()).all()
    rel = bf16_rel(ref, y)
    assert rel <= 2e-2, rel


def test_stack_forward_does_not_modify_input_and_inplace_agrees():
    m, _ = make_stack(2, 64, 16)
    x = torch.randn(2, 40, 64, device="cuda")
    x0 = x.clone()
    with torch.no_grad():
        y = m(x)
        assert torch.equal(x, x0)
        z = m.forward_(x)
    assert z is x
    assert torch.equal(y, x)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_stack_forward_host_equals_forward(dtype):
    """Every slice (300 rows) and the whole batch (900) take the tensor-core
    projections: bit-equal.  With slices below 256 rows the CUDA-core GEMM
    runs instead: equal to within the projections' rounding."""
    m, _ = make_stack(2, 64, 16, dtype=dtype)
    x = torch.randn(3, 300, 64).to(dtype).pin_memory()
    with torch.no_grad():
        ref = m(x.cuda()).cpu()
        y = m.forward_host(x, chunks=3)
    assert torch.equal(y, ref)
    x = torch.randn(5, 60, 64).to(dtype).pin_memory()
    with torch.no_grad():
        ref = m(x.cuda()).cpu()
        y = m.forward_host(x, chunks=3)
    if dtype == torch.float32:
        assert (y - ref).abs().max().item() <= 2e-5
    else:
        assert bf16_rel(ref, y) <= 1e-2


def test_fold_norm_is_columnwise_product():
    from cpu_mamba_b200 import ops
    w = torch.randn(48, 40, device="cuda")
    g = torch.rand(40, device="cuda") + 0.5
    assert torch.equal(ops.fold_norm(w, g), w * g)
    wb, gb = w.bfloat16(), g.bfloat16()
    assert torch.equal(ops.fold_norm(wb, gb), (wb.float() * gb.float()).bfloat16())
