"""Host-side API of the package (no GPU): the reference's module surface,
state_dict layout (tests/test_parity.py:30-49 of the reference), helpers, and
the rule that there is no CPU fallback."""
import pytest
import torch

from cpu_mamba_b200 import (CPUMamba, QuantConfig, assert_state_dict_compatible,
                            memory_footprint, selective_scan)


def test_state_dict_keys_and_shapes():
    block = CPUMamba(d_model=384, d_state=24, d_conv=4, expand=2)
    sd = block.state_dict()
    assert set(sd) == {"A_log", "D", "in_proj.weight", "conv1d.weight", "conv1d.bias",
                       "x_proj.weight", "dt_proj.weight", "dt_proj.bias", "out_proj.weight"}
    assert sd["A_log"].shape == (768, 24)
    assert sd["D"].shape == (768,)
    assert sd["in_proj.weight"].shape == (1536, 384)
    assert sd["conv1d.weight"].shape == (768, 1, 4)
    assert sd["x_proj.weight"].shape == (24 + 48, 768)
    assert sd["dt_proj.weight"].shape == (768, 24)
    assert sd["out_proj.weight"].shape == (384, 768)
    assert torch.equal(sd["A_log"][0], torch.log(torch.arange(1, 25, dtype=torch.float32)))


def test_loads_reference_state_dict(golden):
    case = golden("block.pt")["fp32"][0]
    block = CPUMamba(d_model=case["d_model"], d_state=case["d_state"])
    block.load_state_dict(case["params"], strict=True)


def test_state_dict_compatibility_helper():
    block = CPUMamba(64, 8)
    sd = block.state_dict()
    assert_state_dict_compatible(block, sd)
    bad = dict(sd)
    bad["A_log"] = torch.zeros(100, 8)
    with pytest.raises(ValueError, match="shape mismatch"):
        assert_state_dict_compatible(block, bad)
    bad = dict(sd)
    bad["extra_key"] = torch.zeros(1)
    with pytest.raises(ValueError, match="unexpected keys"):
        assert_state_dict_compatible(block, bad)
    bad = dict(sd)
    del bad["D"]
    with pytest.raises(ValueError, match="missing keys"):
        assert_state_dict_compatible(block, bad)


def test_quant_config_validation():
    assert QuantConfig().scheme == "int8"
    for s in ("int8", "int4", "nf4"):
        QuantConfig(scheme=s)
    with pytest.raises(ValueError, match="unknown scheme"):
        QuantConfig(scheme="fp8")


def test_init_state_shapes_and_dtypes():
    block = CPUMamba(d_model=64, d_state=8, d_conv=4, expand=2)
    st = block.init_state(batch_size=4)
    assert st["h"].shape == (4, 128, 8) and st["h"].dtype == torch.float32
    assert st["conv_state"].shape == (4, 128, 3)
    st16 = block.to(torch.bfloat16).init_state(2)
    assert st16["h"].dtype == torch.float32 and st16["conv_state"].dtype == torch.bfloat16


def test_no_cpu_fallback():
    block = CPUMamba(64, 8).eval()
    x = torch.randn(1, 4, 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        block(x)
    with pytest.raises(RuntimeError, match="CUDA"):
        block.forward_step(x[:, 0], block.init_state(1))
    t = torch.zeros(1, 2, 3)
    with pytest.raises(RuntimeError, match="CUDA"):
        selective_scan(t, t, torch.zeros(3, 4), torch.zeros(1, 2, 4), torch.zeros(1, 2, 4),
                       torch.zeros(3))


def test_selective_scan_contract_errors():
    t = torch.zeros(1, 2, 3)
    A, Bm, D = torch.zeros(3, 4), torch.zeros(1, 2, 4), torch.zeros(3)
    with pytest.raises(RuntimeError, match="contiguous"):
        selective_scan(t.transpose(1, 2), t, A, Bm, Bm, D)
    with pytest.raises(RuntimeError, match="fp32 only"):
        selective_scan(t.double(), t, A, Bm, Bm, D)
    with pytest.raises(RuntimeError, match="shape mismatch"):
        selective_scan(t, t, A, Bm, Bm, D.view(1, 3))


def test_bf16_params_half_the_bytes_and_footprint():
    fp = CPUMamba(128, 16)
    bf = CPUMamba(128, 16).to(torch.bfloat16)
    fb = sum(p.numel() * p.element_size() for p in fp.parameters())
    bb = sum(p.numel() * p.element_size() for p in bf.parameters())
    assert bb == fb // 2
    m = memory_footprint(fp)
    assert m["quant_buffer_bytes"] == 0 and m["total_bytes"] == fb


def test_backend_attributes_tolerated():
    block = CPUMamba(64, 8)
    block._scan_backend = "assoc"
    block._assoc_chunk_T = 16
    block._force_time_loop = True
    assert set(block.state_dict()) == set(CPUMamba(64, 8).state_dict())


def test_stack_state_dict_layout_and_slices():
    """MambaStack keeps mamba_ssm's MixerModel names; forward_host's slices
    cover the batch with small end slices."""
    from cpu_mamba_b200 import MambaStack
    from cpu_mamba_b200.streaming import slice_bounds
    st = MambaStack(3, 64, d_state=16)
    sd = st.state_dict()
    assert sd["layers.2.norm.weight"].shape == (64,)
    assert sd["layers.0.mixer.in_proj.weight"].shape == (256, 64)
    assert len([k for k in sd if k.startswith("layers.1.")]) == 10
    with pytest.raises(RuntimeError, match="CUDA"):
        st(torch.randn(1, 4, 64))
    for B, n in [(151, 6), (7, 7), (10, 9), (5, 2), (1, 1), (151, 3)]:
        b = slice_bounds(B, n, 0.5)
        assert len(b) == n and b[0][0] == 0 and b[-1][1] == B
        assert all(lo < hi for lo, hi in b)
        assert all(b[i][1] == b[i + 1][0] for i in range(n - 1))
    b = slice_bounds(151, 6, 0.5)
    assert b[0][1] - b[0][0] < b[2][1] - b[2][0]


def test_surgery_stub_and_swap(monkeypatch):
    """surgery.py's two routes: the mamba_ssm stub hands out this package's
    block; the swap replaces foreign blocks and keeps their weights."""
    import sys
    import types

    import torch.nn as nn

    from cpu_mamba_b200 import surgery

    monkeypatch.delitem(sys.modules, "mamba_ssm", raising=False)
    surgery.install_mamba_ssm_stub()
    from mamba_ssm import Mamba
    assert Mamba is CPUMamba
    assert surgery.swap_mamba_to_cpu is surgery.swap_mamba_to_b200
    assert surgery.swap_mamba_to_b200(nn.Sequential(CPUMamba(32))) == 0   # nothing foreign

    class ForeignMamba(nn.Module):
        """Stands in for mamba_ssm.Mamba: same attributes and parameter names."""

        def __init__(self, d_model, d_state=16, d_conv=4, expand=2):
            super().__init__()
            src = CPUMamba(d_model, d_state=d_state, d_conv=d_conv, expand=expand)
            for k, v in src._modules.items():
                self.add_module(k, v)
            for k, v in src._parameters.items():
                self.register_parameter(k, v)
            self.d_model, self.d_state, self.d_conv, self.expand = d_model, d_state, d_conv, expand

    fake = types.ModuleType("mamba_ssm")
    fake.Mamba = ForeignMamba
    monkeypatch.setitem(sys.modules, "mamba_ssm", fake)
    model = nn.Sequential(ForeignMamba(32, d_state=8), nn.Linear(32, 32),
                          nn.ModuleList([ForeignMamba(32).eval()]))
    before = {k: v.clone() for k, v in model.state_dict().items()}
    assert surgery.swap_mamba_to_b200(model) == 2
    assert isinstance(model[0], CPUMamba) and isinstance(model[2][0], CPUMamba)
    assert model[0].d_state == 8 and not model[2][0].training
    after = model.state_dict()
    assert set(after) == set(before)
    assert all(torch.equal(after[k], before[k]) for k in before)


def test_quantize_block_finds_every_named_linear_once():
    """quantize_block's site walk (no quantisation, so no GPU): the linears
    named like a block's projections at any depth, each parent visited once,
    nothing found inside a matching linear, other names left alone."""
    from cpu_mamba_b200.quant import _QUANTIZABLE_LINEARS, _linear_sites
    inner = CPUMamba(32, 8)
    outer = torch.nn.Module()
    outer.a = inner
    outer.b = inner                      # the same block under two names: one visit
    outer.c = torch.nn.Sequential(CPUMamba(32, 8))
    outer.in_proj = torch.nn.Sequential(torch.nn.Linear(4, 4))   # not a Linear itself
    outer.head = torch.nn.Linear(4, 4)                          # not a target name
    sites = _linear_sites(outer, _QUANTIZABLE_LINEARS)
    assert len(sites) == 8
    assert sorted({a for _, a, _ in sites}) == sorted(_QUANTIZABLE_LINEARS)
    assert all(isinstance(lin, torch.nn.Linear) and getattr(p, a) is lin for p, a, lin in sites)


def test_memory_footprint_splits_quantised_buffers():
    m = torch.nn.Module()
    m.lin = torch.nn.Linear(8, 4, bias=True)                  # 36 floats
    q = torch.nn.Module()
    q.register_buffer("weight_q", torch.zeros(4, 8, dtype=torch.int8))
    q.register_buffer("scale", torch.zeros(4))
    q.register_buffer("other", torch.zeros(3))
    m.q = q
    assert memory_footprint(m) == {"param_bytes": 36 * 4 + 12, "quant_buffer_bytes": 32 + 16,
                                   "total_bytes": 36 * 4 + 12 + 48}
