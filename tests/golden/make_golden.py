"""Write the golden fixtures in tests/golden/ by running the reference itself.

Run in a container that has the reference source tree (it cannot travel):

    MB2_REFERENCE_DIR=<cpu-mamba checkout> python tests/golden/make_golden.py

(or --ref <checkout>/src; without either, a ``reference`` directory beside this
repository is used when it exists).

The reference's JIT C++ scan op is built and REQUIRED: the reference silently
falls back to its Python time loop when the build fails
(src/cpu_mamba/_mamba.py:44-45), so this script asserts the op loaded.

Fixtures (torch.save dicts, all CPU tensors):
  scan.pt      selective_scan_cpu(x, dt, A, B, C, D) on ragged / edge shapes
  block.pt     CPUMamba.forward fp32 and bf16, and the time-loop output
  stateful.pt  forward_with_final_state + forward_step chains
  quant.pt     quantize_/dequantize_{int8,int4,nf4}, QuantizedLinear, quantised block
"""
from __future__ import annotations

import argparse
import math
import os
import pathlib
import sys
import tempfile

import torch

HERE = pathlib.Path(__file__).resolve().parent
REPO = HERE.parent.parent


def _import_reference(ref_src: str):
    if os.path.exists("/usr/bin/g++"):       # /opt/gcc cannot link OpenMP here
        os.environ["CXX"] = "/usr/bin/g++"
    # the op's JIT build goes to a throwaway directory, never into the repository
    os.environ.setdefault("TORCH_EXTENSIONS_DIR", tempfile.mkdtemp(prefix="mb2_golden_ext_"))
    sys.path.insert(0, ref_src)
    import cpu_mamba  # noqa: F401
    from cpu_mamba import _mamba, quant
    op = _mamba._try_load_cpp_scan()
    assert op is not None, "reference C++ scan op failed to build; refusing to write goldens"
    return _mamba, quant, op


def _params(d_model, d_state, d_conv=4, expand=2, seed=0, **kw):
    sys.path.insert(0, str(REPO))
    from oracle.mamba_oracle import make_block_params
    return make_block_params(d_model, d_state, d_conv, expand, seed=seed, **kw)


def _module(_mamba, p, d_model, d_state, dtype=torch.float32):
    m = _mamba.CPUMamba(d_model=d_model, d_state=d_state, d_conv=4, expand=2).eval()
    m.load_state_dict({k: v.float() for k, v in p.items()}, strict=True)
    return m.to(dtype)


def scan_cases(op):
    g = torch.Generator().manual_seed(1234)
    shapes = [(2, 33, 40, 24), (3, 17, 37, 16), (1, 5, 8, 1), (2, 9, 16, 64),
              (1, 3, 4, 256), (1, 1, 8, 8), (2, 0, 8, 4), (4, 64, 96, 24)]
    out = []
    for (b, t, di, s) in shapes:
        x = torch.randn(b, t, di, generator=g)
        dt = torch.nn.functional.softplus(torch.randn(b, t, di, generator=g) - 3.0)
        A = -torch.exp(torch.log(torch.arange(1, s + 1, dtype=torch.float32)).repeat(di, 1)
                       + 0.1 * torch.randn(di, s, generator=g))
        Bm = torch.randn(b, t, s, generator=g)
        Cm = torch.randn(b, t, s, generator=g)
        D = 1.0 + 0.1 * torch.randn(di, generator=g)
        y = op.selective_scan_cpu(x, dt, A, Bm, Cm, D)
        out.append(dict(x=x, dt=dt, A=A, B=Bm, C=Cm, D=D, y=y.clone()))
    return out


def block_cases(_mamba):
    cases = []
    g = torch.Generator().manual_seed(99)
    for (dm, S, b, t, seed) in [(64, 24, 3, 37, 0), (48, 16, 2, 5, 1), (32, 8, 1, 3, 2)]:
        p = _params(dm, S, seed=seed)
        m = _module(_mamba, p, dm, S)
        x = torch.randn(b, t, dm, generator=g)
        with torch.no_grad():
            y = m(x)
            m._force_time_loop = True
            y_loop = m(x)
        cases.append(dict(d_model=dm, d_state=S, params=p, x=x, y=y.clone(), y_loop=y_loop.clone()))
    # bf16 pair with shared weights (test_bf16.py style)
    p = _params(64, 16, seed=3)
    m32 = _module(_mamba, p, 64, 16)
    m16 = _module(_mamba, p, 64, 16, torch.bfloat16)
    x = torch.randn(2, 32, 64, generator=g)
    with torch.no_grad():
        y32 = m32(x)
        y16 = m16(x.to(torch.bfloat16))
    bf16 = dict(d_model=64, d_state=16, params=p, x=x, y_fp32=y32.clone(), y_bf16=y16.clone())
    return dict(fp32=cases, bf16=bf16)


def stateful_cases(_mamba):
    g = torch.Generator().manual_seed(5)
    p = _params(64, 8, seed=4)
    m = _module(_mamba, p, 64, 8)
    B, T, T_pref = 2, 16, 8
    x = torch.randn(B, T, 64, generator=g)
    with torch.no_grad():
        y_full = m(x)
        y_pref, st = m.forward_with_final_state(x[:, :T_pref])
        pref_state = {k: v.clone() for k, v in st.items()}
        y_steps = []
        for t in range(T_pref, T):
            ys, st = m.forward_step(x[:, t], st)
            y_steps.append(ys.clone())
        st0 = m.init_state(B)
        y_init_steps = []
        for t in range(4):
            ys, st0 = m.forward_step(x[:, t].unsqueeze(1), st0)
            y_init_steps.append(ys.clone())
    return dict(params=p, d_model=64, d_state=8, x=x, T_pref=T_pref, y_full=y_full,
                y_pref=y_pref, pref_state=pref_state, y_steps=torch.stack(y_steps, 1),
                final_state={k: v.clone() for k, v in st.items()},
                y_init_steps=torch.stack(y_init_steps, 1),
                init_steps_state={k: v.clone() for k, v in st0.items()})


def quant_cases(_mamba, quant):
    g = torch.Generator().manual_seed(77)
    w_normal = torch.randn(64, 256, generator=g)
    w_out = torch.randn(48, 33, generator=g) * 0.02
    mask = torch.rand(48, 33, generator=g) < 0.05
    w_out = torch.where(mask, torch.where(torch.rand(48, 33, generator=g) < 0.5, -0.5, 0.5), w_out)
    w_out[3] = 0.0                                   # all-zero row: amax clamps to 1e-8
    lut = torch.tensor(quant._NF4_LUT_VALUES, dtype=torch.float32)
    mids = (lut[:-1] + lut[1:]) / 2
    ties = torch.cat([mids, torch.tensor([1.0, 0.5, -0.5, 2.5 / 127, -3.5 / 127])])
    w_tie = torch.zeros(4, ties.numel())
    w_tie[0] = ties
    w_tie[1] = torch.tensor([127.0, 2.5, -3.5, 0.5, -0.5, 1.5, 126.5] + [0.0] * (ties.numel() - 7))
    w_tie[2] = torch.tensor([7.0, 2.5, -3.5, 0.5, -0.5, 1.5, 6.5] + [0.0] * (ties.numel() - 7))
    w_tie[3] = -w_tie[0]
    weights = dict(normal=w_normal, outlier_odd=w_out, ties=w_tie)
    prims = {}
    for name, w in weights.items():
        q8, s8 = quant.quantize_int8(w)
        p4, s4, d4 = quant.quantize_int4(w)
        pn, sn, dn = quant.quantize_nf4(w)
        prims[name] = dict(
            w=w, int8=(q8, s8, quant.dequantize_int8(q8, s8)),
            int4=(p4, s4, d4, quant.dequantize_int4(p4, s4, d4)),
            nf4=(pn, sn, dn, quant.dequantize_nf4(pn, sn, dn)))
    lin = torch.nn.Linear(33, 40)
    torch.nn.init.normal_(lin.weight, std=0.05, generator=g)
    torch.nn.init.normal_(lin.bias, std=0.1, generator=g)
    xl = torch.randn(5, 33, generator=g)
    qlin = {}
    for scheme in ("int8", "int4", "nf4"):
        ql = quant.QuantizedLinear(lin.weight.detach(), lin.bias.detach(), scheme)
        with torch.no_grad():
            qlin[scheme] = ql(xl).clone()
    p = _params(64, 16, seed=6, weight_std=0.02, outlier_frac=0.01)
    xb = torch.randn(2, 16, 64, generator=g)
    qblock = {}
    for scheme in ("int8", "int4", "nf4"):
        m = _module(_mamba, p, 64, 16)
        n = quant.quantize_block(m, quant.QuantConfig(scheme=scheme))
        assert n == 4
        with torch.no_grad():
            qblock[scheme] = dict(y=m(xb).clone(), footprint=quant.memory_footprint(m),
                                  buffers={k: v.clone() for k, v in m.state_dict().items()})
    return dict(lut=lut, prims=prims, lin_weight=lin.weight.detach().clone(),
                lin_bias=lin.bias.detach().clone(), lin_x=xl, qlin=qlin,
                block_params=p, block_x=xb, qblock=qblock)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=None, help="the reference's src/ directory")
    args = ap.parse_args()
    ref = args.ref
    if ref is None:
        sys.path.insert(0, str(REPO / "oracle"))
        from refpath import reference_root
        root = reference_root()
        if root is None:
            sys.exit("reference tree not found: pass --ref or set MB2_REFERENCE_DIR")
        ref = str(root / "src")
    torch.manual_seed(0)
    _mamba, quant, op = _import_reference(ref)
    torch.save(scan_cases(op), HERE / "scan.pt")
    torch.save(block_cases(_mamba), HERE / "block.pt")
    torch.save(stateful_cases(_mamba), HERE / "stateful.pt")
    torch.save(quant_cases(_mamba, quant), HERE / "quant.pt")
    for f in sorted(HERE.glob("*.pt")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
