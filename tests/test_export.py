"""The MB2W export format (cpu_mamba_b200.export): dense and quantised blocks
and stacks round-trip bit for bit through save / load, the records match the
documented layout, and a C program reading the file with include/mb2w_file.h
sees the same tensors (names, shapes, offsets, byte hashes)."""
import pathlib
import subprocess

import pytest
import torch

import oracle
from cpu_mamba_b200 import CPUMamba, MambaStack, QuantizedLinear, export

ROOT = pathlib.Path(__file__).resolve().parent.parent


def _block(dtype=torch.float32, bias=False, seed=0):
    p = oracle.make_block_params(32, 8, seed=seed)
    m = CPUMamba(32, 8, bias=bias)
    sd = dict(p)
    if bias:
        sd["in_proj.bias"] = torch.randn(128)
        sd["out_proj.bias"] = torch.randn(32)
    m.load_state_dict(sd)
    return m.to(dtype)


def _quantise(m, scheme, group=None):
    """Quantised projections built from the oracle's codes (no GPU needed)."""
    for name in ("in_proj", "x_proj", "dt_proj", "out_proj"):
        lin = getattr(m, name)
        w = lin.weight.detach().float()
        if group:
            q, s = oracle.quant_grouped(scheme, w, group)
        else:
            q, s = {"int8": oracle.quant_int8, "int4": oracle.quant_int4,
                    "nf4": oracle.quant_nf4}[scheme](w)[:2]
        b = lin.bias.detach() if lin.bias is not None else None
        setattr(m, name, QuantizedLinear.from_packed(q, s, b, scheme, w.shape[1], group))
    return m


def _same_state(a, b):
    sa, sb = a.state_dict(), b.state_dict()
    assert list(sa) == list(sb)
    for k in sa:
        assert sa[k].dtype == sb[k].dtype and torch.equal(sa[k], sb[k]), k


@pytest.mark.parametrize("dtype,bias", [(torch.float32, False), (torch.bfloat16, True)])
def test_dense_block_round_trip(tmp_path, dtype, bias):
    m = _block(dtype, bias)
    path = tmp_path / "b.mb2w"
    size = export.save(m, str(path))
    assert path.stat().st_size == size and size % 64 == 0
    meta, recs = export.read_header(str(path))
    assert meta["kind"] == 0 and meta["d_model"] == 32 and meta["d_inner"] == 64
    assert meta["bias"] == int(bias) and meta["dtype"] == export.DTYPES[dtype]
    assert all(r["offset"] % 64 == 0 for r in recs)
    m2 = export.load(str(path))
    _same_state(m, m2)
    assert m2.d_state == 8 and m2.dt_rank == m.dt_rank


@pytest.mark.parametrize("scheme,group", [("int8", None), ("int4", None), ("nf4", 16),
                                          ("int4", 8)])
def test_quantised_block_round_trip(tmp_path, scheme, group):
    m = _quantise(_block(), scheme, group)
    path = tmp_path / "q.mb2w"
    export.save(m, str(path))
    _, recs = export.read_header(str(path))
    wq = {r["name"]: r for r in recs if r["name"].endswith(".weight_q")}
    assert set(wq) == {f"{n}.weight_q" for n in ("in_proj", "x_proj", "dt_proj", "out_proj")}
    assert all(r["scheme"] == scheme and r["group_size"] == group for r in wq.values())
    m2 = export.load(str(path))
    _same_state(m, m2)
    for n in ("in_proj", "x_proj", "dt_proj", "out_proj"):
        a, b = getattr(m, n), getattr(m2, n)
        assert isinstance(b, QuantizedLinear)
        assert (b.scheme, b.group_size, b.in_features) == (a.scheme, a.group_size, a.in_features)


def test_stack_round_trip(tmp_path):
    s = MambaStack(3, 32, d_state=8, eps=1e-6)
    g = torch.Generator().manual_seed(4)
    with torch.no_grad():
        for p in s.parameters():
            p.copy_(torch.randn(p.shape, generator=g))
    path = tmp_path / "s.mb2w"
    export.save(s, str(path))
    meta, _ = export.read_header(str(path))
    assert meta["kind"] == 1 and meta["n_layers"] == 3 and meta["eps_1e12"] == 1_000_000
    s2 = export.load(str(path))
    assert isinstance(s2, MambaStack) and len(s2.layers) == 3 and s2.eps == 1e-6
    _same_state(s, s2)


def test_rejects_foreign_and_truncated_files(tmp_path):
    bad = tmp_path / "x.bin"
    bad.write_bytes(b"GGUF" + bytes(60))
    with pytest.raises(ValueError):
        export.read_header(str(bad))
    path = tmp_path / "b.mb2w"
    export.save(_block(), str(path))
    data = path.read_bytes()
    path.write_bytes(data[: len(data) - 64])
    with pytest.raises(ValueError):
        export.load(str(path))


def test_c_reader_sees_the_same_tensors(tmp_path):
    exe = tmp_path / "read_mb2w"
    r = subprocess.run(["gcc", "-std=c99", "-O1", "-Wall", "-Werror", "-o", str(exe),
                        str(ROOT / "tests" / "c" / "read_mb2w.c")], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    s = MambaStack(2, 32, d_state=8)
    path = tmp_path / "s.mb2w"
    export.save(s, str(path))
    out = subprocess.run([str(exe), str(path)], capture_output=True, text=True, check=True)
    lines = out.stdout.splitlines()
    assert lines[0] == "d_model 32" and lines[1] == "n_layers 2" and lines[-1] == "found_A_log 1"
    _, recs = export.read_header(str(path))
    raw = path.read_bytes()
    assert len(lines) == len(recs) + 3
    for line, rec in zip(lines[2:], recs):
        f = line.split()
        shape = [int(v) for v in f[3:7]][: int(f[2])]
        h = 1469598103934665603
        for byte in raw[rec["offset"]: rec["offset"] + rec["nbytes"]]:
            h = ((h ^ byte) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
        assert f[0] == rec["name"] and tuple(shape) == rec["shape"]
        assert int(f[7]) == rec["offset"] and int(f[8]) == rec["nbytes"]
        assert int(f[12], 16) == h
    # the C reader rejects a truncated file
    path.write_bytes(raw[:100])
    out = subprocess.run([str(exe), str(path)], capture_output=True, text=True, check=True)
    assert out.stdout.strip() == "error -2"


@pytest.mark.gpu
@pytest.mark.parametrize("scheme,group", [(None, None), ("int4", None), ("nf4", 16)])
def test_loaded_file_runs_like_the_original(tmp_path, scheme, group):
    m = _block()
    if scheme:
        m = _quantise(m, scheme, group)
    path = tmp_path / "g.mb2w"
    export.save(m, str(path))
    m2 = export.load(str(path), device="cuda:0")
    m = m.to("cuda:0")
    x = torch.randn(2, 40, 32, generator=torch.Generator().manual_seed(3)).cuda()
    with torch.no_grad():
        assert torch.equal(m(x), m2(x))
