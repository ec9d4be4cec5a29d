"""Host logic of the d_inner channel shards (cpu_mamba_b200.shard) on CPU.

The shards' arithmetic is restated here with torch ops over the oracle's scan
(the GPU library is not needed): every rank runs in_proj -> conv -> SiLU ->
its partial x_proj, the ranks sum x_dbl, every rank runs dt_proj -> scan ->
gate -> its partial out_proj, the ranks sum the output.  That composition
over shard_state_dict's slices must reproduce the unsharded block (the
oracle), in one process over emulated ranks and across two gloo ranks."""
import multiprocessing as mp
import os
import socket

import pytest
import torch
import torch.nn.functional as F

import oracle
from cpu_mamba_b200 import shard


def _head(p, x):
    di, S = p["A_log"].shape
    K = p["conv1d.weight"].shape[-1]
    T = x.shape[1]
    xz = F.linear(x, p["in_proj.weight"], p.get("in_proj.bias"))
    x_pre, z = xz.chunk(2, dim=-1)
    xc = F.conv1d(x_pre.transpose(1, 2), p["conv1d.weight"], p.get("conv1d.bias"),
                  padding=K - 1, groups=di)[..., :T]
    xc = F.silu(xc.transpose(1, 2))
    return xc, z, F.linear(xc, p["x_proj.weight"])


def _tail(p, xc, z, x_dbl):
    S = p["A_log"].shape[1]
    R = p["dt_proj.weight"].shape[1]
    dt_low, Bm, Cm = torch.split(x_dbl, [R, S, S], dim=-1)
    dt = F.softplus(F.linear(dt_low, p["dt_proj.weight"], p["dt_proj.bias"]))
    A = -torch.exp(p["A_log"].float())
    y = oracle.selective_scan(xc.contiguous(), dt.contiguous(), A, Bm.contiguous(),
                              Cm.contiguous(), p["D"])
    return F.linear(y * F.silu(z), p["out_proj.weight"], p.get("out_proj.bias"))


def _params(dm=32, S=8, seed=3, bias=False):
    p = oracle.make_block_params(dm, S, seed=seed)
    if bias:
        g = torch.Generator().manual_seed(seed + 1)
        p["in_proj.bias"] = torch.randn(p["in_proj.weight"].shape[0], generator=g) * 0.1
        p["out_proj.bias"] = torch.randn(dm, generator=g) * 0.1
    return p


@pytest.mark.parametrize("world", [1, 2, 3, 4])
@pytest.mark.parametrize("bias", [False, True])
def test_emulated_ranks_reproduce_the_block(world, bias):
    p = _params(bias=bias)
    di = p["A_log"].shape[0]
    x = torch.randn(3, 11, 32, generator=torch.Generator().manual_seed(0))
    shards = [shard.shard_state_dict(p, di, world, r) for r in range(world)]
    heads = [_head(s, x) for s in shards]
    x_dbl = sum(h[2] for h in heads)                      # all-reduce 1
    y = sum(_tail(s, h[0], h[1], x_dbl) for s, h in zip(shards, heads))   # all-reduce 2
    ref = oracle.block_forward(p, x)       # its linear() applies the biases in p
    assert (y - ref).abs().max().item() <= 1e-5


def test_shards_partition_the_weights():
    p = _params(bias=True)
    di = p["A_log"].shape[0]
    for world in (1, 2, 3, 5):
        sh = [shard.shard_state_dict(p, di, world, r) for r in range(world)]
        assert set(sh[0]) == set(p)
        xh = torch.cat([s["in_proj.weight"][: s["D"].shape[0]] for s in sh])
        zh = torch.cat([s["in_proj.weight"][s["D"].shape[0]:] for s in sh])
        assert torch.equal(torch.cat([xh, zh]), p["in_proj.weight"])
        for k in ("conv1d.weight", "conv1d.bias", "dt_proj.weight", "dt_proj.bias", "A_log", "D"):
            assert torch.equal(torch.cat([s[k] for s in sh]), p[k]), k
        for k in ("x_proj.weight", "out_proj.weight"):
            assert torch.equal(torch.cat([s[k] for s in sh], dim=1), p[k]), k
        assert torch.equal(sum(s["out_proj.bias"] for s in sh), p["out_proj.bias"])
        sizes = [s["D"].shape[0] for s in sh]
        assert max(sizes) - min(sizes) <= 1 and sum(sizes) == di
    with pytest.raises(KeyError):
        shard.shard_state_dict({"norm.weight": torch.ones(4)}, 4, 2, 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                          WORLD_SIZE=str(world), RANK=str(rank), LOCAL_RANK=str(rank))
        torch.set_num_threads(1)
        from cpu_mamba_b200 import dist as d
        d.init("gloo", timeout_s=60)
        reduce = shard._allreduce(None)              # the shards' reduction, over gloo
        p = _params()
        di = p["A_log"].shape[0]
        x = torch.randn(2, 9, 32, generator=torch.Generator().manual_seed(1))
        s = shard.shard_state_dict(p, di, world, rank)
        xc, z, x_dbl = _head(s, x)
        reduce(x_dbl)
        y = _tail(s, xc, z, x_dbl)
        reduce(y)
        d.shutdown()
        q.put(("ok", rank, (y - oracle.block_forward(p, x)).abs().max().item()))
    except Exception as e:
        q.put(("err", rank, f"{type(e).__name__}: {e}"))


def test_two_gloo_ranks_channel_sharded_forward():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_rank, args=(r, 2, port, q)) for r in range(2)]
    for pr in procs:
        pr.start()
    try:
        res = [q.get(timeout=120) for _ in procs]
    finally:
        for pr in procs:
            pr.join(timeout=30)
            if pr.is_alive():
                pr.kill()
    for r in res:
        assert r[0] == "ok", r
        assert r[2] <= 1e-5, r          # every rank holds the whole output
