"""d_inner channel shards on the GPU (cpu_mamba_b200.shard).

On one GPU the ranks are emulated: every shard runs its head, the test sums
x_dbl over the shards (in rank order) and writes the sum back into every
shard's workspace, every shard runs its tail, the test sums the outputs.
That is the library's shard path with the all-reduces done by hand; it must
match the oracle (fp32 1e-5 max abs, bf16 mean rel err 2e-2) and, for one
shard, the unsharded block bit for bit.  On two GPUs the same runs as two
processes over NCCL and over the library's peer-memory all-reduce (skipped
with fewer GPUs); that all-reduce's bounded wait is checked on one GPU with a
peer that never arrives."""
import ctypes
import multiprocessing as mp
import os
import socket

import pytest
import torch

import oracle
from cpu_mamba_b200 import CPUMamba, QuantConfig, StepGraph, quantize_block
from cpu_mamba_b200._lib import PeerGroup, check, lib
from cpu_mamba_b200.shard import ChannelShardedMamba, PeerReducer

PEER_TIMEOUT = 0x7e01

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _block(dm, S, dtype=torch.float32, seed=3, bias=False):
    p = oracle.make_block_params(dm, S, seed=seed)
    m = CPUMamba(dm, S, bias=bias)
    sd = dict(p)
    if bias:
        g = torch.Generator().manual_seed(seed + 1)
        sd["in_proj.bias"] = torch.randn(2 * m.d_inner, generator=g) * 0.1
        sd["out_proj.bias"] = torch.randn(dm, generator=g) * 0.1
    m.load_state_dict(sd)
    return m.to(DEV, dtype), {k: v.float() for k, v in sd.items()}


def _shards(m, world):
    return [ChannelShardedMamba(m, world=world, rank=r) for r in range(world)]


def _sum_into(ts):
    s = ts[0].clone()
    for t in ts[1:]:
        s += t
    return s


def _emulated_forward(shards, x, want_state=False):
    ctxs = [s.head(x, want_state) for s in shards]
    xd = _sum_into([c["x_dbl"] for c in ctxs])
    for c in ctxs:
        c["x_dbl"].copy_(xd)
    return _sum_into([s.tail(c) for s, c in zip(shards, ctxs)]), ctxs


def _emulated_step(shards, x, states):
    ctxs = [s.step_head(x, st) for s, st in zip(shards, states)]
    xd = _sum_into([c["x_dbl"] for c in ctxs])
    for c in ctxs:
        c["x_dbl"].copy_(xd)
    return _sum_into([s.tail(c) for s, c in zip(shards, ctxs)])


def _rel(y, ref):
    return ((y.float().cpu() - ref).abs() / (ref.abs().clamp(min=1e-3) + 1e-6)).mean().item()


@pytest.mark.parametrize("world", [1, 2, 3, 4])
@pytest.mark.parametrize("B,T,dm", [(3, 37, 64), (4, 100, 128)])
def test_emulated_shards_match_oracle(world, B, T, dm):
    m, p = _block(dm, 16, bias=(world == 3))
    x = torch.randn(B, T, dm, generator=torch.Generator().manual_seed(5))
    xd = x.to(DEV)
    with torch.no_grad():
        y, _ = _emulated_forward(_shards(m, world), xd)
        full = m(xd)
    ref = oracle.block_forward(p, x)
    assert (y.cpu() - ref).abs().max().item() <= 1e-5
    if world == 1:
        assert torch.equal(y, full)      # one shard is the block: same kernels, same bits


def test_emulated_shards_final_state_and_steps():
    dm, S, B, T, world = 64, 16, 4, 29, 2
    m, p = _block(dm, S)
    x = torch.randn(B, T + 6, dm, generator=torch.Generator().manual_seed(6))
    shards = _shards(m, world)
    with torch.no_grad():
        y, ctxs = _emulated_forward(shards, x[:, :T].to(DEV), want_state=True)
        y_ref, st_ref = oracle.block_forward_with_final_state(p, x[:, :T])
        assert (y.cpu() - y_ref).abs().max().item() <= 1e-5
        h = torch.cat([c["h"] for c in ctxs], dim=1).cpu()
        conv = torch.cat([c["conv_state"] for c in ctxs], dim=1).cpu()
        assert (h - st_ref["h"]).abs().max().item() <= 1e-5
        assert (conv - st_ref["conv_state"]).abs().max().item() <= 1e-5
        states = [{"h": c["h"], "conv_state": c["conv_state"]} for c in ctxs]
        full_state = {"h": h.to(DEV), "conv_state": conv.to(DEV)}
        st = st_ref
        for t in range(T, T + 6):
            ys = _emulated_step(shards, x[:, t].to(DEV), states)
            yf, _ = m.forward_step(x[:, t].to(DEV), full_state)
            yo, st = oracle.block_step(p, x[:, t], st)
            assert (ys.cpu() - yo).abs().max().item() <= 1e-5
            assert (ys - yf).abs().max().item() <= 1e-5
        h = torch.cat([s["h"] for s in states], dim=1).cpu()
        assert (h - st["h"]).abs().max().item() <= 1e-5


def test_emulated_shards_bf16():
    dm, B, T = 128, 2, 300
    m, p = _block(dm, 16, dtype=torch.bfloat16)
    x = torch.randn(B, T, dm, generator=torch.Generator().manual_seed(7))
    with torch.no_grad():
        y, _ = _emulated_forward(_shards(m, 2), x.to(DEV, torch.bfloat16))
    assert _rel(y, oracle.block_forward(p, x)) <= 2e-2


def test_quantised_block_is_not_channel_sharded():
    m, _ = _block(64, 16)
    quantize_block(m, QuantConfig("int8"))
    with pytest.raises(NotImplementedError):
        ChannelShardedMamba(m, world=2, rank=0)


def test_peer_reducer_single_rank_is_identity():
    red = PeerReducer(max_elems=4096)
    try:
        for dtype in (torch.float32, torch.bfloat16):
            for n in (1, 7, 1024, 4096):
                t = torch.randn(n, device=DEV).to(dtype)
                ref = t.clone()
                red(t)
                torch.cuda.synchronize()
                assert torch.equal(t, ref)
        assert red.status() == 0
    finally:
        red.close()


def test_peer_wait_times_out_without_hanging():
    """A two-rank group whose second rank never runs: rank 0's kernel waits
    for flags nothing sets, gives up after the group's 50 ms bound, records
    MB2_PEER_TIMEOUT, and the context stays usable."""
    L = lib()
    nbytes = L.mb2_peer_buffer_bytes(2, 1024)
    ptrs = []
    try:
        for _ in range(2):
            p, h = ctypes.c_void_p(), ctypes.create_string_buffer(64)
            check(L.mb2_peer_alloc(nbytes, ctypes.byref(p), h), "alloc")
            ptrs.append(p.value)
        g = PeerGroup()
        g.world, g.rank, g.slot_elems, g.timeout_ns = 2, 0, 1024, 50_000_000
        g.bufs[0], g.bufs[1] = ptrs
        t = torch.ones(1000, device=DEV)
        torch.cuda.synchronize()
        check(L.mb2_peer_allreduce(0, t.data_ptr(), t.numel(), ctypes.byref(g),
                                   torch.cuda.current_stream().cuda_stream), "allreduce")
        torch.cuda.synchronize()
        code = ctypes.c_int()
        check(L.mb2_peer_status(ctypes.byref(g), ctypes.byref(code), 1), "status")
        assert code.value == PEER_TIMEOUT
        check(L.mb2_peer_status(ctypes.byref(g), ctypes.byref(code), 0), "status")
        assert code.value == 0                          # cleared
        assert torch.ones(4, device=DEV).sum().item() == 4.0
        bad = PeerGroup()
        bad.world, bad.rank, bad.slot_elems, bad.timeout_ns = 2, 0, 1024, 1
        bad.bufs[0] = ptrs[0]                           # rank 1's buffer missing
        assert L.mb2_peer_allreduce(0, t.data_ptr(), 10, ctypes.byref(bad), None) != 0
        g.slot_elems = 10
        assert L.mb2_peer_allreduce(0, t.data_ptr(), 11, ctypes.byref(g), None) != 0
    finally:
        for p in ptrs:
            check(L.mb2_peer_free(p), "free")


# ------------------------------------------------------------ two GPUs ---
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_rank(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world),
                          RANK=str(rank), LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        from cpu_mamba_b200 import dist as d
        d.init("nccl", device=dev, timeout_s=60)
        dm, S, B, T = 128, 16, 3, 64
        p = oracle.make_block_params(dm, S, seed=11)
        m = CPUMamba(dm, S)
        m.load_state_dict(p)
        m = m.to(dev)
        sh = ChannelShardedMamba(m, world=world, rank=rank)
        x = torch.randn(B, T + 4, dm, generator=torch.Generator().manual_seed(2))
        with torch.no_grad():
            y, st = sh.forward_with_final_state(x[:, :T].to(dev))
            errs = [(y.cpu() - oracle.block_forward(p, x[:, :T])).abs().max().item()]
            full_state = m.forward_with_final_state(x[:, :T].to(dev))[1]
            for t in range(T, T + 4):
                ys, _ = sh.forward_step(x[:, t].to(dev), st)
                yf, _ = m.forward_step(x[:, t].to(dev), full_state)
                errs.append((ys - yf).abs().max().item())
            # the peer-memory all-reduce: exact rank-order sums, eager and in a graph
            import torch.distributed as td
            red = PeerReducer(max_elems=1 << 16, timeout_s=10.0)
            for dtype in (torch.float32, torch.bfloat16):
                for n in (1, 1000, 4099, 1 << 16):
                    t = torch.randn(n, generator=torch.Generator().manual_seed(n + rank)).to(dev, dtype)
                    parts = [torch.empty_like(t) for _ in range(world)]
                    td.all_gather(parts, t)
                    want = parts[0].float()
                    for pt in parts[1:]:
                        want = want + pt.float()
                    red(t)
                    errs.append(0.0 if torch.equal(t, want.to(dtype)) else float("inf"))
            shp = ChannelShardedMamba(m, world=world, rank=rank, reduce=red)
            y2, st2 = shp.forward_with_final_state(x[:, :T].to(dev))
            errs.append((y2.cpu() - oracle.block_forward(p, x[:, :T])).abs().max().item())
            full_state = m.forward_with_final_state(x[:, :T].to(dev))[1]
            graph = StepGraph(shp, st2, x[:, T].to(dev))
            for t in range(T, T + 4):
                ys = graph(x[:, t].to(dev)).clone()
                yf, _ = m.forward_step(x[:, t].to(dev), full_state)
                errs.append((ys - yf).abs().max().item())
            torch.cuda.synchronize()
            if red.status() != 0:
                errs.append(float("inf"))
            del graph
            red.close()
        torch.cuda.synchronize()
        d.shutdown()
        q.put(("ok", rank, max(errs)))
    except Exception as e:
        q.put(("err", rank, f"{type(e).__name__}: {e}"))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpus_nccl_channel_shards():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_rank, args=(r, 2, port, q)) for r in range(2)]
    for pr in procs:
        pr.start()
    try:
        res = [q.get(timeout=300) for _ in procs]
    finally:
        for pr in procs:
            pr.join(timeout=60)
            if pr.is_alive():
                pr.kill()
    for r in res:
        assert r[0] == "ok", r
        assert r[2] <= 1e-5, r
