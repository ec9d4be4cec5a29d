"""The multi-GPU host logic (cpu_mamba_b200.dist) on CPU: two ``gloo`` ranks
in spawned processes.  Batch shards are disjoint and cover the batch, the
sharded block forward (the oracle stands in for the GPU compute) reassembles
to the unsharded result, the timing reductions take the slowest rank, and a
rank that leaves early makes its peer's next collective fail instead of hang."""
import multiprocessing as mp
import os
import socket

import pytest
import torch

from cpu_mamba_b200 import dist


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _env(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world),
                      RANK=str(rank), LOCAL_RANK=str(rank))


def _sharded_forward(rank, world, port, q):
    try:
        _env(rank, world, port)
        import torch.distributed as td
        import oracle
        from cpu_mamba_b200 import dist as d
        torch.set_num_threads(1)
        d.init("gloo", timeout_s=60)
        assert d.env() == (world, rank, rank)
        B, T, dm = 7, 9, 32
        p = oracle.make_block_params(dm, 8, seed=3)
        x = torch.randn(B, T, dm, generator=torch.Generator().manual_seed(0))
        lo, hi = d.shard(B, world, rank)
        y_local = oracle.block_forward(p, x[lo:hi])          # this rank's shard only
        parts = [None] * world
        td.all_gather_object(parts, (lo, hi, y_local))        # test-side reassembly
        t_max = d.max_over_ranks(1.5 + rank)
        n_all = d.sum_over_ranks(hi - lo)
        d.shutdown()
        if rank == 0:
            parts.sort(key=lambda e: e[0])
            assert [e[0] for e in parts] == [0] + [e[1] for e in parts[:-1]]
            y = torch.cat([e[2] for e in parts])
            ref = oracle.block_forward(p, x)
            q.put(("ok", (y - ref).abs().max().item(), t_max, n_all))
    except Exception as e:  # report to the parent instead of hanging it
        q.put(("err", f"rank {rank}: {type(e).__name__}: {e}"))


def _early_exit(rank, world, port, q):
    try:
        _env(rank, world, port)
        from cpu_mamba_b200 import dist as d
        d.init("gloo", timeout_s=10)
        if rank == 1:
            return                                     # leaves between steps
        try:
            d.barrier()
            q.put(("err", "barrier returned although the peer left"))
        except Exception as e:
            q.put(("ok", type(e).__name__))
    except Exception as e:
        q.put(("err", f"rank {rank}: {type(e).__name__}: {e}"))


def _run(target, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = q.get(timeout=timeout)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return res


def test_shards_are_disjoint_and_cover():
    for total in (0, 1, 7, 8, 1024, 1025):
        for world in (1, 2, 3, 8):
            s = [dist.shard(total, world, r) for r in range(world)]
            assert s[0][0] == 0 and s[-1][1] == total
            assert all(s[i][1] == s[i + 1][0] for i in range(world - 1))
            sizes = [b - a for a, b in s]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        dist.shard(4, 2, 2)


def test_single_process_reductions_are_identity():
    assert dist.max_over_ranks(3.25) == 3.25
    assert dist.sum_over_ranks(4) == 4.0


def test_two_gloo_ranks_sharded_forward_and_timing():
    res = _run(_sharded_forward)
    assert res[0] == "ok", res
    _, err, t_max, n_all = res
    assert err <= 1e-6
    assert t_max == 2.5          # the slower rank's time
    assert n_all == 7            # all shards' rows


def test_peer_leaving_fails_the_next_collective():
    res = _run(_early_exit)
    assert res[0] == "ok", res
