"""Multi-rank host logic of compactlogic_b200.parallel, run as world_size-2 gloo process groups on CPU:
per-layer gradient all-reduce hooks, broadcast of rank 0's buffers after resampling, sample sharding
of packed inference with the final count gather, and a bounded error when a rank disappears."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from compactlogic_b200 import parallel as P


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _spawn(target, world, *args, attempts=2):
    """Run `target(rank, world, port, *args, q)` on `world` spawned ranks; returns {rank: payload}.  A fresh
    rendezvous port per attempt: the port is picked free, then released before the ranks bind it, so another
    process can take it in between; one retry covers that race."""
    ctx = mp.get_context("spawn")
    for attempt in range(attempts):
        port = _port()
        q = ctx.Queue()
        procs = [ctx.Process(target=target, args=(r, world, port, *args, q)) for r in range(world)]
        for p in procs:
            p.start()
        try:
            res = dict(q.get(timeout=120) for _ in range(world))
        except Exception:
            res = None
        for p in procs:
            p.join(60)
            if p.is_alive():
                p.kill()
        if res is not None and all(p.exitcode == 0 for p in procs):
            return res
    raise AssertionError(f"{target.__name__}: ranks failed on {attempts} attempts")


def _init(rank, world, port, timeout_s=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _grad_worker(rank, world, port, q):
    _init(rank, world, port)
    torch.manual_seed(0)
    params = [torch.nn.Parameter(torch.randn(5, 4)) for _ in range(3)]
    sync = P.GradAllReduce(params)
    torch.manual_seed(100 + rank)
    x = torch.randn(4, 7)
    loss = sum(((p @ x) ** 2).sum() * (i + 1) for i, p in enumerate(params))
    loss.backward()
    sync.finish()
    q.put((rank, ([p.grad.clone() for p in params], x)))
    dist.destroy_process_group()


def test_grad_allreduce_averages_per_layer():
    world = 2
    res = _spawn(_grad_worker, world)
    torch.manual_seed(0)
    params = [torch.randn(5, 4) for _ in range(3)]
    for i, w in enumerate(params):
        expect = sum(2 * (i + 1) * (w @ res[r][1]) @ res[r][1].T for r in range(world)) / world
        for r in range(world):
            torch.testing.assert_close(res[r][0][i], expect)


def _bcast_worker(rank, world, port, q):
    _init(rank, world, port)
    import compactlogic_b200 as cl
    torch.manual_seed(rank)  # different replicas on purpose
    m = torch.nn.Sequential(cl.LogicLayer(10, 12, num_gates=4))
    P.broadcast_layer_buffers(m)
    q.put((rank, {k: v.clone() for k, v in m.state_dict().items()}))
    dist.destroy_process_group()


def test_broadcast_makes_replicas_identical():
    res = _spawn(_bcast_worker, 2)
    for k in res[0]:
        assert torch.equal(res[0][k], res[1][k]), k


def _gather_worker(rank, world, port, n, q):
    _init(rank, world, port)
    lo, hi = P.shard_range(n, rank, world)
    local = torch.arange(lo, hi, dtype=torch.int32).unsqueeze(1).repeat(1, 3) * (torch.arange(3, dtype=torch.int32) + 1)
    full = P.gather_counts(local, n)
    q.put((rank, full))
    dist.destroy_process_group()


@pytest.mark.parametrize("n", [1, 64, 130, 1000])
def test_shard_and_gather_counts(n):
    world = 2
    res = _spawn(_gather_worker, world, n)
    expect = torch.arange(n, dtype=torch.int32).unsqueeze(1).repeat(1, 3) * (torch.arange(3, dtype=torch.int32) + 1)
    for r in range(world):
        assert torch.equal(res[r], expect)


def test_shard_range_covers_whole_words():
    for n in (1, 63, 64, 65, 4096, 1 << 22):
        for world in (1, 2, 3, 8):
            parts = [P.shard_range(n, r, world) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            for (lo, hi), (lo2, _) in zip(parts[:-1], parts[1:]):
                assert hi == lo2 and lo % 64 == 0


def _dead_rank_worker(rank, world, port, q):
    _init(rank, world, port, timeout_s=5)
    if rank == 1:
        os._exit(0)  # leaves between steps, nothing in flight
    t = torch.ones(4)
    try:
        dist.all_reduce(t)
        q.put((rank, "no error"))
    except Exception as e:  # the surviving rank gets a bounded error instead of hanging
        q.put((rank, type(e).__name__))


def test_missing_rank_raises_bounded_error():
    world, port = 2, _port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_dead_rank_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    rank, outcome = q.get(timeout=120)
    for p in procs:
        p.join(60)
    assert rank == 0 and outcome != "no error"


def _flat_worker(rank, world, port, q):
    _init(rank, world, port)
    torch.manual_seed(0)
    params = [torch.nn.Parameter(torch.randn(5, 4)) for _ in range(3)]
    res = {}
    for bucket in ("layer", "flat"):
        for p in params:
            p.grad = None
        sync = P.GradAllReduce(params, bucket=bucket)
        torch.manual_seed(100 + rank)
        x = torch.randn(4, 7)
        sum(((p @ x) ** 2).sum() * (i + 1) for i, p in enumerate(params)).backward()
        sync.finish()
        sync.remove()
        res[bucket] = [p.grad.clone() for p in params]
    q.put((rank, res))
    dist.destroy_process_group()


def test_flat_bucket_equals_per_layer_buckets():
    res = _spawn(_flat_worker, 2)
    for r in range(2):
        for a, b in zip(res[r]["layer"], res[r]["flat"]):
            torch.testing.assert_close(a, b)
        for a, b in zip(res[r]["flat"], res[0]["flat"]):
            assert torch.equal(a, b)
