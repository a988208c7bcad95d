"""Data-parallel training over NCCL on 2 GPUs: after one step with the batch split across the ranks and
the per-layer gradient all-reduce, the gate-logit gradients equal those of the whole batch on one GPU.
Skipped when fewer than 2 GPUs are visible."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _model():
    import compactlogic_b200 as cl
    torch.manual_seed(0)
    m = torch.nn.Sequential(torch.nn.Flatten(), cl.LogicLayer(64, 256, num_gates=16), cl.LogicLayer(256, 200, num_gates=16),
                            cl.GroupSum(10, tau=4.0))
    return cl.fuse_groupsum(m)


def _data():
    g = torch.Generator().manual_seed(1)
    return (torch.rand(128, 64, generator=g) < 0.5).float(), torch.randint(0, 10, (128,), generator=g)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    from compactlogic_b200.parallel import GradAllReduce
    model = _model().cuda()
    params = [p for p in model.parameters()]
    sync = GradAllReduce(params)
    x, y = _data()
    per = x.shape[0] // world
    xs, ys = x[rank * per:(rank + 1) * per].cuda(), y[rank * per:(rank + 1) * per].cuda()
    torch.nn.functional.cross_entropy(model(xs), ys).backward()
    sync.finish()
    q.put((rank, [p.grad.cpu() for p in params]))
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_dp_gradients_match_single_gpu():
    world, port = 2, _port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    model = _model().cuda()
    x, y = _data()
    torch.nn.functional.cross_entropy(model(x.cuda()), y.cuda()).backward()
    for i, p in enumerate(model.parameters()):
        ref = p.grad.cpu()
        for r in range(world):
            torch.testing.assert_close(res[r][i], ref, rtol=1e-5, atol=1e-6 * ref.abs().max().item())
