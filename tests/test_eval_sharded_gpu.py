"""Float eval (argmax gates, compactlogic.py:120-130) sharded by batch across 2 GPUs: every rank evaluates
its slice of the batch; the all-gathered class scores equal the single-GPU scores of the whole batch bit
for bit.  Skipped when fewer than 2 GPUs are visible."""
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
    torch.manual_seed(6)
    m = torch.nn.Sequential(cl.ConvLayer((3, 8, 8), 1, 12, 3, 2, num_gates=16), torch.nn.Flatten(),
                            cl.LogicLayer(192, 500, num_gates=16), cl.LogicLayer(500, 300, num_gates=16),
                            cl.GroupSum(10, 3.0))
    return cl.fuse_groupsum(m).eval()


def _data():
    g = torch.Generator().manual_seed(2)
    return (torch.rand(256, 3, 8, 8, generator=g) < 0.5).float()


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    model = _model().cuda()
    x = _data()
    per = x.shape[0] // world
    with torch.no_grad():
        local = model(x[rank * per:(rank + 1) * per].cuda()).contiguous()
    out = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(out, local)
    q.put((rank, torch.cat(out).cpu()))
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_eval_batch_sharded_equals_single_gpu():
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
    with torch.no_grad():
        ref = _model().cuda()(_data().cuda()).cpu()
    for r in range(world):
        assert torch.equal(res[r], ref)
