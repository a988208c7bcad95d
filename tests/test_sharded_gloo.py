"""Host logic of width-sharded training (compactlogic_b200.sharded) as world_size-2 gloo process
groups on CPU: the neuron shares partition every layer, the shards hold rank 0's rows after
shard_width, and unshard_into gathers them back into the reference layout."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from compactlogic_b200.sharded import shard_rows


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_rows_partition():
    for n in (1, 7, 64000, 1_000_000):
        for world in (1, 2, 3, 8):
            spans = [shard_rows(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert max(h - l for l, h in spans) - min(h - l for l, h in spans) <= 1


def _model(seed):
    import compactlogic_b200 as cl
    torch.manual_seed(seed)
    return torch.nn.Sequential(torch.nn.Flatten(), cl.LogicLayer(20, 30, num_gates=4), cl.LogicLayer(30, 17, num_gates=4),
                               cl.GroupSum(5, tau=2.0))


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from compactlogic_b200 import sharded as S
    ref = _model(10)                     # what rank 0 holds
    model = S.shard_width(_model(rank + 10), None)   # every rank starts from different values
    layers = [m for m in model.modules() if isinstance(m, S.WidthShardedLogicLayer)]
    refl = [ref[1], ref[2]]
    ok = True
    for s, r in zip(layers, refl):
        lo, hi = S.shard_rows(r.out_dim, rank, world)
        ok &= (s.lo, s.hi, s.full_out_dim, s.out_dim) == (lo, hi, r.out_dim, hi - lo)
        ok &= torch.equal(s.weights.detach(), r.weights.detach()[lo:hi])
        ok &= torch.equal(s.indices, r.indices[:, lo:hi]) and torch.equal(s.gate_sequence, r.gate_sequence[lo:hi])
        ok &= "weights" in s.state_dict() and "indices" in s.state_dict()
    plain = S.unshard_into(model, _model(99), None)
    for p, r in zip([plain[1], plain[2]], refl):
        ok &= torch.equal(p.weights.detach(), r.weights.detach()) and torch.equal(p.indices, r.indices)
        ok &= torch.equal(p.gate_sequence, r.gate_sequence)
        ok &= torch.equal(p.given_x_indices_of_y_start, r.given_x_indices_of_y_start)
    q.put((rank, bool(ok)))
    dist.destroy_process_group()


def test_shard_and_unshard_two_ranks():
    from test_parallel_gloo import _spawn
    assert _spawn(_worker, 2) == {0: True, 1: True}
