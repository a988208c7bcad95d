"""Width-sharded training kernels and module (compactlogic_b200.sharded).

* Two ranks emulated on one GPU through the C ABI: each half of a layer's neurons stores its rows into
  both ranks' activation buffers (forward all-gather fused into the epilogue) and sums both ranks'
  partial grad_x buffers in its grad_y load (backward reduce-scatter); results against the CPU oracle.
  The two halves run one after the other: nothing waits on anything, the ordering is the stream's.
* The module as one process (world 1, NCCL) and as two processes on two GPUs: forward, loss and the
  gate-logit gradients of two successive training steps equal the unsharded model's; eval output
  equal.  The 2-GPU case is skipped when fewer than 2 GPUs are visible.
"""
import ctypes
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import compactlogic_b200 as cl
from compactlogic_b200 import _lib as L
from oracle import oracle as O

from helpers import assert_close

pytestmark = pytest.mark.gpu


def _arr(ptrs):
    return (ctypes.c_void_p * len(ptrs))(*ptrs)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_peer_kernels_two_virtual_ranks(dtype):
    torch.manual_seed(3)
    B, K = 160, 16
    l1 = cl.LogicLayer(64, 256, num_gates=K)
    l2 = cl.LogicLayer(256, 256, num_gates=K)
    with torch.no_grad():
        for l in (l1, l2):
            l.gate_sequence.copy_(torch.randint(0, 16, l.gate_sequence.shape, dtype=torch.uint8))
    ref = [(l.indices.numpy(), l.gate_sequence.numpy(), O.softmax(l.weights.detach().double().numpy())) for l in (l1, l2)]
    l1, l2 = l1.cuda(), l2.cuda()
    dev = torch.device("cuda")
    s1, s2 = l1._layer_spec(dev), l2._layer_spec(dev)
    rng = np.random.default_rng(4)
    xt = torch.from_numpy(rng.random((64, B))).to(dev, dtype).contiguous()
    e = xt.element_size()
    dt = L.dtype_code(dtype)
    st = L.stream(dev)
    halves = [(0, 128), (128, 256)]

    # forward of layer 1: each half writes its rows into both ranks' buffers
    Y = [torch.full((256, B), float("nan"), dtype=dtype, device=dev) for _ in range(2)]
    for lo, hi in halves:
        L.call("clb_logic_forward_peers", dt, L.ptr(xt), B, B, 64, L.ptr(s1.slots[lo:hi]), hi - lo, K, L.W_LOGITS,
               L.ptr(l1.weights[lo:hi]), L.ptr(s1.gates[lo:hi]), 0, _arr([L.ptr(y) + lo * B * e for y in Y]), 2, B, st)
    torch.cuda.synchronize()
    assert torch.equal(Y[0], Y[1])
    xr = xt.double().cpu().numpy()
    (i1, g1, p1), (i2, g2, p2) = ref
    y1 = O.dense_forward(xr, i1[0], i1[1], p1, g1)
    assert_close(Y[0], y1, 1e-5 if dtype == torch.float32 else 1e-2, "forward")

    # backward of layer 2 (replicated grad_y): each half produces its partial grad_x
    gy2 = torch.from_numpy(rng.standard_normal((256, B))).to(dev, torch.float32)
    P = [torch.empty(256, B, dtype=torch.float32, device=dev) for _ in range(2)]
    gw2 = []
    for (lo, hi), part_x in zip(halves, P):
        g = gy2[lo:hi].contiguous()
        ch = int(L.lib().clb_logic_backward_chunks(dt, L.ptr(Y[0]), B, B, 256, L.ptr(g), B, 0, 0, L.ptr(part_x), B))
        part = torch.empty(ch, hi - lo, K, dtype=torch.float32, device=dev)
        L.call("clb_logic_backward_peers", dt, L.ptr(Y[0]), B, B, L.ptr(s2.slots[lo:hi]), hi - lo, K, L.W_LOGITS,
               L.ptr(l2.weights[lo:hi]), L.ptr(s2.gates[lo:hi]), 0, _arr([L.ptr(g)]), 1, B, L.ptr(part_x), B, 1, 256,
               L.ptr(part), ch, st)
        gw = torch.empty(hi - lo, K, dtype=torch.float32, device=dev)
        L.call("clb_logic_grad_finalize", dt, L.ptr(part), ch, hi - lo, K, 1, L.W_LOGITS, L.ptr(l2.weights[lo:hi]),
               L.ptr(gw), st)
        gw2.append(gw)
    torch.cuda.synchronize()
    yr = Y[0].double().cpu().numpy()
    gyr = gy2.double().cpu().numpy()
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    gx2 = O.dense_backward_x(yr, i2[0], i2[1], p2, g2, gyr)
    assert_close(P[0] + P[1], gx2, tol, "grad_x partial sum")
    assert_close(torch.cat(gw2), O.softmax_backward(p2, O.dense_backward_w(yr, i2[0], i2[1], g2, gyr)), tol, "gw2")

    # backward of layer 1: grad_y rows summed over both ranks' partials inside the kernel
    gw1 = []
    for lo, hi in halves:
        peers = _arr([L.ptr(p) + lo * B * 4 for p in P])
        ch = int(L.lib().clb_logic_backward_chunks(dt, L.ptr(xt), B, B, 64, peers[0], B, 0, 0, 0, B))
        part = torch.empty(ch, hi - lo, K, dtype=torch.float32, device=dev)
        L.call("clb_logic_backward_peers", dt, L.ptr(xt), B, B, L.ptr(s1.slots[lo:hi]), hi - lo, K, L.W_LOGITS,
               L.ptr(l1.weights[lo:hi]), L.ptr(s1.gates[lo:hi]), 0, peers, 2, B, 0, B, 0, 64, L.ptr(part), ch, st)
        gw = torch.empty(hi - lo, K, dtype=torch.float32, device=dev)
        L.call("clb_logic_grad_finalize", dt, L.ptr(part), ch, hi - lo, K, 1, L.W_LOGITS, L.ptr(l1.weights[lo:hi]),
               L.ptr(gw), st)
        gw1.append(gw)
    torch.cuda.synchronize()
    assert_close(torch.cat(gw1), O.softmax_backward(p1, O.dense_backward_w(xr, i1[0], i1[1], g1, gx2)), tol, "gw1")


def test_peer_entry_points_validate():
    dev = torch.device("cuda")
    l1 = cl.LogicLayer(8, 8, num_gates=4).cuda()
    s = l1._layer_spec(dev)
    x = torch.rand(8, 16, device=dev)
    y = torch.empty(8, 16, device=dev)
    args = (L.CLB_F32, L.ptr(x), 16, 16, 8, L.ptr(s.slots), 8, 4, L.W_LOGITS, L.ptr(l1.weights), L.ptr(s.gates), 0)
    assert L.lib().clb_logic_forward_peers(*args, _arr([L.ptr(y)] * 9), 9, 16, L.stream(dev)) == L.CLB_ERR_INVALID
    assert L.lib().clb_logic_forward_peers(*args, _arr([L.ptr(y), L.ptr(y) + 4]), 2, 16,
                                           L.stream(dev)) == L.CLB_ERR_INVALID
    assert L.lib().clb_logic_forward_peers(*args, _arr([L.ptr(y), 0]), 2, 16, L.stream(dev)) == L.CLB_ERR_INVALID
    assert L.lib().clb_logic_forward_peers(*args, _arr([L.ptr(y)]), 1, 16, L.stream(dev)) == L.CLB_OK


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _model():
    torch.manual_seed(0)
    return torch.nn.Sequential(torch.nn.Flatten(), cl.LogicLayer(64, 256, num_gates=16),
                               cl.LogicLayer(256, 256, num_gates=16), cl.LogicLayer(256, 200, num_gates=16),
                               cl.GroupSum(10, tau=4.0))


def _worker(rank, world, port, dtype, q):
    import torch.distributed as dist
    from compactlogic_b200 import sharded as S
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        g = torch.Generator().manual_seed(1)
        x = (torch.rand(192, 64, generator=g) < 0.5).to(dtype).cuda()
        y = torch.randint(0, 10, (192,), generator=g).cuda()
        plain = _model().cuda()
        sharded = S.shard_width(_model().cuda())
        errs = {}
        popt = torch.optim.SGD(plain.parameters(), lr=0.5)
        sopt = torch.optim.SGD(sharded.parameters(), lr=0.5)
        for step in range(2):
            popt.zero_grad()
            sopt.zero_grad()
            lp = torch.nn.functional.cross_entropy(plain(x).float(), y)
            ls = torch.nn.functional.cross_entropy(sharded(x).float(), y)
            lp.backward()
            ls.backward()
            errs[f"loss{step}"] = abs(float(lp) - float(ls)) / abs(float(lp))
            for i, (pl, sl) in enumerate(zip([m for m in plain if type(m) is cl.LogicLayer],
                                             [m for m in sharded if isinstance(m, S.WidthShardedLogicLayer)])):
                ref = pl.weights.grad[sl.lo:sl.hi]
                errs[f"grad{step}.{i}"] = float((sl.weights.grad - ref).abs().max() / ref.abs().max())
            popt.step()
            sopt.step()
        plain.eval()
        sharded.eval()
        with torch.no_grad():
            errs["eval"] = float((plain(x).float() - sharded(x).float()).abs().max())
        for m in sharded:
            if isinstance(m, S.WidthShardedLogicLayer):
                m.release_buffers()
        q.put((rank, errs))
    finally:
        dist.destroy_process_group()


def _run(world, dtype):
    port = _port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, dtype, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    for rank, errs in res.items():
        for k, v in errs.items():
            limit = 0.0 if k == "eval" else tol
            assert v <= limit, (rank, k, v)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_width_sharded_module_one_rank(dtype):
    _run(1, dtype)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_width_sharded_matches_single_gpu_two_ranks(dtype):
    _run(2, dtype)
