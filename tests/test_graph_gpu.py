"""CUDA-graph capture of the training step (compactlogic_b200.graph): replaying the captured step gives
the same losses and parameters as issuing the same steps op by op."""
import copy

import pytest
import torch

import compactlogic_b200 as cl
from compactlogic_b200.graph import GraphedLayerPass, GraphedTrainStep

pytestmark = pytest.mark.gpu


def _model():
    torch.manual_seed(2)
    m = torch.nn.Sequential(cl.ConvLayer((3, 8, 8), 1, 12, 3, 2, num_gates=16), cl.ConvLayer((12, 4, 4), 1, 24, 3, 2,
                                                                                           num_gates=8),
                            torch.nn.Flatten(), cl.LogicLayer(96, 400, num_gates=16), cl.GroupSum(10, 4.0))
    return cl.fuse_groupsum(m).cuda()


def test_graphed_train_step_matches_eager():
    g = torch.Generator().manual_seed(0)
    xs = [(torch.rand(64, 3, 8, 8, generator=g) < 0.5).float().cuda() for _ in range(6)]
    ys = [torch.randint(0, 10, (64,), generator=g).cuda() for _ in range(6)]
    eager, graphed = _model(), _model()
    opt_e = torch.optim.Adam(eager.parameters(), lr=0.01, capturable=True)
    opt_g = torch.optim.Adam(graphed.parameters(), lr=0.01, capturable=True)
    # the captured step runs 1 eager warm-up step on its inputs first: mirror it
    step = GraphedTrainStep(graphed, opt_g, torch.nn.functional.cross_entropy, xs[0], ys[0], clip=10.0, warmup=1)
    losses_e, losses_g = [], []
    for it in range(6):
        opt_e.zero_grad(set_to_none=True)
        loss = torch.nn.functional.cross_entropy(eager(xs[0] if it < 2 else xs[it - 1]), ys[0] if it < 2 else ys[it - 1])
        loss.backward()
        torch.nn.utils.clip_grad_norm_(list(eager.parameters()), 10.0)
        opt_e.step()
        losses_e.append(loss.item())
    losses_g = [None, step().item()] + [step(xs[i], ys[i]).item() for i in range(1, 5)]
    assert losses_g[1] == pytest.approx(losses_e[1], rel=1e-5)
    for a, b in zip(losses_g[2:], losses_e[2:]):
        assert a == pytest.approx(b, rel=1e-4)
    for pe, pg in zip(eager.parameters(), graphed.parameters()):
        torch.testing.assert_close(pg, pe, rtol=1e-4, atol=1e-5)


def test_graphed_layer_pass_matches_autograd():
    torch.manual_seed(3)
    layer = cl.LogicLayer(100, 300, num_gates=16).cuda()
    x = torch.rand(32, 100, device="cuda")
    gy = torch.randn(32, 300, device="cuda")
    gpass = GraphedLayerPass(layer, x, gy)
    x2, gy2 = torch.rand(32, 100, device="cuda"), torch.randn(32, 300, device="cuda")
    gx, gw = (t.clone() for t in gpass(x2, gy2))
    xr = x2.clone().requires_grad_(True)
    ref = torch.autograd.grad(layer(xr), [xr, layer.weights], gy2)
    torch.testing.assert_close(gx, ref[0], rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(gw, ref[1], rtol=1e-5, atol=1e-6)
