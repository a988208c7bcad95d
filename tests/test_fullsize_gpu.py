"""Parity at the BASELINE configurations' full layer sizes.

- c2: one 64000 -> 64000 LogicLayer (K=16, batch 1024, fp32) forward and backward against the CPU oracle.
- c5: one 3072 -> 1,000,000 LogicLayer (K=4, bf16 activations, random gate ids) against the oracle on the
  bf16-rounded input, on a 128-sample batch.
- c4: the full 784 -> 8 x 256000 frozen network: packed class counts equal the counts of the float eval
  path (the reference's eval semantics) on 4096 samples, and every count is within [0, class size].
"""
import numpy as np
import pytest
import torch

import compactlogic_b200 as cl
from oracle import oracle as O

from helpers import assert_close, cuda

pytestmark = pytest.mark.gpu


def _layer_case(in_dim, out, K, B, dtype, seed, random_gates):
    torch.manual_seed(seed)
    layer = cl.LogicLayer(in_dim, out, num_gates=K)
    if random_gates:
        with torch.no_grad():
            layer.gate_sequence.copy_(torch.randint(0, 16, layer.gate_sequence.shape, dtype=torch.uint8))
    idx, g = layer.indices.numpy(), layer.gate_sequence.numpy()
    logits = layer.weights.detach().numpy().astype(np.float64)
    layer = layer.cuda()
    rng = np.random.default_rng(seed)
    x = rng.random((B, in_dim)).astype(np.float32)
    xt = torch.from_numpy(x).cuda().to(dtype).requires_grad_(True)
    y = layer(xt)
    xr = xt.detach().double().cpu().numpy().T
    p = O.softmax(logits)
    y_ref = O.dense_forward(xr, idx[0], idx[1], p, g)
    gy = rng.standard_normal((out, B))
    return layer, xt, y, xr, idx, g, p, y_ref, gy


def test_c2_full_layer():
    layer, xt, y, xr, idx, g, p, y_ref, gy = _layer_case(64000, 64000, 16, 1024, torch.float32, 2, False)
    assert_close(y.t(), y_ref, 1e-5, "c2 y")
    y.backward(cuda(gy.T.copy(), torch.float32))
    assert_close(layer.weights.grad, O.softmax_backward(p, O.dense_backward_w(xr, idx[0], idx[1], g, gy)), 1e-5,
                 "c2 grad_logits")
    assert_close(xt.grad.t(), O.dense_backward_x(xr, idx[0], idx[1], p, g, gy), 1e-5, "c2 grad_x")


def test_c5_full_width_layer_bf16():
    layer, xt, y, xr, idx, g, p, y_ref, gy = _layer_case(3072, 1_000_000, 4, 128, torch.bfloat16, 5, True)
    assert_close(y.t(), y_ref, 1e-2, "c5 y")
    gyb = torch.from_numpy(gy.T.copy()).cuda().bfloat16()
    y.backward(gyb)
    gyr = gyb.double().cpu().numpy().T
    assert_close(layer.weights.grad, O.softmax_backward(p, O.dense_backward_w(xr, idx[0], idx[1], g, gyr)), 1e-2,
                 "c5 grad_logits")


def test_c4_full_network_packed_equals_float_eval():
    torch.manual_seed(4)
    widths = [784] + [256000] * 8
    layers = []
    for i in range(8):
        layer = cl.LogicLayer(widths[i], widths[i + 1], num_gates=1)
        with torch.no_grad():
            layer.gate_sequence.copy_(torch.randint(0, 16, layer.gate_sequence.shape, dtype=torch.uint8))
        layer.freeze()
        layers.append(layer)
    model = torch.nn.Sequential(*layers, cl.GroupSum(10, 1.0)).cuda().eval()
    x = (torch.rand(4096, 784, device="cuda") < 0.5).float()
    counts = cl.PackedLogicNet(model)(x)
    pruned = cl.PackedLogicNet(model, prune="exact")
    assert torch.equal(pruned(x), counts) and pruned.prune_stats["kept"] < pruned.prune_stats["gates"]
    with torch.no_grad():
        float_counts = torch.round(model(x)).to(torch.int32)
    assert torch.equal(counts, float_counts)
    assert int(counts.min()) >= 0 and int(counts.max()) <= 25600
