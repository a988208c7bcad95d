"""Parity at the BASELINE configurations' full layer sizes.

- c2: one 64000 -> 64000 LogicLayer (K=16, batch 1024, fp32) forward and backward against the CPU oracle.
- c5: one 3072 -> 1,000,000 LogicLayer (K=4, bf16 activations, random gate ids) against the oracle on the
  bf16-rounded input, on a 128-sample batch.
- c4: the full 784 -> 8 x 256000 frozen network: packed class counts equal the counts of the float eval
  path (the reference's eval semantics) on 4096 samples, and the oracle's packed evaluator on 256.
- c1: the LogicLayer(784, 12000, K=16) layer forward and backward at batch 256.
- c3: the whole conv -> conv -> dense -> GroupSum model at batch 512 (logits and every logit gradient).
- c5: grad_x of the 1M-wide bf16 layer.
"""
import numpy as np
import pytest
import torch

import compactlogic_b200 as cl
from oracle import oracle as O

from helpers import ELEM_RTOL, assert_close, assert_close_elem, assert_close_logit_grad, cuda

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


def test_c1_layer_fwd_bwd():
    """c1: LogicLayer(784, 12000, K=16) built under seed 0, batch 256, per-feature Bernoulli inputs."""
    torch.manual_seed(0)
    layer = cl.LogicLayer(784, 12000, num_gates=16)
    idx, g = layer.indices.numpy(), layer.gate_sequence.numpy()
    logits = layer.weights.detach().numpy().astype(np.float64)
    layer = layer.cuda()
    rng = np.random.default_rng(0)
    pf = rng.uniform(0.1, 0.9, 784)
    x = (rng.random((256, 784)) < pf).astype(np.float32)
    xt = cuda(x).requires_grad_(True)
    y = layer(xt)
    p = O.softmax(logits)
    xr = x.T.astype(np.float64)
    assert_close_elem(y.t(), O.dense_forward(xr, idx[0], idx[1], p, g), 1e-5, ELEM_RTOL[torch.float32], "c1 y")
    gy = rng.standard_normal((12000, 256))
    y.backward(cuda(gy.T.copy(), torch.float32))
    assert_close_elem(layer.weights.grad, O.softmax_backward(p, O.dense_backward_w(xr, idx[0], idx[1], g, gy)), 1e-5,
                      ELEM_RTOL[torch.float32], "c1 grad_logits")
    assert_close_elem(xt.grad.t(), O.dense_backward_x(xr, idx[0], idx[1], p, g, gy), 1e-5, ELEM_RTOL[torch.float32],
                      "c1 grad_x")


def test_c3_full_model_batch_512():
    """c3: (9,32,32) -> Conv(128) -> Conv(256) -> LogicLayer(128000) -> GroupSum(10, 20) at batch 512 with
    cross-entropy: logits and every layer's logit gradient against the oracle chain."""
    torch.manual_seed(1)
    conv1 = cl.ConvLayer((9, 32, 32), 1, 128, 3, 2, num_gates=16)
    conv2 = cl.ConvLayer((128, 16, 16), 1, 256, 3, 2, num_gates=16)
    dense = cl.LogicLayer(256 * 8 * 8, 128000, num_gates=16)
    tabs = [(m.offsets_ch.numpy(), m.offsets_h.numpy(), m.offsets_w.numpy(), m.gate_sequence.numpy(),
             O.softmax(m.weights.detach().numpy().astype(np.float64))) for m in (conv1, conv2)]
    didx, dg = dense.indices.numpy(), dense.gate_sequence.numpy()
    dp = O.softmax(dense.weights.detach().numpy().astype(np.float64))
    model = cl.fuse_groupsum(torch.nn.Sequential(conv1, conv2, torch.nn.Flatten(), dense, cl.GroupSum(10, 20.0)).cuda())
    g = torch.Generator().manual_seed(3)
    px = torch.rand(512, 3, 32, 32, generator=g)
    x = torch.cat([(px > (i + 1) / 4).float() for i in range(3)], dim=1)
    labels = torch.randint(0, 10, (512,), generator=g)
    logits = model(x.cuda())
    torch.nn.functional.cross_entropy(logits, labels.cuda()).backward()

    xn = x.numpy().astype(np.float64)
    h1 = O.conv_forward(xn, *tabs[0][:3], tabs[0][4], tabs[0][3], 2, 1, 3)
    h2 = O.conv_forward(h1, *tabs[1][:3], tabs[1][4], tabs[1][3], 2, 1, 3)
    hf = h2.reshape(512, -1).T
    y3 = O.dense_forward(hf, didx[0], didx[1], dp, dg)
    ref_logits = O.group_sum(y3.T, 10, 20.0)
    assert_close_elem(logits, ref_logits, 1e-5, ELEM_RTOL[torch.float32], "c3 logits")
    gl = O.cross_entropy_grad(ref_logits, labels.numpy())
    gy3 = O.group_sum_backward(gl, 128000, 10, 20.0).T
    assert_close_logit_grad(dense.weights.grad, dp, O.dense_backward_w(hf, didx[0], didx[1], dg, gy3), 1e-5,
                            "c3 dense grad_logits")
    gh2 = O.dense_backward_x(hf, didx[0], didx[1], dp, dg, gy3).T.reshape(h2.shape)
    och, oh, ow, g2, p2 = tabs[1]
    assert_close_logit_grad(conv2.weights.grad, p2, O.conv_backward_w(h1, och, oh, ow, g2, gh2, 2), 1e-5,
                            "c3 conv2 grad_logits", gp_abs=O.conv_backward_w(h1, och, oh, ow, g2, np.abs(gh2), 2))
    gh1 = O.conv_backward_x(h1, och, oh, ow, p2, g2, gh2, 2)
    och, oh, ow, g1, p1 = tabs[0]
    assert_close_logit_grad(conv1.weights.grad, p1, O.conv_backward_w(xn, och, oh, ow, g1, gh1, 2), 1e-5,
                            "c3 conv1 grad_logits", gp_abs=O.conv_backward_w(xn, och, oh, ow, g1, np.abs(gh1), 2))


def test_c4_full_network_vs_oracle_columns():
    """c4: the full 784 -> 8 x 256000 frozen network on 4 packed words (256 samples) against the oracle's
    packed evaluator: class counts bit-exact."""
    torch.manual_seed(4)
    widths = [784] + [256000] * 8
    layers = []
    for i in range(8):
        layer = cl.LogicLayer(widths[i], widths[i + 1], num_gates=1)
        with torch.no_grad():
            layer.gate_sequence.copy_(torch.randint(0, 16, layer.gate_sequence.shape, dtype=torch.uint8))
        layer.freeze()
        layers.append(layer)
    tabs = [O.frozen_tables(m.indices.numpy(), m.gate_sequence.numpy(), m.w.numpy()) for m in layers]
    model = torch.nn.Sequential(*layers, cl.GroupSum(10, 1.0)).cuda().eval()
    x = (torch.rand(256, 784, generator=torch.Generator().manual_seed(44)) < 0.5).float()
    counts = cl.PackedLogicNet(model)(x.cuda()).cpu().numpy()
    np.testing.assert_array_equal(counts, O.packed_network_counts(x.numpy(), tabs, 10))


def test_c5_full_width_grad_x_bf16():
    """c5: grad_x of one 3072 -> 1,000,000 layer (K=4, bf16 activations, random gate ids), the scatter
    path this config stresses, against the oracle on the bf16-rounded operands."""
    layer, xt, y, xr, idx, g, p, y_ref, gy = _layer_case(3072, 1_000_000, 4, 128, torch.bfloat16, 6, True)
    gyb = torch.from_numpy(gy.T.copy()).cuda().bfloat16()
    y.backward(gyb)
    gyr = gyb.double().cpu().numpy().T
    assert_close(xt.grad.t(), O.dense_backward_x(xr, idx[0], idx[1], p, g, gyr), 1e-2, "c5 grad_x")
