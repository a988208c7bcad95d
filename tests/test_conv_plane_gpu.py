"""Receptive-field-staged conv kernels (clb_conv_plane_*) against the CPU oracle.

Every case uses the default num_chn == 1 connections (each output channel reads one input channel),
the layout the staged kernels take; batch sizes are multiples of 4 and include a partial 128-column
chunk.  The staged path must actually run (the spec carries a plan and the launches are recorded
under the conv kinds), and it must agree with the slot-table path on the same inputs.
"""
import os

import numpy as np
import pytest
import torch

import compactlogic_b200 as cl
from compactlogic_b200.functional import TIMER
from oracle import oracle as O

from helpers import assert_close, cuda

pytestmark = pytest.mark.gpu

CASES = [  # (in_shape, pad, c_out, ks, stride, K, N)
    ((9, 32, 32), 1, 128, 3, 2, 16, 132),   # c3 conv1, two column chunks (128 + 4)
    ((128, 16, 16), 1, 256, 3, 2, 16, 8),   # c3 conv2
    ((6, 10, 10), 1, 12, 3, 1, 8, 20),      # stride 1
    ((5, 9, 7), 0, 7, 2, 2, 4, 64),         # ks 2, no padding, ragged tiles
    ((12, 6, 6), 1, 5, 3, 2, 16, 4),        # fewer output than input channels: empty groups
    ((3, 12, 12), 2, 40, 5, 1, 4, 12),      # wide padding, 13+ channels per group
]


def _layer(case, seed):
    in_shape, pad, c_out, ks, stride, K, _ = case
    torch.manual_seed(seed)
    return cl.ConvLayer(in_shape, pad, c_out, ks, stride, num_chn=1, num_gates=K)


def _ref(layer):
    return (layer.offsets_ch.cpu().numpy(), layer.offsets_h.cpu().numpy(), layer.offsets_w.cpu().numpy(),
            layer.gate_sequence.cpu().numpy(), layer.weights.detach().cpu().numpy().astype(np.float64))


@pytest.mark.parametrize("case", CASES)
def test_conv_plane_vs_oracle(case):
    in_shape, pad, c_out, ks, stride, K, N = case
    layer = _layer(case, 11)
    och, oh, ow, g, logits = _ref(layer)
    layer = layer.cuda()
    assert layer._layer_spec(torch.device("cuda", torch.cuda.current_device())).conv is not None
    x = np.random.default_rng(12).random((N,) + tuple(in_shape)).astype(np.float32)
    xt = cuda(x).requires_grad_(True)
    TIMER.reset()
    TIMER.enabled = True
    try:
        y = layer(xt)
        p = O.softmax(logits)
        y_ref = O.conv_forward(x, och, oh, ow, p, g, stride, pad, ks)
        assert_close(y, y_ref, 1e-5, "conv y")
        gy = np.random.default_rng(13).standard_normal(y_ref.shape)
        y.backward(cuda(gy, torch.float32))
        torch.cuda.synchronize()
        kinds = {r[0] for r in TIMER.records}
    finally:
        TIMER.enabled = False
    assert {"conv_forward", "conv_backward"} <= kinds, kinds
    assert_close(xt.grad, O.conv_backward_x(x, och, oh, ow, p, g, gy, stride), 1e-5, "conv grad_x")
    assert_close(layer.weights.grad, O.softmax_backward(p, O.conv_backward_w(x, och, oh, ow, g, gy, stride)), 1e-5,
                 "conv grad_logits")
    layer.eval()
    xb = (x > 0.5).astype(np.float32)
    np.testing.assert_array_equal(layer(cuda(xb)).cpu().numpy(),
                                  O.conv_eval(xb, och, oh, ow, O.argmax_first(logits), g, stride, pad, ks))
    assert int(layer._layer_spec(xt.device).conv.err.item()) == 0


def test_conv_plane_first_layer_without_grad_x():
    """The input needs no gradient: the kernel instantiation without the shared grad_x tile."""
    case = CASES[0]
    layer = _layer(case, 21)
    och, oh, ow, g, logits = _ref(layer)
    layer = layer.cuda()
    x = (np.random.default_rng(22).random((36,) + tuple(case[0])) < 0.5).astype(np.float32)
    y = layer(cuda(x))
    gy = np.random.default_rng(23).standard_normal(tuple(y.shape))
    y.backward(cuda(gy, torch.float32))
    p = O.softmax(logits)
    assert_close(layer.weights.grad, O.softmax_backward(p, O.conv_backward_w(x, och, oh, ow, g, gy, case[4])), 1e-5,
                 "grad_logits")


def test_conv_plane_matches_slot_path(monkeypatch):
    case = CASES[1]
    layer = _layer(case, 31).cuda()
    x = torch.rand((16,) + tuple(case[0]), device="cuda")
    gy = torch.randn(16, 256, 8, 8, device="cuda")
    res = {}
    for mode in ("1", "0"):
        monkeypatch.setenv("CLB_CONV_PLANE", mode)
        layer.weights.grad = None
        xt = x.clone().requires_grad_(True)
        y = layer(xt)
        y.backward(gy)
        res[mode] = (y.detach().clone(), xt.grad.clone(), layer.weights.grad.clone())
    for a, b in zip(res["1"], res["0"]):
        assert_close(a, b.double().cpu().numpy(), 1e-5, "plane vs slot path")


def test_conv_plane_rejects_mixed_channels():
    """Random channels per slot (num_chn == 0) keep the slot-table kernels."""
    torch.manual_seed(3)
    layer = cl.ConvLayer((6, 8, 8), 1, 9, 3, 1, num_chn=0, num_gates=8).cuda()
    assert layer._layer_spec(torch.device("cuda", torch.cuda.current_device())).conv is None
