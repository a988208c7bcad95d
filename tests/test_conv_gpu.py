"""ConvLayer on the GPU against the CPU oracle and through the reference API shims."""
import numpy as np
import pytest
import torch

import compactlogic_b200 as cl
from compactlogic_b200 import convlogic_cuda
from oracle import oracle as O

from helpers import RTOL, assert_close, cuda

pytestmark = pytest.mark.gpu

CASES = [  # (in_shape, pad, c_out, ks, stride, num_chn, K, N)
    ((9, 32, 32), 1, 128, 3, 2, 1, 16, 4),
    ((128, 16, 16), 1, 256, 3, 2, 1, 16, 2),
    ((6, 8, 8), 0, 9, 3, 1, 0, 16, 5),
    ((6, 7, 9), 1, 12, 2, 2, 3, 4, 3),
    ((4, 5, 5), 0, 8, 1, 1, 0, 8, 1),
]


def _layer(case, seed):
    in_shape, pad, c_out, ks, stride, num_chn, K, N = case
    torch.manual_seed(seed)
    return cl.ConvLayer(in_shape, pad, c_out, ks, stride, num_chn=num_chn, num_gates=K)


@pytest.mark.parametrize("case", CASES)
def test_conv_module_vs_oracle(case):
    layer = _layer(case, 1)
    N = case[-1]
    och, oh, ow = (layer.offsets_ch.numpy(), layer.offsets_h.numpy(), layer.offsets_w.numpy())
    g = layer.gate_sequence.numpy()
    logits = layer.weights.detach().numpy().astype(np.float64)
    layer = layer.cuda()
    x = np.random.default_rng(2).random((N,) + tuple(case[0])).astype(np.float32)
    xt = cuda(x).requires_grad_(True)
    y = layer(xt)
    p = O.softmax(logits)
    pad, ks, stride = case[1], case[3], case[4]
    y_ref = O.conv_forward(x, och, oh, ow, p, g, stride, pad, ks)
    assert_close(y, y_ref, 1e-5, "conv y")
    gy = np.random.default_rng(3).standard_normal(y_ref.shape)
    y.backward(cuda(gy, torch.float32))
    assert_close(xt.grad, O.conv_backward_x(x, och, oh, ow, p, g, gy, stride), 1e-5, "conv grad_x")
    assert_close(layer.weights.grad, O.softmax_backward(p, O.conv_backward_w(x, och, oh, ow, g, gy, stride)), 1e-5,
                 "conv grad_logits")
    layer.eval()
    xb = (x > 0.5).astype(np.float32)
    np.testing.assert_array_equal(layer(cuda(xb)).cpu().numpy(),
                                  O.conv_eval(xb, och, oh, ow, O.argmax_first(logits), g, stride, pad, ks))


def test_conv_chain_flatten_dense():
    """Conv -> Conv -> Flatten -> LogicLayer: the feature-major views chain without copies and the
    gradient reaches the input."""
    torch.manual_seed(5)
    model = torch.nn.Sequential(cl.ConvLayer((3, 8, 8), 1, 8, 3, 2, num_gates=4),
                                cl.ConvLayer((8, 4, 4), 1, 16, 3, 2, num_gates=4), torch.nn.Flatten(),
                                cl.LogicLayer(64, 40, num_gates=4), cl.GroupSum(4, 2.0)).cuda()
    x = torch.rand(6, 3, 8, 8, device="cuda", requires_grad=True)
    out = model(x)
    assert out.shape == (6, 4)
    out.sum().backward()
    assert x.grad is not None and torch.isfinite(x.grad).all()
    for m in model:
        if hasattr(m, "weights"):
            assert m.weights.grad is not None and torch.isfinite(m.weights.grad).all()


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_conv_reference_api_shims(dtype):
    case = CASES[3]
    layer = _layer(case, 7)
    in_shape, pad, c_out, ks, stride, _, K, N = case
    och, oh, ow = layer.offsets_ch.numpy(), layer.offsets_h.numpy(), layer.offsets_w.numpy()
    g = layer.gate_sequence.numpy()
    p = O.softmax(layer.weights.detach().numpy().astype(np.float64))
    x = np.random.default_rng(8).random((N,) + tuple(in_shape))
    xt = cuda(x, dtype)
    args = (cuda(och), cuda(oh), cuda(ow))
    y = convlogic_cuda.forward(xt, *args, cuda(p, dtype), cuda(g), stride, pad, ks)
    y_ref = O.conv_forward(x, och, oh, ow, p, g, stride, pad, ks)
    assert_close(y, y_ref, RTOL[dtype], "forward")
    gy = np.random.default_rng(9).standard_normal(y_ref.shape)
    gx = convlogic_cuda.backward_x(xt, *args, cuda(p, dtype), cuda(g), cuda(gy, dtype), stride, pad)
    assert_close(gx, O.conv_backward_x(x, och, oh, ow, p, g, gy, stride), RTOL[dtype], "backward_x")
    gw = convlogic_cuda.backward_w(xt, *args, cuda(g), cuda(gy, dtype), stride)
    assert_close(gw, O.conv_backward_w(x, och, oh, ow, g, gy, stride), RTOL[dtype], "backward_w")
    sel = O.argmax_first(layer.weights.detach().numpy())
    xb = (x > 0.5).astype(np.float64)
    ye = convlogic_cuda.eval(cuda(xb, dtype), *args, cuda(sel), cuda(g), stride, pad, ks)
    np.testing.assert_array_equal(ye.cpu().numpy(), O.conv_eval(xb, och, oh, ow, sel, g, stride, pad, ks))
