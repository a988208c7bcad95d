"""Host-side parity of the drop-in API with the reference Python: under the same seeds the layers
hold bit-identical buffers (the checkpoint layout), resampling / index refresh / pruning masks /
freezers behave identically.  No GPU needed (the kernels are not called)."""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

import compactlogic_b200 as cl

from conftest import GOLDEN


def _buffers(layer):
    return {n: t.detach().cpu().numpy() for n, t in list(layer.named_buffers()) + [("weights", layer.weights)]}


def _assert_same(layer, ref, prefix):
    mine = _buffers(layer)
    names = sorted(k[len(prefix) + 1:] for k in ref.files if k.startswith(prefix + ".") and "_flag" not in k)
    assert sorted(mine) == names, (sorted(mine), names)
    for n in names:
        exp = ref[f"{prefix}.{n}"]
        assert mine[n].dtype == exp.dtype and mine[n].shape == exp.shape, n
        np.testing.assert_array_equal(mine[n], exp, err_msg=f"{prefix}.{n}")


def test_dense_construction(golden):
    ref = golden("layer_buffers.npz")
    torch.manual_seed(0)
    _assert_same(cl.LogicLayer(20, 24, num_gates=16), ref, "dense_random")
    torch.manual_seed(1)
    _assert_same(cl.LogicLayer(30, 16, connections="original", num_gates=8), ref, "dense_original")
    torch.manual_seed(2)
    _assert_same(cl.LogicLayer(12, 10, num_gates=4, residual_init=True), ref, "dense_residual")


@pytest.mark.parametrize("seed,num_chn,ks,pad,stride", [(3, 1, 3, 1, 2), (4, 0, 3, 0, 1), (5, 3, 2, 1, 2),
                                                        (6, 0, 1, 0, 1)])
def test_conv_construction(golden, seed, num_chn, ks, pad, stride):
    ref = golden("layer_buffers.npz")
    torch.manual_seed(seed)
    layer = cl.ConvLayer((6, 8, 8), pad, 9, ks, stride, num_chn=num_chn, num_gates=16)
    _assert_same(layer, ref, f"conv_{seed}")


def test_resample_and_refresh(golden):
    ref = golden("layer_buffers.npz")
    torch.manual_seed(7)
    layer = cl.LogicLayer(40, 50, num_gates=16)
    with torch.no_grad():
        layer.weights[0:10] = 0.0
        layer.weights[10:20, 3] = 20.0
    torch.manual_seed(8)
    weak, strong = layer.resample_connections(torch.arange(0, 30), threshold_high=0.9, threshold_low=0.1)
    np.testing.assert_array_equal(weak.numpy(), ref["resample.weak"])
    np.testing.assert_array_equal(strong.numpy(), ref["resample.strong"])
    _assert_same(layer, ref, "resample.after")

    torch.manual_seed(9)
    conv = cl.ConvLayer((4, 6, 6), 1, 8, 3, 1, num_chn=1, num_gates=8)
    with torch.no_grad():
        conv.weights[0:3] = 0.0
        conv.weights[3:6, 1] = 15.0
    torch.manual_seed(10)
    conv.resample_connections(torch.arange(0, 8), threshold_high=0.9, threshold_low=0.2)
    _assert_same(conv, ref, "conv_resample.after")

    torch.manual_seed(11)
    layer = cl.LogicLayer(16, 12, num_gates=4)
    with torch.no_grad():
        layer.indices[0, 3] = torch.tensor([1, 2, 3, 4])
        layer.indices[1, 7] = torch.tensor([5, 5, 5, 5])
    layer.refresh_backward_index(torch.tensor([3, 7]))
    _assert_same(layer, ref, "refresh")


def test_connected_neurons(golden):
    ref = golden("layer_buffers.npz")
    torch.manual_seed(12)
    layer = cl.LogicLayer(30, 20, num_gates=16)
    layer.freeze()
    x_flag, y_flag = layer.connected_neurons(torch.ones(20, dtype=torch.bool))
    _assert_same(layer, ref, "connected")
    np.testing.assert_array_equal(x_flag.numpy(), ref["connected.x_flag"])
    np.testing.assert_array_equal(y_flag.numpy(), ref["connected.y_flag"])


def test_c1_layer_buffers_sha():
    """LogicLayer(784, 12000, 16) under seed 0 (the c1 configuration) is byte-identical to the reference."""
    with open(os.path.join(GOLDEN, "big_layer_sha.json")) as f:
        ref = json.load(f)["sha256"]
    torch.manual_seed(0)
    layer = cl.LogicLayer(784, 12000, num_gates=16)
    for name, t in list(layer.named_buffers()) + [("weights", layer.weights)]:
        assert hashlib.sha256(t.detach().contiguous().numpy().tobytes()).hexdigest() == ref[name], name


class _Fake(torch.nn.Module):
    def __init__(self, rows):
        super().__init__()
        self.weights = torch.nn.Parameter(torch.zeros(rows, 4))
        self.log_k = float(np.log(4))
        self.is_frozen = False

    def weights_entropy(self):
        log_p = torch.log_softmax(self.weights, -1)
        return -(log_p.exp() * log_p).sum(-1) / self.log_k

    def freeze(self):
        self.is_frozen = True


@pytest.mark.parametrize("name,make", [
    ("sequential", lambda m: cl.SequentialEntropyFreezer(m, ema_decay=0.7, eps=1e-2, patience=3, min_iters=2)),
    ("sequential_l2", lambda m: cl.SequentialEntropyFreezer(m, ema_decay=0.7, eps=1e-2, patience=3, l=2)),
    ("fixed", lambda m: cl.FixedSequentialEntropyFreezer(m, N=7, min_iters=5)),
])
def test_freezer_traces(name, make):
    with open(os.path.join(GOLDEN, "freezer_trace.json")) as f:
        ref = json.load(f)[name]
    layers = [_Fake(3) for _ in range(4)]
    fr = make(layers)
    trace = []
    for it in range(90):
        with torch.no_grad():
            for li, layer in enumerate(layers):
                if it < 10 + 8 * li:
                    layer.weights[:, 0] += 0.3
        fr.step(it)
        trace.append([int(layer.is_frozen) for layer in layers])
    assert trace == ref


def test_resampler_resets_adam_state():
    torch.manual_seed(3)
    layer = cl.LogicLayer(10, 12, num_gates=4)
    model = torch.nn.Sequential(layer)
    opt = torch.optim.Adam(model.parameters())
    layer.weights.grad = torch.randn_like(layer.weights)
    opt.step()
    with torch.no_grad():
        layer.weights[:4] = 0.0
    rs = cl.EntropyRowResampler(model, ema_decay=0.5, eps=1.0, patience=1, threshold_low=0.5)
    rs.step(0, opt)
    rs.step(1, opt)
    st = opt.state[layer.weights]
    assert (st["exp_avg"][:4] == 0).all() and (st["exp_avg_sq"][:4] == 0).all()


def test_groupsum_reference_semantics():
    gs = cl.GroupSum(3, tau=2.0, device="cpu")
    x = torch.arange(14, dtype=torch.float32).reshape(2, 7)
    padded = torch.cat([x, torch.zeros(2, 2)], 1)
    torch.testing.assert_close(gs(x), padded.reshape(2, 3, 3).sum(-1) / 2.0)


def test_fuse_groupsum_keeps_state_dict():
    model = torch.nn.Sequential(torch.nn.Flatten(), cl.LogicLayer(8, 12, num_gates=4), cl.GroupSum(3, 1.0))
    keys = list(model.state_dict())
    cl.fuse_groupsum(model)
    assert list(model.state_dict()) == keys
    assert model[1]._fused_groupsum == (3, 1.0) and model[2].absorbed
