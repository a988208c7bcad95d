"""Bit-packed discrete inference on the GPU: bit-exact against the oracle and against the class
counts of the reference's CPU circuit evaluator."""
import numpy as np
import pytest
import torch

import compactlogic_b200 as cl
from compactlogic_b200 import difflogic_cuda
from oracle import oracle as O

from helpers import cuda

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("bits", [8, 16, 32, 64])
@pytest.mark.parametrize("rows,cols,k", [(20, 1, 5), (20, 100, 4), (30, 129, 3), (64, 1000, 8), (10, 0, 2)])
def test_packbits_groupbitsum(bits, rows, cols, k):
    rng = np.random.default_rng(rows * cols + bits)
    t = rng.random((rows, cols)) < 0.3
    words, pad = difflogic_cuda.tensor_packbits_cuda(cuda(t), bits)
    ref_words, ref_pad = O.packbits(t, bits)
    assert pad == ref_pad
    np.testing.assert_array_equal(words.cpu().numpy(), ref_words)
    if rows % k == 0:
        np.testing.assert_array_equal(difflogic_cuda.groupbitsum(words, pad, k).cpu().numpy(),
                                      O.groupbitsum(ref_words, ref_pad, k))
    else:
        with pytest.raises(ValueError):
            difflogic_cuda.groupbitsum(words, pad, k)


def _model_from_fixture(d):
    widths = [int(v) for v in d["widths"]]
    layers = []
    for i in range(1, len(widths)):
        layer = cl.LogicLayer(widths[i - 1], widths[i], num_gates=16)
        with torch.no_grad():
            layer.weights.copy_(torch.from_numpy(d[f"{i}.weights"]))
            layer.indices.copy_(torch.from_numpy(d[f"{i}.indices"]))
            layer.gate_sequence.copy_(torch.from_numpy(d[f"{i}.gate_sequence"]))
        layers.append(layer)
    return torch.nn.Sequential(torch.nn.Flatten(), *layers, cl.GroupSum(int(d["k"]), float(d["tau"]))).cuda()


@pytest.mark.parametrize("chunk_words", [1, 2, 32])
def test_packed_net_matches_reference_circuit(golden, chunk_words):
    d = golden("discrete.npz")
    model = _model_from_fixture(d)
    net = cl.PackedLogicNet(model, chunk_words=chunk_words)
    x = cuda(d["x"].astype(np.float32))
    np.testing.assert_array_equal(net(x).cpu().numpy(), d["counts"])
    # the float eval path of the same model gives the same counts (round(logits * tau))
    model.eval()
    logits = model(x)
    np.testing.assert_array_equal(torch.round(logits * float(d["tau"])).to(torch.int32).cpu().numpy(), d["counts"])
    cl.fuse_groupsum(model)
    np.testing.assert_array_equal(torch.round(model(x) * float(d["tau"])).to(torch.int32).cpu().numpy(), d["counts"])


@pytest.mark.parametrize("B,widths,k", [(1, [50, 40, 33], 4), (65, [100, 64, 64, 40], 10), (1000, [200, 300, 300, 150], 7),
                                        (4096, [784, 2000, 2000, 1000], 10)])
def test_packed_net_vs_oracle(B, widths, k):
    torch.manual_seed(B)
    mods = [cl.LogicLayer(widths[i], widths[i + 1], num_gates=16) for i in range(len(widths) - 1)]
    with torch.no_grad():
        for m in mods:
            m.gate_sequence.copy_(torch.randint(0, 16, m.gate_sequence.shape, dtype=torch.uint8))
    model = torch.nn.Sequential(*mods, cl.GroupSum(k, 1.0)).cuda()
    x = (torch.rand(B, widths[0]) < 0.5).float()
    layers = [O.frozen_tables(m.indices.cpu().numpy(), m.gate_sequence.cpu().numpy(),
                              O.argmax_first(m.weights.detach().cpu().numpy())) for m in mods]
    ref = O.packed_network_counts(x.numpy(), layers, k)
    net = cl.PackedLogicNet(model, chunk_words=4)
    np.testing.assert_array_equal(net(x.cuda()).cpu().numpy(), ref)


def test_packed_conv_net_matches_float_eval():
    torch.manual_seed(3)
    model = torch.nn.Sequential(cl.ConvLayer((3, 8, 8), 1, 16, 3, 2, num_gates=8),
                                cl.ConvLayer((16, 4, 4), 1, 32, 3, 2, num_gates=8), torch.nn.Flatten(),
                                cl.LogicLayer(128, 100, num_gates=8), cl.GroupSum(5, 2.0)).cuda().eval()
    x = (torch.rand(300, 3, 8, 8, device="cuda") < 0.5).float()
    counts = cl.PackedLogicNet(model, chunk_words=2)(x)
    np.testing.assert_array_equal(counts.cpu().numpy(), torch.round(model(x) * 2.0).to(torch.int32).cpu().numpy())


def test_packed_from_checkpoint_state(golden):
    """Checkpoint model_state -> packed network: class counts equal the reference circuit evaluator's."""
    d = golden("discrete.npz")
    state = {f"{i}.{n}": torch.from_numpy(d[f"{i}.{n}"]) for i in range(1, 4) for n in ("weights", "indices",
                                                                                           "gate_sequence")}
    net = cl.packed_from_state_dict(state, input_dim=784, k=int(d["k"]), tau=float(d["tau"]))
    np.testing.assert_array_equal(net(cuda(d["x"].astype(np.float32))).cpu().numpy(), d["counts"])


@pytest.mark.parametrize("B", [1, 100, 333])
def test_fused_threshold_packing(B):
    """Raw pixels -> thresholds -> packed bits in one kernel equals the reference binarisation
    (experiments/experiment_script.py:92) followed by packing, and the network counts agree."""
    torch.manual_seed(B)
    model = torch.nn.Sequential(cl.ConvLayer((9, 8, 8), 1, 16, 3, 2, num_gates=8), torch.nn.Flatten(),
                                cl.LogicLayer(256, 150, num_gates=8), cl.GroupSum(5, 1.0)).cuda().eval()
    net = cl.PackedLogicNet(model)
    px = torch.rand(B, 3, 8, 8)
    binar = torch.cat([(px > (i + 1) / 4).float() for i in range(3)], dim=1)
    np.testing.assert_array_equal(net.pack_raw(px.cuda(), 3).cpu().numpy().view(np.uint64),
                                  O.pack_samples(binar.reshape(B, -1).numpy()))
    np.testing.assert_array_equal(net.forward_raw(px.cuda(), 3).cpu().numpy(), net(binar.cuda()).cpu().numpy())


@pytest.mark.parametrize("keep", ["exact", "reference"])
@pytest.mark.parametrize("chunk_words", [1, 32])
def test_pruned_packed_net_matches_reference_circuit(golden, keep, chunk_words):
    """After the compiler's stage-1 pruning the packed network still gives the reference evaluator's
    counts, with fewer gates (reference liveness: the compiler's BOP count, tests/golden/pruned.npz)."""
    d = golden("discrete.npz")
    net = cl.PackedLogicNet(_model_from_fixture(d), chunk_words=chunk_words, prune=keep)
    np.testing.assert_array_equal(net(cuda(d["x"].astype(np.float32))).cpu().numpy(), d["counts"])
    assert net.prune_stats["gates"] == 1200
    if keep == "reference":
        assert net.prune_stats["kept"] == len(golden("pruned.npz")["d.node"])
    else:
        assert net.prune_stats["kept"] <= len(golden("pruned.npz")["d.node"])


def test_pruned_conv_net_and_checkpoint(golden):
    torch.manual_seed(3)
    model = torch.nn.Sequential(cl.ConvLayer((3, 8, 8), 1, 16, 3, 2, num_gates=8),
                                cl.ConvLayer((16, 4, 4), 1, 32, 3, 2, num_gates=8), torch.nn.Flatten(),
                                cl.LogicLayer(128, 100, num_gates=8), cl.GroupSum(5, 2.0)).cuda().eval()
    x = (torch.rand(300, 3, 8, 8, device="cuda") < 0.5).float()
    counts = cl.PackedLogicNet(model, chunk_words=2, prune="exact")(x)
    np.testing.assert_array_equal(counts.cpu().numpy(), torch.round(model(x) * 2.0).to(torch.int32).cpu().numpy())
    d = golden("discrete.npz")
    state = {f"{i}.{n}": torch.from_numpy(d[f"{i}.{n}"]) for i in range(1, 4) for n in ("weights", "indices",
                                                                                           "gate_sequence")}
    net = cl.packed_from_state_dict(state, input_dim=784, k=int(d["k"]), tau=float(d["tau"]), prune="exact")
    np.testing.assert_array_equal(net(cuda(d["x"].astype(np.float32))).cpu().numpy(), d["counts"])
