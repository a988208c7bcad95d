"""Stage-1 pruning of frozen networks (compactlogic_b200.prune) on CPU.

Pinned against the reference compiler's naive_prune_circuit (compiler/prune.py) run on two networks
(tests/golden/pruned.npz): the kept gates, their folded gate ids and rewired operands, and every class
source.  The tighter "exact" liveness keeps a subset with the same outputs.  The packed plan built from
the pruned circuit reproduces the unpruned network's class counts bit-exactly on the CPU oracle.
"""
import numpy as np
import pytest

from compactlogic_b200 import prune as P
from oracle import oracle as O


def _raw(golden, tag):
    if tag == "d":
        d = golden("discrete.npz")
        keys = [(f"{i}.weights", f"{i}.indices", f"{i}.gate_sequence") for i in range(1, 4)]
    else:
        d = golden("pruned.npz")
        keys = [(f"t.{i}.weights", f"t.{i}.indices", f"t.{i}.gate_sequence") for i in range(1, 3)]
    layers = []
    for wk, ik, gk in keys:
        sel = O.argmax_first(d[wk])
        ab, g = O.frozen_tables(d[ik], d[gk], sel)
        layers.append((ab[:, 0].astype(np.int64), ab[:, 1].astype(np.int64), g.astype(np.int64)))
    return layers


@pytest.mark.parametrize("tag", ["d", "t"])
def test_reference_liveness_matches_compiler(golden, tag):
    ref = golden("pruned.npz")
    layers = _raw(golden, tag)
    pc = P.prune_circuit(layers, 784, 10, keep="reference")
    nodes = np.flatnonzero(pc.kept)
    np.testing.assert_array_equal(nodes, ref[f"{tag}.node"])
    np.testing.assert_array_equal(pc.gate[nodes], ref[f"{tag}.gate"])
    np.testing.assert_array_equal(pc.op_a[nodes], ref[f"{tag}.a"])
    np.testing.assert_array_equal(pc.op_b[nodes], ref[f"{tag}.b"])
    kind, sig, inv = pc.outputs()
    np.testing.assert_array_equal(kind, ref[f"{tag}.src_kind"])
    np.testing.assert_array_equal(sig, ref[f"{tag}.src_sig"])
    np.testing.assert_array_equal(inv, ref[f"{tag}.src_inv"])
    assert pc.bop_count == len(ref[f"{tag}.node"])


def _eval_plan(pc, xw, k, samples):
    layers, (cab, cg), rows = P.packed_plan(pc)
    h = xw
    for ab, g in layers:
        h = np.concatenate([h, O.packed_layer(h, ab, g, fast=True)], 0)
    assert h.shape[0] == rows
    return O.packed_count(O.packed_layer(h, cab, cg, fast=True), k, samples)


@pytest.mark.parametrize("tag", ["d", "t"])
def test_exact_subset_and_counts_equal(golden, tag):
    layers = _raw(golden, tag)
    ref = P.prune_circuit(layers, 784, 10, keep="reference")
    ex = P.prune_circuit(layers, 784, 10, keep="exact")
    assert not (ex.kept & ~ref.kept).any()
    assert ex.bop_count <= ref.bop_count
    for a, b in zip(ref.outputs(), ex.outputs()):
        np.testing.assert_array_equal(a, b)
    rng = np.random.default_rng(7)
    samples = 1000
    x = rng.random((samples, 784)) < rng.random((1, 784))
    want = O.packed_network_counts(x.astype(np.float64), [(np.stack([a, b], 1).astype(np.int32), g.astype(np.uint8))
                                                          for a, b, g in layers], 10)
    xw = O.pack_samples(x.astype(np.float64))
    for pc in (ref, ex):
        np.testing.assert_array_equal(_eval_plan(pc, xw, 10, samples), want)


def test_constant_operands_and_padding():
    # zero-padding operands (-1) and a repeated operand: AND(0, x) = 0, OR(0, x) = x, NAND(x, 0) = 1,
    # XOR(x, y) stays a gate, XNOR(x, x) = 1
    layers = [(np.array([-1, -1, 0, 1, 2]), np.array([0, 1, -1, 2, 2]), np.array([1, 7, 14, 6, 9])),
              (np.array([0, 1, 2, 3, 4, 1]), np.array([1, 2, 3, 4, 0, 0]), np.array([7, 1, 6, 8, 3, 5]))]
    pc = P.prune_circuit(layers, 3, 4, keep="exact")
    lo = pc.offsets[0]
    assert list(pc.kind[lo:lo + 5]) == [P.CONST0, P.REF, P.CONST1, P.GATE, P.CONST1]
    rng = np.random.default_rng(1)
    x = rng.random((200, 3)) < 0.5
    want = O.packed_network_counts(x.astype(np.float64), [(np.stack([a, b], 1).astype(np.int32), g.astype(np.uint8))
                                                          for a, b, g in layers], 4)
    np.testing.assert_array_equal(_eval_plan(pc, O.pack_samples(x.astype(np.float64)), 4, 200), want)
