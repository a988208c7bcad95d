"""Generate the CPU golden fixtures of tests/golden/ from the reference CompactLogic Python code.

Run where the reference tree is checked out (--ref or $COMPACTLOGIC_REF); nothing here runs at test
time.  The reference package imports its CUDA extensions at module level, so they are replaced by
empty placeholder modules (no kernel is called: only host-side code runs), and the class-definition
default arguments that build tensors on 'cuda' are redirected to the CPU during the import.

Fixtures written (all small, npz):
  gate_kat.npz        vendored difflogic functional.bin_op (the reference's CPU relaxation) on a grid of
                      real inputs, and compiler.gates.eval_gate_torch on all boolean inputs;
  layer_buffers.npz   buffers of reference LogicLayer / ConvLayer objects built under fixed seeds, an
                      incremental inverse-index refresh and a resample_connections call;
  big_layer_sha.json  sha256 of the buffers of the c1 configuration LogicLayer(784, 12000, 16), seed 0;
  discrete.npz        a random frozen 784 -> 3x400 -> GroupSum(10) network built by the reference,
                      random boolean inputs, and the class counts of the reference CPU circuit
                      evaluator (simulation/consistency.py:80-130 on compiler/extract.py:200-268);
  freezer_trace.json  freeze steps of SequentialEntropyFreezer / FixedSequentialEntropyFreezer on a
                      scripted entropy schedule;
  pruned.npz          the reference compiler's stage-1 pruning (compiler/prune.py naive_prune_circuit) of
                      the discrete.npz network and of a 784 -> 300 -> 200 network dominated by constant /
                      pass-through / inverter gates with repeated operands: kept gates (node id, gate id,
                      operand signal ids) and every class-group source (constant, signal, inversion).

Usage: python tests/golden/make_golden.py --ref <reference checkout>
"""
import argparse
import hashlib
import json
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def import_reference(ref_root):
    sys.path.insert(0, ref_root)
    for name in ("difflogic_cuda", "convlogic_cuda"):
        sys.modules.setdefault(name, types.ModuleType(name))
    orig = torch.tensor

    def cpu_tensor(*a, **k):
        if str(k.get("device", "")).startswith("cuda"):
            k["device"] = "cpu"
        return orig(*a, **k)

    torch.tensor = cpu_tensor
    try:
        import compactlogic  # noqa: F401
        import compiler.extract  # noqa: F401
        import compiler.gates  # noqa: F401
        import simulation.consistency  # noqa: F401
    finally:
        torch.tensor = orig
    return sys.modules["compactlogic"]


def bufs(layer, prefix, out):
    for name, t in list(layer.named_buffers()) + [("weights", layer.weights)]:
        out[f"{prefix}.{name}"] = t.detach().cpu().numpy()


def gate_kat(ref_root):
    sys.path.insert(0, os.path.join(ref_root, "third_party", "convlogic_source_code", "src"))
    from difflogic.functional import bin_op  # the reference's CPU relaxation (pure torch)
    from compiler.gates import eval_gate_torch
    grid = torch.linspace(0, 1, 11, dtype=torch.float64)
    a, b = torch.meshgrid(grid, grid, indexing="ij")
    a, b = a.reshape(1, -1), b.reshape(1, -1)
    real = np.stack([bin_op(a, b, i).expand_as(a).numpy()[0] for i in range(16)])
    ab = torch.tensor([[0, 0], [0, 1], [1, 0], [1, 1]], dtype=torch.bool)
    boolean = np.stack([np.broadcast_to(np.asarray(eval_gate_torch(i, ab[:, 0], ab[:, 1])), (4,)) for i in range(16)])
    np.savez(os.path.join(HERE, "gate_kat.npz"), grid_a=a.numpy()[0], grid_b=b.numpy()[0], real=real,
             bool_ab=ab.numpy(), boolean=boolean.astype(np.uint8))


def layer_buffers(cl):
    out = {}
    torch.manual_seed(0)
    bufs(cl.LogicLayer(20, 24, num_gates=16), "dense_random", out)
    torch.manual_seed(1)
    bufs(cl.LogicLayer(30, 16, connections="original", num_gates=8), "dense_original", out)
    torch.manual_seed(2)
    bufs(cl.LogicLayer(12, 10, num_gates=4, residual_init=True), "dense_residual", out)
    for seed, num_chn, ks, pad, stride in ((3, 1, 3, 1, 2), (4, 0, 3, 0, 1), (5, 3, 2, 1, 2), (6, 0, 1, 0, 1)):
        torch.manual_seed(seed)
        layer = cl.ConvLayer((6, 8, 8), pad, 9, ks, stride, num_chn=num_chn, num_gates=16)
        bufs(layer, f"conv_{seed}", out)

    # incremental refresh and resampling
    torch.manual_seed(7)
    layer = cl.LogicLayer(40, 50, num_gates=16)
    with torch.no_grad():
        layer.weights[0:10] = 0.0                      # uniform: weak when threshold_low > 1/16
        layer.weights[10:20, 3] = 20.0                  # strongly peaked
    out["resample.before.weights"] = layer.weights.detach().numpy().copy()
    torch.manual_seed(8)
    weak, strong = layer.resample_connections(torch.arange(0, 30), threshold_high=0.9, threshold_low=0.1)
    out["resample.weak"] = weak.numpy()
    out["resample.strong"] = strong.numpy()
    bufs(layer, "resample.after", out)

    torch.manual_seed(9)
    conv = cl.ConvLayer((4, 6, 6), 1, 8, 3, 1, num_chn=1, num_gates=8)
    with torch.no_grad():
        conv.weights[0:3] = 0.0
        conv.weights[3:6, 1] = 15.0
    torch.manual_seed(10)
    conv.resample_connections(torch.arange(0, 8), threshold_high=0.9, threshold_low=0.2)
    bufs(conv, "conv_resample.after", out)

    torch.manual_seed(11)
    layer = cl.LogicLayer(16, 12, num_gates=4)
    with torch.no_grad():
        layer.indices[0, 3] = torch.tensor([1, 2, 3, 4])
        layer.indices[1, 7] = torch.tensor([5, 5, 5, 5])
    layer.refresh_backward_index(torch.tensor([3, 7]))
    bufs(layer, "refresh", out)

    # connected_neurons on a frozen layer
    torch.manual_seed(12)
    layer = cl.LogicLayer(30, 20, num_gates=16)
    layer.freeze()
    y_flag = torch.ones(20, dtype=torch.bool)
    x_flag, y_flag = layer.connected_neurons(y_flag, device="cpu", const_gates=torch.tensor([0, 15]),
                                             trivial_gates_a=torch.tensor([3, 12]),
                                             trivial_gates_b=torch.tensor([5, 10]))
    bufs(layer, "connected", out)
    out["connected.x_flag"] = x_flag.numpy()
    out["connected.y_flag"] = y_flag.numpy()
    np.savez_compressed(os.path.join(HERE, "layer_buffers.npz"), **out)


def big_layer_sha(cl):
    torch.manual_seed(0)
    layer = cl.LogicLayer(784, 12000, num_gates=16)
    res = {}
    for name, t in list(layer.named_buffers()) + [("weights", layer.weights)]:
        res[name] = hashlib.sha256(t.detach().contiguous().numpy().tobytes()).hexdigest()
    with open(os.path.join(HERE, "big_layer_sha.json"), "w") as f:
        json.dump({"config": "torch.manual_seed(0); LogicLayer(784, 12000, num_gates=16)", "sha256": res}, f, indent=1)


def discrete(cl):
    import compiler.extract as ce
    import simulation.consistency as sc
    torch.manual_seed(21)
    widths = [784, 400, 400, 400]
    model = torch.nn.Sequential(torch.nn.Flatten(), *[cl.LogicLayer(widths[i], widths[i + 1], num_gates=16)
                                                       for i in range(3)], cl.GroupSum(10, tau=3.0, device="cpu"))
    with torch.no_grad():
        for m in model:
            if isinstance(m, cl.LogicLayer):
                m.gate_sequence.copy_(torch.randint(0, 16, m.gate_sequence.shape, dtype=torch.uint8))
                m.weights.mul_(3.0)
    state = {k: v for k, v in model.state_dict().items()}
    circuit = ce.extract_circuit_from_state(state, args=None, num_classes=10, tau=3.0, metadata={"dataset": "mnist"})
    gen = torch.Generator().manual_seed(5)
    x = torch.rand((300, 784), generator=gen) < torch.rand((1, 784), generator=gen)
    orig = sc.extract_circuit_from_checkpoint
    sc.extract_circuit_from_checkpoint = lambda *a, **k: circuit
    try:
        res = sc.evaluate_extracted_circuit_torch("unused", x.to(torch.float32), device="cpu")
    finally:
        sc.extract_circuit_from_checkpoint = orig
    out = {"x": x.numpy().astype(np.uint8), "counts": res["class_counts"].numpy().astype(np.int32),
           "logits": res["logits"].numpy(), "widths": np.array(widths), "tau": np.array(3.0), "k": np.array(10)}
    for i in range(1, 4):
        for name in ("weights", "indices", "gate_sequence"):
            out[f"{i}.{name}"] = state[f"{i}.{name}"].numpy()
    np.savez_compressed(os.path.join(HERE, "discrete.npz"), **out)


def _prune_record(circuit, tag, out):
    from compiler.prune import naive_prune_circuit
    pc = naive_prune_circuit(circuit)
    out[f"{tag}.node"] = np.array([n.node_id for n in pc.nodes], np.int64)
    out[f"{tag}.gate"] = np.array([n.gate_id for n in pc.nodes], np.int64)
    out[f"{tag}.a"] = np.array([n.input_a.signal_id for n in pc.nodes], np.int64)
    out[f"{tag}.b"] = np.array([n.input_b.signal_id for n in pc.nodes], np.int64)
    kind, sig, inv = [], [], []
    for group in pc.class_groups:
        for src in group:
            if src.const_value is not None:
                kind.append(src.const_value)
                sig.append(-1)
                inv.append(0)
            else:
                kind.append(2)
                sig.append(src.signal_id)
                inv.append(int(src.inverted))
    shape = (pc.num_classes, -1)
    out[f"{tag}.src_kind"] = np.array(kind, np.int64).reshape(shape)
    out[f"{tag}.src_sig"] = np.array(sig, np.int64).reshape(shape)
    out[f"{tag}.src_inv"] = np.array(inv, np.int64).reshape(shape)


def pruned(cl):
    import compiler.extract as ce
    out = {}
    d = np.load(os.path.join(HERE, "discrete.npz"))
    state = {f"{i}.{n}": torch.from_numpy(d[f"{i}.{n}"]) for i in range(1, 4)
             for n in ("weights", "indices", "gate_sequence")}
    circuit = ce.extract_circuit_from_state(state, args=None, num_classes=10, tau=3.0, metadata={"dataset": "mnist"})
    _prune_record(circuit, "d", out)
    # trivial-heavy network: gates mostly constants / pass-throughs / inverters, many a == b operands
    g = torch.Generator().manual_seed(9)
    widths = [784, 300, 200]
    pool = torch.tensor([0, 15, 3, 5, 10, 12, 3, 5, 1, 6, 7, 9, 14, 2, 4, 8, 11, 13], dtype=torch.uint8)
    state = {}
    for i in range(2):
        n_in, n_out, K = widths[i], widths[i + 1], 4
        idx = torch.randint(0, n_in, (2, n_out, K), generator=g)
        same = torch.rand((n_out, K), generator=g) < 0.2
        idx[1][same] = idx[0][same]
        state[f"{i + 1}.weights"] = torch.randn((n_out, K), generator=g)
        state[f"{i + 1}.indices"] = idx
        state[f"{i + 1}.gate_sequence"] = pool[torch.randint(0, len(pool), (n_out, K), generator=g)]
    for key, t in state.items():
        out["t." + key] = t.numpy()
    circuit = ce.extract_circuit_from_state(state, args=None, num_classes=10, tau=1.0, metadata={"dataset": "mnist"})
    _prune_record(circuit, "t", out)
    np.savez_compressed(os.path.join(HERE, "pruned.npz"), **out)


def freezer_trace(cl):
    class Fake(torch.nn.Module):
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

    def run(make):
        layers = [Fake(3) for _ in range(4)]
        fr = make(layers)
        trace = []
        for it in range(90):
            with torch.no_grad():
                for li, l in enumerate(layers):
                    if it < 10 + 8 * li:
                        l.weights[:, 0] += 0.3  # still changing
            fr.step(it)
            trace.append([int(l.is_frozen) for l in layers])
        return trace

    res = {
        "sequential": run(lambda m: cl.SequentialEntropyFreezer(m, ema_decay=0.7, eps=1e-2, patience=3, min_iters=2)),
        "sequential_l2": run(lambda m: cl.SequentialEntropyFreezer(m, ema_decay=0.7, eps=1e-2, patience=3, l=2)),
        "fixed": run(lambda m: cl.FixedSequentialEntropyFreezer(m, N=7, min_iters=5)),
    }
    with open(os.path.join(HERE, "freezer_trace.json"), "w") as f:
        json.dump(res, f)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("COMPACTLOGIC_REF"))
    args = ap.parse_args()
    if not args.ref:
        ap.error("give --ref or set COMPACTLOGIC_REF to the reference checkout")
    cl = import_reference(args.ref)
    gate_kat(args.ref)
    layer_buffers(cl)
    big_layer_sha(cl)
    discrete(cl)
    freezer_trace(cl)
    pruned(cl)
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
