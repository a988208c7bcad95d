"""Bit-packed discrete inference of a CompactLogic network.

The reference evaluates a trained network in eval mode with one argmax gate per neuron applied to
fp32 activations (compactlogic/compactlogic.py:120-130, compactlogic/cuda/difflogic_kernel.cu:341-369)
and recovers class counts as round(logits * tau) (simulation/paper_stats.py:56).  Here the same
network runs on bits: 64 samples per uint64 word, one gate evaluation per word, and the final
layer is fused with a per-class vertical popcount, producing the exact integer class counts.

Samples are processed in chunks of ``chunk_words`` words (64 samples each): all layers of one chunk
run back to back.  At the default 128 words a 256000-wide layer's chunk activations (262 MB) exceed
the 126 MB L2, so each layer's output streams through HBM once and is read back by the next layer;
measured on a B200, this beats smaller L2-resident chunks, whose per-launch fixed costs dominate.
"""
import math
from typing import List, Optional

import torch

from . import _lib as L
from .compactlogic import GroupSum, LogicLayer


class _Frozen:
    __slots__ = ("sel_ab", "sel_gate", "n_out", "in_features")

    def __init__(self, sel_ab, sel_gate, n_out, in_features):
        self.sel_ab, self.sel_gate, self.n_out, self.in_features = sel_ab, sel_gate, n_out, in_features


class PackedLogicNet:
    """Discrete packed-inference engine for ``Sequential(LogicLayer|ConvLayer|Flatten ..., GroupSum)``.

    forward(x) -> int32 class counts [batch, k]; logits(x) = counts / tau, equal to the reference
    eval-mode output; predict(x) = argmax (first maximum, as torch.argmax).
    prune: None, or "exact" / "reference" to evaluate the network after the compiler's stage-1 pruning
    (same counts, fewer gates; see compactlogic_b200.prune).
    """

    def __init__(self, model: torch.nn.Module, device=None, chunk_words: int = 128, prune: Optional[str] = None):
        mods = list(model)
        if not mods or not isinstance(mods[-1], GroupSum):
            raise ValueError("PackedLogicNet needs a model ending in GroupSum")
        gs = mods[-1]
        self.k, self.tau = int(gs.k), float(gs.tau)
        first = next((m for m in mods if isinstance(m, LogicLayer)), None)
        self.device = torch.device(device) if device is not None else (first.weights.device if first is not None else
                                                                       torch.device('cuda'))
        self.chunk_words = int(chunk_words)
        self.layers: List[_Frozen] = []
        for m in mods[:-1]:
            if isinstance(m, torch.nn.Flatten):
                continue
            if not isinstance(m, LogicLayer):
                raise ValueError(f"PackedLogicNet: unsupported module {type(m).__name__}")
            self.layers.append(self._freeze_tables(m))
        if not self.layers:
            raise ValueError("PackedLogicNet: no logic layers")
        for prev, nxt in zip(self.layers[:-1], self.layers[1:]):
            if prev.n_out != nxt.in_features:
                raise ValueError("PackedLogicNet: layer widths do not chain")
        self.in_features = self.layers[0].in_features
        self.class_size = -(-self.layers[-1].n_out // self.k)
        self.plan = self._prune_plan(model, prune) if prune else None
        self._bufs = None
        self._ws = None
        self.use_graphs = True
        self._graphs = {}
        self.launches_per_pass = 0

    @torch.no_grad()
    def _freeze_tables(self, layer: LogicLayer) -> _Frozen:
        spec = layer._layer_spec(self.device)
        sel = layer._selected().to(self.device)
        n_out = spec.n_out
        sel_ab = torch.empty(n_out, 2, dtype=torch.int32, device=self.device)
        sel_gate = torch.empty(n_out, dtype=torch.uint8, device=self.device)
        L.call("clb_packed_select", L.ptr(spec.slots), L.ptr(spec.gates), L.ptr(sel.contiguous()), n_out, spec.K,
               spec.group, L.ptr(sel_ab), L.ptr(sel_gate), L.stream(self.device))
        in_features = spec.in_features
        return _Frozen(sel_ab, sel_gate, n_out, in_features)

    @torch.no_grad()
    def _prune_plan(self, model, keep: str):
        """Simplify the frozen network first (the compiler's stage-1 pruning, compiler/prune.py:298-310)
        and evaluate only the gates that survive: every kept gate of the inner layers is a row of one
        signal buffer (inputs first), so rewired operands may read any earlier row; the last layer
        becomes the fused count layer with pass-throughs, inverters and constants in place of the
        simplified neurons.  Counts are identical to the unpruned network's."""
        import numpy as np
        from .prune import packed_plan, prune_circuit
        raw = []
        for m in model:
            if not isinstance(m, LogicLayer):
                continue
            spec = m._layer_spec(self.device)
            slots = spec.slots.cpu().numpy()
            sel = m._selected().cpu().numpy().astype(np.int64)
            gates = spec.gates.cpu().numpy().astype(np.int64)
            j = np.arange(spec.n_out)
            r = j // spec.group
            raw.append((slots[j, sel[r], 0].astype(np.int64), slots[j, sel[r], 1].astype(np.int64), gates[r, sel[r]]))
        pc = prune_circuit(raw, self.in_features, self.k, keep=keep)
        layers, (cab, cg), rows = packed_plan(pc)
        dev = self.device
        t = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a)).to(dev, dt)
        self.prune_stats = {"gates": int(sum(len(g) for _, _, g in raw)), "kept": pc.bop_count,
                            "rows": int(rows), "keep": keep}
        return {"layers": [(t(ab, torch.int32), t(g, torch.uint8), len(g)) for ab, g in layers],
                "count": (t(cab, torch.int32), t(cg, torch.uint8), len(cg)), "rows": int(rows)}

    # ------------------------------------------------------------------
    def pack(self, x: torch.Tensor) -> torch.Tensor:
        """[batch, features] (or [batch, C, H, W]) {0,1} -> [features, ceil(batch/64)] uint64."""
        x = x.reshape(x.shape[0], math.prod(x.shape[1:]))
        if x.dtype not in (torch.float32, torch.float64, torch.bfloat16, torch.float16):
            x = x.to(torch.float32)
        if x.stride(1) != 1:
            x = x.contiguous()
        B, F = x.shape
        if F != self.in_features:
            raise ValueError(f"expected {self.in_features} input features, got {F}")
        W = -(-B // 64)
        xw = torch.empty(F, W, dtype=torch.int64, device=self.device)
        L.call("clb_pack_inputs", L.dtype_code(x.dtype), L.ptr(x), B, F, x.stride(0), L.ptr(xw), W,
               L.stream(self.device))
        return xw

    def pack_raw(self, x: torch.Tensor, nthr: int) -> torch.Tensor:
        """Raw inputs [batch, C, H, W] (or [batch, F]) in [0, 1] -> [nthr*F, W] packed words, thresholding at
        (i+1)/(nthr+1) in the reference's order (experiments/experiment_script.py:92) in the same pass."""
        x = x.reshape(x.shape[0], math.prod(x.shape[1:]))
        if x.dtype not in (torch.float32, torch.float64, torch.bfloat16, torch.float16):
            x = x.to(torch.float32)
        if x.stride(1) != 1:
            x = x.contiguous()
        B, F = x.shape
        if F * nthr != self.in_features:
            raise ValueError(f"{F} raw features x {nthr} thresholds != {self.in_features} network inputs")
        W = -(-B // 64)
        xw = torch.empty(F * nthr, W, dtype=torch.int64, device=self.device)
        L.call("clb_pack_thresholds", L.dtype_code(x.dtype), L.ptr(x), B, F, x.stride(0), nthr, L.ptr(xw), W,
               L.stream(self.device))
        return xw

    @torch.no_grad()
    def forward_raw(self, x: torch.Tensor, nthr: int) -> torch.Tensor:
        """Class counts of raw inputs binarised with nthr thresholds (input binarisation fused with packing)."""
        L.require_cuda(x)
        return self.counts_packed(self.pack_raw(x, nthr), x.shape[0])

    def _buffers(self, width: int):
        if self._bufs is None or self._bufs[0].shape[1] < width:
            rows = max(l.n_out for l in self.layers[:-1]) if len(self.layers) > 1 else 1
            self._bufs = tuple(torch.empty(rows, width, dtype=torch.int64, device=self.device) for _ in range(2))
        return self._bufs

    def _count_ws(self, nwords: int) -> torch.Tensor:
        """Workspace of the fused count (per-CTA partial totals, summed without atomics)."""
        need = int(L.lib().clb_packed_count_workspace_bytes(self.k, self.class_size, nwords))
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(max(need, 1), dtype=torch.uint8, device=self.device)
        return self._ws

    def _run_pruned(self, xw: torch.Tensor, batch: int, counts: torch.Tensor) -> None:
        W = xw.shape[1]
        cw = max(1, min(self.chunk_words, W))
        plan = self.plan
        if self._bufs is None or self._bufs[0].shape[1] < cw:
            self._bufs = (torch.empty(plan["rows"], cw, dtype=torch.int64, device=self.device),)
        sig = self._bufs[0]
        ld = sig.stride(0)
        s = L.stream(self.device)
        counts.zero_()
        n = 0
        cab, cg, n_out = plan["count"]
        for w0 in range(0, W, cw):
            nw = min(cw, W - w0)
            sig[:self.in_features, :nw].copy_(xw[:, w0:w0 + nw])
            row = self.in_features
            for ab, g, m in plan["layers"]:
                if m:
                    L.call("clb_packed_layer", L.ptr(sig), ld, nw, L.ptr(ab), L.ptr(g), m, L.ptr(sig) + 8 * row * ld,
                           ld, s)
                    n += 1
                row += m
            nsamp = min(64 * nw, batch - 64 * w0)
            ws = self._count_ws(nw)
            L.call("clb_packed_layer_count", L.ptr(sig), ld, nw, L.ptr(cab), L.ptr(cg), n_out, self.k,
                   self.class_size, L.ptr(counts), 64 * w0, nsamp, L.ptr(ws), ws.numel(), s)
            n += 1
        self.launches_per_pass = n

    def _run(self, xw: torch.Tensor, batch: int, counts: torch.Tensor) -> None:
        """Enqueue one pass: per chunk, every layer then the fused last layer + class count."""
        if self.plan is not None:
            return self._run_pruned(xw, batch, counts)
        W = xw.shape[1]
        cw = max(1, min(self.chunk_words, W))
        bufs = self._buffers(cw)
        s = L.stream(self.device)
        counts.zero_()
        n = 0
        for w0 in range(0, W, cw):
            nw = min(cw, W - w0)
            src, ld_src = xw[:, w0:], xw.stride(0)
            for li, layer in enumerate(self.layers[:-1]):
                dst = bufs[li % 2]
                L.call("clb_packed_layer", L.ptr(src), ld_src, nw, L.ptr(layer.sel_ab), L.ptr(layer.sel_gate),
                       layer.n_out, L.ptr(dst), dst.stride(0), s)
                src, ld_src = dst, dst.stride(0)
            last = self.layers[-1]
            nsamp = min(64 * nw, batch - 64 * w0)
            ws = self._count_ws(nw)
            L.call("clb_packed_layer_count", L.ptr(src), ld_src, nw, L.ptr(last.sel_ab), L.ptr(last.sel_gate),
                   last.n_out, self.k, self.class_size, L.ptr(counts), 64 * w0, nsamp, L.ptr(ws), ws.numel(), s)
            n += len(self.layers) + 1
        self.launches_per_pass = n

    @torch.no_grad()
    def counts_packed(self, xw: torch.Tensor, batch: int, counts: Optional[torch.Tensor] = None,
                      use_graph: Optional[bool] = None) -> torch.Tensor:
        """Class counts [batch, k] of pre-packed inputs xw [features, W] (int64 words, unit column stride).

        With graphs enabled (default) the pass — thousands of launches for large batches — is captured
        once per (input, output) buffer pair into a CUDA graph and replayed, so the host issues one
        launch per pass."""
        if xw.shape[0] != self.in_features or (xw.shape[1] > 1 and xw.stride(1) != 1):
            raise ValueError("xw must be [in_features, words] with unit column stride")
        if counts is None:
            counts = torch.empty(batch, self.k, dtype=torch.int32, device=self.device)
        if batch == 0 or xw.shape[1] == 0:
            return counts.zero_()
        if not (self.use_graphs if use_graph is None else use_graph):
            self._run(xw, batch, counts)
            return counts
        key = (xw.data_ptr(), tuple(xw.shape), xw.stride(0), batch, counts.data_ptr())
        graph = self._graphs.get(key)
        if graph is None:
            side = torch.cuda.Stream(self.device)
            side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(side):  # eager warm-up allocates the chunk buffers outside the capture
                self._run(xw, batch, counts)
            torch.cuda.current_stream(self.device).wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                self._run(xw, batch, counts)
            if len(self._graphs) >= 8:
                self._graphs.pop(next(iter(self._graphs)))
            self._graphs[key] = graph
        graph.replay()
        return counts

    @torch.no_grad()
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        L.require_cuda(x)
        return self.counts_packed(self.pack(x), x.shape[0])

    __call__ = forward

    def logits(self, x: torch.Tensor) -> torch.Tensor:
        return self.forward(x).to(torch.float32) / self.tau

    def predict(self, x: torch.Tensor) -> torch.Tensor:
        return self.forward(x).argmax(-1)


def _state_prefixes(state):
    return sorted({k.split(".")[0] for k in state if k.endswith(".weights") and k.split(".")[0].isdigit()}, key=int)


def packed_from_state_dict(state: dict, input_dim: int, k: int, tau: float = 1.0, device="cuda",
                           chunk_words: int = 128, prune: Optional[str] = None) -> PackedLogicNet:
    """PackedLogicNet straight from a checkpoint's ``model_state`` of dense logic layers (the layout the
    reference writes, experiments/experiment_script.py:520-541, and its compiler reads,
    compiler/extract.py:49-98): per layer ``{i}.weights`` (out, K), ``{i}.indices`` (2, out, K),
    ``{i}.gate_sequence`` (out, K); the gate of neuron j is the one at argmax_k weights[j, k] (first
    maximum), as the compiler and the eval path choose it.  ``input_dim`` is the network's input width
    (not recoverable from the state), ``k`` / ``tau`` the GroupSum parameters."""
    layers = []
    in_dim = int(input_dim)
    for p in _state_prefixes(state):
        w, idx, g = state[f"{p}.weights"], state[f"{p}.indices"], state[f"{p}.gate_sequence"]
        out, K = w.shape
        if tuple(idx.shape) != (2, out, K) or tuple(g.shape) != (out, K):
            raise ValueError(f"layer {p}: unexpected buffer shapes")
        layer = LogicLayer.__new__(LogicLayer)  # buffers only, no RNG-consuming constructor
        torch.nn.Module.__init__(layer)
        layer.in_dim, layer.out_dim, layer.num_gates = in_dim, out, K
        layer.weights = torch.nn.Parameter(torch.as_tensor(w).float().to(device), requires_grad=False)
        layer.register_buffer("indices", torch.as_tensor(idx).long().to(device))
        layer.register_buffer("gate_sequence", torch.as_tensor(g).to(torch.uint8).to(device))
        layer.is_frozen, layer._spec_key, layer._spec, layer._fused_groupsum = False, None, None, None
        layers.append(layer)
        in_dim = out
    if not layers:
        raise ValueError("no dense logic layers in the state dict")
    return PackedLogicNet(torch.nn.Sequential(*layers, GroupSum(k, tau)), device=device, chunk_words=chunk_words,
                          prune=prune)
