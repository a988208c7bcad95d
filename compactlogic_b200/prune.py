"""Stage-1 pruning of a frozen (discrete) CompactLogic network, vectorised over whole layers.

The reference compiler simplifies the extracted circuit gate by gate from the outputs
(compiler/prune.py:159-245, ``naive_prune_circuit``): operands that are inverted references are folded
into the gate id, constants and repeated operands collapse the gate to a constant or to a (possibly
inverted) reference, the pass-through / inverter gates 3, 5, 10, 12 become references and the constant
gates 0, 15 constants; what is left is a real two-input gate ("BOP").  The same rules are applied here
one layer at a time with array operations, so a 256000-wide layer is simplified in milliseconds.

Liveness comes in two flavours:
  * ``"reference"`` keeps exactly the reference's set: every gate reachable from the outputs through
    the original connections (its recursion visits both operands of every node it meets) that does not
    simplify away — the BOP count the reference reports;
  * ``"exact"`` keeps only gates whose value is still read after simplification (a subset of the
    former with identical outputs), which is what an evaluator wants.

Signal numbering follows the reference IR (compiler/extract.py:200-268): inputs 0..in-1, then the
nodes of each layer in order.
"""
from dataclasses import dataclass
from typing import List, Sequence, Tuple

import numpy as np

CONST0, CONST1, REF, GATE = 0, 1, 2, 3


def _truth_table() -> np.ndarray:
    """T[g, a, b]: gate g's output for inputs a, b (bit 3 - (2a + b) of the gate id)."""
    g = np.arange(16)[:, None, None]
    a = np.arange(2)[None, :, None]
    b = np.arange(2)[None, None, :]
    return (g >> (3 - 2 * a - b)) & 1


T = _truth_table()


def _gate_of(table: np.ndarray) -> np.ndarray:
    """Gate ids of truth tables [..., 2, 2]."""
    return (table[..., 0, 0] << 3) | (table[..., 0, 1] << 2) | (table[..., 1, 0] << 1) | table[..., 1, 1]


INV_A = _gate_of(T[:, ::-1, :])  # g(not a, b)
INV_B = _gate_of(T[:, :, ::-1])  # g(a, not b)


@dataclass
class PrunedCircuit:
    in_dim: int
    offsets: np.ndarray   # [layers + 1]: global id of each layer's first node, then the signal count
    kind: np.ndarray      # [signals] CONST0 / CONST1 / REF / GATE: the simplified expression of each signal
    sig: np.ndarray       # REF: the referenced signal; GATE: the node itself
    inv: np.ndarray       # REF: inverted
    gate: np.ndarray      # GATE: gate id after folding operand inversions
    op_a: np.ndarray      # GATE: operand signals (never constants, never inverted)
    op_b: np.ndarray
    kept: np.ndarray      # [signals] bool: gate kept by the chosen liveness
    k: int

    @property
    def bop_count(self) -> int:
        return int(self.kept.sum())

    def layer_nodes(self, layer: int) -> np.ndarray:
        """Global ids of the kept gates of `layer` (0-based), in order."""
        lo, hi = self.offsets[layer], self.offsets[layer + 1]
        return lo + np.flatnonzero(self.kept[lo:hi])

    def outputs(self) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
        """Class-group sources [k, size] as (kind, signal, inverted): the last layer's expressions, a
        GATE node as a reference to itself, GroupSum's zero padding as CONST0 (compiler/ir.py:79-92)."""
        lo, hi = self.offsets[-2], self.offsets[-1]
        n = hi - lo
        size = -(-n // self.k)
        kind = np.full(self.k * size, CONST0, np.int64)
        sig = np.full(self.k * size, -1, np.int64)
        inv = np.zeros(self.k * size, np.int64)
        kind[:n] = np.where(self.kind[lo:hi] == GATE, REF, self.kind[lo:hi])
        sig[:n] = np.where(kind[:n] == REF, self.sig[lo:hi], -1)
        inv[:n] = self.inv[lo:hi] & (kind[:n] == REF)
        return kind.reshape(self.k, size), sig.reshape(self.k, size), inv.reshape(self.k, size)


def _collapse(f0, f1, s):
    """A gate that became a function of one signal s: constant, s, or not s."""
    kind = np.where(f0 == f1, f0, REF)
    inv = (f0 == 1) & (f1 == 0)
    return kind, np.where(kind == REF, s, -1), inv


def prune_circuit(layers: Sequence[Tuple[np.ndarray, np.ndarray, np.ndarray]], in_dim: int, k: int,
                  keep: str = "exact") -> PrunedCircuit:
    """Simplify a frozen network.  `layers[l]` = (a, b, g): per neuron the two operand positions in the
    previous layer's outputs (the inputs for l = 0), -1 for the constant 0 (conv zero padding), and the
    gate id."""
    if keep not in ("exact", "reference"):
        raise ValueError("keep must be 'exact' or 'reference'")
    widths = [len(g) for _, _, g in layers]
    offsets = in_dim + np.concatenate([[0], np.cumsum(widths)]).astype(np.int64)
    n_sig = int(offsets[-1])
    kind = np.full(n_sig, REF, np.int64)
    sig = np.arange(n_sig, dtype=np.int64)
    inv = np.zeros(n_sig, bool)
    gate = np.zeros(n_sig, np.int64)
    op_a = np.full(n_sig, -1, np.int64)
    op_b = np.full(n_sig, -1, np.int64)
    prev_lo = 0
    for l, (a, b, g) in enumerate(layers):
        lo = int(offsets[l])
        n = len(g)
        ids = lo + np.arange(n)
        g = np.asarray(g, np.int64).copy()

        def operand(loc):
            loc = np.asarray(loc, np.int64)
            glob = np.where(loc >= 0, prev_lo + loc, 0)
            kk = np.where(loc >= 0, kind[glob], CONST0)
            ss = np.where(loc >= 0, sig[glob], -1)
            vv = np.where(loc >= 0, inv[glob], False)
            is_gate = kk == GATE  # a real gate is referenced as itself
            return np.where(is_gate, REF, kk), np.where(is_gate, glob, ss), vv & ~is_gate

        ka, sa, va = operand(a)
        kb, sb, vb = operand(b)
        g = np.where((ka == REF) & va, INV_A[g], g)
        g = np.where((kb == REF) & vb, INV_B[g], g)
        ca, cb = ka != REF, kb != REF
        nk = np.empty(n, np.int64)
        ns = np.full(n, -1, np.int64)
        ni = np.zeros(n, bool)
        # both constant
        m = ca & cb
        nk[m] = T[g[m], ka[m], kb[m]]
        # constant a: a function of b
        m = ca & ~cb
        nk[m], ns[m], ni[m] = _collapse(T[g[m], ka[m], 0], T[g[m], ka[m], 1], sb[m])
        # constant b: a function of a
        m = ~ca & cb
        nk[m], ns[m], ni[m] = _collapse(T[g[m], 0, kb[m]], T[g[m], 1, kb[m]], sa[m])
        # one signal on both operands
        refs = ~ca & ~cb
        m = refs & (sa == sb)
        nk[m], ns[m], ni[m] = _collapse(T[g[m], 0, 0], T[g[m], 1, 1], sa[m])
        rest = refs & (sa != sb)
        for gid, use_a, flip in ((3, True, False), (5, False, False), (10, False, True), (12, True, True)):
            m = rest & (g == gid)
            nk[m], ns[m], ni[m] = REF, np.where(use_a, sa[m], sb[m]), flip
        m = rest & ((g == 0) | (g == 15))
        nk[m] = np.where(g[m] == 15, CONST1, CONST0)
        m = rest & ~np.isin(g, (0, 15, 3, 5, 10, 12))
        nk[m], ns[m] = GATE, ids[m]
        gate[ids[m]], op_a[ids[m]], op_b[ids[m]] = g[m], sa[m], sb[m]
        kind[lo:lo + n], sig[lo:lo + n], inv[lo:lo + n] = nk, ns, ni
        prev_lo = lo

    kept = np.zeros(n_sig, bool)
    if keep == "reference":
        reach = np.zeros(n_sig, bool)
        reach[offsets[-2]:] = True
        for l in range(len(layers) - 1, -1, -1):
            lo, hi = int(offsets[l]), int(offsets[l + 1])
            base = 0 if l == 0 else int(offsets[l - 1])
            r = np.flatnonzero(reach[lo:hi])
            for side in (layers[l][0], layers[l][1]):
                loc = np.asarray(side, np.int64)[r]
                reach[base + loc[loc >= 0]] = True
        kept = reach & (kind == GATE)
    else:
        need = np.zeros(n_sig, bool)
        lo = int(offsets[-2])
        last = np.arange(lo, n_sig)
        need[last[kind[last] == GATE]] = True
        need[sig[last[kind[last] == REF]]] = True
        for l in range(len(layers) - 1, -1, -1):
            lo, hi = int(offsets[l]), int(offsets[l + 1])
            live = lo + np.flatnonzero(need[lo:hi] & (kind[lo:hi] == GATE))
            need[op_a[live]] = True
            need[op_b[live]] = True
        kept = need & (kind == GATE)
    return PrunedCircuit(in_dim, offsets, kind, sig, inv, gate, op_a, op_b, kept, int(k))


def packed_plan(pc: PrunedCircuit) -> Tuple[List[Tuple[np.ndarray, np.ndarray]], Tuple[np.ndarray, np.ndarray], int]:
    """Tables for the packed evaluator: the kept gates of every layer but the last are materialised as
    rows of one signal buffer (inputs first, then each layer's kept gates in order), so an operand can
    be any earlier row; the last layer becomes the fused count layer, one entry per output neuron
    (gate, pass-through 3 / inverter 12 of a row, or constant 0 / 15).
    Returns ([(sel_ab [n, 2] int32, gate [n] uint8) per materialised layer], count (sel_ab, gate), rows)."""
    n_layers = len(pc.offsets) - 1
    row = np.full(len(pc.kind), -1, np.int64)
    row[:pc.in_dim] = np.arange(pc.in_dim)
    nxt = pc.in_dim
    layers = []
    for l in range(n_layers - 1):
        nodes = pc.layer_nodes(l)
        row[nodes] = nxt + np.arange(len(nodes))
        nxt += len(nodes)
        ab = np.stack([row[pc.op_a[nodes]], row[pc.op_b[nodes]]], 1)
        assert (ab >= 0).all()
        layers.append((ab.astype(np.int32), pc.gate[nodes].astype(np.uint8)))
    lo, hi = int(pc.offsets[-2]), int(pc.offsets[-1])
    ids = np.arange(lo, hi)
    kd = pc.kind[ids]
    ab = np.full((hi - lo, 2), -1, np.int64)
    gt = np.zeros(hi - lo, np.int64)
    m = kd == GATE
    ab[m, 0], ab[m, 1], gt[m] = row[pc.op_a[ids[m]]], row[pc.op_b[ids[m]]], pc.gate[ids[m]]
    m = kd == REF
    ab[m, 0] = row[pc.sig[ids[m]]]
    gt[m] = np.where(pc.inv[ids[m]], 12, 3)
    gt[kd == CONST1] = 15
    if (ab[(kd == GATE) | (kd == REF)][:, 0] < 0).any():
        raise AssertionError("count layer reads a row that was not materialised")
    return layers, (ab.astype(np.int32), gt.astype(np.uint8)), nxt
