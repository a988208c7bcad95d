"""Drop-in replacement of the reference ``compactlogic`` Python API (compactlogic/compactlogic.py).

Same classes, constructor signatures, buffer names, dtypes and shapes (the checkpoint layout the
reference's compiler reads, compiler/extract.py:49-98), the same train/eval/frozen semantics and the
same transposed-view output convention.  The compute runs on hand-written sm_100a kernels through
the C ABI (compactlogic_b200/_lib.py); there is no CPU path.

Differences from the reference, all internal:
  * the softmax over the gate logits, its backward, grad_w and grad_x of a layer are fused into one
    forward and one backward kernel (the reference runs softmax and its backward in PyTorch and
    three separate kernels);
  * int32 slot tables are derived on the device from the int64 ``indices`` / conv offsets and
    re-derived whenever those buffers change (tracked through the tensors' version counters);
  * conv layers return an (N, C, H, W) view of feature-major storage, so Flatten -> LogicLayer
    needs no copy;
  * ``fuse_groupsum(model)`` fuses a trailing (LogicLayer, GroupSum) pair into the layer's kernel.

Host-side algorithms that consume the torch RNG (connection sampling, conflict resolution,
resampling) follow the reference step by step so that a given seed yields identical buffers.
"""
import numpy as np
import torch

from . import _lib as L
from .functional import ConvPlan, GradSlot, LayerSpec, LogicGroupSumFn, LogicLayerFn, eval_forward, eval_group_sum

__all__ = [
    "LogicLayer", "GroupSum", "LogicLayerCudaFunction", "ConvLayer", "ConvLayerCudaFunction",
    "SequentialEntropyFreezer", "FixedSequentialEntropyFreezer", "EntropyRowResampler", "fuse_groupsum",
]


########################################################################################################################


class LogicLayer(torch.nn.Module):
    """Differentiable logic-gate layer (reference: compactlogic/compactlogic.py:10-444).

    Buffers: ``weights`` (out, K) fp32 logits, ``indices`` (2, out, K) int64, ``gate_sequence``
    (out, K) uint8, inverse index ``given_x_indices_of_y_start`` (in+1) int64,
    ``given_x_indices_of_y`` (2*out*K) int64, ``given_x_indices_of_gate`` (2*out*K) int8 and, once
    frozen, ``w`` (out,) uint8.  Input (batch, in_dim), output (batch, out_dim).
    """

    def __init__(self, in_dim: int, out_dim: int, connections: str = 'random', num_gates=16,
                 residual_init: bool = False):
        super().__init__()
        self.in_dim = in_dim
        self.out_dim = out_dim
        self.connections = connections
        self.num_gates = num_gates
        self.log_k = torch.log(torch.tensor(self.num_gates)).item()
        self.init_weights(residual_init)
        self.init_gate_sequence()

        self.get_connections(device=self.weights.device)
        self.refresh_backward_index()

        self.num_neurons = out_dim
        self.num_weights = out_dim
        self.is_frozen = False
        self._spec_key = None
        self._spec = None
        self._fused_groupsum = None  # (k, tau) when fused with a following GroupSum

    # ------------------------------------------------------------------ forward
    def forward(self, x):
        if getattr(self, "is_frozen", False) or not self.training:
            with torch.no_grad():
                return self.forward_cuda_eval(x)
        return self.forward_cuda(x)

    def _to_feature_major(self, x):
        assert x.ndim == 2, x.ndim
        xt = x.transpose(0, 1)
        if xt.shape[1] > 1 and (xt.stride(1) != 1 or xt.stride(0) < xt.shape[1]):
            xt = xt.contiguous()
        assert xt.shape[0] == self.in_dim, (xt.shape, self.in_dim)
        return xt

    def _weights_for(self, dtype):
        return self.weights.double() if dtype == torch.float64 else self.weights

    def forward_cuda(self, x):
        """Train-mode forward (compactlogic.py:83-118): softmax + gate mix in one kernel."""
        in_slot = getattr(x, "_clb_slot", None)
        xt = self._to_feature_major(x)
        spec = self._layer_spec(xt.device)
        w = self._weights_for(xt.dtype)
        if self._fused_groupsum is not None:
            k, tau = self._fused_groupsum
            acc = LogicGroupSumFn.apply(xt, w, spec, k, _group_size(self.out_dim, k), in_slot)
            return acc.transpose(0, 1) / tau
        out_slot = GradSlot() if xt.dtype in (torch.bfloat16, torch.float16) else None
        y = LogicLayerFn.apply(xt, w, spec, in_slot, out_slot).transpose(0, 1)
        if out_slot is not None:
            y._clb_slot = out_slot
        return y

    @torch.no_grad()
    def forward_cuda_eval(self, x):
        """Discrete eval (compactlogic.py:120-130): the argmax gate (or frozen ``w``) per neuron."""
        assert self.is_frozen or not self.training
        sel = self._selected()
        xt = self._to_feature_major(x)
        spec = self._layer_spec(xt.device)
        if self._fused_groupsum is not None:
            k, tau = self._fused_groupsum
            return eval_group_sum(xt, spec, sel, k, _group_size(self.out_dim, k)).transpose(0, 1) / tau
        return eval_forward(xt, spec, sel).transpose(0, 1)

    def _selected(self):
        w = getattr(self, "w", None)
        if w is None:
            w = self.weights.argmax(-1).to(dtype=torch.uint8, device=self.weights.device)
        return w

    # ------------------------------------------------------------------ device slot table
    def _spec_source(self):
        return (self.indices,)

    def _layer_spec(self, device) -> LayerSpec:
        srcs = self._spec_source() + (self.gate_sequence,)
        key = (device,) + tuple((t.data_ptr(), t._version) for t in srcs)
        if self._spec_key != key:
            self._spec = self._build_spec(device)
            self._spec_key = key
        return self._spec

    def _build_spec(self, device) -> LayerSpec:
        L.require_cuda(self.indices)
        out, K = self.out_dim, self.num_gates
        slots = torch.empty(out, K, 2, dtype=torch.int32, device=device)
        err = torch.zeros(1, dtype=torch.int32, device=device)
        idx = self.indices.contiguous()
        L.call("clb_slots_dense", L.ptr(idx[0]), L.ptr(idx[1]), out, K, self.in_dim, L.ptr(slots), L.ptr(err),
               L.stream(device))
        if int(err.item()):
            raise RuntimeError(f"LogicLayer: connection index outside [0, {self.in_dim})")
        return LayerSpec(slots, self.gate_sequence.contiguous(), out, K, 1, self.in_dim, False)

    # ------------------------------------------------------------------ parameters / buffers
    def extra_repr(self):
        return '{}, {}, {}'.format(self.in_dim, self.out_dim, 'train' if self.training else 'eval')

    def init_weights(self, residual_init: bool = False):
        """Gate logits ~ N(0, 1), or favouring the pass-through gate 3 (compactlogic.py:135-147)."""
        rows = getattr(self, 'c_out', self.out_dim)
        if residual_init:
            w = torch.zeros((rows, self.num_gates))
            w[:, 3] = np.log(9 * (self.num_gates - 1))
        else:
            w = torch.randn([rows, self.num_gates])
        self.weights = torch.nn.parameter.Parameter(w)

    def init_gate_sequence(self):
        """Slot k of every row holds gate id k mod 16 (compactlogic.py:149-158)."""
        rows = getattr(self, 'c_out', self.out_dim)
        ids = torch.arange(self.num_gates, device=self.weights.device, dtype=torch.int64) & 15
        self.register_buffer('gate_sequence', ids.unsqueeze(0).repeat(rows, 1).to(torch.uint8))

    def get_connections(self, device='cuda'):
        """Sample the (a, b) input pair of every slot (compactlogic.py:160-182).

        'random': each of the 2*out rows of a column k draws a distinct position of a random
        permutation, folded onto the inputs through a second per-column permutation, so every input
        is used about equally often.  'original': one pair per neuron shared by all its slots.
        """
        assert self.out_dim * 2 >= self.in_dim, (
            'The number of neurons ({}) must not be smaller than half of the number of inputs ({}) because '
            'otherwise not all inputs could be used or considered.'.format(self.out_dim, self.in_dim))
        if self.connections == 'random':
            order = torch.argsort(torch.rand(2 * self.out_dim, self.num_gates, device=device), dim=0)
            fold = torch.argsort(torch.rand(self.in_dim, self.num_gates, device=device), dim=0)
            c = torch.gather(fold, dim=0, index=order % self.in_dim).view(2, self.out_dim, self.num_gates)
        elif self.connections == 'original':
            pos = torch.randperm(2 * self.out_dim) % self.in_dim
            c = torch.randperm(self.in_dim)[pos]
            c = torch.broadcast_to(c.unsqueeze(-1), (*c.shape, self.num_gates)).reshape(2, self.out_dim,
                                                                                         self.num_gates)
        else:
            raise NotImplementedError(f'self.connections: "{self.connections}" not implemented.')
        self.register_buffer('indices', c.to(torch.int64).to(device))

    def refresh_backward_index(self, changed_rows: torch.Tensor | None = None) -> None:
        """Inverse connection index: for every input, the (neuron, slot, side) entries reading it
        (compactlogic.py:184-274).  Side a is stored as the slot id k, side b as -(k+1).  A full
        rebuild lists all a-side entries in (neuron, slot) order followed by all b-side entries and
        sorts them by input; an incremental rebuild keeps the entries of unchanged rows and appends
        fresh ones for ``changed_rows`` before sorting."""
        if not hasattr(self, "indices") or self.indices.ndim != 3:
            return
        dev = self.indices.device
        n_in = self.in_dim
        n_out, K = self.indices.shape[1], self.indices.shape[2]
        slot_ids = torch.arange(K, device=dev, dtype=torch.int64)

        def entries(rows):
            rows = rows.to(device=dev, dtype=torch.int64).flatten()
            if rows.numel() == 0:
                e64 = torch.empty(0, dtype=torch.int64, device=dev)
                return e64, e64, torch.empty(0, dtype=torch.int8, device=dev)
            ks = slot_ids.unsqueeze(0).expand(rows.numel(), -1).reshape(-1)
            js = rows.unsqueeze(1).expand(-1, K).reshape(-1)
            inputs = torch.cat((self.indices[0, rows].reshape(-1), self.indices[1, rows].reshape(-1)), dim=0)
            neurons = torch.cat((js, js), dim=0)
            codes = torch.cat((ks, -(ks + 1)), dim=0).to(torch.int8)
            return inputs, neurons, codes

        def store(inputs, neurons, codes):
            perm = inputs.argsort()
            counts = torch.bincount(inputs[perm], minlength=n_in)
            starts = torch.empty(n_in + 1, dtype=torch.int64, device=dev)
            starts[0] = 0
            starts[1:] = counts.cumsum(0)
            self._set_or_register_buffer("given_x_indices_of_y_start", starts)
            self._set_or_register_buffer("given_x_indices_of_y", neurons[perm])
            self._set_or_register_buffer("given_x_indices_of_gate", codes[perm])

        if changed_rows is None or "given_x_indices_of_y_start" not in self._buffers:
            store(*entries(torch.arange(n_out, device=dev, dtype=torch.int64)))
            return
        changed_rows = changed_rows.to(device=dev, dtype=torch.int64).flatten()
        if changed_rows.numel() == 0:
            return
        changed_rows = torch.unique(changed_rows)
        is_changed = torch.zeros(n_out, dtype=torch.bool, device=dev)
        is_changed[changed_rows] = True
        starts = self.given_x_indices_of_y_start
        old_neurons = self.given_x_indices_of_y
        old_codes = self.given_x_indices_of_gate
        old_inputs = torch.arange(n_in, device=dev, dtype=torch.int64).repeat_interleave(starts[1:] - starts[:-1])
        keep = ~is_changed[old_neurons]
        new_inputs, new_neurons, new_codes = entries(changed_rows)
        store(torch.cat((old_inputs[keep], new_inputs), dim=0), torch.cat((old_neurons[keep], new_neurons), dim=0),
              torch.cat((old_codes[keep], new_codes), dim=0))

    def _set_or_register_buffer(self, name: str, tensor: torch.Tensor) -> None:
        if name in self._buffers:
            self._buffers[name] = tensor
        else:
            self.register_buffer(name, tensor)

    @torch.no_grad()
    def resample_connections(self, converged_rows, threshold_high: float = 0.95, threshold_low: float = 0.0,
                             update_gate=True, keep_strong_weights=True, draws=None):
        """Re-draw rows whose gate distribution converged (compactlogic.py:282-348).

        Weak rows (max prob < threshold_low): new N(0,1) logits, new random gates and connections for
        every slot.  Strong rows (max prob > threshold_high): keep the winning slot with logit
        log(p (K-1) / (1-p)) (or log(9 (K-1))), zero the others and give them new gates and
        connections.  Returns (weak_mask, strong_mask).

        ``draws`` (optional, from ``resample_draws``): take the random values from these full-size tensors
        at the rewritten positions instead of drawing them in the reference's order; the device path
        (``resample_rows_device``) consumes the same tensors, so both give identical buffers."""
        dev = self.weights.device
        rows = self.weights.shape[0]
        assert len(converged_rows.shape) == 1
        picked = torch.zeros(rows, device=dev, dtype=torch.bool)
        picked[converged_rows.detach().clone().to(dev)] = True

        row_max, row_argmax = torch.nn.functional.softmax(self.weights, dim=-1).max(dim=1)
        strong_mask = (row_max > threshold_high) & picked
        weak_mask = (row_max < threshold_low) & picked
        n_strong = strong_mask.sum().item()
        n_weak = weak_mask.sum().item()
        pool = torch.arange(16, device=dev, dtype=torch.uint8)

        if n_weak:
            self.weights[weak_mask] = (draws["logits"][weak_mask] if draws is not None else
                                       torch.randn((n_weak, self.num_gates), device=dev))
            if update_gate:
                self.gate_sequence[weak_mask] = (draws["gates"][weak_mask] if draws is not None else
                                                 pool[torch.randint(0, len(pool), (n_weak, self.num_gates), device=dev)])
            if draws is not None:
                self._indices_from_draws(weak_mask, draws)
            else:
                self.update_indices_weak(n_weak, weak_mask)

        if n_strong:
            refill = torch.zeros_like(self.weights, dtype=torch.bool, device=dev)
            refill[strong_mask] = True
            strong_rows = strong_mask.nonzero(as_tuple=False).squeeze(-1)
            winners = row_argmax[strong_rows]
            refill[strong_rows, winners] = False
            p = row_max[strong_mask].clamp(min=1e-6, max=1 - 1e-6)
            self.weights[strong_mask] = 0.0
            self.weights[strong_rows, winners] = (torch.log(p * (self.num_gates - 1) / (1 - p)) if keep_strong_weights
                                                  else np.log(9 * (self.num_gates - 1)))
            n_fill = refill.sum().item()
            if update_gate and n_fill > 0:
                self.gate_sequence[refill] = (draws["gates"][refill] if draws is not None else
                                              pool[torch.randint(0, len(pool), (n_fill,), device=dev)])
            if draws is not None:
                self._indices_from_draws(refill, draws)
            else:
                self.update_indices_strong(refill, n_fill)
        if n_weak or n_strong:
            self.refresh_backward_index(
                torch.nonzero(torch.logical_or(weak_mask, strong_mask), as_tuple=False).flatten())
        return weak_mask, strong_mask

    def _indices_from_draws(self, mask, draws):
        if not hasattr(self, "indices"):
            raise NotImplementedError("resampling from pre-drawn tensors is implemented for LogicLayer connections")
        self.indices[0][mask] = draws["a"][mask]
        self.indices[1][mask] = draws["b"][mask]

    @torch.no_grad()
    def resample_draws(self, generator=None):
        """Full-size random tensors for one resampling call: N(0,1) logits, gate ids in [0, 16) and the two
        operands' inputs in [0, in_dim), each [rows, K] on the layer's device."""
        dev = self.weights.device
        shape = tuple(self.weights.shape)
        return {"logits": torch.randn(shape, device=dev, generator=generator),
                "gates": torch.randint(0, 16, shape, device=dev, dtype=torch.uint8, generator=generator),
                "a": torch.randint(0, self.in_dim, shape, device=dev, dtype=torch.int64, generator=generator),
                "b": torch.randint(0, self.in_dim, shape, device=dev, dtype=torch.int64, generator=generator)}

    def device_resample_ok(self) -> bool:
        """Whether ``resample_rows_device`` handles this layer: a dense CUDA layer, fp32 logits, K <= 32."""
        return (type(self) is not ConvLayer and hasattr(self, "indices") and self.weights.is_cuda and
                self.weights.dtype == torch.float32 and self.num_gates <= 32 and self.weights.is_contiguous())

    @torch.no_grad()
    def resample_rows_device(self, picked: torch.Tensor, draws=None, threshold_high: float = 0.95,
                             threshold_low: float = 0.0, update_gate=True, keep_strong_weights=True,
                             adam_state=None, counter=None) -> torch.Tensor:
        """``resample_connections`` for the rows flagged in ``picked`` (uint8 [rows], on the device), as one
        kernel (clb_resample_rows) plus a sort-based inverse-index rebuild: nothing is read back to the host.
        Also zeroes the Adam moments (``adam_state``, the optimizer's state dict of ``weights``) of changed
        rows and resets ``counter`` on picked rows.  Returns the changed-row mask (uint8 [rows])."""
        if not self.device_resample_ok():
            raise RuntimeError("resample_rows_device: needs a dense CUDA layer with fp32 logits and K <= 32")
        draws = draws if draws is not None else self.resample_draws()
        dev = self.weights.device
        rows, K = self.weights.shape
        changed = torch.empty(rows, dtype=torch.uint8, device=dev)
        st = adam_state or {}
        m1, m2 = st.get("exp_avg"), st.get("exp_avg_sq")
        w = self.weights.data
        L.call("clb_resample_rows", L.ptr(w), L.ptr(self.gate_sequence), L.ptr(self.indices[0]),
               L.ptr(self.indices[1]), rows, K, L.ptr(picked), float(threshold_high), float(threshold_low),
               int(bool(keep_strong_weights)), int(bool(update_gate)), L.ptr(draws["logits"]), L.ptr(draws["gates"]),
               L.ptr(draws["a"]), L.ptr(draws["b"]), L.ptr(changed), L.ptr(m1), L.ptr(m2), L.ptr(counter),
               L.stream(dev))
        # the kernel rewrote the buffers in place: bump their versions so the slot table is rebuilt
        self.indices.add_(0)
        self.gate_sequence.add_(0)
        if "max_exp_avg_sq" in st:
            st["max_exp_avg_sq"].masked_fill_(changed.bool()[:, None], 0.0)
        # the native kernels never read the inverse index: rebuild it when something does (the reference-API
        # backward, a checkpoint, a device move), applying the pending refreshes in order
        self.__dict__.setdefault("_csr_pending", []).append(changed)
        return changed

    _CSR_BUFFERS = ("given_x_indices_of_y_start", "given_x_indices_of_y", "given_x_indices_of_gate")

    def _materialize_csr(self) -> None:
        pending = self.__dict__.get("_csr_pending")
        if pending:
            self.__dict__["_csr_pending"] = []
            for changed in pending:
                self.refresh_backward_index_device(changed)

    def __getattr__(self, name):
        if name in LogicLayer._CSR_BUFFERS and self.__dict__.get("_csr_pending"):
            self._materialize_csr()
        return super().__getattr__(name)

    def state_dict(self, *args, **kwargs):
        self._materialize_csr()
        return super().state_dict(*args, **kwargs)

    def _apply(self, fn, *args, **kwargs):
        self._materialize_csr()
        return super()._apply(fn, *args, **kwargs)

    @torch.no_grad()
    def refresh_backward_index_device(self, changed: torch.Tensor = None) -> None:
        """``refresh_backward_index`` with no host synchronisation: one sort of a 64-bit key per (neuron,
        slot, operand) entry, (input << 32) | position, where an entry of an unchanged neuron keeps its
        position in the current index and an entry of a changed neuron (``changed`` uint8 [out], None =
        all) is placed after them in the order the host rebuild appends it (operand a of every changed
        row, then operand b; rows ascending, slots ascending).  The start offsets equal the host path's and
        every input's entries are the same set; within an input the order is the entry list's (a stable
        sort), which the host's unstable argsort (kept for the reference's CPU order) may permute."""
        dev = self.indices.device
        n_out, K = self.indices.shape[1], self.indices.shape[2]
        M = 2 * n_out * K
        eid = torch.arange(M, device=dev, dtype=torch.int64)
        side, rem = eid // (n_out * K), eid % (n_out * K)
        j, k = rem // K, rem % K
        inputs = self.indices.reshape(-1)
        if changed is None or "given_x_indices_of_y_start" not in self._buffers:
            key = eid
        else:
            ch = changed.to(torch.int64)
            rank = torch.cumsum(ch, 0) - ch  # rank of a changed row among the changed rows
            nc = ch.sum()
            codes_old = self.given_x_indices_of_gate.to(torch.int64)
            old_side = (codes_old < 0).to(torch.int64)
            old_k = torch.where(codes_old < 0, -codes_old - 1, codes_old)
            old_eid = old_side * (n_out * K) + self.given_x_indices_of_y * K + old_k
            pos = torch.empty(M, dtype=torch.int64, device=dev)
            pos.scatter_(0, old_eid, eid)
            new_key = M + side * nc * K + rank[j] * K + k
            key = torch.where(ch[j] > 0, new_key, pos)
        order = torch.sort((inputs << 32) | key).indices
        counts = torch.zeros(self.in_dim, dtype=torch.int64, device=dev)
        counts.scatter_add_(0, inputs, torch.ones_like(inputs))
        starts = torch.zeros(self.in_dim + 1, dtype=torch.int64, device=dev)
        starts[1:] = torch.cumsum(counts, 0)
        self._set_or_register_buffer("given_x_indices_of_y_start", starts)
        self._set_or_register_buffer("given_x_indices_of_y", j[order])
        self._set_or_register_buffer("given_x_indices_of_gate",
                                     torch.where(side[order] > 0, -(k[order] + 1), k[order]).to(torch.int8))

    @torch.no_grad()
    def update_indices_weak(self, n_weak, weak_mask):
        """New uniform inputs for both operands of every slot of the weak rows (compactlogic.py:350-359)."""
        dev = self.weights.device
        for side in (0, 1):
            self.indices[side][weak_mask] = torch.randint(0, self.in_dim, (n_weak, self.num_gates), device=dev,
                                                          dtype=torch.int64)

    @torch.no_grad()
    def update_indices_strong(self, mask2d, num_to_fill):
        """New uniform inputs for the refilled slots of strong rows (compactlogic.py:361-368)."""
        dev = self.weights.device
        for side in (0, 1):
            self.indices[side][mask2d] = torch.randint(0, self.in_dim, (num_to_fill,), device=dev, dtype=torch.int64)

    @torch.no_grad()
    def weights_entropy(self, dim: int = -1) -> torch.Tensor:
        """Entropy of the gate distribution per row, divided by log K (compactlogic.py:370-385)."""
        log_p = torch.log_softmax(self.weights, dim=dim)
        return -(log_p.exp() * log_p).sum(dim=dim) / self.log_k

    def freeze(self):
        """Fix every row to its argmax gate (compactlogic.py:387-394)."""
        self.weights.requires_grad = False
        self.register_buffer("w", self.weights.argmax(-1).to(dtype=torch.uint8, device=self.weights.device))
        self.is_frozen = True

    def unfreeze(self):
        self.weights.requires_grad = True
        self.is_frozen = False

    @torch.no_grad()
    def connected_neurons(self, y_flag: torch.Tensor, const_gates=None, trivial_gates_a=None, trivial_gates_b=None,
                          device=None):
        """Masks of inputs that reach active outputs, for pruning (compactlogic.py:400-444).
        Defaults: constant gates {0, 15}, a-only gates {3, 12}, b-only gates {5, 10}."""
        device = self.weights.device if device is None else device
        const_gates = torch.tensor([0, 15], device=device) if const_gates is None else const_gates
        trivial_gates_a = torch.tensor([3, 12], device=device) if trivial_gates_a is None else trivial_gates_a
        trivial_gates_b = torch.tensor([5, 10], device=device) if trivial_gates_b is None else trivial_gates_b
        assert y_flag.shape == (self.out_dim,), f'y_flag shape mismatch: {y_flag.shape}, should be {self.out_dim}'
        x_flag = torch.zeros(self.in_dim, dtype=bool, device=device)
        w = getattr(self, 'w', self.weights.argmax(-1)).to(torch.long)
        pair = torch.gather(self.indices, dim=2, index=w.view(1, -1, 1).expand(2, -1, 1)).squeeze(-1)
        g = torch.gather(self.gate_sequence, dim=1, index=w.unsqueeze(-1)).squeeze(-1)
        is_const = torch.isin(g, const_gates)
        only_a = torch.isin(g, trivial_gates_a)
        only_b = torch.isin(g, trivial_gates_b)
        y_flag[is_const] = False
        uses = torch.cat((pair[0][y_flag & ~is_const & ~only_b], pair[1][y_flag & ~is_const & ~only_a]))
        x_flag[torch.unique(uses)] = True
        y_flag[only_a | only_b] = False
        return x_flag, y_flag


def _group_size(out_dim: int, k: int) -> int:
    """Neurons per class after GroupSum's zero padding of out_dim to a multiple of k."""
    return -(-out_dim // k)


########################################################################################################################


class GroupSum(torch.nn.Module):
    """Sum of k contiguous neuron groups divided by tau (compactlogic/compactlogic.py:450-468).
    When the preceding LogicLayer was fused with it (``fuse_groupsum``) this module passes its input
    (already the class logits) through."""

    def __init__(self, k: int, tau: float = 1., device='cuda'):
        super().__init__()
        self.k = k
        self.tau = tau
        self.device = device
        self.absorbed = False

    def forward(self, x):
        if self.absorbed:
            assert x.shape[-1] == self.k, (x.shape, self.k)
            return x
        if x.shape[-1] % self.k != 0:
            x = torch.cat([x, torch.zeros((x.shape[0], self.k - x.shape[1] % self.k), device=x.device,
                                          dtype=x.dtype)], dim=1)
        return x.reshape(*x.shape[:-1], self.k, x.shape[-1] // self.k).sum(-1) / self.tau

    def extra_repr(self):
        return 'k={}, tau={}'.format(self.k, self.tau)


def fuse_groupsum(model: torch.nn.Sequential) -> torch.nn.Sequential:
    """Fuse every (LogicLayer, GroupSum) pair of a Sequential: the layer then accumulates class sums
    in its kernel and never materialises its (batch, out) output.  Buffers and state_dict keys are
    unchanged.  Returns the model."""
    mods = list(model)
    for prev, nxt in zip(mods[:-1], mods[1:]):
        if isinstance(nxt, GroupSum) and type(prev) is LogicLayer:
            prev._fused_groupsum = (nxt.k, nxt.tau)
            nxt.absorbed = True
    return model


########################################################################################################################


class LogicLayerCudaFunction(torch.autograd.Function):
    """The reference autograd bridge (compactlogic/compactlogic.py:474-508), same signature: takes
    probabilities ``w`` and the inverse index, returns grad w.r.t. x and w.  Runs on the
    reference-compatible kernels of ``compactlogic_b200.difflogic_cuda``."""

    @staticmethod
    def forward(ctx, x, a, b, w, gate_sequence, given_x_indices_of_y_start, given_x_indices_of_y,
                given_x_indices_of_gate):
        from . import difflogic_cuda
        ctx.save_for_backward(x, a, b, w, gate_sequence, given_x_indices_of_y_start, given_x_indices_of_y,
                              given_x_indices_of_gate)
        return difflogic_cuda.forward(x, a, b, w, gate_sequence)

    @staticmethod
    def backward(ctx, grad_y):
        from . import difflogic_cuda
        x, a, b, w, gate_sequence, starts, ys, codes = ctx.saved_tensors
        grad_y = grad_y.contiguous()
        grad_x = grad_w = None
        if ctx.needs_input_grad[0]:
            grad_x = difflogic_cuda.backward_x(x, a, b, w, gate_sequence, grad_y, starts, ys, codes)
        if ctx.needs_input_grad[3]:
            grad_w = difflogic_cuda.backward_w(x, a, b, gate_sequence, grad_y)
        return grad_x, None, None, grad_w, None, None, None, None


########################################################################################################################


class ConvLayer(LogicLayer):
    """Convolutional logic layer (reference: compactlogic/compactlogic.py:514-832).

    Buffers ``offsets_ch`` (2, c_out, K) int32 and ``offsets_h`` / ``offsets_w`` (2, c_out, K) int8,
    the spatial offsets already shifted by -padding.  Input (batch, c_in, h_in, w_in), output
    (batch, c_out, h_out, w_out) — returned as a view of channel-major storage [c_out*h_out*w_out,
    batch]."""

    def __init__(self, in_shape, padding: int, c_out: int, ks: int, stride: int, num_chn: int = 1, **kwargs):
        self.padding = padding
        self.c_in, self.h_in, self.w_in = in_shape[0], in_shape[1] + 2 * padding, in_shape[2] + 2 * padding
        self.in_dim = np.prod((self.c_in, self.h_in, self.w_in))
        self.in_shape = in_shape
        self.c_out = c_out
        self.ks = ks
        self.stride = stride
        self.h_out = (self.h_in - self.ks) // self.stride + 1
        self.w_out = (self.w_in - self.ks) // self.stride + 1
        self.out_shape = (self.c_out, self.h_out, self.w_out)
        self.out_dim = np.prod(self.out_shape)
        self.chn_grp = num_chn if num_chn <= 1 else (self.c_in // num_chn)
        super().__init__(self.in_dim, self.out_dim, **kwargs)

    def _to_feature_major(self, x):
        assert tuple(x.shape[1:]) == tuple(self.in_shape), f'input shape mismatch {x.shape}, {self.in_shape}'
        assert x.ndim == 4, x.ndim
        F = int(np.prod(self.in_shape))
        xt = x.permute(1, 2, 3, 0)
        if not xt.is_contiguous():
            xt = xt.contiguous()
        return xt.reshape(F, x.shape[0])

    def _to_public(self, y):
        return y.view(self.c_out, self.h_out, self.w_out, -1).permute(3, 0, 1, 2)

    def forward_cuda(self, x):
        """Train-mode conv forward (compactlogic.py:598-626)."""
        if self.training:
            assert x.device.type == 'cuda', x.device
        in_slot = getattr(x, "_clb_slot", None)
        xt = self._to_feature_major(x)
        spec = self._layer_spec(xt.device)
        out_slot = GradSlot() if xt.dtype in (torch.bfloat16, torch.float16) else None
        y = self._to_public(LogicLayerFn.apply(xt, self._weights_for(xt.dtype), spec, in_slot, out_slot))
        if out_slot is not None:
            y._clb_slot = out_slot
        return y

    @torch.no_grad()
    def forward_cuda_eval(self, x):
        """Discrete conv eval (compactlogic.py:628-640)."""
        assert self.is_frozen or not self.training
        xt = self._to_feature_major(x)
        return self._to_public(eval_forward(xt, self._layer_spec(xt.device), self._selected()))

    def _spec_source(self):
        return (self.offsets_ch, self.offsets_h, self.offsets_w)

    def _build_spec(self, device) -> LayerSpec:
        L.require_cuda(self.offsets_ch)
        c_in, h, w = (int(v) for v in self.in_shape)
        K = self.num_gates
        n_out = int(self.out_dim)
        slots = torch.empty(n_out, K, 2, dtype=torch.int32, device=device)
        err = torch.zeros(1, dtype=torch.int32, device=device)
        och, oh, ow = self.offsets_ch.contiguous(), self.offsets_h.contiguous(), self.offsets_w.contiguous()
        L.call("clb_slots_conv", L.ptr(och), L.ptr(oh), L.ptr(ow), self.c_out, K, c_in, h, w, self.h_out, self.w_out,
               self.stride, L.ptr(slots), L.ptr(err), L.stream(device))
        if int(err.item()):
            raise RuntimeError(f"ConvLayer: channel offset outside [0, {c_in})")
        return LayerSpec(slots, self.gate_sequence.contiguous(), n_out, K, self.h_out * self.w_out,
                         int(np.prod(self.in_shape)), True, conv=self._plane_plan(och, oh, ow, device))

    def _plane_plan(self, och, oh, ow, device):
        """Channel grouping for the receptive-field-staged kernels, or None when a slot reads another
        channel than its row's first one, or an offset lies outside [-pad, ks-1-pad]."""
        c_in, h, w = (int(v) for v in self.in_shape)
        lo, hi = -self.padding, self.ks - 1 - self.padding
        chan = och[0, :, 0]
        single = bool(((och == chan.view(1, -1, 1)).all()).item())
        in_range = bool((((oh >= lo) & (oh <= hi)).all() & ((ow >= lo) & (ow <= hi)).all()).item())
        if not (single and in_range):
            return None
        chan64 = chan.to(torch.int64)
        order = torch.argsort(chan64, stable=True).to(torch.int32)
        counts = torch.bincount(chan64, minlength=c_in)
        starts = torch.zeros(c_in + 1, dtype=torch.int32, device=device)
        starts[1:] = counts.cumsum(0).to(torch.int32)
        return ConvPlan(c_in, h, w, int(self.c_out), int(self.h_out), int(self.w_out), int(self.stride),
                        int(self.padding), int(self.ks), oh, ow, order, starts, int(counts.max().item()),
                        torch.zeros(1, dtype=torch.int32, device=device))

    def get_connections(self, device='cuda'):
        """Sample channel and spatial offsets of every slot (compactlogic.py:642-698).

        num_chn > 1: channels drawn within groups of input channels; num_chn == 1: channel
        c_out % c_in for both operands; num_chn == 0: any channel.  Spatial offsets are uniform in
        [0, ks); identical operand pairs are re-drawn, then the offsets are shifted by -padding."""
        K = self.num_gates
        shape = (2, self.c_out, K)
        if self.chn_grp > 1:
            assert self.chn_grp <= self.c_in and self.chn_grp <= self.c_out
            offsets_h = torch.randint(0, self.ks, size=shape, device=device, dtype=torch.int8)
            offsets_w = torch.randint(0, self.ks, size=shape, device=device, dtype=torch.int8)
            per_group, extra = self.c_in // self.chn_grp, self.c_in % self.chn_grp
            sizes = torch.full((self.chn_grp,), per_group, device=device)
            sizes[:extra] += 1
            bounds = torch.cat([torch.zeros(1, device=device), sizes.cumsum(0)]).to(torch.int32)
            channels = torch.arange(self.c_in, device=device, dtype=torch.int32)
            members = [channels[bounds[i]:bounds[i + 1]] for i in range(len(bounds) - 1)]
            out_per_group = self.c_out // self.chn_grp
            group_of = torch.clamp(torch.arange(self.c_out, device=device, dtype=torch.int32) // out_per_group, 0,
                                   self.chn_grp - 1)
            offsets_ch = torch.empty(shape, device=device, dtype=torch.int32)
            for gid, chans in enumerate(members):
                outs = (group_of == gid).nonzero(as_tuple=True)[0]
                if outs.numel() > 0:
                    for side in (0, 1):
                        offsets_ch[side, outs] = chans[torch.randint(0, chans.numel(), (outs.numel(), K),
                                                                     device=device)]
        elif self.chn_grp == 1:
            assert self.ks > 1
            offsets_ch = (torch.arange(0, self.c_out, device=device, dtype=torch.int32) % self.c_in
                          ).unsqueeze(-1).expand(2, -1, K)
            offsets_h = torch.randint(0, self.ks, size=shape, device=device, dtype=torch.int8)
            offsets_w = torch.randint(0, self.ks, size=shape, device=device, dtype=torch.int8)
        else:
            offsets_ch = torch.randint(0, self.c_in, size=shape, device=device, dtype=torch.int32)
            offsets_h = torch.randint(0, self.ks, size=shape, device=device, dtype=torch.int8)
            offsets_w = torch.randint(0, self.ks, size=shape, device=device, dtype=torch.int8)

        offsets_ch, offsets_h, offsets_w = self.resolve_conflicts(offsets_ch, offsets_h, offsets_w, self.ks, self.c_in)
        offsets_h -= self.padding
        offsets_w -= self.padding
        self.register_buffer("offsets_ch", offsets_ch.contiguous().to(device))
        self.register_buffer("offsets_h", offsets_h.contiguous().to(device))
        self.register_buffer("offsets_w", offsets_w.contiguous().to(device))

    @staticmethod
    def resolve_conflicts(offsets_ch, offsets_h, offsets_w, ks, c_in):
        """Re-draw operand b of every slot whose two operands coincide (compactlogic.py:700-743)."""

        def clashes():
            return (offsets_ch[0] == offsets_ch[1]) & (offsets_h[0] == offsets_h[1]) & (offsets_w[0] == offsets_w[1])

        conflict = clashes()
        while conflict.any():
            num = conflict.sum()
            if ks > 1:
                offsets_h[1][conflict] = torch.randint(0, ks, size=(num,), device=offsets_h.device, dtype=torch.int8)
                offsets_w[1][conflict] = torch.randint(0, ks, size=(num,), device=offsets_w.device, dtype=torch.int8)
            elif ks == 1:
                offsets_ch[1][conflict] = torch.randint(0, c_in, size=(num,), device=offsets_ch.device,
                                                        dtype=torch.int32)
            conflict = clashes()
        return offsets_ch, offsets_h, offsets_w

    @torch.no_grad()
    def update_indices_weak(self, n_weak, weak_mask):
        """compactlogic.py:745-762."""
        dev = self.weights.device
        if self.ks == 1:
            for side in (0, 1):
                self.offsets_ch[side][weak_mask] = torch.randint(0, self.c_in, size=(n_weak, self.num_gates),
                                                                 device=dev, dtype=torch.int32)
        else:
            for buf in (self.offsets_h[0], self.offsets_h[1], self.offsets_w[0], self.offsets_w[1]):
                buf[weak_mask] = torch.randint(0, self.ks, size=(n_weak, self.num_gates), device=dev,
                                               dtype=torch.int8) - self.padding

    @torch.no_grad()
    def update_indices_strong(self, mask2d, num_to_fill):
        """compactlogic.py:764-779."""
        dev = self.weights.device
        if self.ks == 1:
            for side in (0, 1):
                self.offsets_ch[side][mask2d] = torch.randint(0, self.c_in, size=(num_to_fill,), device=dev,
                                                              dtype=torch.int32)
        else:
            for buf in (self.offsets_h[0], self.offsets_h[1], self.offsets_w[0], self.offsets_w[1]):
                buf[mask2d] = torch.randint(0, self.ks, size=(num_to_fill,), device=dev,
                                            dtype=torch.int8) - self.padding

    def extra_repr(self):
        return 'in_shape={}, out_shape={}, pad={}, kernel_size={}, stride={}, num_chn={}, {}'.format(
            self.in_shape, self.out_shape, self.padding, self.ks, self.stride,
            self.chn_grp if self.chn_grp <= 1 else (self.c_in // self.chn_grp),
            'train' if self.training else 'eval')

    @torch.no_grad()
    def connected_neurons(self, y_flag: torch.Tensor, const_gates=None, trivial_gates=None, device=None):
        """Pruning masks for a conv layer (compactlogic.py:800-832)."""
        device = self.weights.device if device is None else device
        const_gates = torch.tensor([0, 15], device=device) if const_gates is None else const_gates
        trivial_gates = torch.tensor([3, 5, 10, 12], device=device) if trivial_gates is None else trivial_gates
        assert y_flag.shape == self.out_shape, f'y_flag shape mismatch: {y_flag.shape}, should be {self.out_shape}'
        x_flag = torch.zeros(self.in_shape, dtype=bool, device=device)
        w = getattr(self, 'w', self.weights.argmax(-1)).to(torch.long)
        pick = w.view(1, -1, 1).expand(2, -1, 1)
        och = torch.gather(self.offsets_ch, dim=2, index=pick).squeeze(-1)
        oh = torch.gather(self.offsets_h, dim=2, index=pick).squeeze(-1)
        ow = torch.gather(self.offsets_w, dim=2, index=pick).squeeze(-1)
        g = torch.gather(self.gate_sequence, dim=1, index=w.unsqueeze(-1)).squeeze(-1)
        is_const = torch.isin(g, const_gates)
        y_flag[is_const] = False
        for c in torch.nonzero(~is_const, as_tuple=True)[0]:
            gid = int(g[c])
            sides = [s for s, skip in ((0, (5, 10)), (1, (3, 12))) if gid not in skip]
            for coord in torch.nonzero(y_flag[c]):
                for s in sides:
                    hh = coord[0] * self.stride + oh[s][c]
                    ww = coord[1] * self.stride + ow[s][c]
                    if 0 <= hh < self.in_shape[1] and 0 <= ww < self.in_shape[2]:
                        x_flag[och[s][c], hh, ww] |= True
        y_flag[torch.isin(g, trivial_gates)] = False
        return x_flag, y_flag


class ConvLayerCudaFunction(torch.autograd.Function):
    """The reference conv autograd bridge (compactlogic/compactlogic.py:838-867), same signature,
    on ``compactlogic_b200.convlogic_cuda``."""

    @staticmethod
    def forward(ctx, x, offsets_ch, offsets_h, offsets_w, w, gate_sequence, stride, pad, ks):
        from . import convlogic_cuda
        y = convlogic_cuda.forward(x, offsets_ch, offsets_h, offsets_w, w, gate_sequence, stride, pad, ks)
        ctx.save_for_backward(x, offsets_ch, offsets_h, offsets_w, w, gate_sequence)
        ctx.stride = stride
        ctx.pad = pad
        return y

    @staticmethod
    def backward(ctx, grad_y):
        from . import convlogic_cuda
        x, och, oh, ow, w, gate_sequence = ctx.saved_tensors
        grad_y = grad_y.contiguous()
        grad_x = grad_w = None
        if ctx.needs_input_grad[0]:
            grad_x = convlogic_cuda.backward_x(x, och, oh, ow, w, gate_sequence, grad_y, ctx.stride, ctx.pad)
        if ctx.needs_input_grad[4]:
            grad_w = convlogic_cuda.backward_w(x, och, oh, ow, gate_sequence, grad_y, ctx.stride)
        return grad_x, None, None, None, grad_w, None, None, None, None


########################################################################################################################


def _logic_layers(model):
    return [(i, layer) for i, layer in enumerate(model) if hasattr(layer, "freeze")]


class SequentialEntropyFreezer:
    """Freeze logic layers one at a time, in order, once the EMA of their mean normalised gate
    entropy stops moving (compactlogic/compactlogic.py:873-978).

    Per step and for the first unfrozen layer whose predecessors are all frozen: the first
    observation seeds the EMA and ends the step; afterwards |h - ema_old| < eps increments a
    patience counter (else resets it) and the layer freezes when the counter reaches `patience`
    (at most one layer per step).  `l` caps the managed layers (default: all but the last)."""

    def __init__(self, model, ema_decay=0.99, eps=5e-4, patience=200, min_iters=0, l=None):
        self.model = model
        self.ema_decay = ema_decay
        self.eps = eps
        self.patience = patience
        self.min_iters = min_iters
        self.l = l
        layers = _logic_layers(model)
        self.logic_layers = layers[:-1] if l is None else layers[:int(l)]
        self.ema = {}
        self.counter = {}
        self.iter = 0

    def step(self, iter: int):
        self.iter = iter
        if self.iter < self.min_iters:
            return
        for idx, layer in self.logic_layers:
            if not self._can_consider_layer(idx) or layer.is_frozen:
                continue
            h = layer.weights_entropy().mean().item()
            if idx not in self.ema:
                self.ema[idx] = h
                self.counter[idx] = 0
                return
            old = self.ema[idx]
            self.ema[idx] = self.ema_decay * old + (1 - self.ema_decay) * h
            self.counter[idx] = self.counter[idx] + 1 if abs(h - old) < self.eps else 0
            if self.counter[idx] >= self.patience:
                self._freeze_layer(layer)
                break

    def _can_consider_layer(self, idx):
        return all(layer.is_frozen for i, layer in self.logic_layers if i < idx)

    def _freeze_layer(self, layer):
        layer.freeze()

    def __str__(self):
        return 'ema_decay={}, eps={}, patience={}, min_iters={}'.format(self.ema_decay, self.eps, self.patience,
                                                                       self.min_iters)


class FixedSequentialEntropyFreezer:
    """Freeze the n-th managed layer at step min_iters + n*N, one per call, in order
    (compactlogic/compactlogic.py:984-1051)."""

    def __init__(self, model, N: int, min_iters: int = 0, l=None):
        if N <= 0:
            raise ValueError(f'N must be > 0, got {N}.')
        self.model = model
        self.N = int(N)
        self.min_iters = min_iters
        self.l = l
        layers = _logic_layers(model)
        self.logic_layers = layers[:-1] if l is None else layers[:int(l)]
        self.iter = 0

    def step(self, iter: int):
        self.iter = iter
        for order, (_, layer) in enumerate(self.logic_layers, start=1):
            if layer.is_frozen:
                continue
            if self.iter >= self.min_iters + order * self.N:
                layer.freeze()
            break

    def __str__(self):
        return 'N={}, min_iters={}'.format(self.N, self.min_iters)


class EntropyRowResampler:
    """Per-row entropy convergence monitor that re-draws converged rows and clears their Adam moments
    (compactlogic/compactlogic.py:1057-1190)."""

    def __init__(self, model, ema_decay: float = 0.99, eps: float = 5e-4, patience: int = 200, min_iters: int = 0,
                 max_iters=np.inf, only_unfrozen: bool = True, **kwargs):
        self.model = model
        self.ema_decay = ema_decay
        self.eps = eps
        self.patience = patience
        self.min_iters = min_iters
        self.max_iters = max_iters
        self.only_unfrozen = only_unfrozen
        self.resample_kwargs = kwargs
        self.layers = [(i, layer) for i, layer in enumerate(model) if hasattr(layer, "resample_connections")]
        self.ema = {}
        self.counter = {}
        self.iter = 0

    #: on CUDA layers with fp32 logits, run the per-row monitor as one fused kernel per layer and read
    #: the converged counts of all layers with a single host synchronisation per step
    use_device_monitor = True
    #: with the device monitor, rewrite converged rows of dense layers with one kernel per layer and rebuild
    #: the inverse index with a device sort (no further synchronisation).  The random values come from
    #: full-size draws (LogicLayer.resample_draws) instead of the reference's count-sized draws, so the
    #: buffers match the reference's in distribution, not bit for bit under one seed; set False for that.
    use_device_resample = True

    @torch.no_grad()
    def step(self, iter: int, optimizer):
        self.iter = iter
        if self.iter < self.min_iters or self.iter > self.max_iters:
            return
        active = [(idx, layer) for idx, layer in self.layers
                  if not (self.only_unfrozen and getattr(layer, "is_frozen", False))]
        if self.use_device_monitor and active and all(
                l.weights.is_cuda and l.weights.dtype == torch.float32 for _, l in active):
            self._step_device(active, optimizer)
            return
        for idx, layer in active:
            h = layer.weights_entropy().detach()
            assert h.dim() == 1
            if idx not in self.ema:
                self.ema[idx] = h.clone()
                self.counter[idx] = torch.zeros_like(h, dtype=torch.int32, device=h.device)
                continue
            old = self.ema[idx]
            self.ema[idx] = self.ema_decay * old + (1.0 - self.ema_decay) * h
            cnt = self.counter[idx]
            self.counter[idx] = torch.where((h - old).abs() < self.eps, cnt + 1, torch.zeros_like(cnt))
            rows = (self.counter[idx] >= self.patience).nonzero(as_tuple=False).flatten()
            self._resample(idx, layer, rows, optimizer)

    def _resample(self, idx, layer, rows, optimizer):
        if rows.numel() > 0:
            weak, strong = layer.resample_connections(rows, **self.resample_kwargs)
            changed = torch.logical_or(weak, strong)
            self.reset_adam_state_for_mask(optimizer, layer.weights, changed[:, None].expand_as(layer.weights))
            self.counter[idx][rows] = 0

    def _step_device(self, active, optimizer):
        dev = active[0][1].weights.device
        counts = torch.zeros(len(active), dtype=torch.int32, device=dev)
        pending = []
        for i, (idx, layer) in enumerate(active):
            w = layer.weights.detach()
            if w.stride(-1) != 1 or w.stride(0) != w.shape[1]:
                w = w.contiguous()
            rows = w.shape[0]
            first = idx not in self.ema
            if first:
                self.ema[idx] = torch.empty(rows, dtype=torch.float32, device=dev)
                self.counter[idx] = torch.zeros(rows, dtype=torch.int32, device=dev)
            flags = torch.empty(rows, dtype=torch.uint8, device=dev)
            L.call("clb_entropy_monitor", L.ptr(w), rows, w.shape[1], float(self.ema_decay), float(self.eps),
                   int(min(self.patience, 2**31 - 1)), int(first), L.ptr(self.ema[idx]), L.ptr(self.counter[idx]),
                   L.ptr(flags), L.ptr(counts[i:i + 1]), L.stream(dev))
            if not first:
                pending.append((i, idx, layer, flags))
        if not pending:
            return
        host_counts = counts.cpu()  # the one synchronisation of the step
        for i, idx, layer, flags in pending:
            if int(host_counts[i]) == 0:
                continue
            if self.use_device_resample and layer.device_resample_ok():
                layer.resample_rows_device(flags, adam_state=optimizer.state.get(layer.weights, None),
                                           counter=self.counter[idx], **self.resample_kwargs)
            else:
                self._resample(idx, layer, flags.nonzero(as_tuple=False).flatten(), optimizer)

    @torch.no_grad()
    def reset_adam_state_for_mask(self, optimizer, param, mask):
        """Zero the Adam moments of the masked entries (compactlogic.py:1152-1180)."""
        st = optimizer.state.get(param, None)
        if not st:
            return
        for key in ("exp_avg", "exp_avg_sq", "max_exp_avg_sq"):
            if key in st:
                st[key].masked_fill_(mask, 0.0)

    def __str__(self):
        return 'ema_decay={}, eps={}, patience={}, min_iters={}, max_iters={}, resample_kwargs={}'.format(
            self.ema_decay, self.eps, self.patience, self.min_iters, self.max_iters, self.resample_kwargs)
