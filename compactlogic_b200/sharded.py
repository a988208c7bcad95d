"""Width-sharded (neuron-parallel) training of dense logic layers, one process per GPU.

Each rank owns a contiguous share [lo, hi) of every layer's neurons (its rows of ``weights``,
``indices`` and ``gate_sequence``, compactlogic/compactlogic.py:10-182) and runs the whole batch.
Every rank needs the full input activations of a layer, because a neuron reads two arbitrary inputs;
the two exchanges this implies are fused into the layer kernels over NVLink peer memory:

* forward: the kernel's epilogue stores the owned output rows straight into every rank's full
  activation buffer (the all-gather, as peer stores overlapped with the gather-bound compute);
* backward: each rank scatters its neurons' contributions to grad_x into a local partial buffer; the
  previous layer's backward kernel reads its grad_y rows as the sum of all ranks' partials (the
  reduce-scatter, as peer loads inside the grad_y load).

The ranks are ordered by one tiny NCCL all-reduce after each layer kernel (stream-ordered, so a
rank's kernel has finished before any rank passes it).  Gate-logit gradients are local: no all-reduce
of parameters.  The activation buffers are persistent and mapped into all ranks, so a training
forward must be followed by its backward before the next training forward (eval / no-grad forwards
use separate, NCCL-gathered tensors).

Against data parallelism (``parallel.GradAllReduce``) this moves (N-1)/N of the activations and of
the activation gradients of every layer over NVLink per step instead of one fp32 logit gradient per
layer; it pays only when a layer's parameters or the full-batch optimizer state do not fit one GPU.

The reference has no distributed code; this module is new.
"""
import ctypes
from typing import Dict, List, Optional, Tuple

import torch
import torch.distributed as dist

from . import _lib as L
from .compactlogic import LogicLayer, GroupSum
from .functional import TIMER, _param_bytes, _placeholder, GradSlot


def rank_world(group=None) -> Tuple[int, int]:
    """(rank, world size) of `group`; (0, 1) without an initialised process group."""
    if not dist.is_initialized():
        return 0, 1
    return dist.get_rank(group), dist.get_world_size(group)


def shard_rows(n: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous [lo, hi) share of n neurons owned by `rank`."""
    return n * rank // world, n * (rank + 1) // world


class _CudaArray:
    """Minimal __cuda_array_interface__ view of raw device memory (bytes)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3}


class PeerBuffer:
    """A device buffer of `nbytes` on every rank, mapped into every rank's address space (CUDA IPC).

    ``ptrs[p]`` is rank p's buffer as seen from this process; ``view(shape, dtype)`` is this rank's
    own buffer as a tensor."""

    def __init__(self, nbytes: int, device: torch.device, group=None):
        self.group = group
        self.rank, self.world = rank_world(group)
        self.nbytes = max(int(nbytes), 256)
        self.device = device
        p = ctypes.c_void_p()
        with torch.cuda.device(device):
            L.call("clb_peer_alloc", self.nbytes, ctypes.byref(p))
            self.local = int(p.value)
            self._imported: List[int] = []
            self.ptrs: List[int] = [0] * self.world
            self.ptrs[self.rank] = self.local
            if self.world > 1:
                h = (ctypes.c_uint8 * 64)()
                L.call("clb_ipc_export", self.local, h)
                mine = torch.tensor(list(bytes(h)), dtype=torch.uint8, device=device)
                every = [torch.empty_like(mine) for _ in range(self.world)]
                dist.all_gather(every, mine, group=group)
                for r, t in enumerate(every):
                    if r == self.rank:
                        continue
                    hr = (ctypes.c_uint8 * 64)(*t.cpu().tolist())
                    q = ctypes.c_void_p()
                    L.call("clb_ipc_import", hr, ctypes.byref(q))
                    self.ptrs[r] = int(q.value)
                    self._imported.append(int(q.value))
        self._bytes = torch.as_tensor(_CudaArray(self.local, self.nbytes), device=device)

    def view(self, shape, dtype) -> torch.Tensor:
        n = 1
        for s in shape:
            n *= s
        esz = torch.empty((), dtype=dtype).element_size()
        return self._bytes[:n * esz].view(dtype).view(*shape)

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (collective: every rank calls it)."""
        if self.local is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        for q in self._imported:
            L.call("clb_ipc_close", q)
        if self.world > 1:
            dist.barrier(group=self.group)
        self._bytes = None
        L.call("clb_peer_free", self.local)
        self.local = None


class PeerGradSlot:
    """Hand-over between two width-sharded layers: the consumer leaves the PeerBuffer holding its
    partial grad_x (one per rank) here and returns a placeholder to autograd; the producer's backward
    sums the ranks' partials of its own rows inside its kernel."""
    __slots__ = ("gpart",)

    def __init__(self):
        self.gpart: Optional[PeerBuffer] = None


def _peer_array(ptrs: List[int], offset: int):
    return (ctypes.c_void_p * len(ptrs))(*[p + offset for p in ptrs])


class _WidthShardedFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, xt, weights, layer: "WidthShardedLogicLayer", in_slot, out_slot):
        spec = layer._layer_spec(xt.device)
        B = xt.shape[1]
        e = xt.element_size()
        buf = layer._buffer("y", layer.full_out_dim * B * e, xt.device)
        peers = _peer_array(buf.ptrs, layer.lo * B * e)
        nbytes = e * B * (spec.in_features + spec.n_out) + _param_bytes(spec)
        TIMER.launch("forward", nbytes, lambda: L.call(
            "clb_logic_forward_peers", L.dtype_code(xt.dtype), L.ptr(xt), xt.stride(0), B, spec.in_features,
            L.ptr(spec.slots), spec.n_out, spec.K, L.W_LOGITS, L.ptr(weights), L.ptr(spec.gates), int(spec.has_pad),
            peers, len(buf.ptrs), B, L.stream(xt.device)))
        layer._barrier(xt.device)
        ctx.save_for_backward(xt, weights)
        ctx.layer, ctx.in_slot, ctx.out_slot = layer, in_slot, out_slot
        return buf.view((layer.full_out_dim, B), xt.dtype)

    @staticmethod
    def backward(ctx, gy):
        xt, weights = ctx.saved_tensors
        layer = ctx.layer
        spec = layer._layer_spec(xt.device)
        B = xt.shape[1]
        dev = xt.device
        acc = L.acc_dtype(xt.dtype)
        a = torch.empty((), dtype=acc).element_size()
        slot = ctx.out_slot
        keep = None
        if slot is not None and slot.gpart is not None:
            # the following layer is sharded too: grad_y of the owned rows = sum of every rank's partial
            if not _placeholder(gy):
                raise NotImplementedError("a width-sharded layer's output feeds both a sharded layer and other ops")
            gpeers = _peer_array(slot.gpart.ptrs, layer.lo * B * a)
            n_peers = len(slot.gpart.ptrs)
            slot.gpart = None
        else:
            # replicated consumer (GroupSum, loss): every rank holds the same gradient; take the owned rows
            keep = gy[layer.lo:layer.hi].to(acc).contiguous()
            gpeers = _peer_array([keep.data_ptr()], 0)
            n_peers = 1
        need_gx, need_gw = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        gbuf = layer._buffer("gx", spec.in_features * B * a, dev) if need_gx else None
        gx_ptr = gbuf.local if gbuf is not None else 0
        chunks = int(L.lib().clb_logic_backward_chunks(L.dtype_code(xt.dtype), L.ptr(xt), xt.stride(0), B,
                                                       spec.in_features, gpeers[0], B, 0, 0, gx_ptr, B))
        part = torch.empty(max(chunks, 1), spec.n_out, spec.K, dtype=acc, device=dev) if need_gw else None
        nbytes = (xt.element_size() * B * spec.in_features + a * B * spec.n_out +
                  (a * B * spec.in_features if need_gx else 0) + _param_bytes(spec))
        TIMER.launch("backward", nbytes, lambda: L.call(
            "clb_logic_backward_peers", L.dtype_code(xt.dtype), L.ptr(xt), xt.stride(0), B, L.ptr(spec.slots),
            spec.n_out, spec.K, L.W_LOGITS, L.ptr(weights), L.ptr(spec.gates), int(spec.has_pad), gpeers, n_peers, B,
            gx_ptr, B, 1, spec.in_features, L.ptr(part), chunks if need_gw else 0, L.stream(dev)))
        gw = None
        if need_gw:
            gw = torch.empty(spec.n_out, spec.K, dtype=acc, device=dev)
            TIMER.launch("finalize", (max(chunks, 1) * spec.n_out + spec.n_out) * spec.K * a,
                         lambda: L.call("clb_logic_grad_finalize", L.dtype_code(xt.dtype), L.ptr(part),
                                        chunks if B > 0 else 0, spec.n_out, spec.K, 1, L.W_LOGITS, L.ptr(weights),
                                        L.ptr(gw), L.stream(dev)))
        del keep
        gx = None
        if need_gx:
            layer._barrier(dev)  # every rank's partial is complete before any rank reads it
            in_slot = ctx.in_slot
            if isinstance(in_slot, PeerGradSlot):
                in_slot.gpart = gbuf
                gx = torch.zeros((), dtype=xt.dtype, device=dev).expand(xt.shape)
            else:
                full = gbuf.view((spec.in_features, B), acc).clone()
                if rank_world(layer.group)[1] > 1:
                    dist.all_reduce(full, group=layer.group)
                if isinstance(in_slot, GradSlot):
                    in_slot.add(full)
                    gx = torch.zeros((), dtype=xt.dtype, device=dev).expand(xt.shape)
                else:
                    gx = full.to(xt.dtype)
        return gx, gw, None, None, None


class WidthShardedLogicLayer(LogicLayer):
    """This rank's share of a dense LogicLayer (same buffers and state_dict keys, holding rows
    [lo, hi) of ``weights``, ``indices``, ``gate_sequence`` and, once frozen, ``w``).  Input
    (batch, in_dim) replicated on every rank, output (batch, out_dim) — the full layer output, equal
    on every rank.  Build with ``shard_width``; collect with ``unshard_into``."""

    def __init__(self, layer: LogicLayer, group=None):
        torch.nn.Module.__init__(self)
        if type(layer) is not LogicLayer:
            raise TypeError("width sharding applies to dense LogicLayer modules")
        self.group = group
        rank, world = rank_world(group)
        self.lo, self.hi = shard_rows(layer.out_dim, rank, world)
        self.in_dim = layer.in_dim
        self.full_out_dim = layer.out_dim
        self.out_dim = self.hi - self.lo
        self.connections = layer.connections
        self.num_gates = layer.num_gates
        self.log_k = layer.log_k
        self.num_neurons = self.num_weights = self.out_dim
        self.is_frozen = layer.is_frozen
        self._spec_key = None
        self._spec = None
        self._fused_groupsum = None
        self.weights = torch.nn.Parameter(layer.weights.detach()[self.lo:self.hi].clone(),
                                          requires_grad=layer.weights.requires_grad)
        self.register_buffer("indices", layer.indices[:, self.lo:self.hi].clone())
        self.register_buffer("gate_sequence", layer.gate_sequence[self.lo:self.hi].clone())
        if hasattr(layer, "w") and isinstance(getattr(layer, "w"), torch.Tensor):
            self.register_buffer("w", layer.w[self.lo:self.hi].clone())
        self._bufs: Dict[tuple, PeerBuffer] = {}
        self._flag = None

    def extra_repr(self):
        return '{}, {} (rows {}:{}), {}'.format(self.in_dim, self.full_out_dim, self.lo, self.hi,
                                                'train' if self.training else 'eval')

    def refresh_backward_index(self, changed_rows=None):
        pass  # the native path needs no inverse index

    def _buffer(self, kind: str, nbytes: int, device) -> PeerBuffer:
        key = (kind, device)
        b = self._bufs.get(key)
        if b is None or b.nbytes < nbytes:
            if b is not None:
                b.close()
            b = self._bufs[key] = PeerBuffer(nbytes, device, self.group)
        return b

    def _barrier(self, device) -> None:
        if rank_world(self.group)[1] == 1:
            return
        if self._flag is None or self._flag.device != device:
            self._flag = torch.zeros(1, dtype=torch.int32, device=device)
        dist.all_reduce(self._flag, group=self.group)

    def release_buffers(self) -> None:
        """Free the peer-mapped activation / gradient buffers (collective)."""
        for b in self._bufs.values():
            b.close()
        self._bufs = {}

    def forward(self, x):
        if getattr(self, "is_frozen", False) or not self.training:
            with torch.no_grad():
                return self._forward_eval(x)
        in_slot = getattr(x, "_clb_peer_slot", None) or getattr(x, "_clb_slot", None)
        xt = self._to_feature_major(x)
        out_slot = PeerGradSlot()
        y = _WidthShardedFn.apply(xt, self._weights_for(xt.dtype), self, in_slot, out_slot).transpose(0, 1)
        y._clb_peer_slot = out_slot
        return y

    def _forward_eval(self, x):
        y_local = super().forward_cuda_eval(x).transpose(0, 1).contiguous()  # [n_loc, B]
        world = rank_world(self.group)[1]
        if world == 1:
            return y_local.transpose(0, 1)
        B = y_local.shape[1]
        cap = max(h - l for l, h in (shard_rows(self.full_out_dim, r, world) for r in range(world)))
        pad = torch.zeros(cap, B, dtype=y_local.dtype, device=y_local.device)
        pad[:self.out_dim] = y_local
        every = torch.empty(world * cap, B, dtype=y_local.dtype, device=y_local.device)
        dist.all_gather_into_tensor(every, pad, group=self.group)
        rows = [every[r * cap:r * cap + (h - l)] for r, (l, h) in
                enumerate(shard_rows(self.full_out_dim, r, world) for r in range(world))]
        return torch.cat(rows, 0).transpose(0, 1)


def shard_width(model: torch.nn.Module, group=None) -> torch.nn.Module:
    """Replace every dense LogicLayer of `model` by this rank's WidthShardedLogicLayer (in place).

    All ranks must call it on the same architecture; rank 0's parameters and buffers are broadcast
    first so that the shards come from one model.  A GroupSum fused into the last layer is unfused
    (it then runs replicated on the gathered output).  Returns the model."""
    from .parallel import broadcast_layer_buffers
    broadcast_layer_buffers(model, group=group)
    for name, mod in list(model.named_children()):
        if type(mod) is LogicLayer:
            mod._fused_groupsum = None
            setattr(model, name, WidthShardedLogicLayer(mod, group))
        elif isinstance(mod, GroupSum):
            mod.absorbed = False
        elif len(list(mod.children())):
            shard_width(mod, group)
    return model


def _gather_rows(t: torch.Tensor, n: int, dim: int, group) -> torch.Tensor:
    world = rank_world(group)[1]
    if world == 1:
        return t
    sizes = [h - l for l, h in (shard_rows(n, r, world) for r in range(world))]
    cap = max(sizes)
    tm = t.movedim(dim, 0)
    pad = torch.zeros((cap,) + tuple(tm.shape[1:]), dtype=t.dtype, device=t.device)
    pad[:tm.shape[0]] = tm
    every = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(every, pad.contiguous(), group=group)
    return torch.cat([e[:s] for e, s in zip(every, sizes)], 0).movedim(0, dim)


@torch.no_grad()
def unshard_into(sharded: torch.nn.Module, plain: torch.nn.Module, group=None) -> torch.nn.Module:
    """Gather every WidthShardedLogicLayer's rows into the matching LogicLayer of `plain` (same
    architecture), e.g. to save a checkpoint with the reference's layout.  Collective."""
    src = [m for m in sharded.modules() if isinstance(m, WidthShardedLogicLayer)]
    dst = [m for m in plain.modules() if type(m) is LogicLayer]
    if len(src) != len(dst):
        raise ValueError(f"{len(src)} sharded layers vs {len(dst)} LogicLayers")
    for s, d in zip(src, dst):
        n = s.full_out_dim
        d.weights.data.copy_(_gather_rows(s.weights.detach(), n, 0, group).to(d.weights.device))
        d.indices.copy_(_gather_rows(s.indices, n, 1, group).to(d.indices.device))
        d.gate_sequence.copy_(_gather_rows(s.gate_sequence, n, 0, group).to(d.gate_sequence.device))
        if hasattr(s, "w"):
            d.register_buffer("w", _gather_rows(s.w, n, 0, group).to(d.weights.device))
            d.is_frozen = s.is_frozen
        d.refresh_backward_index()
    return plain
