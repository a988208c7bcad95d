"""Autograd functions of the native fast path (softmax, gate mix, GroupSum and their backward fused
into the sm_100a kernels).

Activations live feature-major, ``[features, batch]`` contiguous, as in the reference dense kernels
(compactlogic/cuda/difflogic_kernel.cu:8-12); a layer's public output is the transposed view, so a
chain of layers never copies (compactlogic/compactlogic.py:101-118 uses the same convention).
"""
import os
from dataclasses import dataclass, field
from typing import Optional

import torch

from . import _lib as L

# Forward stage baked once per call (clb_logic_forward_staged) instead of once per column chunk;
# CLB_FWD_STAGE=0 selects the per-CTA stage build of clb_logic_forward.
_FWD_STAGE = os.environ.get("CLB_FWD_STAGE", "1") != "0"


@dataclass
class LayerSpec:
    """Device-side description of one logic layer (a slot table plus its per-row parameters)."""
    slots: torch.Tensor          # int32 [n_out, K, 2]
    gates: torch.Tensor          # uint8 [n_out/group, K]
    n_out: int
    K: int
    group: int
    in_features: int
    has_pad: bool
    # occurrence index of the gather-form backward (built on first use; the spec itself is rebuilt
    # whenever the connection or gate buffers change)
    index: Optional[torch.Tensor] = field(default=None, repr=False)
    # receptive-field-staged conv kernels (clb_conv_plane_*), when every output channel reads one input
    # channel; None for dense layers and for conv layers with mixed channels
    conv: Optional["ConvPlan"] = field(default=None, repr=False)


@dataclass
class ConvPlan:
    """Geometry and channel grouping of a conv layer for the receptive-field-staged kernels."""
    c_in: int
    h_in: int
    w_in: int
    c_out: int
    h_out: int
    w_out: int
    stride: int
    pad: int
    ks: int
    off_h: torch.Tensor   # int8 [2, c_out, K] (the layer's offsets_h buffer)
    off_w: torch.Tensor
    order: torch.Tensor   # int32 [c_out]: output channels grouped by input channel
    starts: torch.Tensor  # int32 [c_in + 1]
    max_group: int
    err: torch.Tensor     # int32 [1]: bit 1 set if a staging wait gave up


def _plane_ok(spec: "LayerSpec", xt: torch.Tensor, *others) -> bool:
    """Whether the staged conv kernels take this call: fp32, 16-byte rows, K in {4, 8, 16}."""
    if spec.conv is None or os.environ.get("CLB_CONV_PLANE", "1") == "0" or xt.dtype != torch.float32:
        return False
    B = xt.shape[1]
    for t in (xt,) + others:
        if t is None:
            continue
        if t.data_ptr() % 16 or (t.dim() == 2 and t.stride(0) % 4):
            return False
    return B % 4 == 0 and spec.K in (4, 8, 16)


def _gather_backward_enabled(spec: "LayerSpec", xt: torch.Tensor) -> bool:
    """Whether a layer that needs grad_x uses the gather-form backward (clb_logic_backward_gather: walked by
    destination, grad_x summed in a fixed order, so bitwise reproducible run to run) instead of the scatter
    form (clb_logic_backward, whose grad_x reductions land in a hardware-dependent order).

    CLB_BWD_GATHER=1 / 0 forces either form.  By default ("auto") the gather form runs for fp32 / bf16 / fp16
    dense layers with at least 16384 (input row x 128-column chunk) warps of work: measured on a B200 it is
    faster there (c2 step 9.33 vs 9.82 ms, c3 2.01 vs 2.17 ms, c5 bf16 20.4 vs 26.0 ms) and slower on small
    layers (c1: 0.143 vs 0.124 ms) and on fp64, which uses its unbaked kernel."""
    mode = os.environ.get("CLB_BWD_GATHER", "auto")
    if mode in ("0", "1"):
        return mode == "1"
    if spec.conv is not None or xt.dtype == torch.float64 or spec.group != 1:
        return False
    B = xt.shape[1]
    return B % 4 == 0 and spec.in_features * -(-B // 128) >= 16384 and spec.n_out * spec.K <= (1 << 24)


def layer_index(spec: LayerSpec, device) -> Optional[torch.Tensor]:
    """The spec's occurrence index (None when the layer is too large for it)."""
    if spec.index is None:
        nbytes = int(L.lib().clb_logic_index_bytes(spec.n_out, spec.K, spec.in_features))
        if nbytes < 0:
            return None
        idx = torch.empty(nbytes, dtype=torch.uint8, device=device)
        L.call("clb_logic_index_build", L.ptr(spec.slots), spec.n_out, spec.K, spec.group, L.ptr(spec.gates),
               spec.in_features, L.ptr(idx), nbytes, L.stream(device))
        spec.index = idx
    return spec.index


class KernelTimer:
    """Optional per-launch CUDA-event timing of the layer kernels (used by bench.py for the roofline).

    While enabled, every forward / backward kernel launch is bracketed by events on the launching
    stream and recorded with its algorithmic (compulsory) byte count:
      forward  = e*B*(in + out) + n_out*K*8 + rows*K*5        (y not written when GroupSum is fused)
      backward = e*B*in + a*B*out + a*B*in + n_out*K*8 + rows*K*5
                 (gy term dropped when synthesised from the fused GroupSum, gx term when not needed)
    with e the activation element size, a the gradient element size, slots int32 pairs, gate ids
    uint8 and logits fp32.  Each record also carries the launch's L2 gather / reduction bytes: one
    e-byte read per used operand and column (operands a gate ignores are never touched), plus, in the
    backward, one a-byte reduction per used operand and column when grad_x is produced."""

    def __init__(self):
        self.enabled = False
        self.records = []

    def reset(self):
        self.records = []

    def launch(self, kind, nbytes, fn, l2_bytes=0):
        if not self.enabled:
            return fn()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        out = fn()
        e.record()
        self.records.append((kind, s, e, nbytes, l2_bytes))
        return out

    def summary(self):
        """{kind: (launches, total_ms, total_bytes, total_l2_bytes)} (call after a synchronize)."""
        res = {}
        for kind, s, e, nb, l2 in self.records:
            n, ms, b, c = res.get(kind, (0, 0.0, 0, 0))
            res[kind] = (n + 1, ms + s.elapsed_time(e), b + nb, c + l2)
        return res


TIMER = KernelTimer()


_USED_A = [1 if (((g >> 1) & 1) != ((g >> 3) & 1)) or (((g >> 3) & 1) - ((g >> 2) & 1) - ((g >> 1) & 1) + (g & 1)) else 0
           for g in range(16)]
_USED_B = [1 if (((g >> 2) & 1) != ((g >> 3) & 1)) or (((g >> 3) & 1) - ((g >> 2) & 1) - ((g >> 1) & 1) + (g & 1)) else 0
           for g in range(16)]


def used_operands(spec: "LayerSpec") -> int:
    """Operands the layer's gates read, over all n_out * K slots (gates 0 / 15 read none, 3 / 5 / 10 / 12
    one), cached on the spec."""
    n = getattr(spec, "_used_ops", None)
    if n is None:
        tab = torch.tensor([a + b for a, b in zip(_USED_A, _USED_B)], dtype=torch.int64, device=spec.gates.device)
        n = int(tab[(spec.gates.to(torch.int64) & 15)].sum().item()) * spec.group
        spec._used_ops = n
    return n


def _bwd_l2(spec: "LayerSpec", xt: torch.Tensor, need_gx: bool) -> int:
    """L2 gather + reduction bytes of a backward launch (see KernelTimer)."""
    if not TIMER.enabled:
        return 0
    a = 8 if xt.dtype == torch.float64 else 4
    return used_operands(spec) * xt.shape[1] * (xt.element_size() + (a if need_gx else 0))


def _param_bytes(spec: "LayerSpec") -> int:
    return spec.n_out * spec.K * 8 + (spec.n_out // spec.group) * spec.K * 5


def _check_x(xt: torch.Tensor, spec: LayerSpec) -> None:
    L.require_cuda(xt)
    if xt.dim() != 2 or xt.shape[0] != spec.in_features or (xt.shape[1] > 1 and xt.stride(1) != 1):
        raise RuntimeError(f"expected feature-major activations [{spec.in_features}, batch] with unit column stride, "
                           f"got shape {tuple(xt.shape)} strides {xt.stride()}")


def forward_into(xt: torch.Tensor, weights: Optional[torch.Tensor], spec: LayerSpec, mode: int,
                 select: Optional[torch.Tensor] = None, y: Optional[torch.Tensor] = None,
                 gs_acc: Optional[torch.Tensor] = None, gs_size: int = 0) -> None:
    _check_x(xt, spec)
    B = xt.shape[1]
    e = xt.element_size()
    nbytes = e * B * (spec.in_features + (spec.n_out if y is not None else 0)) + _param_bytes(spec)
    l2 = used_operands(spec) * B * e if TIMER.enabled else 0
    if gs_acc is None and y is not None and _plane_ok(spec, xt, y):
        c = spec.conv
        TIMER.launch("conv_forward" if mode != L.W_SELECT else "conv_eval", nbytes, lambda: L.call(
            "clb_conv_plane_forward", L.CLB_F32, L.ptr(xt), xt.stride(0), B, c.c_in, c.h_in, c.w_in, c.c_out,
            c.h_out, c.w_out, c.stride, c.pad, c.ks, spec.K, L.ptr(c.off_h), L.ptr(c.off_w), L.ptr(c.order),
            L.ptr(c.starts), c.max_group, mode, L.ptr(weights), L.ptr(spec.gates), L.ptr(select), L.ptr(y),
            y.stride(0), L.ptr(c.err), L.stream(xt.device)), l2)
        return
    stage, stage_bytes = None, 0
    # with 4+ column chunks (32 x 16-byte columns each) bake the stage once instead of once per chunk
    # (measured: c2 forward 35.8 -> 34.4 ms over 78 launches; with 2 chunks, c1 and c5, the extra launch costs more)
    if _FWD_STAGE and B >= 4 * 32 * (16 // xt.element_size()):
        stage_bytes = L.lib().clb_logic_forward_stage_bytes(L.dtype_code(xt.dtype), spec.n_out, spec.K)
        stage = torch.empty(stage_bytes, dtype=torch.uint8, device=xt.device)
    TIMER.launch("forward" if mode != L.W_SELECT else "eval", nbytes, lambda: L.call(
        "clb_logic_forward_staged", L.dtype_code(xt.dtype), L.ptr(xt), xt.stride(0), B, spec.in_features,
        L.ptr(spec.slots), spec.n_out,
        spec.K, spec.group, mode, L.ptr(weights), L.ptr(spec.gates), L.ptr(select), int(spec.has_pad), L.ptr(y),
        y.stride(0) if y is not None else 0, L.ptr(gs_acc), gs_acc.shape[0] if gs_acc is not None else 0, gs_size,
        gs_acc.stride(0) if gs_acc is not None else 0, L.ptr(stage), stage_bytes, L.stream(xt.device)), l2)


def backward_into(xt: torch.Tensor, weights: torch.Tensor, spec: LayerSpec, mode: int,
                  gy: Optional[torch.Tensor], gs_grad: Optional[torch.Tensor], gs_size: int, gs_scale: float,
                  need_gx: bool, need_gw: bool):
    """Returns (grad_x [in, B] or None, grad_weights [rows, K] or None)."""
    if need_gx and mode in (L.W_LOGITS, L.W_PROBS) and _gather_backward_enabled(spec, xt):
        index = layer_index(spec, xt.device)
        if index is not None:
            return _backward_gather(xt, weights, spec, mode, gy, gs_grad, gs_size, gs_scale, need_gw, index)
    B = xt.shape[1]
    acc = L.acc_dtype(xt.dtype)
    dev = xt.device
    if gs_grad is None and mode in (L.W_LOGITS, L.W_PROBS) and _plane_ok(spec, xt, gy):
        return _backward_conv_plane(xt, weights, spec, mode, gy, need_gx, need_gw)
    gx = torch.empty(spec.in_features, B, dtype=acc, device=dev) if need_gx else None
    gy_ptr, ldgy = (L.ptr(gy), gy.stride(0)) if gy is not None else (0, 0)
    gs_ptr, ld_gs, gs_k = (L.ptr(gs_grad), gs_grad.stride(0), gs_grad.shape[0]) if gs_grad is not None else (0, 0, 0)
    part = None
    chunks = 0
    if need_gw:
        chunks = int(L.lib().clb_logic_backward_chunks(L.dtype_code(xt.dtype), L.ptr(xt), xt.stride(0), B,
                                                       spec.in_features, gy_ptr,
                                                       ldgy, gs_ptr, ld_gs, L.ptr(gx), B))
        part = torch.empty(max(chunks, 1), spec.n_out, spec.K, dtype=acc, device=dev)
    a = torch.empty((), dtype=acc).element_size()
    nbytes = (xt.element_size() * B * spec.in_features + (a * B * spec.n_out if gy is not None else 0) +
              (a * B * spec.in_features if need_gx else 0) + _param_bytes(spec))
    TIMER.launch("backward", nbytes, lambda: L.call(
        "clb_logic_backward", L.dtype_code(xt.dtype), L.ptr(xt), xt.stride(0), B, L.ptr(spec.slots), spec.n_out,
        spec.K, spec.group, mode, L.ptr(weights), L.ptr(spec.gates), int(spec.has_pad), gy_ptr, ldgy, gs_ptr, gs_k,
        gs_size, ld_gs, float(gs_scale), L.ptr(gx), B, 1, spec.in_features, L.ptr(part), chunks, L.stream(dev)),
        _bwd_l2(spec, xt, need_gx))
    gw = None
    if need_gw:
        gw = torch.empty(spec.n_out // spec.group, spec.K, dtype=acc, device=dev)
        TIMER.launch("finalize", (max(chunks, 1) * spec.n_out + spec.n_out // spec.group) * spec.K * a,
                     lambda: L.call("clb_logic_grad_finalize", L.dtype_code(xt.dtype), L.ptr(part),
                                    chunks if B > 0 else 0, spec.n_out, spec.K, spec.group, mode, L.ptr(weights),
                                    L.ptr(gw), L.stream(dev)))
    return gx, gw


def _backward_conv_plane(xt, weights, spec, mode, gy, need_gx, need_gw):
    """Conv layer backward on the receptive-field-staged kernel (clb_conv_plane_backward): grad_x
    (accumulated from shared-memory tiles) and per-(tile, column chunk) partials of d loss / d p,
    folded with the softmax backward by clb_logic_grad_finalize over the c_out parameter rows."""
    c = spec.conv
    B = xt.shape[1]
    dev = xt.device
    gx = torch.empty(spec.in_features, B, dtype=torch.float32, device=dev) if need_gx else None
    nparts = int(L.lib().clb_conv_plane_parts(c.h_out, c.w_out, c.stride, c.ks, B))
    part = torch.empty(max(nparts, 1), c.c_out, spec.K, dtype=torch.float32, device=dev)
    nbytes = 4 * B * (spec.in_features + spec.n_out + (spec.in_features if need_gx else 0)) + _param_bytes(spec)
    TIMER.launch("conv_backward", nbytes, lambda: L.call(
        "clb_conv_plane_backward", L.CLB_F32, L.ptr(xt), xt.stride(0), B, c.c_in, c.h_in, c.w_in, c.c_out, c.h_out,
        c.w_out, c.stride, c.pad, c.ks, spec.K, L.ptr(c.off_h), L.ptr(c.off_w), L.ptr(c.order), L.ptr(c.starts),
        c.max_group, mode, L.ptr(weights), L.ptr(spec.gates), L.ptr(gy), gy.stride(0), L.ptr(gx), B, 1, L.ptr(part),
        nparts, L.ptr(c.err), L.stream(dev)), _bwd_l2(spec, xt, need_gx))
    gw = None
    if need_gw:
        gw = torch.empty(c.c_out, spec.K, dtype=torch.float32, device=dev)
        TIMER.launch("finalize", (nparts + 1) * c.c_out * spec.K * 4, lambda: L.call(
            "clb_logic_grad_finalize", L.CLB_F32, L.ptr(part), nparts if B > 0 else 0, c.c_out, spec.K, 1, mode,
            L.ptr(weights), L.ptr(gw), L.stream(dev)))
    return gx, gw


def _backward_gather(xt, weights, spec, mode, gy, gs_grad, gs_size, gs_scale, need_gw, index):
    B = xt.shape[1]
    acc = L.acc_dtype(xt.dtype)
    dev = xt.device
    gx = torch.empty(spec.in_features, B, dtype=acc, device=dev)
    gy_ptr, ldgy = (L.ptr(gy), gy.stride(0)) if gy is not None else (0, 0)
    gs_ptr, ld_gs, gs_k = (L.ptr(gs_grad), gs_grad.stride(0), gs_grad.shape[0]) if gs_grad is not None else (0, 0, 0)
    chunks = int(L.lib().clb_logic_backward_gather_chunks(L.dtype_code(xt.dtype), L.ptr(xt), xt.stride(0), B, gy_ptr,
                                                          ldgy, gs_ptr, ld_gs, L.ptr(gx), B))
    part = torch.empty(max(chunks, 1), spec.n_out, spec.K, dtype=acc, device=dev) if need_gw else None
    probs = torch.empty(spec.n_out // spec.group, spec.K, dtype=acc, device=dev)
    a = torch.empty((), dtype=acc).element_size()
    nbytes = (xt.element_size() * B * spec.in_features + (a * B * spec.n_out if gy is not None else 0) +
              a * B * spec.in_features + _param_bytes(spec))
    # L2 bytes: per occurrence (used operand) one read of the other operand's row and one of grad_y's
    l2 = used_operands(spec) * B * (xt.element_size() + a) if TIMER.enabled else 0
    TIMER.launch("backward_gather", nbytes, lambda: L.call(
        "clb_logic_backward_gather", L.dtype_code(xt.dtype), L.ptr(xt), xt.stride(0), B, spec.in_features,
        spec.n_out, spec.K, spec.group, mode, L.ptr(weights), L.ptr(index), gy_ptr, ldgy, gs_ptr, gs_k, gs_size,
        ld_gs, float(gs_scale), L.ptr(gx), B, L.ptr(probs), L.ptr(part), chunks if need_gw else 0, L.stream(dev)), l2)
    gw = None
    if need_gw:
        gw = torch.empty(spec.n_out // spec.group, spec.K, dtype=acc, device=dev)
        TIMER.launch("finalize", (max(chunks, 1) * spec.n_out + spec.n_out // spec.group) * spec.K * a,
                     lambda: L.call("clb_logic_grad_finalize", L.dtype_code(xt.dtype), L.ptr(part),
                                    chunks if B > 0 else 0, spec.n_out, spec.K, spec.group, mode, L.ptr(weights),
                                    L.ptr(gw), L.stream(dev)))
    return gx, gw


class GradSlot:
    """fp32 gradient hand-over between two logic layers whose activations are low precision (bf16 / fp16).

    Autograd casts a gradient to the dtype of the tensor it belongs to, which would round every
    inter-layer gradient to bf16.  A producing layer attaches a slot to its output; a logic layer that
    consumes that output deposits its fp32 grad_x in the slot and hands autograd a zero-stride
    placeholder instead; the producer's backward adds the slot's fp32 gradient to whatever autograd
    delivers (other consumers' contributions, if any).  fp32 and fp64 activations do not use slots."""
    __slots__ = ("grad",)

    def __init__(self):
        self.grad = None

    def add(self, g):
        self.grad = g if self.grad is None else self.grad + g


def _placeholder(g: torch.Tensor) -> bool:
    return all(s == 0 for s in g.stride())


def _incoming_grad(gy: torch.Tensor, slot, acc_dtype) -> torch.Tensor:
    if slot is not None and slot.grad is not None:
        g, slot.grad = slot.grad, None
        return g if _placeholder(gy) else g + gy.to(acc_dtype)
    return gy.to(acc_dtype)


def _outgoing_grad(gx, xt: torch.Tensor, in_slot):
    if gx is not None and in_slot is not None:
        in_slot.add(gx)
        return torch.zeros((), dtype=xt.dtype, device=xt.device).expand(xt.shape)
    return gx


class LogicLayerFn(torch.autograd.Function):
    """y [n_out, B] = soft logic layer of xt [in, B] with gate logits `weights` [rows, K].

    Fuses the reference's ``softmax(weights)`` (compactlogic/compactlogic.py:108), the kernel
    forward (difflogic_kernel.cu:39-78) and, in backward, grad_x, grad_w and the softmax backward
    (compactlogic.py:488-508 + torch autograd).  in_slot / out_slot: see GradSlot."""

    @staticmethod
    def forward(ctx, xt, weights, spec: LayerSpec, in_slot=None, out_slot=None):
        y = torch.empty(spec.n_out, xt.shape[1], dtype=xt.dtype, device=xt.device)
        forward_into(xt, weights, spec, L.W_LOGITS, y=y)
        ctx.save_for_backward(xt, weights)
        ctx.spec, ctx.in_slot, ctx.out_slot = spec, in_slot, out_slot
        return y

    @staticmethod
    def backward(ctx, gy):
        xt, weights = ctx.saved_tensors
        spec = ctx.spec
        gy = _incoming_grad(gy, ctx.out_slot, L.acc_dtype(xt.dtype))
        if gy.stride(1) != 1 or gy.stride(0) < gy.shape[1]:
            gy = gy.contiguous()
        gx, gw = backward_into(xt, weights, spec, L.W_LOGITS, gy, None, 0, 1.0, ctx.needs_input_grad[0],
                               ctx.needs_input_grad[1])
        return _outgoing_grad(gx, xt, ctx.in_slot), gw, None, None, None


class LogicGroupSumFn(torch.autograd.Function):
    """Last logic layer with GroupSum fused (compactlogic/compactlogic.py:450-468): returns the raw
    class sums [k, B]; the layer output [n_out, B] is never materialised, and the backward
    synthesises grad_y[j, n] = grad[class(j), n] on the fly."""

    @staticmethod
    def forward(ctx, xt, weights, spec: LayerSpec, k: int, gs_size: int, in_slot=None):
        acc = torch.zeros(k, xt.shape[1], dtype=L.acc_dtype(xt.dtype), device=xt.device)
        forward_into(xt, weights, spec, L.W_LOGITS, gs_acc=acc, gs_size=gs_size)
        ctx.save_for_backward(xt, weights)
        ctx.spec, ctx.gs_size, ctx.in_slot = spec, gs_size, in_slot
        return acc

    @staticmethod
    def backward(ctx, gacc):
        xt, weights = ctx.saved_tensors
        gacc = gacc.contiguous().to(L.acc_dtype(xt.dtype))
        gx, gw = backward_into(xt, weights, ctx.spec, L.W_LOGITS, None, gacc, ctx.gs_size, 1.0,
                               ctx.needs_input_grad[0], ctx.needs_input_grad[1])
        return _outgoing_grad(gx, xt, ctx.in_slot), gw, None, None, None, None


def eval_forward(xt: torch.Tensor, spec: LayerSpec, select: torch.Tensor) -> torch.Tensor:
    """Discrete float eval (difflogic_kernel.cu:341-369): y [n_out, B]."""
    y = torch.empty(spec.n_out, xt.shape[1], dtype=xt.dtype, device=xt.device)
    forward_into(xt, None, spec, L.W_SELECT, select=select, y=y)
    return y


def eval_group_sum(xt: torch.Tensor, spec: LayerSpec, select: torch.Tensor, k: int, gs_size: int) -> torch.Tensor:
    acc = torch.zeros(k, xt.shape[1], dtype=L.acc_dtype(xt.dtype), device=xt.device)
    forward_into(xt, None, spec, L.W_SELECT, select=select, gs_acc=acc, gs_size=gs_size)
    return acc
