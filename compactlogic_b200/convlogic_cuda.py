"""Drop-in for the reference extension module ``convlogic_cuda`` (compactlogic/cuda/convlogic.cpp:49-110).

NCHW tensors in and out, as in the reference; internally the activations are transposed to
feature-major storage in a workspace and run through the shared logic-layer kernels.
"""
import torch

from . import _lib as L
from .difflogic_cuda import _check

__all__ = ["forward", "backward_x", "backward_w", "eval"]


def _ws(x, c_out, h_out, w_out, K):
    n, c, h, w = x.shape
    nb = int(L.lib().clb_convlogic_workspace_bytes(n, c, h, w, c_out, h_out, w_out, K, L.dtype_code(x.dtype)))
    return torch.empty(nb, dtype=torch.uint8, device=x.device)


def _out_hw(x, pad, ks, stride):
    h_out = (x.shape[2] + 2 * pad - ks) // stride + 1
    w_out = (x.shape[3] + 2 * pad - ks) // stride + 1
    if h_out <= 0 or w_out <= 0:
        raise RuntimeError(f"Invalid output shape: h_out={h_out}, w_out={w_out}")
    return h_out, w_out


def forward(x, offsets_ch, offsets_h, offsets_w, w, gate_seq, stride, pad, ks):
    """convlogic_kernel.cu:140-188."""
    _check(x=x, offsets_ch=offsets_ch, offsets_h=offsets_h, offsets_w=offsets_w, w=w, gate_seq=gate_seq)
    c_out, K = w.shape
    h_out, w_out = _out_hw(x, pad, ks, stride)
    y = torch.empty(x.shape[0], c_out, h_out, w_out, dtype=x.dtype, device=x.device)
    ws = _ws(x, c_out, h_out, w_out, K)
    L.call("clb_convlogic_forward", L.dtype_code(x.dtype), L.ptr(x), *x.shape, L.ptr(offsets_ch), L.ptr(offsets_h),
           L.ptr(offsets_w), L.ptr(w), L.ptr(gate_seq), c_out, K, stride, pad, ks, L.ptr(y), L.ptr(ws), ws.numel(),
           L.stream(x.device))
    return y


def backward_x(x, offsets_ch, offsets_h, offsets_w, w, gate_seq, grad_y, stride, pad):
    """convlogic_kernel.cu:248-293."""
    _check(x=x, offsets_ch=offsets_ch, offsets_h=offsets_h, offsets_w=offsets_w, w=w, gate_seq=gate_seq,
           grad_y=grad_y)
    c_out, K = w.shape
    h_out, w_out = grad_y.shape[2], grad_y.shape[3]
    gx = torch.empty_like(x)
    ws = _ws(x, c_out, h_out, w_out, K)
    L.call("clb_convlogic_backward_x", L.dtype_code(x.dtype), L.ptr(x), *x.shape, L.ptr(offsets_ch), L.ptr(offsets_h),
           L.ptr(offsets_w), L.ptr(w), L.ptr(gate_seq), L.ptr(grad_y), c_out, h_out, w_out, K, stride, pad, L.ptr(gx),
           L.ptr(ws), ws.numel(), L.stream(x.device))
    return gx


def backward_w(x, offsets_ch, offsets_h, offsets_w, gate_seq, grad_y, stride):
    """convlogic_kernel.cu:385-430."""
    _check(x=x, offsets_ch=offsets_ch, offsets_h=offsets_h, offsets_w=offsets_w, gate_seq=gate_seq, grad_y=grad_y)
    c_out, K = gate_seq.shape
    h_out, w_out = grad_y.shape[2], grad_y.shape[3]
    gw = torch.empty(c_out, K, dtype=x.dtype, device=x.device)
    ws = _ws(x, c_out, h_out, w_out, K)
    L.call("clb_convlogic_backward_w", L.dtype_code(x.dtype), L.ptr(x), *x.shape, L.ptr(offsets_ch), L.ptr(offsets_h),
           L.ptr(offsets_w), L.ptr(gate_seq), L.ptr(grad_y), c_out, h_out, w_out, K, stride, L.ptr(gw), L.ptr(ws),
           ws.numel(), L.stream(x.device))
    return gw


def eval(x, offsets_ch, offsets_h, offsets_w, w, gate_seq, stride, pad, ks):  # noqa: A001
    """convlogic_kernel.cu:479-530: the selected gate per output channel, w uint8 [c_out]."""
    _check(x=x, offsets_ch=offsets_ch, offsets_h=offsets_h, offsets_w=offsets_w, w=w, gate_seq=gate_seq)
    c_out, K = gate_seq.shape
    h_out, w_out = _out_hw(x, pad, ks, stride)
    y = torch.empty(x.shape[0], c_out, h_out, w_out, dtype=x.dtype, device=x.device)
    ws = _ws(x, c_out, h_out, w_out, K)
    L.call("clb_convlogic_eval", L.dtype_code(x.dtype), L.ptr(x), *x.shape, L.ptr(offsets_ch), L.ptr(offsets_h),
           L.ptr(offsets_w), L.ptr(w), L.ptr(gate_seq), c_out, K, stride, pad, ks, L.ptr(y), L.ptr(ws), ws.numel(),
           L.stream(x.device))
    return y
