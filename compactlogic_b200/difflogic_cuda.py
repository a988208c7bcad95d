"""Drop-in for the reference extension module ``difflogic_cuda`` (compactlogic/cuda/difflogic.cpp:60-105).

Same function names, argument order, layouts, dtypes and results; each call goes through the C ABI
(clb_difflogic_*, clb_tensor_packbits, clb_groupbitsum).  Inputs must be contiguous CUDA tensors
(the reference's CHECK_INPUT, compactlogic/cuda/utils.cuh:10-14); outputs are allocated here, as in
the reference.  fp32, fp64 and fp16 activations are supported, as in the reference.
"""
import ctypes

import torch

from . import _lib as L

__all__ = ["forward", "backward_w", "backward_x", "eval", "tensor_packbits_cuda", "groupbitsum",
           "backward_x_atomicAdd"]


def _check(**tensors):
    for name, t in tensors.items():
        if not t.is_cuda:
            raise RuntimeError(f"{name} must be a CUDA tensor")
        if not t.is_contiguous():
            raise RuntimeError(f"{name} must be contiguous")


def _ws(in_dim, out_dim, K, batch, dtype, device):
    n = int(L.lib().clb_difflogic_workspace_bytes(in_dim, out_dim, K, batch, L.dtype_code(dtype)))
    return torch.empty(n, dtype=torch.uint8, device=device)


def forward(x, a, b, w, gate_seq):
    """y [out, batch] = sum_k w[j,k] f_{g[j,k]}(x[a[j,k]], x[b[j,k]])  (difflogic_kernel.cu:197-236)."""
    _check(x=x, a=a, b=b, w=w, gate_seq=gate_seq)
    out_dim, K = w.shape
    y = torch.empty(out_dim, x.shape[1], dtype=x.dtype, device=x.device)
    ws = _ws(x.shape[0], out_dim, K, x.shape[1], x.dtype, x.device)
    L.call("clb_difflogic_forward", L.dtype_code(x.dtype), L.ptr(x), x.shape[0], x.shape[1], L.ptr(a), L.ptr(b),
           L.ptr(w), L.ptr(gate_seq), out_dim, K, L.ptr(y), L.ptr(ws), ws.numel(), L.stream(x.device))
    return y


def backward_w(x, a, b, gate_seq, grad_y):
    """d loss / d w (probabilities) [out, K]  (difflogic_kernel.cu:239-282)."""
    _check(x=x, a=a, b=b, gate_seq=gate_seq, grad_y=grad_y)
    out_dim, K = a.shape
    gw = torch.empty(out_dim, K, dtype=x.dtype, device=x.device)
    ws = _ws(x.shape[0], out_dim, K, x.shape[1], x.dtype, x.device)
    L.call("clb_difflogic_backward_w", L.dtype_code(x.dtype), L.ptr(x), x.shape[0], x.shape[1], L.ptr(a), L.ptr(b),
           L.ptr(gate_seq), L.ptr(grad_y), out_dim, K, L.ptr(gw), L.ptr(ws), ws.numel(), L.stream(x.device))
    return gw


def backward_x(x, a, b, w, gate_seq, grad_y, given_x_indices_of_y_start, given_x_indices_of_y,
               given_x_types_of_gate):
    """grad_x [in, batch] by a gather over the inverse connection index (difflogic_kernel.cu:285-333)."""
    _check(x=x, a=a, b=b, w=w, gate_seq=gate_seq, grad_y=grad_y, given_x_indices_of_y_start=given_x_indices_of_y_start,
           given_x_indices_of_y=given_x_indices_of_y, given_x_types_of_gate=given_x_types_of_gate)
    out_dim, K = w.shape
    gx = torch.empty_like(x)
    ws = _ws(x.shape[0], out_dim, K, x.shape[1], x.dtype, x.device)
    L.call("clb_difflogic_backward_x", L.dtype_code(x.dtype), L.ptr(x), x.shape[0], x.shape[1], L.ptr(a), L.ptr(b),
           L.ptr(w), L.ptr(gate_seq), L.ptr(grad_y), L.ptr(given_x_indices_of_y_start), L.ptr(given_x_indices_of_y),
           L.ptr(given_x_types_of_gate), out_dim, K, L.ptr(gx), L.ptr(ws), ws.numel(), L.stream(x.device))
    return gx


def backward_x_atomicAdd(x, a, b, w, gate_seq, grad_y):
    """grad_x [in, batch] by scattering (difflogic_kernel.cu:613-656)."""
    _check(x=x, a=a, b=b, w=w, gate_seq=gate_seq, grad_y=grad_y)
    out_dim, K = w.shape
    gx = torch.empty_like(x)
    ws = _ws(x.shape[0], out_dim, K, x.shape[1], x.dtype, x.device)
    L.call("clb_difflogic_backward_x_atomic", L.dtype_code(x.dtype), L.ptr(x), x.shape[0], x.shape[1], L.ptr(a),
           L.ptr(b), L.ptr(w), L.ptr(gate_seq), L.ptr(grad_y), out_dim, K, L.ptr(gx), L.ptr(ws), ws.numel(),
           L.stream(x.device))
    return gx


def eval(x, a, b, w, gate_seq):  # noqa: A001 - the reference's name
    """Discrete eval: the real polynomial of the selected gate, w uint8 [out]  (difflogic_kernel.cu:371-411)."""
    _check(x=x, a=a, b=b, w=w, gate_seq=gate_seq)
    out_dim, K = a.shape
    y = torch.empty(out_dim, x.shape[1], dtype=x.dtype, device=x.device)
    ws = _ws(x.shape[0], out_dim, K, x.shape[1], x.dtype, x.device)
    L.call("clb_difflogic_eval", L.dtype_code(x.dtype), L.ptr(x), x.shape[0], x.shape[1], L.ptr(a), L.ptr(b),
           L.ptr(w), L.ptr(gate_seq), out_dim, K, L.ptr(y), L.ptr(ws), ws.numel(), L.stream(x.device))
    return y


_WORD = {8: torch.int8, 16: torch.int16, 32: torch.int32, 64: torch.int64}


def tensor_packbits_cuda(t, bit_count):
    """bool [rows, cols] -> (words [rows, ceil(cols/bit_count)], pad_len)  (difflogic_kernel.cu:453-494)."""
    _check(t=t)
    if bit_count not in _WORD:
        raise ValueError("`bit_count` has to be in { 8, 16, 32, 64 }")
    rows, cols = t.shape
    words = torch.empty(rows, -(-cols // bit_count), dtype=_WORD[bit_count], device=t.device)
    pad = ctypes.c_int64(0)
    L.call("clb_tensor_packbits", L.ptr(t), rows, cols, bit_count, L.ptr(words), ctypes.byref(pad),
           L.stream(t.device))
    return words, int(pad.value)


def groupbitsum(b, pad_len, k):
    """Per-class bit counts [batch, k] int32 (difflogic_kernel.cu:535-568); ValueError if rows % k."""
    _check(b=b)
    if b.shape[0] % k != 0:
        raise ValueError(f"in_dim ({b.shape[0]}) has to be divisible by k ({k}) but it is not")
    bits = 8 * b.element_size()
    counts = torch.empty(b.shape[1] * bits - pad_len, k, dtype=torch.int32, device=b.device)
    L.call("clb_groupbitsum", L.ptr(b), b.shape[0], b.shape[1], bits, pad_len, k, L.ptr(counts), L.stream(b.device))
    return counts
