"""The allocation-free backward_w entry point, called through the C ABI.

Callers that cannot allocate device memory where they need the gate-probability gradient (no
allocator of their own to provide a workspace, or an allocator that forbids cudaMalloc there) use
clb_difflogic_backward_w_noalloc, which works in an 8 MiB scratch array compiled into the library.
It must give the same result as the workspace entry point clb_difflogic_backward_w, also when called
twice in a row (the scratch keeps the previous call's contents), and reject calls that do not fit.
This file is collected last so a failure here cannot hide any other test's result.
"""

import numpy as np
import pytest
import torch

from compactlogic_b200 import _lib as L
from oracle import oracle as O

from helpers import RTOL, assert_close, cuda, rand_dense

pytestmark = pytest.mark.gpu

def _with_workspace(x, a, b, g, gy, dtype):
    out, K = a.shape
    ws = torch.empty(int(L.lib().clb_difflogic_workspace_bytes(x.shape[0], out, K, x.shape[1], L.dtype_code(dtype))),
                     dtype=torch.uint8, device="cuda")
    gw = torch.empty(out, K, dtype=dtype, device="cuda")
    st = L.lib().clb_difflogic_backward_w(L.dtype_code(dtype), x.data_ptr(), x.shape[0], x.shape[1], a.data_ptr(),
                                          b.data_ptr(), g.data_ptr(), gy.data_ptr(), out, K, gw.data_ptr(),
                                          ws.data_ptr(), ws.numel(), L.stream())
    assert st == L.CLB_OK, L.lib().clb_last_error()
    return gw

def _no_alloc(x, a, b, g, gy, dtype):
    out, K = a.shape
    gw = torch.empty(out, K, dtype=dtype, device="cuda")
    st = L.lib().clb_difflogic_backward_w_noalloc(L.dtype_code(dtype), x.data_ptr(), x.shape[0], x.shape[1],
                                                  a.data_ptr(), b.data_ptr(), g.data_ptr(), gy.data_ptr(), out, K,
                                                  gw.data_ptr(), L.stream())
    assert st == L.CLB_OK, L.lib().clb_last_error()
    return gw

@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_no_alloc_matches_workspace_entry_twice(dtype):
    shapes = [(784, 1200, 16, 256), (300, 400, 4, 33)]  # the second call is smaller than the first
    for seed, (in_dim, out, K, B) in enumerate(shapes):
        x, a, b, _, g, gy = rand_dense(100 + seed, in_dim, out, K, B)
        xt, at, bt, gt, gyt = cuda(x, dtype), cuda(a), cuda(b), cuda(g), cuda(gy, dtype)
        ref = _with_workspace(xt, at, bt, gt, gyt, dtype)
        got = _no_alloc(xt, at, bt, gt, gyt, dtype)
        torch.cuda.synchronize()
        assert_close(got, ref.cpu().numpy(), RTOL[dtype], f"call {seed}")
        assert_close(got, O.dense_backward_w(x, a, b, g, gy), RTOL[dtype], f"call {seed} vs oracle")

def test_no_alloc_rejects_oversize():
    out, K, B = 200000, 16, 64  # slot table alone is 25.6 MB > 8 MiB
    x = torch.zeros(10, B, device="cuda")
    idx = torch.zeros(out, K, dtype=torch.int64, device="cuda")
    g = torch.zeros(out, K, dtype=torch.uint8, device="cuda")
    gy = torch.zeros(out, B, device="cuda")
    gw = torch.empty(out, K, device="cuda")
    st = L.lib().clb_difflogic_backward_w_noalloc(L.CLB_F32, x.data_ptr(), 10, B, idx.data_ptr(), idx.data_ptr(),
                                                  g.data_ptr(), gy.data_ptr(), out, K, gw.data_ptr(), L.stream())
    assert st == L.CLB_ERR_WORKSPACE
    assert b"8 MiB" in L.lib().clb_last_error()


def _chunks(x, gy):
    return int(L.lib().clb_logic_backward_chunks(L.CLB_F32, x.data_ptr(), x.shape[1], x.shape[1], x.shape[0],
                                                 gy.data_ptr(), gy.shape[1], None, 0, None, x.shape[1]))


def _r256(v):
    return (v + 255) // 256 * 256


@pytest.mark.parametrize("extra_chunk", [0, 1])
def test_no_alloc_limit_counts_partials(extra_chunk):
    """The slot table fits; the per-chunk partials decide.  A call sized to fill the 8 MiB exactly runs and
    matches the workspace entry point; one column chunk more is rejected."""
    in_dim, out, K = 64, 4096, 16
    slot_bytes = _r256(out * K * 8)
    probe = 4096
    cols_per_chunk = probe // _chunks(torch.zeros(in_dim, probe, device="cuda"), torch.zeros(out, probe, device="cuda"))
    fit = ((8 << 20) - slot_bytes) // (out * K * 4)
    B = (fit + extra_chunk) * cols_per_chunk
    x, a, b, _, g, gy = rand_dense(7, in_dim, out, K, B)
    xt, at, bt, gt, gyt = cuda(x), cuda(a), cuda(b), cuda(g), cuda(gy)
    assert slot_bytes + _r256(_chunks(xt, gyt) * out * K * 4) == (8 << 20) + extra_chunk * out * K * 4
    gw = torch.empty(out, K, device="cuda")
    st = L.lib().clb_difflogic_backward_w_noalloc(L.CLB_F32, xt.data_ptr(), in_dim, B, at.data_ptr(), bt.data_ptr(),
                                                  gt.data_ptr(), gyt.data_ptr(), out, K, gw.data_ptr(), L.stream())
    if extra_chunk:
        assert st == L.CLB_ERR_WORKSPACE
        return
    assert st == L.CLB_OK, L.lib().clb_last_error()
    ref = _with_workspace(xt, at, bt, gt, gyt, torch.float32)
    torch.cuda.synchronize()
    assert_close(gw, ref.cpu().numpy(), RTOL[torch.float32], "exactly 8 MiB of scratch")


def test_no_alloc_rejects_fp16():
    x = torch.zeros(8, 32, dtype=torch.float16, device="cuda")
    idx = torch.zeros(4, 2, dtype=torch.int64, device="cuda")
    g = torch.zeros(4, 2, dtype=torch.uint8, device="cuda")
    gy = torch.zeros(4, 32, dtype=torch.float16, device="cuda")
    gw = torch.empty(4, 2, dtype=torch.float16, device="cuda")
    st = L.lib().clb_difflogic_backward_w_noalloc(L.CLB_F16, x.data_ptr(), 8, 32, idx.data_ptr(), idx.data_ptr(),
                                                  g.data_ptr(), gy.data_ptr(), 4, 2, gw.data_ptr(), L.stream())
    assert st == L.CLB_ERR_DTYPE
