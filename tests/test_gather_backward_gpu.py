"""Gather-form fused backward (clb_logic_backward_gather) against the CPU oracle and the scatter-form
kernel (clb_logic_backward) on the same inputs."""
import numpy as np
import pytest
import torch

from compactlogic_b200 import _lib as L
from compactlogic_b200.functional import LayerSpec, LogicGroupSumFn, LogicLayerFn, layer_index
from oracle import oracle as O

from helpers import RTOL, assert_close, cuda, rand_dense

import test_conv_gpu

pytestmark = pytest.mark.gpu


def _spec(a, b, g, in_dim):
    out, K = a.shape
    idx = cuda(np.stack([a, b]).astype(np.int64))
    slots = torch.empty(out, K, 2, dtype=torch.int32, device="cuda")
    L.call("clb_slots_dense", L.ptr(idx[0]), L.ptr(idx[1]), out, K, in_dim, L.ptr(slots), 0, L.stream())
    return LayerSpec(slots, cuda(g), out, K, 1, in_dim, False)


def _grads(x, logits, spec, gy, dtype, gather, monkeypatch):
    monkeypatch.setenv("CLB_BWD_GATHER", "1" if gather else "0")
    xt = cuda(x, dtype).requires_grad_(True)
    w = cuda(logits, torch.float64 if dtype == torch.float64 else torch.float32).requires_grad_(True)
    y = LogicLayerFn.apply(xt, w, spec)
    y.backward(cuda(gy, L.acc_dtype(dtype)))
    return xt.grad, w.grad


SHAPES = [  # in, out, K, B
    (16, 24, 16, 1), (40, 30, 16, 3), (64, 64, 4, 64), (100, 80, 7, 130), (784, 512, 16, 256),
    (33, 20, 1, 8), (50, 64, 8, 96), (20, 12, 32, 40), (1000, 3, 2, 128),  # most rows read by nobody
    (128, 1024, 16, 256), (96, 600, 8, 384),  # >= 64 occurrences per row: the 8-lanes-per-occurrence walk (fp32)
]


@pytest.mark.parametrize("in_dim,out,K,B", SHAPES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_gather_vs_oracle_and_scatter(in_dim, out, K, B, dtype, monkeypatch):
    x, a, b, logits, g, gy = rand_dense(in_dim * 3 + K + B, in_dim, out, K, B)
    spec = _spec(a, b, g, in_dim)
    gx, gw = _grads(x, logits, spec, gy, dtype, True, monkeypatch)
    assert spec.index is not None, "gather path not taken"
    p = O.softmax(logits)
    assert_close(gx, O.dense_backward_x(x, a, b, p, g, gy), RTOL[dtype], "grad_x")
    assert_close(gw, O.softmax_backward(p, O.dense_backward_w(x, a, b, g, gy)), RTOL[dtype], "grad_logits")
    gx_s, gw_s = _grads(x, logits, spec, gy, dtype, False, monkeypatch)
    assert_close(gx, gx_s.double().cpu().numpy(), RTOL[dtype], "grad_x vs scatter")
    assert_close(gw, gw_s.double().cpu().numpy(), RTOL[dtype], "grad_logits vs scatter")


@pytest.mark.parametrize("gate_set", [(0, 15), (3, 5, 10, 12), (0, 3, 6, 15)])
def test_constant_and_one_operand_gates(gate_set, monkeypatch):
    """Slots with no occurrence (constant gates) and one-occurrence slots (gates A, B, not A, not B)."""
    x, a, b, logits, _, gy = rand_dense(11, 50, 70, 8, 64)
    g = np.random.default_rng(12).choice(np.array(gate_set, np.uint8), size=a.shape)
    b[:5] = a[:5]  # both operands of some slots read the same row
    spec = _spec(a, b, g, 50)
    gx, gw = _grads(x, logits, spec, gy, torch.float32, True, monkeypatch)
    p = O.softmax(logits)
    assert_close(gx, O.dense_backward_x(x, a, b, p, g, gy), 1e-5, "grad_x")
    assert_close(gw, O.softmax_backward(p, O.dense_backward_w(x, a, b, g, gy)), 1e-5, "grad_logits")


def test_gather_bf16(monkeypatch):
    x, a, b, logits, g, gy = rand_dense(5, 256, 300, 4, 512)
    spec = _spec(a, b, g, 256)
    xb = cuda(x, torch.bfloat16)
    xr = xb.double().cpu().numpy()
    gx, gw = _grads(xr, logits, spec, gy, torch.bfloat16, True, monkeypatch)
    p = O.softmax(logits)
    assert_close(gx, O.dense_backward_x(xr, a, b, p, g, gy), 1e-2, "grad_x bf16")
    assert_close(gw, O.softmax_backward(p, O.dense_backward_w(xr, a, b, g, gy)), 1e-2, "grad_logits bf16")


@pytest.mark.parametrize("in_dim,out,K,B,k", [(50, 40, 16, 64, 10), (30, 33, 4, 7, 4), (784, 1000, 16, 256, 10)])
def test_gather_groupsum_fused(in_dim, out, K, B, k, monkeypatch):
    monkeypatch.setenv("CLB_BWD_GATHER", "1")
    x, a, b, logits, g, _ = rand_dense(in_dim + out + 1, in_dim, out, K, B)
    spec = _spec(a, b, g, in_dim)
    xt = cuda(x, torch.float32).requires_grad_(True)
    w = cuda(logits, torch.float32).requires_grad_(True)
    acc = LogicGroupSumFn.apply(xt, w, spec, k, -(-out // k))
    gl = np.random.default_rng(0).standard_normal((B, k))
    (acc.t() / 2.0).backward(cuda(gl, torch.float32))
    assert spec.index is not None
    p = O.softmax(logits)
    gy = O.group_sum_backward(gl, out, k, 2.0).T
    assert_close(xt.grad, O.dense_backward_x(x, a, b, p, g, gy), 1e-5, "grad_x")
    assert_close(w.grad, O.softmax_backward(p, O.dense_backward_w(x, a, b, g, gy)), 1e-5, "grad_logits")


def test_gather_is_deterministic(monkeypatch):
    """grad_x is summed in the index's fixed order: identical bits on every call and every rebuild."""
    x, a, b, logits, g, gy = rand_dense(21, 2000, 4000, 16, 512)
    spec = _spec(a, b, g, 2000)
    gx1, gw1 = _grads(x, logits, spec, gy, torch.float32, True, monkeypatch)
    spec.index = None  # rebuild the index (its fill uses atomics; the sort fixes the order)
    gx2, gw2 = _grads(x, logits, spec, gy, torch.float32, True, monkeypatch)
    assert torch.equal(gx1, gx2) and torch.equal(gw1, gw2)


def test_index_covers_every_slot():
    """The index holds one record per used, unpadded operand, plus one per slot without any."""
    x, a, b, logits, g, gy = rand_dense(31, 97, 120, 16, 4)
    spec = _spec(a, b, g, 97)
    idx = layer_index(spec, torch.device("cuda"))
    starts = idx[: 4 * 98].view(torch.int32).cpu().numpy()
    t00, t01, t10, t11 = (g >> 3) & 1, (g >> 2) & 1, (g >> 1) & 1, g & 1
    c1, c2, c3 = t10.astype(int) - t00, t01.astype(int) - t00, t00.astype(int) - t01 - t10 + t11
    ua, ub = (c1 != 0) | (c3 != 0), (c2 != 0) | (c3 != 0)
    none = ~(ua | ub)
    assert starts[0] == 0 and starts[-1] == int(ua.sum() + ub.sum() + none.sum())
    counts = np.bincount(a[ua], minlength=97) + np.bincount(b[ub], minlength=97)
    jj = np.nonzero(none)[0]
    counts += np.bincount(jj % 97, minlength=97)
    np.testing.assert_array_equal(np.diff(starts), counts)


@pytest.mark.parametrize("gather", [True, False])
def test_conv_both_backward_forms(gather, monkeypatch):
    monkeypatch.setenv("CLB_BWD_GATHER", "1" if gather else "0")
    for case in test_conv_gpu.CASES:
        test_conv_gpu.test_conv_module_vs_oracle(case)


def test_index_rejects_oversize():
    assert L.lib().clb_logic_index_bytes(1 << 21, 16, 100) == -1
    assert L.lib().clb_logic_index_build(None, 1 << 21, 16, 1, None, 100, None, 0, None) == L.CLB_ERR_INVALID


@pytest.mark.parametrize("in_dim,out,K,B", [(784, 512, 16, 256), (300, 1000, 4, 128), (64, 64, 8, 36)])
def test_gather_bf16_vs_oracle_and_scatter(in_dim, out, K, B, monkeypatch):
    """bf16 activations (fp32 gradients) on the baked gather path, against the oracle on the bf16-rounded
    input and against the scatter form."""
    x, a, b, logits, g, gy = rand_dense(in_dim + 5 * K + B, in_dim, out, K, B)
    xr = torch.from_numpy(x).to(torch.bfloat16).double().numpy()
    gy = torch.from_numpy(gy).to(torch.bfloat16).double().numpy()  # autograd hands the bf16 output a bf16 gradient
    spec = _spec(a, b, g, in_dim)
    gx, gw = _grads(x, logits, spec, gy, torch.bfloat16, True, monkeypatch)
    assert spec.index is not None, "gather path not taken"
    p = O.softmax(logits)
    assert_close(gx, O.dense_backward_x(xr, a, b, p, g, gy), RTOL[torch.bfloat16], "grad_x")
    assert_close(gw, O.softmax_backward(p, O.dense_backward_w(xr, a, b, g, gy)), 1e-4, "grad_logits")
    gx_s, gw_s = _grads(x, logits, spec, gy, torch.bfloat16, False, monkeypatch)
    assert_close(gw, gw_s.double().cpu().numpy(), 1e-4, "grad_logits vs scatter")
