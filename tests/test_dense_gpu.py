"""Dense soft / eval logic layer on the GPU against the CPU oracle (and the reference API shims)."""
import numpy as np
import pytest
import torch

import compactlogic_b200 as cl
from compactlogic_b200 import _lib as L
from compactlogic_b200 import difflogic_cuda
from compactlogic_b200.functional import LayerSpec, LogicGroupSumFn, LogicLayerFn, eval_forward
from oracle import oracle as O

from helpers import RTOL, assert_close, cuda, rand_dense

pytestmark = pytest.mark.gpu


def _spec(a, b, g, in_dim):
    out, K = a.shape
    idx = cuda(np.stack([a, b]).astype(np.int64))
    slots = torch.empty(out, K, 2, dtype=torch.int32, device="cuda")
    L.call("clb_slots_dense", L.ptr(idx[0]), L.ptr(idx[1]), out, K, in_dim, L.ptr(slots), 0, L.stream())
    return LayerSpec(slots, cuda(g), out, K, 1, in_dim, False)


SHAPES = [(16, 24, 16, 1), (40, 30, 16, 3), (64, 64, 4, 64), (100, 80, 7, 130), (784, 512, 16, 256),
          (33, 20, 1, 8), (50, 64, 8, 96), (20, 12, 32, 40)]


@pytest.mark.parametrize("in_dim,out,K,B", SHAPES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_forward_backward_vs_oracle(in_dim, out, K, B, dtype):
    x, a, b, logits, g, gy = rand_dense(in_dim * 7 + K, in_dim, out, K, B)
    spec = _spec(a, b, g, in_dim)
    xt = cuda(x, dtype).requires_grad_(True)
    w = cuda(logits, dtype).requires_grad_(True)
    y = LogicLayerFn.apply(xt, w, spec)
    p = O.softmax(logits)
    assert_close(y, O.dense_forward(x, a, b, p, g), RTOL[dtype], "y")
    y.backward(cuda(gy, dtype))
    assert_close(xt.grad, O.dense_backward_x(x, a, b, p, g, gy), RTOL[dtype], "grad_x")
    assert_close(w.grad, O.softmax_backward(p, O.dense_backward_w(x, a, b, g, gy)), RTOL[dtype], "grad_logits")


@pytest.mark.parametrize("in_dim,out,K,B,k", [(50, 40, 16, 64, 10), (30, 33, 4, 7, 4), (784, 1000, 16, 256, 10)])
def test_groupsum_fused_vs_oracle(in_dim, out, K, B, k):
    x, a, b, logits, g, _ = rand_dense(in_dim + out, in_dim, out, K, B)
    spec = _spec(a, b, g, in_dim)
    xt = cuda(x, torch.float32).requires_grad_(True)
    w = cuda(logits, torch.float32).requires_grad_(True)
    size = -(-out // k)
    acc = LogicGroupSumFn.apply(xt, w, spec, k, size)
    p = O.softmax(logits)
    y = O.dense_forward(x, a, b, p, g)
    assert_close(acc.t() / 2.0, O.group_sum(y.T, k, 2.0), 1e-5, "logits")
    gl = np.random.default_rng(0).standard_normal((B, k))
    (acc.t() / 2.0).backward(cuda(gl, torch.float32))
    gy = O.group_sum_backward(gl, out, k, 2.0).T
    assert_close(xt.grad, O.dense_backward_x(x, a, b, p, g, gy), 1e-5, "grad_x")
    assert_close(w.grad, O.softmax_backward(p, O.dense_backward_w(x, a, b, g, gy)), 1e-5, "grad_logits")


@pytest.mark.parametrize("B", [1, 5, 64, 200])
def test_eval_select_bitexact(B):
    x, a, b, logits, g, _ = rand_dense(B, 60, 70, 16, B, binary_input=True)
    spec = _spec(a, b, g, 60)
    sel = O.argmax_first(logits)
    y = eval_forward(cuda(x, torch.float32), spec, cuda(sel))
    np.testing.assert_array_equal(y.cpu().numpy(), O.dense_eval(x, a, b, sel, g))


def test_bf16_activations():
    x, a, b, logits, g, gy = rand_dense(5, 256, 300, 4, 512)
    spec = _spec(a, b, g, 256)
    xb = cuda(x, torch.bfloat16)
    xr = xb.double().cpu().numpy()  # the oracle sees the bf16-rounded inputs
    xt = xb.clone().requires_grad_(True)
    w = cuda(logits, torch.float32).requires_grad_(True)
    y = LogicLayerFn.apply(xt, w, spec)
    p = O.softmax(logits)
    assert_close(y, O.dense_forward(xr, a, b, p, g), 1e-2, "y bf16")
    y.backward(cuda(gy, torch.bfloat16))
    gyr = cuda(gy, torch.bfloat16).double().cpu().numpy()
    assert_close(w.grad, O.softmax_backward(p, O.dense_backward_w(xr, a, b, g, gyr)), 1e-2, "grad_logits bf16")


def test_gradcheck_float64():
    x, a, b, logits, g, _ = rand_dense(9, 7, 6, 3, 4)
    spec = _spec(a, b, g, 7)
    xt = cuda(x, torch.float64).requires_grad_(True)
    w = cuda(logits, torch.float64).requires_grad_(True)
    assert torch.autograd.gradcheck(lambda xx, ww: LogicLayerFn.apply(xx, ww, spec), (xt, w), eps=1e-6, atol=1e-8)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_reference_api_shims(dtype):
    in_dim, out, K, B = 70, 90, 16, 48
    x, a, b, logits, g, gy = rand_dense(3, in_dim, out, K, B)
    p = O.softmax(logits)
    xt, at, bt, pt, gt, gyt = cuda(x, dtype), cuda(a), cuda(b), cuda(p, dtype), cuda(g), cuda(gy, dtype)
    assert_close(difflogic_cuda.forward(xt, at, bt, pt, gt), O.dense_forward(x, a, b, p, g), RTOL[dtype], "forward")
    assert_close(difflogic_cuda.backward_w(xt, at, bt, gt, gyt), O.dense_backward_w(x, a, b, g, gy), RTOL[dtype],
                 "backward_w")
    starts, ys, codes = O.inverse_index(a, b, in_dim)
    gx_ref = O.dense_backward_x(x, a, b, p, g, gy)
    gx = difflogic_cuda.backward_x(xt, at, bt, pt, gt, gyt, cuda(starts), cuda(ys), cuda(codes))
    assert_close(gx, gx_ref, RTOL[dtype], "backward_x")
    assert_close(difflogic_cuda.backward_x_atomicAdd(xt, at, bt, pt, gt, gyt), gx_ref, RTOL[dtype], "backward_x_atomic")
    sel = O.argmax_first(logits)
    xb = (x > 0.5).astype(np.float64)
    np.testing.assert_array_equal(difflogic_cuda.eval(cuda(xb, dtype), at, bt, cuda(sel), gt).cpu().numpy(),
                                  O.dense_eval(xb, a, b, sel, g))


def test_shim_input_checks():
    x = torch.rand(4, 3)
    with pytest.raises(RuntimeError, match="CUDA"):
        difflogic_cuda.forward(x, x, x, x, x)
    xt = torch.rand(3, 4, device="cuda").t()
    with pytest.raises(RuntimeError, match="contiguous"):
        difflogic_cuda.forward(xt, xt, xt, xt, xt)


def test_layer_module_matches_reference_math():
    """LogicLayer module (train mode, then eval) on the GPU vs the oracle restatement of the reference
    LogicLayer.forward_cuda / forward_cuda_eval (compactlogic.py:74-130)."""
    torch.manual_seed(0)
    layer = cl.LogicLayer(96, 120, num_gates=16)
    idx = layer.indices.numpy()
    g = layer.gate_sequence.numpy()
    logits = layer.weights.detach().numpy().astype(np.float64)
    layer = layer.cuda()
    x = (np.random.default_rng(1).random((40, 96)) < 0.5).astype(np.float32)
    xt = cuda(x).requires_grad_(True)
    y = layer(xt)
    p = O.softmax(logits)
    y_ref = O.dense_forward(x.T, idx[0], idx[1], p, g).T
    assert_close(y, y_ref, 1e-5, "module y")
    gy = np.random.default_rng(2).standard_normal(y_ref.shape)
    y.backward(cuda(gy, torch.float32))
    assert_close(layer.weights.grad, O.softmax_backward(p, O.dense_backward_w(x.T, idx[0], idx[1], g, gy.T)), 1e-5,
                 "module grad")
    assert_close(xt.grad, O.dense_backward_x(x.T, idx[0], idx[1], p, g, gy.T).T, 1e-5, "module grad_x")
    layer.eval()
    ye = layer(cuda(x))
    np.testing.assert_array_equal(ye.cpu().numpy(), O.dense_eval(x.T, idx[0], idx[1], O.argmax_first(logits), g).T)
    # indices changed in place -> slot table rebuilt
    with torch.no_grad():
        layer.indices[0, :, :] = 0
    ye2 = layer(cuda(x))
    idx2 = layer.indices.cpu().numpy()
    np.testing.assert_array_equal(ye2.cpu().numpy(),
                                  O.dense_eval(x.T, idx2[0], idx2[1], O.argmax_first(logits), g).T)


def test_frozen_layer_runs_eval_in_train_mode():
    torch.manual_seed(4)
    layer = cl.LogicLayer(30, 40, num_gates=8).cuda()
    layer.freeze()
    layer.train()
    x = (torch.rand(10, 30, device="cuda") < 0.5).float()
    idx = layer.indices.cpu().numpy()
    ref = O.dense_eval(x.cpu().numpy().T, idx[0], idx[1], layer.w.cpu().numpy(), layer.gate_sequence.cpu().numpy()).T
    np.testing.assert_array_equal(layer(x).cpu().numpy(), ref)


def _bf16(a):
    return torch.from_numpy(np.asarray(a, np.float32)).bfloat16().double().numpy()


def test_bf16_chain_keeps_fp32_gradients():
    """bf16 activations, fp32 logits and gradients (BASELINE config c5 regime): a 3-layer chain with
    fused GroupSum against the oracle run on the bf16-rounded activations, 1e-2 relative."""
    torch.manual_seed(3)
    layers = [cl.LogicLayer(96, 256, num_gates=4), cl.LogicLayer(256, 256, num_gates=4), cl.LogicLayer(256, 200, num_gates=4)]
    model = cl.fuse_groupsum(torch.nn.Sequential(*layers, cl.GroupSum(10, 3.0))).cuda()
    x = (torch.rand(64, 96) < 0.5).float()
    labels = torch.randint(0, 10, (64,))
    logits = model(x.cuda().bfloat16())
    torch.nn.functional.cross_entropy(logits, labels.cuda()).backward()
    tabs = [(m.indices.cpu().numpy(), m.gate_sequence.cpu().numpy(), O.softmax(m.weights.detach().cpu().numpy()))
            for m in layers]
    h = [x.numpy().T.astype(np.float64)]
    for li, (idx, g, p) in enumerate(tabs):
        y = O.dense_forward(h[-1], idx[0], idx[1], p, g)
        h.append(_bf16(y) if li < len(tabs) - 1 else y)
    ref_logits = O.group_sum(h[-1].T, 10, 3.0)
    assert_close(logits, ref_logits, 1e-2, "bf16 logits")
    gy = O.group_sum_backward(O.cross_entropy_grad(ref_logits, labels.numpy()), 200, 10, 3.0).T
    for li in range(len(tabs) - 1, -1, -1):
        idx, g, p = tabs[li]
        gw = O.softmax_backward(p, O.dense_backward_w(h[li], idx[0], idx[1], g, gy))
        assert_close(layers[li].weights.grad, gw, 1e-2, f"bf16 grad layer {li}")
        gy = O.dense_backward_x(h[li], idx[0], idx[1], p, g, gy)


def _narrow_case(dtype_name, in_dim, out, K, B):
    dtype = getattr(torch, dtype_name)
    x, a, b, logits, g, gy = rand_dense(11, in_dim, out, K, B)
    spec = _spec(a, b, g, in_dim)
    xt = cuda(x, dtype)
    wide_chunks = B // (32 * (16 // xt.element_size()))
    n = L.lib().clb_logic_backward_chunks(L.dtype_code(dtype), xt.data_ptr(), B, B, in_dim, 1, B, None, 0, 1, B)
    assert n > wide_chunks  # the narrow geometry is in use
    xt.requires_grad_(True)
    w = cuda(logits, torch.float32).requires_grad_(True)
    y = LogicLayerFn.apply(xt, w, spec)
    xr = xt.detach().double().cpu().numpy()
    p = O.softmax(logits)
    tol = RTOL[dtype]
    assert_close(y, O.dense_forward(xr, a, b, p, g), tol, "narrow y")
    y.backward(cuda(gy, dtype))
    gyr = cuda(gy, dtype).double().cpu().numpy()
    assert_close(w.grad, O.softmax_backward(p, O.dense_backward_w(xr, a, b, g, gyr)), tol, "narrow grad_logits")
    if dtype == torch.float32:
        assert_close(xt.grad, O.dense_backward_x(xr, a, b, p, g, gyr), tol, "narrow grad_x")


@pytest.mark.parametrize("dtype,in_dim,out,K,B,lpn", [("float32", 30000, 20000, 4, 256, 2),
                                                     ("float32", 30000, 20000, 16, 200, 8),
                                                     ("bfloat16", 60000, 30000, 4, 128, 4)])
def test_narrow_chunks_opt_in(dtype, in_dim, out, K, B, lpn):
    """The opt-in narrow-chunk kernels (several neurons per warp; CLB_FWD_LPN / CLB_BWD_LPN, read once per
    process, hence a child process) give the same results."""
    import os
    import subprocess
    import sys
    env = dict(os.environ, CLB_FWD_LPN=str(lpn), CLB_BWD_LPN=str(lpn))
    code = ("import sys; sys.path[:0] = ['tests', '.']; import test_dense_gpu as t; "
            f"t._narrow_case({dtype!r}, {in_dim}, {out}, {K}, {B})")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", code], cwd=root, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]


def test_reference_autograd_bridges():
    """LogicLayerCudaFunction / ConvLayerCudaFunction (the reference bridges, compactlogic.py:474-508,
    838-867) driven exactly as the reference's forward_cuda drives them give the native layers' results."""
    torch.manual_seed(6)
    layer = cl.LogicLayer(50, 60, num_gates=16).cuda()
    x = torch.rand(12, 50, device="cuda")
    xr = x.clone().requires_grad_(True)
    w = torch.nn.functional.softmax(layer.weights, dim=-1)
    y_ref = cl.LogicLayerCudaFunction.apply(xr.t().contiguous(), layer.indices[0], layer.indices[1], w,
                                            layer.gate_sequence, layer.given_x_indices_of_y_start,
                                            layer.given_x_indices_of_y, layer.given_x_indices_of_gate).t()
    gy = torch.randn_like(y_ref)
    y_ref.backward(gy)
    g_ref, gx_ref = layer.weights.grad.clone(), xr.grad.clone()
    layer.weights.grad = None
    xn = x.clone().requires_grad_(True)
    y = layer(xn)
    y.backward(gy)
    torch.testing.assert_close(y, y_ref, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(layer.weights.grad, g_ref, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(xn.grad, gx_ref, rtol=1e-5, atol=1e-6)

    conv = cl.ConvLayer((4, 6, 6), 1, 8, 3, 2, num_gates=8).cuda()
    xc = torch.rand(3, 4, 6, 6, device="cuda", requires_grad=True)
    wc = torch.nn.functional.softmax(conv.weights, dim=-1)
    yc_ref = cl.ConvLayerCudaFunction.apply(xc, conv.offsets_ch, conv.offsets_h, conv.offsets_w, wc,
                                            conv.gate_sequence, conv.stride, conv.padding, conv.ks)
    gyc = torch.randn_like(yc_ref)
    yc_ref.backward(gyc)
    gc_ref, gxc_ref = conv.weights.grad.clone(), xc.grad.clone()
    conv.weights.grad, xc.grad = None, None
    yc = conv(xc)
    yc.backward(gyc)
    torch.testing.assert_close(yc, yc_ref, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(conv.weights.grad, gc_ref, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(xc.grad, gxc_ref, rtol=1e-5, atol=1e-6)


def test_fp16_reference_api_and_layers():
    """fp16 activations (the reference dense kernels dispatch half, difflogic_kernel.cu:222): the
    reference-API shims and the native layers, against the oracle on fp16-rounded inputs (2e-3)."""
    in_dim, out, K, B = 64, 80, 16, 48
    x, a, b, logits, g, gy = rand_dense(21, in_dim, out, K, B)
    h = lambda v: cuda(v, torch.float16)
    r = lambda t: t.double().cpu().numpy()
    xh, ph, gyh = h(x), h(O.softmax(logits)), h(gy)
    xr, pr, gyr = r(xh), r(ph), r(gyh)
    at, bt, gt = cuda(a), cuda(b), cuda(g)
    y = difflogic_cuda.forward(xh, at, bt, ph, gt)
    assert y.dtype == torch.float16
    assert_close(y, O.dense_forward(xr, a, b, pr, g), 2e-3, "fp16 forward")
    assert_close(difflogic_cuda.backward_w(xh, at, bt, gt, gyh), O.dense_backward_w(xr, a, b, g, gyr), 2e-3, "fp16 gw")
    starts, ys, codes = O.inverse_index(a, b, in_dim)
    gx_ref = O.dense_backward_x(xr, a, b, pr, g, gyr)
    assert_close(difflogic_cuda.backward_x(xh, at, bt, ph, gt, gyh, cuda(starts), cuda(ys), cuda(codes)), gx_ref, 2e-3,
                 "fp16 gx csr")
    assert_close(difflogic_cuda.backward_x_atomicAdd(xh, at, bt, ph, gt, gyh), gx_ref, 2e-3, "fp16 gx atomic")
    sel = O.argmax_first(logits)
    xb = (x > 0.5).astype(np.float64)
    np.testing.assert_array_equal(difflogic_cuda.eval(h(xb), at, bt, cuda(sel), gt).cpu().numpy(),
                                  O.dense_eval(xb, a, b, sel, g))
    # native layers with fp16 activations keep fp32 gradients between layers
    torch.manual_seed(2)
    layers = [cl.LogicLayer(64, 128, num_gates=8), cl.LogicLayer(128, 100, num_gates=8)]
    model = cl.fuse_groupsum(torch.nn.Sequential(*layers, cl.GroupSum(5, 2.0))).cuda()
    xin = (torch.rand(32, 64) < 0.5).float()
    out = model(xin.cuda().half())
    out.sum().backward()
    tabs = [(m.indices.cpu().numpy(), m.gate_sequence.cpu().numpy(), O.softmax(m.weights.detach().cpu().numpy()))
            for m in layers]
    h1 = r(cuda(O.dense_forward(xin.numpy().T.astype(np.float64), tabs[0][0][0], tabs[0][0][1], tabs[0][2],
                                tabs[0][1]), torch.float16))
    lg = O.group_sum(O.dense_forward(h1, tabs[1][0][0], tabs[1][0][1], tabs[1][2], tabs[1][1]).T, 5, 2.0)
    assert_close(out, lg, 2e-3, "fp16 model")
    gy2 = O.group_sum_backward(np.ones_like(lg), 100, 5, 2.0).T
    assert_close(layers[1].weights.grad, O.softmax_backward(tabs[1][2], O.dense_backward_w(h1, tabs[1][0][0], tabs[1][0][1],
                                                                                           tabs[1][1], gy2)), 2e-3, "fp16 g2")


@pytest.mark.parametrize("K", [128, 33])
def test_many_candidate_gates(K):
    """K beyond the specialised 4/8/16 paths (the reference's LogicLayer docstring default is 128)."""
    x, a, b, logits, g, gy = rand_dense(K, 90, 70, K, 40)
    spec = _spec(a, b, g, 90)
    xt = cuda(x, torch.float32).requires_grad_(True)
    w = cuda(logits, torch.float32).requires_grad_(True)
    y = LogicLayerFn.apply(xt, w, spec)
    p = O.softmax(logits)
    assert_close(y, O.dense_forward(x, a, b, p, g), 1e-5, "y")
    y.backward(cuda(gy, torch.float32))
    assert_close(xt.grad, O.dense_backward_x(x, a, b, p, g, gy), 1e-5, "gx")
    assert_close(w.grad, O.softmax_backward(p, O.dense_backward_w(x, a, b, g, gy)), 1e-5, "gw")


def test_empty_batch():
    torch.manual_seed(0)
    model = cl.fuse_groupsum(torch.nn.Sequential(cl.LogicLayer(20, 30, num_gates=4), cl.LogicLayer(30, 24, num_gates=4),
                                                 cl.GroupSum(4, 1.0))).cuda()
    x = torch.zeros(0, 20, device="cuda", requires_grad=True)
    out = model(x)
    assert out.shape == (0, 4)
    out.sum().backward()
    assert torch.count_nonzero(model[0].weights.grad) == 0
    model.eval()
    assert model(torch.zeros(0, 20, device="cuda")).shape == (0, 4)
    assert cl.PackedLogicNet(model)(torch.zeros(0, 20, device="cuda")).shape == (0, 4)


def _fwd_call(name, xt, w, spec, mode, sel, y, gs=None, gs_size=0, stage=None):
    args = [L.dtype_code(xt.dtype), L.ptr(xt), xt.stride(0), xt.shape[1], spec.in_features, L.ptr(spec.slots),
            spec.n_out, spec.K, spec.group, mode, L.ptr(w), L.ptr(spec.gates), L.ptr(sel), 0,
            L.ptr(y), y.stride(0) if y is not None else 0, L.ptr(gs), gs.shape[0] if gs is not None else 0, gs_size,
            gs.stride(0) if gs is not None else 0]
    if name == "clb_logic_forward_staged":
        args += [L.ptr(stage), stage.numel() if stage is not None else 0]
    return getattr(L.lib(), name)(*args, L.stream())


@pytest.mark.parametrize("in_dim,out,K,B", [(784, 1000, 16, 512), (300, 517, 7, 640), (64, 96, 4, 1024)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float64])
def test_staged_forward_matches_per_chunk_stage(in_dim, out, K, B, dtype):
    """clb_logic_forward_staged (stage baked once per call) gives bitwise the forward of clb_logic_forward,
    in soft mode, select mode and with the fused GroupSum; a short stage buffer is rejected."""
    x, a, b, logits, g, _ = rand_dense(in_dim + 3 * K, in_dim, out, K, B)
    spec = _spec(a, b, g, in_dim)
    xt = cuda(x, dtype)
    w = cuda(logits, L.acc_dtype(dtype))
    sel = cuda(O.argmax_first(logits))
    nbytes = L.lib().clb_logic_forward_stage_bytes(L.dtype_code(dtype), out, K)
    stage = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    for mode in (L.W_LOGITS, L.W_SELECT):
        y0 = torch.empty(out, B, dtype=dtype, device="cuda")
        y1 = torch.full_like(y0, float("nan"))
        assert _fwd_call("clb_logic_forward", xt, w, spec, mode, sel, y0) == L.CLB_OK
        assert _fwd_call("clb_logic_forward_staged", xt, w, spec, mode, sel, y1, stage=stage) == L.CLB_OK
        torch.cuda.synchronize()
        assert torch.equal(y0, y1), mode
    k = 10
    acc0 = torch.zeros(k, B, dtype=L.acc_dtype(dtype), device="cuda")
    acc1 = torch.zeros_like(acc0)
    size = -(-out // k)
    assert _fwd_call("clb_logic_forward", xt, w, spec, L.W_LOGITS, None, None, acc0, size) == L.CLB_OK
    assert _fwd_call("clb_logic_forward_staged", xt, w, spec, L.W_LOGITS, None, None, acc1, size, stage) == L.CLB_OK
    torch.cuda.synchronize()
    torch.testing.assert_close(acc0, acc1, rtol=1e-6, atol=1e-5)  # class sums: atomic order may differ
    short = stage[: nbytes - 256]
    y1 = torch.empty(out, B, dtype=dtype, device="cuda")
    assert _fwd_call("clb_logic_forward_staged", xt, w, spec, L.W_LOGITS, sel, y1, stage=short) == L.CLB_ERR_WORKSPACE
