"""CPU oracle of the CompactLogic logic-layer hot path — TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline / reference arm use this module,
and only as the checker or the timed CPU baseline.  The product package ``compactlogic_b200``
never imports it.

Real-valued kernels are restated in C (``oracle.c``, double accumulation, OpenMP) and wrapped
here with numpy; the reference's Python-side algebra around the kernels (softmax placement,
GroupSum padding, argmax eval, autograd softmax backward) is restated in numpy.  Each function names
the reference code it follows (paths relative to the CompactLogic repository).

Parity status: pinned.  The gate algebra is checked against the reference's coefficient tables
and the vendored difflogic known-answer tests; kernel outputs are checked against fixtures produced
by the reference's own CUDA extensions (tests/golden/).
"""
import ctypes
import os
import subprocess
from concurrent.futures import ThreadPoolExecutor

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")
_lib = None


def build(force: bool = False) -> str:
    src = os.path.join(HERE, "oracle.c")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE, "-B" if force else "all"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = ctypes.CDLL(_LIB_PATH)
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _f64(a):
    return np.ascontiguousarray(a, dtype=np.float64)


def _i64(a):
    return np.ascontiguousarray(a, dtype=np.int64)


def _u8(a):
    return np.ascontiguousarray(a, dtype=np.uint8)


I = ctypes.c_int64

#: host threads the oracle uses (rows are split across threads; ctypes releases the GIL)
THREADS = int(os.environ.get("ORACLE_THREADS", os.cpu_count() or 1))


def _par(n, fn, threads=None):
    """Run fn(lo, hi) over [0, n) split into contiguous ranges on `threads` host threads."""
    t = max(1, min(threads or THREADS, n))
    if t == 1:
        fn(0, n)
        return
    bounds = np.linspace(0, n, t + 1).astype(np.int64)
    with ThreadPoolExecutor(t) as ex:
        list(ex.map(lambda i: fn(int(bounds[i]), int(bounds[i + 1])), range(t)))

# ---------------------------------------------------------------------------------------------
# gate algebra
# ---------------------------------------------------------------------------------------------


def gate_coefficients() -> np.ndarray:
    """[16, 4] coefficients (c0, c1, c2, c3) of f = c0 + c1 a + c2 b + c3 ab (utils.cuh:180-202)."""
    out = np.zeros((16, 4), np.float64)
    lib().orc_gate_coefficients(_p(out))
    return out


def gate_bool(g: int, a, b):
    """Truth table of gate g on bool arrays (utils.cuh:122-139 table)."""
    a = np.asarray(a, bool)
    b = np.asarray(b, bool)
    idx = 3 - (2 * a.astype(np.int64) + b.astype(np.int64))
    return ((g >> idx) & 1).astype(bool)


# ---------------------------------------------------------------------------------------------
# Python-side algebra of compactlogic/compactlogic.py
# ---------------------------------------------------------------------------------------------


def softmax(w):
    """torch.softmax(weights, -1) (compactlogic.py:108)."""
    w = np.asarray(w, np.float64)
    e = np.exp(w - w.max(-1, keepdims=True))
    return e / e.sum(-1, keepdims=True)


def softmax_backward(p, gp):
    """Autograd of softmax: dL/dw = p * (gp - sum(p * gp))."""
    return p * (gp - (p * gp).sum(-1, keepdims=True))


def group_sum(y_bt, k, tau):
    """GroupSum.forward on [batch, out] (compactlogic.py:460-465): zero-pad out to a multiple of k,
    split into k contiguous groups, sum, divide by tau."""
    y = np.asarray(y_bt, np.float64)
    pad = (-y.shape[1]) % k
    if pad:
        y = np.concatenate([y, np.zeros((y.shape[0], pad))], 1)
    return y.reshape(y.shape[0], k, -1).sum(-1) / tau


def group_sum_backward(g_logits, out_dim, k, tau):
    """d GroupSum / d y: [batch, out]."""
    size = -(-out_dim // k)
    cls = np.arange(out_dim) // size
    return np.asarray(g_logits, np.float64)[:, cls] / tau


def argmax_first(w):
    """weights.argmax(-1) as uint8 (compactlogic.py:126): the first maximum on ties."""
    return np.argmax(np.asarray(w), axis=-1).astype(np.uint8)


def cross_entropy_grad(logits, labels):
    """d mean CE / d logits."""
    p = softmax(logits)
    p[np.arange(len(labels)), labels] -= 1
    return p / len(labels)


# ---------------------------------------------------------------------------------------------
# dense layer kernels (difflogic_kernel.cu)
# ---------------------------------------------------------------------------------------------


def dense_forward(x, a, b, w, g):
    """x [in, B], a/b [out, K], w probs [out, K], g uint8 -> y [out, B] (difflogic_kernel.cu:39-78)."""
    x, a, b, w, g = _f64(x), _i64(a), _i64(b), _f64(w), _u8(g)
    out, K = a.shape
    y = np.empty((out, x.shape[1]), np.float64)
    _par(out, lambda lo, hi: lib().orc_dense_forward(_p(x), I(x.shape[0]), I(x.shape[1]), _p(a[lo:hi]), _p(b[lo:hi]),
                                                     _p(w[lo:hi]), _p(g[lo:hi]), I(hi - lo), I(K), _p(y[lo:hi])))
    return y


def dense_backward_w(x, a, b, g, gy):
    """d loss / d prob [out, K] (difflogic_kernel.cu:82-137)."""
    x, a, b, g, gy = _f64(x), _i64(a), _i64(b), _u8(g), _f64(gy)
    out, K = a.shape
    gw = np.empty((out, K), np.float64)
    _par(out, lambda lo, hi: lib().orc_dense_backward_w(_p(x), I(x.shape[0]), I(x.shape[1]), _p(a[lo:hi]), _p(b[lo:hi]),
                                                        _p(g[lo:hi]), _p(gy[lo:hi]), I(hi - lo), I(K), _p(gw[lo:hi])))
    return gw


def dense_backward_x_csr(x, a, b, w, g, gy, starts, ys, codes):
    """grad_x [in, B] over the inverse index (difflogic_kernel.cu:140-194)."""
    x, a, b, w, g, gy = _f64(x), _i64(a), _i64(b), _f64(w), _u8(g), _f64(gy)
    starts, ys, codes = _i64(starts), _i64(ys), np.ascontiguousarray(codes, np.int8)
    out, K = a.shape
    gx = np.empty_like(x)
    _par(x.shape[0], lambda lo, hi: lib().orc_dense_backward_x_csr(
        _p(x), I(hi - lo), I(x.shape[1]), _p(a), _p(b), _p(w), _p(g), _p(gy), _p(starts[lo:]), _p(ys), _p(codes),
        I(out), I(K), _p(gx[lo:hi])))
    return gx


def dense_backward_x(x, a, b, w, g, gy):
    """grad_x [in, B] by scattering (difflogic_kernel.cu:574-610)."""
    x, a, b, w, g, gy = _f64(x), _i64(a), _i64(b), _f64(w), _u8(g), _f64(gy)
    out, K = a.shape
    gx = np.empty_like(x)
    lib().orc_dense_backward_x_scatter(_p(x), I(x.shape[0]), I(x.shape[1]), _p(a), _p(b), _p(w), _p(g), _p(gy), I(out),
                                       I(K), _p(gx))
    return gx


def dense_eval(x, a, b, sel, g):
    """Discrete float eval [out, B] (difflogic_kernel.cu:341-369)."""
    x, a, b, sel, g = _f64(x), _i64(a), _i64(b), _u8(sel), _u8(g)
    out, K = a.shape
    y = np.empty((out, x.shape[1]), np.float64)
    _par(out, lambda lo, hi: lib().orc_dense_eval(_p(x), I(x.shape[0]), I(x.shape[1]), _p(a[lo:hi]), _p(b[lo:hi]),
                                                  _p(sel[lo:hi]), _p(g[lo:hi]), I(hi - lo), I(K), _p(y[lo:hi])))
    return y


def inverse_index(a, b, in_dim):
    """The (starts, ys, codes) inverse connection index of LogicLayer.refresh_backward_index
    (compactlogic.py:184-274) for a full rebuild: entries sorted by input id (stable within an input:
    all a-side entries in (j, k) order, then all b-side entries)."""
    a, b = _i64(a), _i64(b)
    out, K = a.shape
    jj = np.repeat(np.arange(out), K)
    kk = np.tile(np.arange(K), out)
    flat_in = np.concatenate([a.reshape(-1), b.reshape(-1)])
    flat_y = np.concatenate([jj, jj])
    flat_code = np.concatenate([kk, -(kk + 1)]).astype(np.int8)
    order = np.argsort(flat_in, kind="stable")
    counts = np.bincount(flat_in, minlength=in_dim)
    starts = np.zeros(in_dim + 1, np.int64)
    starts[1:] = np.cumsum(counts)
    return starts, flat_y[order].astype(np.int64), flat_code[order]


# ---------------------------------------------------------------------------------------------
# conv layer kernels (convlogic_kernel.cu); x NCHW
# ---------------------------------------------------------------------------------------------


def conv_out_hw(h, w, pad, ks, stride):
    """convlogic_kernel.cu:159-160."""
    return (h + 2 * pad - ks) // stride + 1, (w + 2 * pad - ks) // stride + 1


def _conv_args(x, och, oh, ow):
    x = _f64(x)
    return (x, np.ascontiguousarray(och, np.int32), np.ascontiguousarray(oh, np.int8),
            np.ascontiguousarray(ow, np.int8))


def conv_forward(x, och, oh, ow, w, g, stride, pad, ks):
    x, och, oh, ow = _conv_args(x, och, oh, ow)
    w, g = _f64(w), _u8(g)
    N, C, H, W = x.shape
    Cout, K = w.shape
    Ho, Wo = conv_out_hw(H, W, pad, ks, stride)
    y = np.empty((N, Cout, Ho, Wo), np.float64)
    _par(N, lambda lo, hi: lib().orc_conv_forward(_p(x[lo:hi]), I(hi - lo), I(C), I(H), I(W), _p(och), _p(oh), _p(ow),
                                                  _p(w), _p(g), I(Cout), I(K), ctypes.c_int(stride), I(Ho), I(Wo),
                                                  _p(y[lo:hi])))
    return y


def conv_eval(x, och, oh, ow, sel, g, stride, pad, ks):
    x, och, oh, ow = _conv_args(x, och, oh, ow)
    sel, g = _u8(sel), _u8(g)
    N, C, H, W = x.shape
    Cout, K = g.shape
    Ho, Wo = conv_out_hw(H, W, pad, ks, stride)
    y = np.empty((N, Cout, Ho, Wo), np.float64)
    _par(N, lambda lo, hi: lib().orc_conv_eval(_p(x[lo:hi]), I(hi - lo), I(C), I(H), I(W), _p(och), _p(oh), _p(ow),
                                               _p(sel), _p(g), I(Cout), I(K), ctypes.c_int(stride), I(Ho), I(Wo),
                                               _p(y[lo:hi])))
    return y


def conv_backward_x(x, och, oh, ow, w, g, gy, stride):
    x, och, oh, ow = _conv_args(x, och, oh, ow)
    w, g, gy = _f64(w), _u8(g), _f64(gy)
    N, C, H, W = x.shape
    Cout, K = w.shape
    gx = np.empty_like(x)
    _par(N, lambda lo, hi: lib().orc_conv_backward_x(
        _p(x[lo:hi]), I(hi - lo), I(C), I(H), I(W), _p(och), _p(oh), _p(ow), _p(w), _p(g), _p(gy[lo:hi]), I(Cout),
        I(K), ctypes.c_int(stride), I(gy.shape[2]), I(gy.shape[3]), _p(gx[lo:hi])))
    return gx


def conv_backward_w(x, och, oh, ow, g, gy, stride):
    x, och, oh, ow = _conv_args(x, och, oh, ow)
    g, gy = _u8(g), _f64(gy)
    N, C, H, W = x.shape
    Cout, K = g.shape
    t = max(1, min(THREADS, N))
    parts = np.zeros((t, Cout, K), np.float64)
    bounds = np.linspace(0, N, t + 1).astype(np.int64)

    def run(i):
        lo, hi = int(bounds[i]), int(bounds[i + 1])
        lib().orc_conv_backward_w(_p(x[lo:hi]), I(hi - lo), I(C), I(H), I(W), _p(och), _p(oh), _p(ow), _p(g),
                                  _p(gy[lo:hi]), I(Cout), I(K), ctypes.c_int(stride), I(gy.shape[2]), I(gy.shape[3]),
                                  _p(parts[i]))

    with ThreadPoolExecutor(t) as ex:
        list(ex.map(run, range(t)))
    return parts.sum(0)


# ---------------------------------------------------------------------------------------------
# bit packing (difflogic_kernel.cu:417-568) and packed inference
# ---------------------------------------------------------------------------------------------
_NP_WORD = {8: np.int8, 16: np.int16, 32: np.int32, 64: np.int64}


def packbits(t, bits):
    """tensor_packbits_cuda: bool [rows, cols] -> (words [rows, ceil(cols/bits)] signed ints, pad_len)."""
    t = np.ascontiguousarray(t, np.uint8)
    rows, cols = t.shape
    nwords = -(-cols // bits)
    out = np.zeros((rows, nwords * bits // 8), np.uint8)
    lib().orc_packbits(_p(t), I(rows), I(cols), ctypes.c_int(bits), _p(out))
    return out.view(_NP_WORD[bits]).reshape(rows, nwords), (bits - cols % bits) % bits


def groupbitsum(words, pad_len, k):
    """groupbitsum: words [rows, nwords] -> counts [batch, k] int32."""
    words = np.ascontiguousarray(words)
    rows, nwords = words.shape
    if rows % k:
        raise ValueError(f"in_dim ({rows}) has to be divisible by k ({k}) but it is not")
    bits = words.dtype.itemsize * 8
    samples = nwords * bits - pad_len
    counts = np.zeros((samples, k), np.int32)
    raw = words.view(np.uint8).reshape(rows, nwords * bits // 8)
    lib().orc_groupbitsum(_p(raw), I(rows), I(raw.shape[1]), I(samples), I(k), _p(counts))
    return counts


def pack_samples(x_bt):
    """[batch, features] {0,1} -> [features, ceil(batch/64)] uint64, bit i of word w = sample 64w+i."""
    x = np.asarray(x_bt) > 0.5
    B, F = x.shape
    W = -(-B // 64)
    padded = np.zeros((W * 64, F), bool)
    padded[:B] = x
    bits = padded.T.reshape(F, W, 64).astype(np.uint64)
    return (bits << np.arange(64, dtype=np.uint64)).sum(-1, dtype=np.uint64)


def packed_layer(xw, ab, gate, fast=False):
    """One frozen layer on uint64 words: xw [in, W], ab int32 [out, 2] (-1 = constant 0), gate [out]."""
    xw = np.ascontiguousarray(xw, np.uint64)
    ab = np.ascontiguousarray(ab, np.int32)
    gate = _u8(gate)
    y = np.empty((ab.shape[0], xw.shape[1]), np.uint64)
    fn = lib().orc_packed_layer_fast if fast else lib().orc_packed_layer
    _par(ab.shape[0], lambda lo, hi: fn(_p(xw), I(xw.shape[0]), I(xw.shape[1]), _p(ab[lo:hi]), _p(gate[lo:hi]),
                                        I(hi - lo), _p(y[lo:hi])))
    return y


def packed_count(words, k, samples):
    """Packed GroupSum with zero padding: [samples, k] int32."""
    words = np.ascontiguousarray(words, np.uint64)
    rows, W = words.shape
    size = -(-rows // k)
    counts = np.zeros((samples, k), np.int32)
    lib().orc_packed_count(_p(words), I(rows), I(W), I(k), I(size), I(samples), _p(counts))
    return counts


def frozen_tables(indices, gate_sequence, sel):
    """Per-neuron (a, b, gate) of a frozen dense layer: the slot chosen by `sel` (compactlogic.py:126)."""
    idx = np.asarray(indices)
    sel = np.asarray(sel, np.int64)
    j = np.arange(idx.shape[1])
    ab = np.stack([idx[0, j, sel], idx[1, j, sel]], 1).astype(np.int32)
    return ab, np.asarray(gate_sequence)[j, sel].astype(np.uint8)


def packed_network_counts(x_bt, layers, k):
    """Class counts of a frozen dense network: layers = [(ab, gate)], input x [batch, features]."""
    B = np.asarray(x_bt).shape[0]
    h = pack_samples(x_bt)
    for ab, gate in layers:
        h = packed_layer(h, ab, gate, fast=True)
    return packed_count(h, k, B)
