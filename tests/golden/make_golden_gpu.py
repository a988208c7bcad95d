"""Generate tests/golden/ref_cuda.npz by running the reference's own CUDA extensions on a GPU.

The reference kernels (compactlogic/cuda/{difflogic,convlogic}{.cpp,_kernel.cu}) are compiled
unmodified for sm_100 by oracle/build_ref.py into oracle/_ref/.  This script loads them, runs every
entry point of both pybind modules on small seeded inputs, and stores inputs and outputs.  The
fixture then pins the CPU oracle to the reference's real kernels (tests/test_oracle_pins.py) and is
a second parity target for the B200 kernels (tests/test_ref_cuda_gpu.py).

Usage (on a GPU box, from the repository root):
    python tests/golden/make_golden_gpu.py [--out tests/golden/ref_cuda.npz]
"""
import argparse
import importlib.util
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def load_ref(name):
    path = os.path.join(ROOT, "oracle", "_ref", name + ".so")
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=os.path.join(ROOT, "tests", "golden", "ref_cuda.npz"))
    args = ap.parse_args()
    dl, cv = load_ref("difflogic_cuda"), load_ref("convlogic_cuda")
    dev = torch.device("cuda")
    rng = np.random.default_rng(2024)
    out = {}

    # dense layer: in 50, out 70, K 16, batch 40 (fp64 so the fixture is precise)
    in_dim, n, K, B = 50, 70, 16, 40
    x = rng.random((in_dim, B))
    a = rng.integers(0, in_dim, (n, K))
    b = rng.integers(0, in_dim, (n, K))
    logits = rng.standard_normal((n, K))
    w = np.exp(logits - logits.max(1, keepdims=True))
    w /= w.sum(1, keepdims=True)
    g = rng.integers(0, 16, (n, K)).astype(np.uint8)
    gy = rng.standard_normal((n, B))
    T = lambda v, dt=None: torch.from_numpy(np.ascontiguousarray(v)).to(dev) if dt is None else \
        torch.from_numpy(np.ascontiguousarray(v)).to(dev, dt)
    xt, at, bt, wt, gt, gyt = T(x), T(a), T(b), T(w), T(g), T(gy)
    out.update(dense_x=x, dense_a=a, dense_b=b, dense_w=w, dense_g=g, dense_gy=gy)
    out["dense_y"] = dl.forward(xt, at, bt, wt, gt).cpu().numpy()
    out["dense_gw"] = dl.backward_w(xt, at, bt, gt, gyt).cpu().numpy()
    # inverse index exactly as LogicLayer.refresh_backward_index builds it
    jj = np.repeat(np.arange(n), K)
    kk = np.tile(np.arange(K), n)
    flat_in = np.concatenate([a.reshape(-1), b.reshape(-1)])
    flat_y = np.concatenate([jj, jj])
    flat_code = np.concatenate([kk, -(kk + 1)]).astype(np.int8)
    order = np.argsort(flat_in, kind="stable")
    starts = np.zeros(in_dim + 1, np.int64)
    starts[1:] = np.cumsum(np.bincount(flat_in, minlength=in_dim))
    ys, codes = flat_y[order].astype(np.int64), flat_code[order]
    out.update(dense_starts=starts, dense_ys=ys, dense_codes=codes)
    out["dense_gx"] = dl.backward_x(xt, at, bt, wt, gt, gyt, T(starts), T(ys), T(codes)).cpu().numpy()
    out["dense_gx_atomic"] = dl.backward_x_atomicAdd(xt, at, bt, wt, gt, gyt).cpu().numpy()
    sel = rng.integers(0, K, n).astype(np.uint8)
    xb = (x > 0.5).astype(np.float64)
    out.update(dense_sel=sel, dense_xb=xb)
    out["dense_eval"] = dl.eval(T(xb), at, bt, T(sel), gt).cpu().numpy()
    # fp32 forward too (the reference's own float rounding)
    out["dense_y_f32"] = dl.forward(T(x, torch.float32), at, bt, T(w, torch.float32), gt).cpu().numpy()

    # packbits / groupbitsum
    tb = rng.random((30, 200)) < 0.4
    out["pack_t"] = tb.astype(np.uint8)
    for bits in (8, 16, 32, 64):
        words, pad = dl.tensor_packbits_cuda(T(tb), bits)
        out[f"pack_words_{bits}"] = words.cpu().numpy()
        out[f"pack_pad_{bits}"] = np.array(pad)
        out[f"groupbitsum_{bits}"] = dl.groupbitsum(words, pad, 5).cpu().numpy()

    # conv layer: x (3, 6, 8, 8), c_out 9, ks 3, stride 2, pad 1, K 8, random channels
    N, C, H, W, Co, Kc, ks, stride, pad = 3, 6, 8, 8, 9, 8, 3, 2, 1
    cx = rng.random((N, C, H, W))
    och = rng.integers(0, C, (2, Co, Kc)).astype(np.int32)
    oh = (rng.integers(0, ks, (2, Co, Kc)) - pad).astype(np.int8)
    ow = (rng.integers(0, ks, (2, Co, Kc)) - pad).astype(np.int8)
    cl = rng.standard_normal((Co, Kc))
    cw = np.exp(cl - cl.max(1, keepdims=True))
    cw /= cw.sum(1, keepdims=True)
    cg = rng.integers(0, 16, (Co, Kc)).astype(np.uint8)
    args_c = (T(och), T(oh), T(ow))
    cy = cv.forward(T(cx), *args_c, T(cw), T(cg), stride, pad, ks)
    cgy = rng.standard_normal(tuple(cy.shape))
    out.update(conv_x=cx, conv_och=och, conv_oh=oh, conv_ow=ow, conv_w=cw, conv_g=cg, conv_gy=cgy,
               conv_meta=np.array([stride, pad, ks]))
    out["conv_y"] = cy.cpu().numpy()
    out["conv_gx"] = cv.backward_x(T(cx), *args_c, T(cw), T(cg), T(cgy), stride, pad).cpu().numpy()
    out["conv_gw"] = cv.backward_w(T(cx), *args_c, T(cg), T(cgy), stride).cpu().numpy()
    csel = rng.integers(0, Kc, Co).astype(np.uint8)
    cxb = (cx > 0.5).astype(np.float64)
    out.update(conv_sel=csel, conv_xb=cxb)
    out["conv_eval"] = cv.eval(T(cxb), *args_c, T(csel), T(cg), stride, pad, ks).cpu().numpy()
    torch.cuda.synchronize()
    os.makedirs(os.path.dirname(os.path.abspath(args.out)), exist_ok=True)
    np.savez_compressed(args.out, **out)
    print("wrote", args.out, file=sys.stderr)


if __name__ == "__main__":
    main()
