"""The B200 kernels, called through the reference-API shims, against outputs of the reference's own
CUDA extensions (tests/golden/ref_cuda.npz, produced by tests/golden/make_golden_gpu.py).
Discrete outputs are bit-exact; real outputs agree to 1e-6 of each output's scale (the reference's
fp64 path rounds through float, see tests/test_oracle_pins.py)."""
import numpy as np
import pytest
import torch

from compactlogic_b200 import convlogic_cuda, difflogic_cuda

from helpers import assert_close, cuda

pytestmark = pytest.mark.gpu


def test_dense_vs_reference_kernels(golden):
    d = golden("ref_cuda.npz")
    x, a, b, w, g, gy = (cuda(d[k]) for k in ("dense_x", "dense_a", "dense_b", "dense_w", "dense_g", "dense_gy"))
    assert_close(difflogic_cuda.forward(x, a, b, w, g), d["dense_y"], 1e-6, "forward")
    assert_close(difflogic_cuda.forward(x.float(), a, b, w.float(), g), d["dense_y_f32"], 1e-5, "forward f32")
    assert_close(difflogic_cuda.backward_w(x, a, b, g, gy), d["dense_gw"], 1e-6, "backward_w")
    gx = difflogic_cuda.backward_x(x, a, b, w, g, gy, cuda(d["dense_starts"]), cuda(d["dense_ys"]),
                                   cuda(d["dense_codes"]))
    assert_close(gx, d["dense_gx"], 1e-6, "backward_x")
    assert_close(difflogic_cuda.backward_x_atomicAdd(x, a, b, w, g, gy), d["dense_gx_atomic"], 1e-6, "atomic")
    np.testing.assert_array_equal(difflogic_cuda.eval(cuda(d["dense_xb"]), a, b, cuda(d["dense_sel"]), g).cpu().numpy(),
                                  d["dense_eval"])


def test_packbits_groupbitsum_vs_reference_kernels(golden):
    d = golden("ref_cuda.npz")
    t = cuda(d["pack_t"].astype(bool))
    for bits in (8, 16, 32, 64):
        words, pad = difflogic_cuda.tensor_packbits_cuda(t, bits)
        np.testing.assert_array_equal(words.cpu().numpy(), d[f"pack_words_{bits}"])
        assert pad == int(d[f"pack_pad_{bits}"])
        np.testing.assert_array_equal(difflogic_cuda.groupbitsum(words, pad, 5).cpu().numpy(), d[f"groupbitsum_{bits}"])


def test_conv_vs_reference_kernels(golden):
    d = golden("ref_cuda.npz")
    stride, pad, ks = (int(v) for v in d["conv_meta"])
    x, och, oh, ow, w, g, gy = (cuda(d[k]) for k in ("conv_x", "conv_och", "conv_oh", "conv_ow", "conv_w", "conv_g",
                                                      "conv_gy"))
    assert_close(convlogic_cuda.forward(x, och, oh, ow, w, g, stride, pad, ks), d["conv_y"], 1e-6, "conv forward")
    assert_close(convlogic_cuda.backward_x(x, och, oh, ow, w, g, gy, stride, pad), d["conv_gx"], 1e-6, "conv gx")
    assert_close(convlogic_cuda.backward_w(x, och, oh, ow, g, gy, stride), d["conv_gw"], 1e-6, "conv gw")
    ye = convlogic_cuda.eval(cuda(d["conv_xb"]), och, oh, ow, cuda(d["conv_sel"]), g, stride, pad, ks)
    np.testing.assert_array_equal(ye.cpu().numpy(), d["conv_eval"])
