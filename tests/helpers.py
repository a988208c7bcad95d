"""Shared parity helpers for the GPU tests."""
import numpy as np
import torch

# Tolerances (the parity bar of the task): fp32 soft mode 1e-5 relative, bf16 activations 1e-2
# relative, fp64 1e-10; discrete outputs bit-exact.  "Relative" is elementwise rtol plus an absolute
# floor of rtol times the largest reference magnitude, so entries that cancel to ~0 are judged on
# the scale of the quantity.
RTOL = {torch.float32: 1e-5, torch.float64: 1e-10, torch.bfloat16: 1e-2}


def assert_close(got, ref, rtol, what=""):
    got = got.detach().double().cpu().numpy() if isinstance(got, torch.Tensor) else np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    scale = max(float(np.abs(ref).max()) if ref.size else 0.0, 1e-30)
    np.testing.assert_allclose(got, ref, rtol=rtol, atol=rtol * scale, err_msg=what)


def rand_dense(seed, in_dim, out, K, B, p_lo=0.1, p_hi=0.9, binary_input=False):
    rng = np.random.default_rng(seed)
    if binary_input:
        p = rng.uniform(p_lo, p_hi, (in_dim, 1))
        x = (rng.random((in_dim, B)) < p).astype(np.float64)
    else:
        x = rng.random((in_dim, B))
    a = rng.integers(0, in_dim, (out, K))
    b = rng.integers(0, in_dim, (out, K))
    logits = rng.standard_normal((out, K))
    g = rng.integers(0, 16, (out, K)).astype(np.uint8)
    gy = rng.standard_normal((out, B))
    return x, a, b, logits, g, gy


def cuda(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t if dtype is None else t.to(dtype)
