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


# Per-element check of the full-size tests, on top of assert_close: every entry whose reference magnitude
# is at least 1e-3 of the largest must also be within ELEM_RTOL of itself.  fp32 sums of 10^4-10^5
# products with cancellation lose up to ~1e-4 of a small entry's own size (1.4e-4 measured on c1 grad_x),
# hence the separate, looser bound.
ELEM_RTOL = {torch.float32: 1e-3, torch.float64: 1e-9, torch.bfloat16: 2e-2}


def assert_close_elem(got, ref, rtol, elem_rtol, what=""):
    """assert_close, then the per-element relative bound on entries above 1e-3 of the largest."""
    assert_close(got, ref, rtol, what)
    got = got.detach().double().cpu().numpy() if isinstance(got, torch.Tensor) else np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    big = np.abs(ref) >= 1e-3 * np.abs(ref).max()
    rel = np.abs(got[big] - ref[big]) / np.abs(ref[big])
    assert rel.size == 0 or rel.max() <= elem_rtol, f"{what}: per-element rel err {rel.max():.3g} > {elem_rtol}"


def assert_close_logit_grad(got, p, gp, rtol, what="", gp_abs=None):
    """Gradient w.r.t. the gate logits, p * (gp - sum_k p gp) with gp = d loss / d p.  The subtraction cancels
    (gp is typically 10-100x larger than the result), so fp32 arithmetic, the reference's included, is only
    accurate to rtol of the terms p * gp: the absolute floor is rtol * max |p * gp| (at least rtol * max |ref|).
    gp_abs (optional): the same gradient summed over the absolute values of its terms (sum_n |gy| f, f >= 0
    for inputs in [0, 1]); for reductions over 10^5 terms with cancellation the floor becomes
    rtol * max |p * gp_abs|, the backward-error scale of an fp32 sum."""
    from oracle import oracle as O
    ref = O.softmax_backward(p, gp)
    got = got.detach().double().cpu().numpy() if isinstance(got, torch.Tensor) else np.asarray(got, np.float64)
    scale = max(float(np.abs(p * (gp if gp_abs is None else gp_abs)).max()), float(np.abs(ref).max()), 1e-30)
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
