"""Pin the CPU oracle to the reference: coefficient tables, the reference's CPU gate relaxation,
the reference's CPU circuit evaluator, and the reference's own known-answer / gradient tests."""
import numpy as np
import pytest

from oracle import oracle as O

# The relaxation coefficient tables of the reference (compactlogic/cuda/utils.cuh:180-202, C0..C3) and
# the derivative tables (utils.cuh:209-243): GRAD_A_C0 = C1, GRAD_A_C1 = C3, GRAD_B_C0 = C2, GRAD_B_C1 = C3.
REF_C = np.array([
    [0, 0, 0, 0, 0, 0, 0, 0, 1, 1, 1, 1, 1, 1, 1, 1],
    [0, 0, 1, 1, 0, 0, 1, 1, -1, -1, 0, 0, -1, -1, 0, 0],
    [0, 0, 0, 0, 1, 1, 1, 1, -1, -1, -1, -1, 0, 0, 0, 0],
    [0, 1, -1, 0, -1, 0, -2, -1, 1, 2, 0, 1, 0, 1, -1, 0],
], dtype=np.float64)


def test_coefficients_match_reference_tables():
    np.testing.assert_array_equal(O.gate_coefficients().T, REF_C)


def test_relaxation_matches_reference_cpu_bin_op(golden):
    kat = golden("gate_kat.npz")
    x = np.stack([kat["grid_a"], kat["grid_b"]])
    a = np.zeros((16, 1), np.int64)
    b = np.ones((16, 1), np.int64)
    y = O.dense_forward(x, a, b, np.ones((16, 1)), np.arange(16).reshape(16, 1))
    np.testing.assert_allclose(y, kat["real"], rtol=0, atol=1e-12)


def test_boolean_truth_table_matches_compiler_gates(golden):
    kat = golden("gate_kat.npz")
    ab = kat["bool_ab"]
    for g in range(16):
        np.testing.assert_array_equal(O.gate_bool(g, ab[:, 0], ab[:, 1]), kat["boolean"][g].astype(bool))


def test_all_gates_kat():
    """The vendored difflogic all-gates KAT (tests/difflogic/test_difflogic_forward.py:74-100): one-hot
    weights pick each gate; inputs pairs (0,0),(0,1),(1,0),(1,1)."""
    flat = np.array([0, 0, 0, 1, 1, 0, 1, 1], np.float64)
    x = flat.reshape(8, 1)
    a = np.tile(np.array([0, 2, 4, 6]), 16).reshape(64, 1)
    b = a + 1
    g = np.repeat(np.arange(16), 4).reshape(64, 1)
    y = O.dense_forward(x, a, b, np.ones((64, 1)), g)[:, 0]
    expect = np.array([O.gate_bool(gg, flat[0::2][i], flat[1::2][i]) for gg in range(16) for i in range(4)], float)
    np.testing.assert_array_equal(y, expect)


def _rand_layer(rng, in_dim, out, K, B):
    x = rng.random((in_dim, B))
    a = rng.integers(0, in_dim, (out, K))
    b = rng.integers(0, in_dim, (out, K))
    w = O.softmax(rng.standard_normal((out, K)))
    g = rng.integers(0, 16, (out, K)).astype(np.uint8)
    return x, a, b, w, g


def test_gradients_by_finite_differences():
    """float64 gradient check of the restated backward formulas (the reference's gradcheck strategy,
    third_party/convlogic_source_code/tests/difflogic/test_difflogic_autograd.py:31-54)."""
    rng = np.random.default_rng(0)
    x, a, b, w, g = _rand_layer(rng, 6, 5, 3, 4)
    gy = rng.standard_normal((5, 4))
    f = lambda xx, ww: (O.dense_forward(xx, a, b, ww, g) * gy).sum()
    gx = O.dense_backward_x(x, a, b, w, g, gy)
    gw = O.dense_backward_w(x, a, b, g, gy)
    eps = 1e-6
    for idx in np.ndindex(*x.shape):
        d = np.zeros_like(x)
        d[idx] = eps
        assert abs((f(x + d, w) - f(x - d, w)) / (2 * eps) - gx[idx]) < 1e-7
    for idx in np.ndindex(*w.shape):
        d = np.zeros_like(w)
        d[idx] = eps
        assert abs((f(x, w + d) - f(x, w - d)) / (2 * eps) - gw[idx]) < 1e-7


def test_csr_and_scatter_grad_x_agree():
    rng = np.random.default_rng(1)
    x, a, b, w, g = _rand_layer(rng, 30, 40, 8, 7)
    gy = rng.standard_normal((40, 7))
    starts, ys, codes = O.inverse_index(a, b, 30)
    np.testing.assert_allclose(O.dense_backward_x_csr(x, a, b, w, g, gy, starts, ys, codes),
                               O.dense_backward_x(x, a, b, w, g, gy), rtol=1e-12, atol=1e-12)


def test_conv_gradients_by_finite_differences():
    rng = np.random.default_rng(2)
    N, C, H, W, Cout, K, ks, pad, stride = 2, 3, 5, 5, 4, 3, 3, 1, 2
    x = rng.random((N, C, H, W))
    och = rng.integers(0, C, (2, Cout, K))
    oh = rng.integers(0, ks, (2, Cout, K)) - pad
    ow = rng.integers(0, ks, (2, Cout, K)) - pad
    w = O.softmax(rng.standard_normal((Cout, K)))
    g = rng.integers(0, 16, (Cout, K))
    y = O.conv_forward(x, och, oh, ow, w, g, stride, pad, ks)
    gy = rng.standard_normal(y.shape)
    f = lambda xx, ww: (O.conv_forward(xx, och, oh, ow, ww, g, stride, pad, ks) * gy).sum()
    gx = O.conv_backward_x(x, och, oh, ow, w, g, gy, stride)
    gw = O.conv_backward_w(x, och, oh, ow, g, gy, stride)
    eps = 1e-6
    for idx in list(np.ndindex(*x.shape))[::7]:
        d = np.zeros_like(x)
        d[idx] = eps
        assert abs((f(x + d, w) - f(x - d, w)) / (2 * eps) - gx[idx]) < 1e-7
    for idx in np.ndindex(*w.shape):
        d = np.zeros_like(w)
        d[idx] = eps
        assert abs((f(x, w + d) - f(x, w - d)) / (2 * eps) - gw[idx]) < 1e-7


def test_discrete_counts_match_reference_circuit_evaluator(golden):
    """Packed and float-eval restatements reproduce the class counts of the reference's CPU circuit
    evaluator (simulation/consistency.py:80-130) bit-exactly."""
    d = golden("discrete.npz")
    x = d["x"].astype(np.float64)
    layers = []
    for i in range(1, 4):
        sel = O.argmax_first(d[f"{i}.weights"])
        layers.append(O.frozen_tables(d[f"{i}.indices"], d[f"{i}.gate_sequence"], sel))
    counts = O.packed_network_counts(x, layers, int(d["k"]))
    np.testing.assert_array_equal(counts, d["counts"])
    # float eval chain + GroupSum, then round(logits * tau) as simulation/paper_stats.py:56
    h = x.T
    for i in range(1, 4):
        sel = O.argmax_first(d[f"{i}.weights"])
        h = O.dense_eval(h, d[f"{i}.indices"][0], d[f"{i}.indices"][1], sel, d[f"{i}.gate_sequence"])
    logits = O.group_sum(h.T, int(d["k"]), float(d["tau"]))
    np.testing.assert_array_equal(np.rint(logits * float(d["tau"])).astype(np.int32), d["counts"])
    np.testing.assert_allclose(logits, d["logits"], rtol=0, atol=1e-6)


@pytest.mark.parametrize("bits", [8, 16, 32, 64])
@pytest.mark.parametrize("cols", [1, 7, 64, 100, 129])
def test_packbits_groupbitsum_semantics(bits, cols):
    rng = np.random.default_rng(cols)
    rows, k = 20, 5
    t = rng.random((rows, cols)) < 0.4
    words, pad = O.packbits(t, bits)
    assert words.shape == (rows, -(-cols // bits)) and pad == (bits - cols % bits) % bits
    raw = words.view(np.uint8).reshape(rows, -1)
    unpacked = np.unpackbits(raw, axis=1, bitorder="little")[:, :cols].astype(bool)
    np.testing.assert_array_equal(unpacked, t)
    counts = O.groupbitsum(words, pad, k)
    np.testing.assert_array_equal(counts, t.reshape(k, rows // k, cols).sum(1).T)
    with pytest.raises(ValueError):
        O.groupbitsum(words, pad, 3)


def test_packed_layer_fast_equals_bitwise():
    rng = np.random.default_rng(3)
    xw = rng.integers(0, 2**63, (50, 9), dtype=np.int64).astype(np.uint64)
    ab = rng.integers(-1, 50, (70, 2)).astype(np.int32)
    gate = rng.integers(0, 16, 70)
    np.testing.assert_array_equal(O.packed_layer(xw, ab, gate), O.packed_layer(xw, ab, gate, fast=True))


def test_oracle_matches_reference_cuda_kernels(golden):
    """The oracle reproduces the outputs of the reference's own CUDA extensions (run on a B200 by
    tests/golden/make_golden_gpu.py): dense forward / backward_w / backward_x (CSR and atomic) / eval,
    packbits / groupbitsum at every word width, conv forward / backward_x / backward_w / eval."""
    d = golden("ref_cuda.npz")
    x, a, b, w, g, gy = (d[k] for k in ("dense_x", "dense_a", "dense_b", "dense_w", "dense_g", "dense_gy"))
    # The fixture ran the reference in fp64, but its gate polynomial goes through fmaf with float
    # coefficients (compactlogic/cuda/utils.cuh:189-195) and its derivatives are computed in float
    # (utils.cuh:219-241), and backward_w sums in float (difflogic_kernel.cu:92-110): its fp64 results
    # carry float rounding, so compare at 1e-6 relative to the largest magnitude of each output.
    def close(got, ref, rtol=1e-6):
        np.testing.assert_allclose(got, ref, rtol=rtol, atol=rtol * np.abs(ref).max())

    close(O.dense_forward(x, a, b, w, g), d["dense_y"])
    close(O.dense_forward(x, a, b, w, g), d["dense_y_f32"], 1e-5)
    close(O.dense_backward_w(x, a, b, g, gy), d["dense_gw"])
    starts, ys, codes = O.inverse_index(a, b, x.shape[0])
    for name, ref in (("starts", starts), ("ys", ys), ("codes", codes)):
        np.testing.assert_array_equal(ref, d[f"dense_{name}"])
    close(O.dense_backward_x_csr(x, a, b, w, g, gy, starts, ys, codes), d["dense_gx"])
    close(O.dense_backward_x(x, a, b, w, g, gy), d["dense_gx_atomic"])
    np.testing.assert_array_equal(O.dense_eval(d["dense_xb"], a, b, d["dense_sel"], g), d["dense_eval"])
    t = d["pack_t"].astype(bool)
    for bits in (8, 16, 32, 64):
        words, pad = O.packbits(t, bits)
        np.testing.assert_array_equal(words, d[f"pack_words_{bits}"])
        assert pad == int(d[f"pack_pad_{bits}"])
        np.testing.assert_array_equal(O.groupbitsum(words, pad, 5), d[f"groupbitsum_{bits}"])
    stride, pad, ks = (int(v) for v in d["conv_meta"])
    cx, och, oh, ow, cw, cg, cgy = (d[k] for k in ("conv_x", "conv_och", "conv_oh", "conv_ow", "conv_w", "conv_g",
                                                     "conv_gy"))
    close(O.conv_forward(cx, och, oh, ow, cw, cg, stride, pad, ks), d["conv_y"])
    close(O.conv_backward_x(cx, och, oh, ow, cw, cg, cgy, stride), d["conv_gx"])
    close(O.conv_backward_w(cx, och, oh, ow, cg, cgy, stride), d["conv_gw"])
    np.testing.assert_array_equal(O.conv_eval(d["conv_xb"], och, oh, ow, d["conv_sel"], cg, stride, pad, ks),
                                  d["conv_eval"])
