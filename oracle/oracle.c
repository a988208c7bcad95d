/*
 * CPU oracle for the CompactLogic logic-layer hot path — TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference algorithms, used by tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference arm of bench.py as the checker and the CPU baseline.  The product
 * (compactlogic_b200) never links or calls this file.
 *
 * Every real-valued routine accumulates in double and is single-threaded; oracle.py runs row ranges
 * on several threads (ctypes releases the GIL).  Each function cites the reference code it
 * restates (paths relative to the CompactLogic repository).
 *
 * Gate algebra (compactlogic/cuda/utils.cuh:122-243): gate id g has truth table bits
 * t00 = g>>3&1, t01 = g>>2&1, t10 = g>>1&1, t11 = g&1 (t_ab is the output for inputs a, b).
 * Relaxation: f(a,b) = sum_ab t_ab * P(a) * P(b) with P(1)=v, P(0)=1-v; derivatives by hand.
 */
#include <stdint.h>
#include <string.h>

static inline int bit_of(int g, int a, int b) { return (g >> (3 - (2 * a + b))) & 1; }

/* f_g(a, b) evaluated directly from the truth table (multilinear extension). */
static inline double gate_real(int g, double a, double b) {
    return bit_of(g, 0, 0) * (1 - a) * (1 - b) + bit_of(g, 0, 1) * (1 - a) * b + bit_of(g, 1, 0) * a * (1 - b) +
           bit_of(g, 1, 1) * a * b;
}
static inline double gate_da(int g, double b) {
    return -bit_of(g, 0, 0) * (1 - b) - bit_of(g, 0, 1) * b + bit_of(g, 1, 0) * (1 - b) + bit_of(g, 1, 1) * b;
}
static inline double gate_db(int g, double a) {
    return -bit_of(g, 0, 0) * (1 - a) + bit_of(g, 0, 1) * (1 - a) - bit_of(g, 1, 0) * a + bit_of(g, 1, 1) * a;
}

/* Relaxation coefficients c0..c3 of f = c0 + c1 a + c2 b + c3 ab, for KAT comparison with the
 * reference tables C0..C3 (utils.cuh:180-202). */
void orc_gate_coefficients(double* out /* [16*4] */) {
    for (int g = 0; g < 16; ++g) {
        double f00 = gate_real(g, 0, 0), f01 = gate_real(g, 0, 1), f10 = gate_real(g, 1, 0), f11 = gate_real(g, 1, 1);
        out[4 * g + 0] = f00;
        out[4 * g + 1] = f10 - f00;
        out[4 * g + 2] = f01 - f00;
        out[4 * g + 3] = f11 - f10 - f01 + f00;
    }
}

/* ---------------------------------------------------------------------------------------------
 * Dense layer, x [in, B], y [out, B], a/b int64 [out, K], w probs [out, K], g uint8 [out, K].
 * ------------------------------------------------------------------------------------------- */

/* compactlogic/cuda/difflogic_kernel.cu:39-78 */
void orc_dense_forward(const double* x, int64_t in_dim, int64_t B, const int64_t* a, const int64_t* b, const double* w,
                       const uint8_t* g, int64_t out, int64_t K, double* y) {
    (void)in_dim;
    for (int64_t j = 0; j < out; ++j) {
        double* yr = y + j * B;
        for (int64_t n = 0; n < B; ++n) yr[n] = 0;
        for (int64_t k = 0; k < K; ++k) {
            const double* xa = x + a[j * K + k] * B;
            const double* xb = x + b[j * K + k] * B;
            const double p = w[j * K + k];
            const int gg = g[j * K + k] & 15;
            for (int64_t n = 0; n < B; ++n) yr[n] += p * gate_real(gg, xa[n], xb[n]);
        }
    }
}

/* compactlogic/cuda/difflogic_kernel.cu:82-137 : d loss / d prob */
void orc_dense_backward_w(const double* x, int64_t in_dim, int64_t B, const int64_t* a, const int64_t* b,
                          const uint8_t* g, const double* gy, int64_t out, int64_t K, double* gw) {
    (void)in_dim;
    for (int64_t j = 0; j < out; ++j) {
        for (int64_t k = 0; k < K; ++k) {
            const double* xa = x + a[j * K + k] * B;
            const double* xb = x + b[j * K + k] * B;
            const int gg = g[j * K + k] & 15;
            double s = 0;
            for (int64_t n = 0; n < B; ++n) s += gy[j * B + n] * gate_real(gg, xa[n], xb[n]);
            gw[j * K + k] = s;
        }
    }
}

/* compactlogic/cuda/difflogic_kernel.cu:140-194 : gather over the inverse index (starts/ys/codes,
 * compactlogic/compactlogic.py:184-274; code >= 0 means operand a of slot code, -(k+1) operand b). */
void orc_dense_backward_x_csr(const double* x, int64_t in_dim, int64_t B, const int64_t* a, const int64_t* b,
                              const double* w, const uint8_t* g, const double* gy, const int64_t* starts,
                              const int64_t* ys, const int8_t* codes, int64_t out, int64_t K, double* gx) {
    (void)out;
    for (int64_t i = 0; i < in_dim; ++i) {
        double* gr = gx + i * B;
        for (int64_t n = 0; n < B; ++n) gr[n] = 0;
        for (int64_t o = starts[i]; o < starts[i + 1]; ++o) {
            const int64_t j = ys[o];
            const int code = codes[o];
            const int side_a = code >= 0;
            const int64_t k = side_a ? code : -code - 1;
            const double p = w[j * K + k];
            const int gg = g[j * K + k] & 15;
            const double* other = x + (side_a ? b[j * K + k] : a[j * K + k]) * B;
            for (int64_t n = 0; n < B; ++n) {
                const double d = side_a ? gate_da(gg, other[n]) : gate_db(gg, other[n]);
                gr[n] += p * d * gy[j * B + n];
            }
        }
    }
}

/* compactlogic/cuda/difflogic_kernel.cu:574-610 : same result by scattering from each slot. */
void orc_dense_backward_x_scatter(const double* x, int64_t in_dim, int64_t B, const int64_t* a, const int64_t* b,
                                  const double* w, const uint8_t* g, const double* gy, int64_t out, int64_t K,
                                  double* gx) {
    memset(gx, 0, sizeof(double) * in_dim * B);
    for (int64_t j = 0; j < out; ++j)
        for (int64_t k = 0; k < K; ++k) {
            const int64_t ia = a[j * K + k], ib = b[j * K + k];
            const double p = w[j * K + k];
            const int gg = g[j * K + k] & 15;
            for (int64_t n = 0; n < B; ++n) {
                const double t = p * gy[j * B + n];
                const double va = x[ia * B + n], vb = x[ib * B + n];
                gx[ia * B + n] += t * gate_da(gg, vb);
                gx[ib * B + n] += t * gate_db(gg, va);
            }
        }
}

/* compactlogic/cuda/difflogic_kernel.cu:341-369 : chosen slot only. */
void orc_dense_eval(const double* x, int64_t in_dim, int64_t B, const int64_t* a, const int64_t* b, const uint8_t* sel,
                    const uint8_t* g, int64_t out, int64_t K, double* y) {
    (void)in_dim;
    for (int64_t j = 0; j < out; ++j) {
        const int64_t k = sel[j];
        const double* xa = x + a[j * K + k] * B;
        const double* xb = x + b[j * K + k] * B;
        const int gg = g[j * K + k] & 15;
        for (int64_t n = 0; n < B; ++n) y[j * B + n] = gate_real(gg, xa[n], xb[n]);
    }
}

/* ---------------------------------------------------------------------------------------------
 * Conv layer, x [N, Cin, H, W] NCHW, y [N, Cout, Ho, Wo]; offsets [2, Cout, K] pre-shifted by -pad;
 * a coordinate outside [0,H)x[0,W) reads 0 (compactlogic/cuda/convlogic_kernel.cu:110-137).
 * ------------------------------------------------------------------------------------------- */
static inline double conv_read(const double* x, int64_t n, int64_t C, int64_t H, int64_t W, int64_t ch, int64_t yy,
                               int64_t xx, int* valid) {
    *valid = yy >= 0 && yy < H && xx >= 0 && xx < W;
    return *valid ? x[((n * C + ch) * H + yy) * W + xx] : 0.0;
}

/* compactlogic/cuda/convlogic_kernel.cu:86-138 (mode 0: probs w) and :433-476 (mode 1: select). */
static void conv_fwd(const double* x, int64_t N, int64_t C, int64_t H, int64_t W, const int32_t* och, const int8_t* oh,
                     const int8_t* ow, const double* w, const uint8_t* sel, const uint8_t* g, int64_t Cout, int64_t K,
                     int stride, int64_t Ho, int64_t Wo, double* y) {
    for (int64_t n = 0; n < N; ++n)
        for (int64_t c = 0; c < Cout; ++c)
            for (int64_t oy = 0; oy < Ho; ++oy)
                for (int64_t ox = 0; ox < Wo; ++ox) {
                    double acc = 0;
                    const int64_t k0 = sel ? sel[c] : 0, k1 = sel ? sel[c] + 1 : K;
                    for (int64_t k = k0; k < k1; ++k) {
                        const int64_t o0 = c * K + k, o1 = Cout * K + c * K + k;
                        int v;
                        const double va = conv_read(x, n, C, H, W, och[o0], oy * stride + oh[o0], ox * stride + ow[o0], &v);
                        const double vb = conv_read(x, n, C, H, W, och[o1], oy * stride + oh[o1], ox * stride + ow[o1], &v);
                        const double f = gate_real(g[c * K + k] & 15, va, vb);
                        acc += sel ? f : w[c * K + k] * f;
                    }
                    y[((n * Cout + c) * Ho + oy) * Wo + ox] = acc;
                }
}

void orc_conv_forward(const double* x, int64_t N, int64_t C, int64_t H, int64_t W, const int32_t* och, const int8_t* oh,
                      const int8_t* ow, const double* w, const uint8_t* g, int64_t Cout, int64_t K, int stride,
                      int64_t Ho, int64_t Wo, double* y) {
    conv_fwd(x, N, C, H, W, och, oh, ow, w, NULL, g, Cout, K, stride, Ho, Wo, y);
}

void orc_conv_eval(const double* x, int64_t N, int64_t C, int64_t H, int64_t W, const int32_t* och, const int8_t* oh,
                   const int8_t* ow, const uint8_t* sel, const uint8_t* g, int64_t Cout, int64_t K, int stride,
                   int64_t Ho, int64_t Wo, double* y) {
    conv_fwd(x, N, C, H, W, och, oh, ow, NULL, sel, g, Cout, K, stride, Ho, Wo, y);
}

/* compactlogic/cuda/convlogic_kernel.cu:190-246 : scatter into zeroed grad_x. */
void orc_conv_backward_x(const double* x, int64_t N, int64_t C, int64_t H, int64_t W, const int32_t* och,
                         const int8_t* oh, const int8_t* ow, const double* w, const uint8_t* g, const double* gy,
                         int64_t Cout, int64_t K, int stride, int64_t Ho, int64_t Wo, double* gx) {
    memset(gx, 0, sizeof(double) * N * C * H * W);
    for (int64_t n = 0; n < N; ++n)  /* samples are independent: no race across n */
        for (int64_t c = 0; c < Cout; ++c)
            for (int64_t oy = 0; oy < Ho; ++oy)
                for (int64_t ox = 0; ox < Wo; ++ox) {
                    const double gyv = gy[((n * Cout + c) * Ho + oy) * Wo + ox];
                    for (int64_t k = 0; k < K; ++k) {
                        const int64_t o0 = c * K + k, o1 = Cout * K + c * K + k;
                        const int64_t ya = oy * stride + oh[o0], xa = ox * stride + ow[o0];
                        const int64_t yb = oy * stride + oh[o1], xb = ox * stride + ow[o1];
                        int va_ok, vb_ok;
                        const double va = conv_read(x, n, C, H, W, och[o0], ya, xa, &va_ok);
                        const double vb = conv_read(x, n, C, H, W, och[o1], yb, xb, &vb_ok);
                        const double p = w[c * K + k];
                        const int gg = g[c * K + k] & 15;
                        if (va_ok) gx[((n * C + och[o0]) * H + ya) * W + xa] += p * gate_da(gg, vb) * gyv;
                        if (vb_ok) gx[((n * C + och[o1]) * H + yb) * W + xb] += p * gate_db(gg, va) * gyv;
                    }
                }
}

/* compactlogic/cuda/convlogic_kernel.cu:295-382 */
void orc_conv_backward_w(const double* x, int64_t N, int64_t C, int64_t H, int64_t W, const int32_t* och,
                         const int8_t* oh, const int8_t* ow, const uint8_t* g, const double* gy, int64_t Cout,
                         int64_t K, int stride, int64_t Ho, int64_t Wo, double* gw) {
    for (int64_t c = 0; c < Cout; ++c)
        for (int64_t k = 0; k < K; ++k) {
            const int64_t o0 = c * K + k, o1 = Cout * K + c * K + k;
            const int gg = g[c * K + k] & 15;
            double s = 0;
            for (int64_t n = 0; n < N; ++n)
                for (int64_t oy = 0; oy < Ho; ++oy)
                    for (int64_t ox = 0; ox < Wo; ++ox) {
                        int v;
                        const double va = conv_read(x, n, C, H, W, och[o0], oy * stride + oh[o0], ox * stride + ow[o0], &v);
                        const double vb = conv_read(x, n, C, H, W, och[o1], oy * stride + oh[o1], ox * stride + ow[o1], &v);
                        s += gate_real(gg, va, vb) * gy[((n * Cout + c) * Ho + oy) * Wo + ox];
                    }
            gw[c * K + k] = s;
        }
}

/* ---------------------------------------------------------------------------------------------
 * Bit packing and packed GroupSum.
 * ------------------------------------------------------------------------------------------- */

/* compactlogic/cuda/difflogic_kernel.cu:417-451 : bit i of word c = t[row, c*bits + i], LSB first.
 * Words are written as little-endian bytes, row_bytes = ceil(cols/bits)*bits/8. */
void orc_packbits(const uint8_t* t, int64_t rows, int64_t cols, int bits, uint8_t* out) {
    const int64_t nwords = (cols + bits - 1) / bits, row_bytes = nwords * bits / 8;
    memset(out, 0, rows * row_bytes);
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t c = 0; c < cols; ++c)
            if (t[r * cols + c]) out[r * row_bytes + c / 8] |= (uint8_t)(1u << (c % 8));
}

/* compactlogic/cuda/difflogic_kernel.cu:500-533 : counts[n, c] = sum_{i<cs} bit n of row c*cs+i. */
void orc_groupbitsum(const uint8_t* words, int64_t rows, int64_t row_bytes, int64_t samples, int64_t k,
                     int32_t* counts) {
    const int64_t cs = rows / k;
    for (int64_t n = 0; n < samples; ++n)
        for (int64_t c = 0; c < k; ++c) {
            int32_t s = 0;
            for (int64_t i = 0; i < cs; ++i) s += (words[(c * cs + i) * row_bytes + n / 8] >> (n % 8)) & 1;
            counts[n * k + c] = s;
        }
}

/* One frozen layer on packed words: bit by bit from the truth table (utils.cuh:141-178 semantics). */
void orc_packed_layer(const uint64_t* x, int64_t in_dim, int64_t W, const int32_t* ab, const uint8_t* gate,
                      int64_t out, uint64_t* y) {
    (void)in_dim;
    for (int64_t j = 0; j < out; ++j) {
        const int gg = gate[j] & 15;
        for (int64_t w = 0; w < W; ++w) {
            const uint64_t va = ab[2 * j] >= 0 ? x[ab[2 * j] * W + w] : 0;
            const uint64_t vb = ab[2 * j + 1] >= 0 ? x[ab[2 * j + 1] * W + w] : 0;
            uint64_t r = 0;
            for (int i = 0; i < 64; ++i) r |= (uint64_t)bit_of(gg, (int)((va >> i) & 1), (int)((vb >> i) & 1)) << i;
            y[j * W + w] = r;
        }
    }
}

/* Same layer with the word-parallel multiplexer (used to time a fair packed CPU baseline). */
void orc_packed_layer_fast(const uint64_t* x, int64_t in_dim, int64_t W, const int32_t* ab, const uint8_t* gate,
                           int64_t out, uint64_t* y) {
    (void)in_dim;
    for (int64_t j = 0; j < out; ++j) {
        const int gg = gate[j] & 15;
        const uint64_t t00 = 0 - (uint64_t)bit_of(gg, 0, 0), t01 = 0 - (uint64_t)bit_of(gg, 0, 1);
        const uint64_t t10 = 0 - (uint64_t)bit_of(gg, 1, 0), t11 = 0 - (uint64_t)bit_of(gg, 1, 1);
        const uint64_t* xa = ab[2 * j] >= 0 ? x + ab[2 * j] * W : NULL;
        const uint64_t* xb = ab[2 * j + 1] >= 0 ? x + ab[2 * j + 1] * W : NULL;
        for (int64_t w = 0; w < W; ++w) {
            const uint64_t va = xa ? xa[w] : 0, vb = xb ? xb[w] : 0;
            y[j * W + w] = (t00 & ~va & ~vb) | (t01 & ~va & vb) | (t10 & va & ~vb) | (t11 & va & vb);
        }
    }
}

/* Packed GroupSum with the reference's zero padding (compactlogic/compactlogic.py:460-465):
 * class(j) = j / class_size; counts[n, c] += popcount of bit n over the class's rows. */
void orc_packed_count(const uint64_t* words, int64_t rows, int64_t W, int64_t k, int64_t class_size, int64_t samples,
                      int32_t* counts) {
    for (int64_t n = 0; n < samples; ++n) {
        for (int64_t c = 0; c < k; ++c) counts[n * k + c] = 0;
        for (int64_t r = 0; r < rows; ++r) counts[n * k + r / class_size] += (int32_t)((words[r * W + n / 64] >> (n % 64)) & 1);
    }
}
