// Receptive-field-staged convolutional logic layers (ConvLayer forward, eval and backward, fp32).
//
// Reference: conv_layer_cuda_forward / _backward_x / _backward_w / eval
// (compactlogic/cuda/convlogic_kernel.cu:86-188, 190-430, 433-530).  Output (c, oy, ox) of a conv
// logic layer reads, for each of its K candidate gates, the two input elements
// (ch, oy*stride + dh, ox*stride + dw), with per-(c, k, operand) offsets shared by all positions and
// out-of-frame coordinates reading 0 (the offsets are pre-shifted by -padding, compactlogic.py:690).
//
// Plane mode.  When every slot of output channel c reads one input channel ch(c) (the default
// num_chn == 1 connection scheme, ch = c mod c_in, compactlogic.py:678-683), all output channels with
// the same ch read the same input plane.  A CTA owns one input channel, one TH x TW tile of output
// positions and one chunk of 128 batch columns (activations are feature-major, [c*h*w, batch]):
//   1. the tile's receptive field, THI x TWI input positions with THI = (TH-1)*stride + ks, is copied
//      into shared memory: one bulk asynchronous copy (cp.async.bulk, 512 bytes = 128 columns) per
//      in-frame position, all completing on one mbarrier; zero-padding positions are cleared, and
//      one extra all-zero position serves the operands a gate ignores;
//   2. every output channel of the group and every tile position is evaluated from shared memory
//      (2K operand reads per output, none through L1/L2), one warp per (channel, position), lanes on
//      consecutive 4-column groups;
//   3. backward: operands come from the staged tile; the activation gradient leaves as one
//      red.global.add.v4.f32 per operand and 4 columns into the pre-zeroed grad_x (its slab of one
//      column chunk stays in L2; measured on a B200, a shared-memory gradient tile with per-element
//      shared atomics was 2x slower); d loss / d p is reduced per warp with a butterfly
//      reduce-scatter and per CTA in shared memory into partials [parts, c_out, K]
//      (parts = column chunks x tiles), folded with the softmax backward by the finalize kernel.
// Layers whose slots read several channels use the slot-table kernels (logic_layer.cu).
#include <cuda_runtime.h>
#include <float.h>
#include <stdint.h>

#include "common.cuh"
#include "gates.cuh"
#include "kernels.h"

namespace clb {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kCols = 128;     // batch columns per CTA: 32 lanes x float4
constexpr int kRowBytes = 512; // shared bytes per staged position
constexpr int kChanBatch = 32; // output channels whose parameters are staged at once

struct PlaneArgs {
    const float* x;
    int64_t ldx;
    int64_t ncols;
    int c_in, h_in, w_in, c_out, h_out, w_out, stride, pad, ks, K;
    const int8_t* oh;  // [2, c_out, K], shifted by -pad
    const int8_t* ow;
    const int32_t* order;   // output channels grouped by input channel
    const int32_t* starts;  // [c_in + 1] group boundaries in `order`
    int cg;                 // output channels staged per batch (min(kChanBatch, largest group))
    int mode;
    const float* weights;   // [c_out, K]
    const uint8_t* gates;   // [c_out, K]
    const uint8_t* select;  // [c_out] (CLB_W_SELECT)
    int TH, TW, THI, TWI, tiles_x, ntiles;
    int32_t* err;           // optional: set to 2 when a staging wait gave up
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

// ---------------------------------------------------------------------------------------------
// Receptive-field staging through the bulk-copy engine.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

// Bounded wait: gives up after about a second (each try_wait itself suspends for a bounded time).
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
    const unsigned long long t0 = clock64();
    for (int i = 0; i < (1 << 24); ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (clock64() - t0 > 2000000000ull) break;  // ~1 s at 2 GHz
    }
    return false;
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

// Stage input channel ch's receptive field of the tile at output (oy0, ox0), columns [col0, col0+128):
// xs[p] for p = r * TWI + c is input (oy0*stride - pad + r, ox0*stride - pad + c); xs[THI*TWI] is the
// zero position.  Returns false (after a second bounded wait) if the copies did not complete.
__device__ bool stage_tile(const PlaneArgs& a, int ch, int oy0, int ox0, int64_t col0, float4* xs, uint64_t* bar) {
    const int npi = a.THI * a.TWI;
    const int64_t left = a.ncols - col0;
    const uint32_t nbytes = (uint32_t)((left < kCols ? left : kCols) * 4);  // ncols % 4 == 0: multiple of 16
    const int iy0 = oy0 * a.stride - a.pad, ix0 = ox0 * a.stride - a.pad;
    const uint32_t sbar = smem_u32(bar);
    if (threadIdx.x == 0) {
        mbar_init(sbar, 1);
        const int r_lo = iy0 < 0 ? -iy0 : 0, r_hi = min(a.THI, a.h_in - iy0);
        const int c_lo = ix0 < 0 ? -ix0 : 0, c_hi = min(a.TWI, a.w_in - ix0);
        const int n_in = max(r_hi - r_lo, 0) * max(c_hi - c_lo, 0);
        mbar_expect_tx(sbar, (uint32_t)n_in * nbytes);
    }
    __syncthreads();
    const float* plane = a.x + (int64_t)ch * a.h_in * a.w_in * a.ldx + col0;
    for (int p = threadIdx.x; p <= npi; p += blockDim.x) {
        const int r = p / a.TWI, c = p - r * a.TWI;
        const int iy = iy0 + r, ix = ix0 + c;
        if (p < npi && iy >= 0 && iy < a.h_in && ix >= 0 && ix < a.w_in) {
            bulk_g2s(smem_u32(xs + p * 32), plane + ((int64_t)iy * a.w_in + ix) * a.ldx, nbytes, sbar);
        } else {
            float4* z = xs + p * 32;
#pragma unroll 8
            for (int l = 0; l < 32; ++l) z[l] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    bool ok = mbar_wait_bounded(sbar, 0);
    if (!ok) ok = mbar_wait_bounded(sbar, 0);  // copies in flight must not outlive the CTA's shared memory
    ok = __syncthreads_and(ok);
    if (!ok && threadIdx.x == 0 && a.err != nullptr) atomicOr(a.err, 2);
    return ok;
}

// Offset of operand (dh, dw) from the tile-relative output base, in staged positions.
__device__ __forceinline__ int rel_off(const PlaneArgs& a, int dh, int dw) {
    return (dh + a.pad) * a.TWI + (dw + a.pad);
}


// ---------------------------------------------------------------------------------------------
// Forward (soft: softmax over the K logits + gate mix, convlogic_kernel.cu:86-188) and select mode
// (discrete eval, convlogic_kernel.cu:433-530).  Per channel, the stage holds the two-operand gates
// first (ns of them: offsets, p*c1, p*c2, p*c3), the one-operand gates at the end (n1 of them) and the
// constant part sum_k p*c0.
// ---------------------------------------------------------------------------------------------
template <bool SELECT>
__global__ void __launch_bounds__(kThreads) conv_plane_forward_kernel(const PlaneArgs a, float* __restrict__ y,
                                                                      const int64_t ldy) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int ch = blockIdx.y;
    const int g0 = a.starts[ch], g1 = a.starts[ch + 1];
    if (g0 >= g1) return;
    const int K = a.K;
    const int npi = a.THI * a.TWI;
    float4* xs = reinterpret_cast<float4*>(smem);
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + (size_t)(npi + 1) * kRowBytes);
    float4* cf = reinterpret_cast<float4*>(bar + 2);
    int2* off = reinterpret_cast<int2*>(cf + a.cg * K);
    float* c0 = reinterpret_cast<float*>(off + a.cg * K);
    int* ns = reinterpret_cast<int*>(c0 + a.cg);
    int* n1 = ns + a.cg;
    int* chan = n1 + a.cg;

    const int ty = blockIdx.x / a.tiles_x, tx = blockIdx.x - ty * a.tiles_x;
    const int oy0 = ty * a.TH, ox0 = tx * a.TW;
    const int64_t col0 = (int64_t)blockIdx.z * kCols;
    if (!stage_tile(a, ch, oy0, ox0, col0, xs, bar)) return;

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t col = col0 + lane * 4;
    const bool active = col < a.ncols;
    const int64_t hw = (int64_t)a.h_out * a.w_out;
    const int TP = a.TH * a.TW;
    const float4* xl = xs + lane;

    for (int cb = g0; cb < g1; cb += a.cg) {
        const int ncl = min(a.cg, g1 - cb);
        if (cb > g0) __syncthreads();  // previous batch's parameters are no longer read
        // one thread per (channel, slot), the K slots of a channel in K adjacent lanes (K = 4, 8 or 16):
        // softmax and the compaction by segmented warp shuffles / ballots
        const int rounds = (ncl * K + blockDim.x - 1) / blockDim.x;
        for (int r = 0; r < rounds; ++r) {
            const int e = r * blockDim.x + threadIdx.x;  // warp-uniform trip count keeps the shuffles legal
            const int t = e / K, k = e - t * K;
            const bool valid = e < ncl * K;
            const int c = valid ? a.order[cb + t] : 0;
            const int64_t ia = (int64_t)c * K + k, ib = ((int64_t)a.c_out + c) * K + k;
            float p = 0.f;
            GatePoly gp{0.f, 0.f, 0.f, 0.f};
            int oa = 0, ob = 0;
            if (valid) {
                gp = gate_poly(a.gates[ia] & 15);
                oa = rel_off(a, a.oh[ia], a.ow[ia]);
                ob = rel_off(a, a.oh[ib], a.ow[ib]);
            }
            if (SELECT) {
                p = valid && a.select[c] == k ? 1.f : 0.f;
            } else if (a.mode == CLB_W_LOGITS) {
                const float wv = valid ? a.weights[ia] : -FLT_MAX;
                float m = wv;
                for (int o = K >> 1; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
                const float ex = valid ? expf(wv - m) : 0.f;
                float sum = ex;
                for (int o = K >> 1; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
                p = valid ? ex / sum : 0.f;
            } else if (valid) {
                p = a.weights[ia];
            }
            const bool use = valid && (!SELECT || p != 0.f);
            const bool ua = use && (gp.c1 != 0.f || gp.c3 != 0.f), ub = use && (gp.c2 != 0.f || gp.c3 != 0.f);
            const bool two = ua && ub, one = ua != ub;
            const unsigned tm = __ballot_sync(0xffffffffu, two), om = __ballot_sync(0xffffffffu, one);
            const int lane = threadIdx.x & 31;
            const unsigned seg = ((1u << K) - 1u) << (lane & ~(K - 1));
            const unsigned below = seg & ((1u << lane) - 1u);
            const int np = __popc(tm & seg), no = __popc(om & seg);
            if (two) {
                const int pos = t * K + __popc(tm & below);
                off[pos] = make_int2(oa, ob);
                cf[pos] = make_float4(p * gp.c1, p * gp.c2, p * gp.c3, 0.f);
            } else if (one) {
                const int pos = t * K + K - 1 - __popc(om & below);
                off[pos] = make_int2(ua ? oa : ob, 0);
                cf[pos] = make_float4(p * (ua ? gp.c1 : gp.c2), 0.f, 0.f, 0.f);
            }
            float cs = use ? p * gp.c0 : 0.f;
            for (int o = K >> 1; o > 0; o >>= 1) cs += __shfl_xor_sync(0xffffffffu, cs, o);
            if (valid && k == 0) {
                chan[t] = c;
                ns[t] = np;
                n1[t] = no;
                c0[t] = cs;
            }
        }
        __syncthreads();

        for (int it = warp; it < ncl * TP; it += kWarps) {
            const int t = it / TP, pp = it - t * TP;
            const int oyl = pp / a.TW, oxl = pp - oyl * a.TW;
            const int oy = oy0 + oyl, ox = ox0 + oxl;
            if (oy >= a.h_out || ox >= a.w_out) continue;
            const int base = oyl * a.stride * a.TWI + oxl * a.stride;
            const float4* xb = xl + base * 32;
            const float cz = c0[t];
            float4 acc = make_float4(cz, cz, cz, cz);
            const int2* of = off + t * K;
            const float4* cc = cf + t * K;
            const int n = ns[t];
            int s = 0;
            for (; s + 2 <= n; s += 2) {  // the shared loads of two slots issued before their arithmetic
                const int2 o0 = of[s], o1 = of[s + 1];
                const float4 a0 = xb[o0.x * 32], b0 = xb[o0.y * 32], a1 = xb[o1.x * 32], b1 = xb[o1.y * 32];
                const float4 c = cc[s], d = cc[s + 1];
                acc.x = fmaf(fmaf(c.z, a0.x, c.y), b0.x, fmaf(c.x, a0.x, acc.x));
                acc.y = fmaf(fmaf(c.z, a0.y, c.y), b0.y, fmaf(c.x, a0.y, acc.y));
                acc.z = fmaf(fmaf(c.z, a0.z, c.y), b0.z, fmaf(c.x, a0.z, acc.z));
                acc.w = fmaf(fmaf(c.z, a0.w, c.y), b0.w, fmaf(c.x, a0.w, acc.w));
                acc.x = fmaf(fmaf(d.z, a1.x, d.y), b1.x, fmaf(d.x, a1.x, acc.x));
                acc.y = fmaf(fmaf(d.z, a1.y, d.y), b1.y, fmaf(d.x, a1.y, acc.y));
                acc.z = fmaf(fmaf(d.z, a1.z, d.y), b1.z, fmaf(d.x, a1.z, acc.z));
                acc.w = fmaf(fmaf(d.z, a1.w, d.y), b1.w, fmaf(d.x, a1.w, acc.w));
            }
            for (; s < n; ++s) {
                const int2 o = of[s];
                const float4 c = cc[s];
                const float4 va = xb[o.x * 32], vb = xb[o.y * 32];
                acc.x = fmaf(fmaf(c.z, va.x, c.y), vb.x, fmaf(c.x, va.x, acc.x));
                acc.y = fmaf(fmaf(c.z, va.y, c.y), vb.y, fmaf(c.x, va.y, acc.y));
                acc.z = fmaf(fmaf(c.z, va.z, c.y), vb.z, fmaf(c.x, va.z, acc.z));
                acc.w = fmaf(fmaf(c.z, va.w, c.y), vb.w, fmaf(c.x, va.w, acc.w));
            }
            for (int s = K - n1[t]; s < K; ++s) {
                const float c = cc[s].x;
                const float4 va = xb[of[s].x * 32];
                acc.x = fmaf(c, va.x, acc.x);
                acc.y = fmaf(c, va.y, acc.y);
                acc.z = fmaf(c, va.z, acc.z);
                acc.w = fmaf(c, va.w, acc.w);
            }
            if (active)
                *reinterpret_cast<float4*>(y + ((int64_t)chan[t] * hw + (int64_t)oy * a.w_out + ox) * ldy + col) = acc;
        }
    }
}

// Butterfly reduce-scatter of N per-lane values: afterwards lane l holds the warp sum of value
// (l >> (5 - log2 N)) & (N - 1).
template <int N, int OFF> struct PlaneRS {
    static __device__ __forceinline__ void run(float* v, int lane) {
        const bool up = (lane & OFF) != 0;
#pragma unroll
        for (int i = 0; i < N / 2; ++i) {
            const float send = up ? v[i] : v[i + N / 2];
            const float keep = up ? v[i + N / 2] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, OFF);
        }
        PlaneRS<N / 2, OFF / 2>::run(v, lane);
    }
};
template <int OFF> struct PlaneRS<1, OFF> {
    static __device__ __forceinline__ void run(float* v, int lane) {
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], OFF);
        PlaneRS<1, OFF / 2>::run(v, lane);
    }
};
template <> struct PlaneRS<1, 0> {
    static __device__ __forceinline__ void run(float*, int) {}
};

constexpr int log2i(int n) { return n <= 1 ? 0 : 1 + log2i(n / 2); }

// Add the warp's K per-lane partial dot products into the CTA's partials of local channel t.
template <int KT>
__device__ __forceinline__ void flush_dots(float (&pk)[KT], float* spart, int t, int lane) {
    PlaneRS<KT, 16>::run(pk, lane);
    constexpr int SH = 5 - log2i(KT);
    if ((lane & ((1 << SH) - 1)) == 0) atomicAdd(spart + t * KT + ((lane >> SH) & (KT - 1)), pk[0]);
#pragma unroll
    for (int k = 0; k < KT; ++k) pk[k] = 0.f;
}

// ---------------------------------------------------------------------------------------------
// Backward: per slot and output, from the staged operands,
//   d loss / d p[c, k]  += gy * f(a, b)                         (convlogic_kernel.cu:333-355)
//   grad_x[a] += p (c1 + c3 b) gy,  grad_x[b] += p (c2 + c3 a) gy  (convlogic_kernel.cu:227-245)
// GX = false when the layer's input needs no gradient.
// ---------------------------------------------------------------------------------------------
template <int KT, bool GX>
__global__ void __launch_bounds__(kThreads) conv_plane_backward_kernel(const PlaneArgs a, const float* __restrict__ gy,
                                                                       const int64_t ldgy, float* __restrict__ gx,
                                                                       const int64_t ldgx, float* __restrict__ part) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int ch = blockIdx.y;
    const int g0 = a.starts[ch], g1 = a.starts[ch + 1];
    if (g0 >= g1) return;
    const int npi = a.THI * a.TWI;
    float4* xs = reinterpret_cast<float4*>(smem);
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + (size_t)(npi + 1) * kRowBytes);
    float4* cf = reinterpret_cast<float4*>(bar + 2);
    int2* off = reinterpret_cast<int2*>(cf + a.cg * KT);
    float* pw = reinterpret_cast<float*>(off + a.cg * KT);
    float* spart = pw + a.cg * KT;
    int2* rcs = reinterpret_cast<int2*>(spart + a.cg * KT);  // (dh+pad, dw+pad) of operand a | b, packed 16:16
    int* chan = reinterpret_cast<int*>(rcs + a.cg * KT);

    const int ty = blockIdx.x / a.tiles_x, tx = blockIdx.x - ty * a.tiles_x;
    const int oy0 = ty * a.TH, ox0 = tx * a.TW;
    const int64_t col0 = (int64_t)blockIdx.z * kCols;
    if (!stage_tile(a, ch, oy0, ox0, col0, xs, bar)) return;

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t col = col0 + lane * 4;
    const bool active = col < a.ncols;
    const int64_t hw = (int64_t)a.h_out * a.w_out;
    const int TP = a.TH * a.TW;
    const int64_t pidx = (int64_t)blockIdx.z * a.ntiles + blockIdx.x;
    const int iy0 = oy0 * a.stride - a.pad, ix0 = ox0 * a.stride - a.pad;
    float* gplane = GX ? gx + (int64_t)ch * a.h_in * a.w_in * ldgx + col : nullptr;
    const float4 zero4 = make_float4(0.f, 0.f, 0.f, 0.f);

    for (int cb = g0; cb < g1; cb += a.cg) {
        const int ncl = min(a.cg, g1 - cb);
        if (cb > g0) __syncthreads();
        const int rounds = (ncl * KT + blockDim.x - 1) / blockDim.x;
        for (int r = 0; r < rounds; ++r) {
            const int e = r * blockDim.x + threadIdx.x;  // warp-uniform trip count keeps the shuffles legal
            const int t = e / KT, k = e - t * KT;
            const bool valid = e < ncl * KT;
            const int c = valid ? a.order[cb + t] : 0;
            const int64_t ia = (int64_t)c * KT + k, ib = ((int64_t)a.c_out + c) * KT + k;
            float p = 0.f;
            if (a.mode == CLB_W_LOGITS) {
                const float wv = valid ? a.weights[ia] : -FLT_MAX;
                float m = wv;
#pragma unroll
                for (int o = KT >> 1; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
                const float ex = valid ? expf(wv - m) : 0.f;
                float sum = ex;
#pragma unroll
                for (int o = KT >> 1; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
                p = valid ? ex / sum : 0.f;
            } else if (valid && a.weights != nullptr) {
                p = a.weights[ia];
            }
            if (!valid) continue;
            if (k == 0) chan[t] = c;
            const GatePoly gp = gate_poly(a.gates[ia] & 15);
            const bool ua = gp.c1 != 0.f || gp.c3 != 0.f, ub = gp.c2 != 0.f || gp.c3 != 0.f;
            off[e] = make_int2(ua ? rel_off(a, a.oh[ia], a.ow[ia]) : -1, ub ? rel_off(a, a.oh[ib], a.ow[ib]) : -1);
            rcs[e] = make_int2(((a.oh[ia] + a.pad) << 16) | (a.ow[ia] + a.pad), ((a.oh[ib] + a.pad) << 16) | (a.ow[ib] + a.pad));
            cf[e] = make_float4(gp.c0, gp.c1, gp.c2, gp.c3);
            pw[e] = p;
            spart[e] = 0.f;
        }
        __syncthreads();

        float pk[KT];
#pragma unroll
        for (int k = 0; k < KT; ++k) pk[k] = 0.f;
        int cur = -1;
        for (int it = warp; it < ncl * TP; it += kWarps) {
            const int t = it / TP, pp = it - t * TP;
            if (t != cur) {
                if (cur >= 0) flush_dots<KT>(pk, spart, cur, lane);
                cur = t;
            }
            const int oyl = pp / a.TW, oxl = pp - oyl * a.TW;
            const int oy = oy0 + oyl, ox = ox0 + oxl;
            if (oy >= a.h_out || ox >= a.w_out) continue;
            const int base = oyl * a.stride * a.TWI + oxl * a.stride;
            const int by = iy0 + oyl * a.stride, bx = ix0 + oxl * a.stride;  // input coordinates of offset (0, 0)
            float4 g = zero4;
            if (active) g = *reinterpret_cast<const float4*>(gy + ((int64_t)chan[t] * hw + (int64_t)oy * a.w_out + ox) * ldgy + col);
            const int2* of = off + t * KT;
            const float4* cc = cf + t * KT;
            const float* pp_ = pw + t * KT;
#pragma unroll
            for (int k = 0; k < KT; ++k) {
                const int2 o = of[k];
                const float4 c = cc[k];
                const int ia = o.x >= 0 ? base + o.x : npi, ib = o.y >= 0 ? base + o.y : npi;
                float4 va = xs[ia * 32 + lane], vb = xs[ib * 32 + lane];
                if (!active) va = vb = zero4;
                const float fa[4] = {va.x, va.y, va.z, va.w}, fb[4] = {vb.x, vb.y, vb.z, vb.w};
                const float gg[4] = {g.x, g.y, g.z, g.w};
                float dot = 0.f;
                float da[4], db[4];
                const float p = pp_[k];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float dfdb = fmaf(c.w, fa[i], c.z);  // c2 + c3 a
                    const float f = fmaf(dfdb, fb[i], fmaf(c.y, fa[i], c.x));
                    dot = fmaf(gg[i], f, dot);
                    if (GX) {
                        const float pg = p * gg[i];
                        da[i] = fmaf(c.w, fb[i], c.y) * pg;
                        db[i] = dfdb * pg;
                    }
                }
                pk[k] += dot;
                if (GX && active) {  // activation gradient straight into L2 (fire-and-forget vector reductions)
                    const int2 rc = rcs[t * KT + k];
                    if (o.x >= 0) {
                        const int iy = by + (rc.x >> 16), ix = bx + (rc.x & 0xffff);
                        if ((unsigned)iy < (unsigned)a.h_in && (unsigned)ix < (unsigned)a.w_in)
                            red_add<4>(gplane + (int64_t)(iy * a.w_in + ix) * ldgx, da);
                    }
                    if (o.y >= 0) {
                        const int iy = by + (rc.y >> 16), ix = bx + (rc.y & 0xffff);
                        if ((unsigned)iy < (unsigned)a.h_in && (unsigned)ix < (unsigned)a.w_in)
                            red_add<4>(gplane + (int64_t)(iy * a.w_in + ix) * ldgx, db);
                    }
                }
            }
        }
        if (cur >= 0) flush_dots<KT>(pk, spart, cur, lane);
        __syncthreads();
        for (int e = threadIdx.x; e < ncl * KT; e += blockDim.x) {
            const int t = e / KT, k = e - t * KT;
            part[(pidx * a.c_out + chan[t]) * KT + k] = spart[e];
        }
    }
}

void plane_tile(int h_out, int w_out, int stride, int ks, int& TH, int& TW) {
    TH = h_out < 4 ? h_out : 4;
    TW = w_out < 4 ? w_out : 4;
    while (((TH - 1) * stride + ks) * ((TW - 1) * stride + ks) > 144 && (TH > 1 || TW > 1)) {
        if (TW >= TH && TW > 1) TW = (TW + 1) / 2; else TH = (TH + 1) / 2;
    }
}

int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

struct Geometry {
    int TH, TW, THI, TWI, tiles_x, ntiles;
    int64_t chunks;
};

Geometry geometry(int64_t h_out, int64_t w_out, int stride, int ks, int64_t ncols) {
    Geometry g{};
    plane_tile((int)h_out, (int)w_out, stride, ks, g.TH, g.TW);
    g.THI = (g.TH - 1) * stride + ks;
    g.TWI = (g.TW - 1) * stride + ks;
    g.tiles_x = (int)cdiv(w_out, g.TW);
    g.ntiles = (int)(cdiv(h_out, g.TH) * g.tiles_x);
    g.chunks = cdiv(ncols, kCols);
    return g;
}

size_t fwd_smem(const Geometry& g, int cg, int K) {
    return (size_t)(g.THI * g.TWI + 1) * kRowBytes + 16 + (size_t)cg * K * (16 + 8) + (size_t)cg * 16;
}

size_t bwd_smem(const Geometry& g, int cg, int K, bool gx) {
    (void)gx;
    return (size_t)(g.THI * g.TWI + 1) * kRowBytes + 16 +
           (size_t)cg * K * (16 + 8 + 4 + 4 + 8) + (size_t)cg * 4;
}

constexpr size_t kMaxSmem = 200 * 1024;

int check_plane(int dtype, const void* x, int64_t ldx, int64_t ncols, int64_t c_in, int64_t h_in, int64_t w_in,
                int64_t c_out, int64_t h_out, int64_t w_out, int stride, int pad, int ks, int64_t K,
                const int8_t* oh, const int8_t* ow, const int32_t* order, const int32_t* starts, int64_t max_group,
                int mode, const void* weights, const uint8_t* gates) {
    if (dtype != CLB_F32) return set_error(CLB_ERR_DTYPE, "conv plane kernels: fp32 only");
    if (c_in < 1 || h_in < 1 || w_in < 1 || c_out < 1 || h_out < 1 || w_out < 1 || stride < 1 || ks < 1 || pad < 0 ||
        K < 1 || max_group < 1 || ncols < 0 || ldx < ncols || c_in > 65535)
        return set_error(CLB_ERR_INVALID, "conv plane: bad geometry");
    if ((h_out - 1) * stride + ks > h_in + 2 * pad || (w_out - 1) * stride + ks > w_in + 2 * pad)
        return set_error(CLB_ERR_INVALID, "conv plane: output larger than the padded input allows");
    if (ncols % 4 || ldx % 4 || (uintptr_t)x % 16) return set_error(CLB_ERR_INVALID, "conv plane: x needs 16-byte rows");
    if (!oh || !ow || !order || !starts || !gates) return set_error(CLB_ERR_INVALID, "conv plane: null table");
    if (mode != CLB_W_SELECT && !weights) return set_error(CLB_ERR_INVALID, "conv plane: null weights");
    if (cdiv(ncols, kCols) > 65535) return set_error(CLB_ERR_INVALID, "conv plane: too many columns");
    return CLB_OK;
}

PlaneArgs plane_args(const void* x, int64_t ldx, int64_t ncols, int64_t c_in, int64_t h_in, int64_t w_in,
                     int64_t c_out, int64_t h_out, int64_t w_out, int stride, int pad, int ks, int64_t K,
                     const int8_t* oh, const int8_t* ow, const int32_t* order, const int32_t* starts,
                     int64_t max_group, int mode, const void* weights, const uint8_t* gates, const uint8_t* select,
                     const Geometry& g, int32_t* err) {
    PlaneArgs a{};
    a.x = reinterpret_cast<const float*>(x);
    a.ldx = ldx;
    a.ncols = ncols;
    a.c_in = (int)c_in;
    a.h_in = (int)h_in;
    a.w_in = (int)w_in;
    a.c_out = (int)c_out;
    a.h_out = (int)h_out;
    a.w_out = (int)w_out;
    a.stride = stride;
    a.pad = pad;
    a.ks = ks;
    a.K = (int)K;
    a.oh = oh;
    a.ow = ow;
    a.order = order;
    a.starts = starts;
    a.cg = (int)(max_group < kChanBatch ? max_group : kChanBatch);
    a.mode = mode;
    a.weights = reinterpret_cast<const float*>(weights);
    a.gates = gates;
    a.select = select;
    a.TH = g.TH;
    a.TW = g.TW;
    a.THI = g.THI;
    a.TWI = g.TWI;
    a.tiles_x = g.tiles_x;
    a.ntiles = g.ntiles;
    a.err = err;
    return a;
}

template <int KT, bool GX>
cudaError_t bwd_launch(const PlaneArgs& a, const Geometry& g, const float* gy, int64_t ldgy, float* gx, int64_t ldgx,
                       float* part, cudaStream_t s) {
    const size_t smem = bwd_smem(g, a.cg, KT, GX);
    auto k = conv_plane_backward_kernel<KT, GX>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k<<<dim3((unsigned)g.ntiles, (unsigned)a.c_in, (unsigned)g.chunks), kThreads, smem, s>>>(a, gy, ldgy, gx, ldgx,
                                                                                           part);
    return cudaGetLastError();
}

}  // namespace

}  // namespace clb

using namespace clb;

extern "C" int64_t clb_conv_plane_parts(int64_t h_out, int64_t w_out, int stride, int ks, int64_t ncols) {
    if (h_out < 1 || w_out < 1 || stride < 1 || ks < 1 || ncols < 0) return -1;
    const Geometry g = geometry(h_out, w_out, stride, ks, ncols);
    return g.chunks * g.ntiles;
}

extern "C" int clb_conv_plane_forward(int dtype, const void* x, int64_t ldx, int64_t ncols, int64_t c_in, int64_t h_in,
                                      int64_t w_in, int64_t c_out, int64_t h_out, int64_t w_out, int stride, int pad,
                                      int ks, int64_t K, const int8_t* off_h, const int8_t* off_w,
                                      const int32_t* order, const int32_t* starts, int64_t max_group,
                                      int weight_mode, const void* weights, const uint8_t* gates,
                                      const uint8_t* select, void* y, int64_t ldy, int32_t* err,
                                      clb_stream_t stream) {
    int st = check_plane(dtype, x, ldx, ncols, c_in, h_in, w_in, c_out, h_out, w_out, stride, pad, ks, K, off_h,
                         off_w, order, starts, max_group, weight_mode, weights, gates);
    if (st) return st;
    if (weight_mode == CLB_W_SELECT && !select) return set_error(CLB_ERR_INVALID, "conv plane: null select");
    if (K != 2 && K != 4 && K != 8 && K != 16 && K != 32)
        return set_error(CLB_ERR_INVALID, "conv plane forward: K must be a power of two <= 32");
    if (!y || ldy < ncols || ldy % 4 || (uintptr_t)y % 16) return set_error(CLB_ERR_INVALID, "conv plane: bad y");
    if (ncols == 0) return CLB_OK;
    const Geometry g = geometry(h_out, w_out, stride, ks, ncols);
    const PlaneArgs a = plane_args(x, ldx, ncols, c_in, h_in, w_in, c_out, h_out, w_out, stride, pad, ks, K, off_h,
                                   off_w, order, starts, max_group, weight_mode, weights, gates, select, g, err);
    const size_t smem = fwd_smem(g, a.cg, (int)K);
    if (smem > kMaxSmem) return set_error(CLB_ERR_INVALID, "conv plane: receptive field too large for shared memory");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const dim3 grid((unsigned)g.ntiles, (unsigned)c_in, (unsigned)g.chunks);
    auto k = weight_mode == CLB_W_SELECT ? conv_plane_forward_kernel<true> : conv_plane_forward_kernel<false>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k<<<grid, kThreads, smem, s>>>(a, reinterpret_cast<float*>(y), ldy);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(CLB_ERR_CUDA, cudaGetErrorString(e));
    count_launches(1);
    return CLB_OK;
}

extern "C" int clb_conv_plane_backward(int dtype, const void* x, int64_t ldx, int64_t ncols, int64_t c_in,
                                       int64_t h_in, int64_t w_in, int64_t c_out, int64_t h_out, int64_t w_out,
                                       int stride, int pad, int ks, int64_t K, const int8_t* off_h,
                                       const int8_t* off_w, const int32_t* order, const int32_t* starts,
                                       int64_t max_group, int weight_mode, const void* weights, const uint8_t* gates,
                                       const void* grad_y, int64_t ldgy, void* grad_x, int64_t ldgx, int zero_grad_x,
                                       void* partials, int64_t nparts, int32_t* err, clb_stream_t stream) {
    int st = check_plane(dtype, x, ldx, ncols, c_in, h_in, w_in, c_out, h_out, w_out, stride, pad, ks, K, off_h,
                         off_w, order, starts, max_group, weight_mode, weights, gates);
    if (st) return st;
    if (weight_mode == CLB_W_SELECT) return set_error(CLB_ERR_INVALID, "conv plane backward: select mode has no gradient");
    if (K != 4 && K != 8 && K != 16) return set_error(CLB_ERR_INVALID, "conv plane backward: K must be 4, 8 or 16");
    if (!grad_y || ldgy < ncols || ldgy % 4 || (uintptr_t)grad_y % 16)
        return set_error(CLB_ERR_INVALID, "conv plane backward: bad grad_y");
    if (grad_x && (ldgx < ncols || ldgx % 4 || (uintptr_t)grad_x % 16))
        return set_error(CLB_ERR_INVALID, "conv plane backward: bad grad_x");
    const Geometry g = geometry(h_out, w_out, stride, ks, ncols);
    if (!partials || nparts != g.chunks * g.ntiles)
        return set_error(CLB_ERR_INVALID, "conv plane backward: partials must hold clb_conv_plane_parts() blocks");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (grad_x && zero_grad_x) {
        const cudaError_t e = cudaMemsetAsync(grad_x, 0, sizeof(float) * (size_t)(c_in * h_in * w_in) * (size_t)ldgx, s);
        if (e != cudaSuccess) return set_error(CLB_ERR_CUDA, cudaGetErrorString(e));
    }
    if (ncols == 0) {
        const cudaError_t e = cudaMemsetAsync(partials, 0, sizeof(float) * (size_t)(nparts * c_out * K), s);
        return e == cudaSuccess ? CLB_OK : set_error(CLB_ERR_CUDA, cudaGetErrorString(e));
    }
    const PlaneArgs a = plane_args(x, ldx, ncols, c_in, h_in, w_in, c_out, h_out, w_out, stride, pad, ks, K, off_h,
                                   off_w, order, starts, max_group, weight_mode, weights, gates, nullptr, g, err);
    if (bwd_smem(g, a.cg, (int)K, grad_x != nullptr) > kMaxSmem)
        return set_error(CLB_ERR_INVALID, "conv plane: receptive field too large for shared memory");
    const float* gyp = reinterpret_cast<const float*>(grad_y);
    float* gxp = reinterpret_cast<float*>(grad_x);
    float* pp = reinterpret_cast<float*>(partials);
    cudaError_t e;
    switch (K) {
        case 4: e = gxp ? bwd_launch<4, true>(a, g, gyp, ldgy, gxp, ldgx, pp, s) : bwd_launch<4, false>(a, g, gyp, ldgy, gxp, ldgx, pp, s); break;
        case 8: e = gxp ? bwd_launch<8, true>(a, g, gyp, ldgy, gxp, ldgx, pp, s) : bwd_launch<8, false>(a, g, gyp, ldgy, gxp, ldgx, pp, s); break;
        default: e = gxp ? bwd_launch<16, true>(a, g, gyp, ldgy, gxp, ldgx, pp, s) : bwd_launch<16, false>(a, g, gyp, ldgy, gxp, ldgx, pp, s); break;
    }
    if (e != cudaSuccess) return set_error(CLB_ERR_CUDA, cudaGetErrorString(e));
    count_launches(1);
    return CLB_OK;
}
