// Gather-form fused backward of a logic layer: destination-sorted, no scatter reductions.
//
// The scatter backward (logic_layer.cu) walks slots and adds each slot's activation gradient into
// grad_x with L2 reductions.  Here the work is walked by destination instead: a per-layer index lists,
// for every input feature i, the slot operands that read it ("occurrences", sorted owners first, then by slot, so the
// summation order is fixed for a given index).  One warp owns one input row and one column chunk;
// for each occurrence it gathers the other operand's row and grad_y of the slot's neuron, and
//   grad_x[i, n]        += p * (c_self + c3 * x_other) * gy[j, n]       (difflogic_kernel.cu:140-194)
//   d loss / d p[j, k]  = sum_n gy[j, n] * f(a, b)                      (difflogic_kernel.cu:82-137)
// the second written by exactly one occurrence per slot (its "owner"), into the same per-chunk
// partials [nchunks, n_out, K] the scatter backward produces, so clb_logic_grad_finalize folds both.
// grad_x is stored once per element (no pre-zeroing, no atomics).
//
// Occurrence record: int2 {other operand row or -1, meta}, meta = slot << 7 | zero << 6 | owner << 5 |
// side << 4 | gate id.  side 0 = the occurrence is operand a of the slot, 1 = operand b.  Operands a
// gate ignores get no occurrence (and read as -1 when they are the other operand).  A slot with no
// occurrence at all (a constant gate, or every used operand is zero padding) still needs its
// d loss / d p = c0 * sum_n gy[j, n]: it gets one "virtual" occurrence on row j % in_features with
// the zero flag set, which evaluates the gate with its own operand read as 0 and adds nothing to
// grad_x.
//
// Index layout (bytes, each part 256-aligned): starts int32 [in + 1], tmp int2 [2 * n_out * K] (the
// unsorted fill), recs int2 [2 * n_out * K], cursor int32 [in], baked 2 x int4 [2 * n_out * K] (rewritten every
// step by the fp32 path: see bake_kernel).
#include <cuda_runtime.h>
#include <float.h>
#include <stdint.h>
#include <stdlib.h>

#include <type_traits>

#include "common.cuh"
#include "gates.cuh"
#include "kernels.h"

namespace clb {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int64_t kMaxSlots = int64_t(1) << 24;  // slot id field of the record

size_t round256(size_t v) { return (v + 255) & ~size_t(255); }

struct IndexParts {
    int32_t* starts;
    int2* tmp;
    int2* recs;
    int32_t* cursor;
    int4* baked;  // per-step records of the fast fp32 path (see bake_kernel)
    size_t bytes;
};

IndexParts index_parts(void* base, int64_t n_out, int64_t K, int64_t in_features) {
    IndexParts p{};
    unsigned char* b = reinterpret_cast<unsigned char*>(base);
    const size_t s_starts = round256(sizeof(int32_t) * (size_t)(in_features + 1));
    const size_t s_recs = round256(sizeof(int2) * (size_t)(2 * n_out * K));
    const size_t s_cursor = round256(sizeof(int32_t) * (size_t)in_features);
    p.starts = reinterpret_cast<int32_t*>(b);
    p.tmp = reinterpret_cast<int2*>(b + s_starts);
    p.recs = reinterpret_cast<int2*>(b + s_starts + s_recs);
    p.cursor = reinterpret_cast<int32_t*>(b + s_starts + 2 * s_recs);
    p.baked = reinterpret_cast<int4*>(b + s_starts + 2 * s_recs + s_cursor);
    p.bytes = s_starts + 2 * s_recs + s_cursor + round256(2 * sizeof(int4) * (size_t)(2 * n_out * K));
    return p;
}

__device__ __forceinline__ bool uses_a(const GatePoly& g) { return g.c1 != 0.f || g.c3 != 0.f; }
__device__ __forceinline__ bool uses_b(const GatePoly& g) { return g.c2 != 0.f || g.c3 != 0.f; }

// The occurrences of slot (j, k): up to two records, each with its destination row.
__device__ __forceinline__ int slot_occurrences(const int2* slots, const uint8_t* gates, int64_t j, int K, int64_t k,
                                                int64_t group, int64_t in_features, int (&row)[2], int2 (&rec)[2]) {
    const int64_t slot = j * K + k;
    const int g = gates[(j / group) * K + k] & 15;
    const GatePoly gp = gate_poly(g);
    const int2 s = slots[slot];
    const bool ha = uses_a(gp) && s.x >= 0, hb = uses_b(gp) && s.y >= 0;
    const int oa = uses_b(gp) ? s.y : -1, ob = uses_a(gp) ? s.x : -1;  // the other operand, if it is used
    const int base = (int)(slot << 7) | g;
    int n = 0;
    if (ha) {
        row[n] = s.x;
        rec[n++] = make_int2(oa, base | (1 << 5));
    }
    if (hb) {
        row[n] = s.y;
        rec[n++] = make_int2(ob, base | (ha ? 0 : 1 << 5) | (1 << 4));
    }
    if (n == 0) {
        row[n] = (int)(j % in_features);
        rec[n++] = make_int2(-1, base | (1 << 6) | (1 << 5));
    }
    return n;
}

__global__ void index_count_kernel(const int2* slots, const uint8_t* gates, int64_t n_out, int K, int64_t group,
                                   int64_t in_features, int32_t* counts) {
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= n_out * K) return;
    int row[2];
    int2 rec[2];
    const int n = slot_occurrences(slots, gates, e / K, K, e % K, group, in_features, row, rec);
    for (int i = 0; i < n; ++i) atomicAdd(counts + row[i], 1);
}

// Exclusive scan of counts[0, n) into starts[0, n], one CTA.
__global__ void __launch_bounds__(1024) index_scan_kernel(const int32_t* counts, int64_t n, int32_t* starts,
                                                          int32_t* cursor) {
    __shared__ int32_t part[1024];
    const int t = threadIdx.x;
    const int64_t per = (n + 1023) / 1024;
    const int64_t lo = t * per < n ? t * per : n, hi = lo + per < n ? lo + per : n;
    int32_t s = 0;
    for (int64_t i = lo; i < hi; ++i) s += counts[i];
    part[t] = s;
    __syncthreads();
    for (int o = 1; o < 1024; o <<= 1) {
        const int32_t v = t >= o ? part[t - o] : 0;
        __syncthreads();
        part[t] += v;
        __syncthreads();
    }
    int32_t run = part[t] - s;
    for (int64_t i = lo; i < hi; ++i) {
        const int32_t c = counts[i];  // counts may alias cursor
        starts[i] = run;
        cursor[i] = run;
        run += c;
    }
    if (t == 1023) starts[n] = part[1023];
}

__global__ void index_fill_kernel(const int2* slots, const uint8_t* gates, int64_t n_out, int K, int64_t group,
                                  int64_t in_features, int32_t* cursor, int2* tmp) {
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= n_out * K) return;
    int row[2];
    int2 rec[2];
    const int n = slot_occurrences(slots, gates, e / K, K, e % K, group, in_features, row, rec);
    for (int i = 0; i < n; ++i) tmp[atomicAdd(cursor + row[i], 1)] = rec[i];
}

// Sort key of a record: owners (bit 5 of meta) first, then by meta (unique per slot and side).
__device__ __forceinline__ uint64_t occ_key(int meta) {
    return ((uint64_t)(((meta >> 5) & 1) ^ 1) << 32) | (uint32_t)meta;
}

// Order each row's occurrences by record key, owners first: rank sort, one warp per row.
__global__ void index_sort_kernel(const int32_t* starts, int64_t in_features, const int2* tmp, int2* recs) {
    const int64_t row = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= in_features) return;
    const int beg = starts[row], end = starts[row + 1];
    for (int e = beg + lane; e < end; e += 32) {
        const int2 r = tmp[e];
        const uint64_t key = occ_key(r.y);
        int rank = 0;
        for (int q = beg; q < end; ++q) rank += occ_key(tmp[q].y) < key;
        recs[beg + rank] = r;
    }
}

__device__ __forceinline__ float exp_acc(float v) { return expf(v); }
__device__ __forceinline__ double exp_acc(double v) { return exp(v); }

// Per-step probabilities p[r, k]: softmax of the logits (compactlogic.py:108), or the probabilities as given.
template <typename A>
__global__ void softmax_rows_kernel(const A* w, int64_t rows, int K, int mode, A* probs) {
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    const A* wr = w + r * K;
    A* pr = probs + r * K;
    if (mode != CLB_W_LOGITS) {
        for (int k = 0; k < K; ++k) pr[k] = wr[k];
        return;
    }
    A m = wr[0];
    for (int k = 1; k < K; ++k) m = wr[k] > m ? wr[k] : m;
    A s = 0;
    for (int k = 0; k < K; ++k) s += exp_acc(wr[k] - m);
    for (int k = 0; k < K; ++k) pr[k] = exp_acc(wr[k] - m) / s;
}

// Butterfly reduce-scatter of N per-lane values: afterwards lane l holds the warp sum of value
// (l >> (5 - log2 N)) & (N - 1).
template <typename A, int N, int OFF> struct RS {
    static __device__ __forceinline__ void run(A* v, int lane) {
        const bool up = (lane & OFF) != 0;
#pragma unroll
        for (int i = 0; i < N / 2; ++i) {
            const A send = up ? v[i] : v[i + N / 2];
            const A keep = up ? v[i + N / 2] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, OFF);
        }
        RS<A, N / 2, OFF / 2>::run(v, lane);
    }
};
template <typename A, int OFF> struct RS<A, 1, OFF> {
    static __device__ __forceinline__ void run(A* v, int lane) {
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], OFF);
        RS<A, 1, OFF / 2>::run(v, lane);
    }
};
template <typename A> struct RS<A, 1, 0> {
    static __device__ __forceinline__ void run(A*, int) {}
};

struct GatherArgs {
    const void* x;
    int64_t ldx;
    int64_t ncols;
    const void* gy;   // arithmetic type [n_out, ldgy], or null with the fused GroupSum
    int64_t ldgy;
    const void* gs_grad;
    int64_t gs_size;
    int64_t ld_gs;
    double gs_scale;
    void* gx;         // arithmetic type [in, ldgx], written
    int64_t ldgx;
    void* part;       // arithmetic type [nchunks, n_out, K] or null
    const void* probs;
    const int32_t* starts;
    const int2* recs;
    int4* baked;
    int2* tmp;  // the build's scratch: owner slot ids of the fast path
    int64_t in_features;
    int64_t n_out;
    int K;
    int64_t group;
    int split;  // gather2: light loop for non-owner occurrences (CLB_GATHER_SPLIT=0 turns it off)
};

// Gate coefficients of one occurrence, from the point of view of its own operand ("s", the row the
// warp owns) and the other operand ("o"): f = c0 + cs s + co o + c3 s o.  Indexed by
// gate | side << 4 | zero << 5 | absent << 6 (absent: the other operand is not read, the warp reads its
// own row in its place).  zero clears cs and c3 (the own operand reads as 0 and receives no gradient);
// absent clears co and c3 (the other operand is 0 or ignored).
template <typename A> struct Coef { A c0, cs, co, c3; };

__device__ __forceinline__ int occ_code(int meta, bool absent) { return (meta & 15) | ((meta >> 4 & 1) << 4) | ((meta >> 6 & 1) << 5) | (absent ? 64 : 0); }

// One warp per (input row, column chunk); U occurrences in flight per step.  I is the index type of
// element offsets (int when every operand fits 2^31 elements).
template <typename T, int VEC, int U, typename I>
__global__ void __launch_bounds__(kThreads, U == 4 ? 3 : 1) logic_backward_gather_kernel(const GatherArgs a) {
    using Ac = typename Acc<T>::type;
    __shared__ Coef<Ac> tab[128];
    if (threadIdx.x < 128) {
        const int c = threadIdx.x;
        const GatePoly gp = gate_poly(c & 15);
        const bool side_b = c >> 4 & 1, zero = c >> 5 & 1, absent = c >> 6 & 1;
        Coef<Ac> e;
        e.c0 = (Ac)gp.c0;
        e.cs = zero ? (Ac)0 : (Ac)(side_b ? gp.c2 : gp.c1);
        e.co = absent ? (Ac)0 : (Ac)(side_b ? gp.c1 : gp.c2);
        e.c3 = (zero || absent) ? (Ac)0 : (Ac)gp.c3;
        tab[c] = e;
    }
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const I row = (I)((int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5));
    if (row >= (I)a.in_features) return;
    const int chunk = blockIdx.y;
    const I col = (I)chunk * (32 * VEC) + lane * VEC;
    const bool active = col < (I)a.ncols;
    const I lcol = active ? col : 0;  // inactive lanes read column 0 with a zero weight
    const T* __restrict__ x = reinterpret_cast<const T*>(a.x);
    const bool use_gs = a.gs_grad != nullptr;
    const Ac* __restrict__ gsrc = reinterpret_cast<const Ac*>(use_gs ? a.gs_grad : a.gy);
    const I ldg = (I)(use_gs ? a.ld_gs : a.ldgy), ldx = (I)a.ldx;
    const Ac* __restrict__ probs = reinterpret_cast<const Ac*>(a.probs);
    // grad_y scale (the fused GroupSum's): 0 on inactive lanes, whose column-0 reads then contribute
    // nothing (a non-finite value there is also read by lane 0 itself)
    const Ac gscale = active ? (Ac)(use_gs ? a.gs_scale : 1.0) : (Ac)0;
    const int K = a.K, group = (int)a.group, gs_size = (int)a.gs_size;

    Ac xi[VEC], acc[VEC];
#pragma unroll
    for (int i = 0; i < VEC; ++i) xi[i] = acc[i] = 0;
    if (active) load_acc<T, VEC>(x + row * ldx + col, xi);

    const int beg = a.starts[row], end = a.starts[row + 1];
    for (int base = beg; base < end; base += 32) {
        const int n = end - base < 32 ? end - base : 32;
        // per-lane decode of one record: other row (own row when absent), grad_y row, p, table code
        int lo = (int)row, lg = 0, lcode = 0, lmeta = 0;
        Ac lp = 0;
        if (lane < n) {
            const int2 rec = a.recs[base + lane];
            lmeta = rec.y;
            const int slot = (int)((uint32_t)rec.y >> 7);
            const int j = slot / K;
            lp = probs[(group == 1 ? j : j / group) * K + (slot - j * K)];
            lg = use_gs ? j / gs_size : j;
            lo = rec.x >= 0 ? rec.x : (int)row;
            lcode = occ_code(rec.y, rec.x < 0) | (rec.y & (1 << 5) ? 128 : 0);
        }
        for (int e = 0; e < n; e += U) {
            // phase 1: issue every gather of the U occurrences before any arithmetic
            Ac g[U][VEC], xo[U][VEC];
            int code[U];
            Ac pu[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int src = (e + u) & 31;
                const int o = __shfl_sync(0xffffffffu, lo, src);
                const int gr = __shfl_sync(0xffffffffu, lg, src);
                code[u] = __shfl_sync(0xffffffffu, lcode, src);
                pu[u] = __shfl_sync(0xffffffffu, lp, src);
                if (e + u < n) {  // warp-uniform
                    load_acc<Ac, VEC>(gsrc + (I)gr * ldg + lcol, g[u]);
                    load_acc<T, VEC>(x + (I)o * ldx + lcol, xo[u]);
                } else {
#pragma unroll
                    for (int i = 0; i < VEC; ++i) g[u][i] = xo[u][i] = 0;
                    code[u] = 0;  // gate 0: every coefficient zero
                }
            }
            // phase 2: the arithmetic
            Ac dot[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const Coef<Ac> c = tab[code[u] & 127];
                const Ac pcs = pu[u] * c.cs, pc3 = pu[u] * c.c3;
                Ac d = 0;
#pragma unroll
                for (int i = 0; i < VEC; ++i) {
                    const Ac gi = g[u][i] * gscale;
                    const Ac f = fma(fma(c.c3, xi[i], c.co), xo[u][i], fma(c.cs, xi[i], c.c0));
                    d = fma(gi, f, d);
                    acc[i] = fma(fma(pc3, xo[u][i], pcs), gi, acc[i]);
                }
                dot[u] = (code[u] & 128) ? d : (Ac)0;
            }
            if (a.part != nullptr) {
                constexpr int L = U == 8 ? 3 : U == 4 ? 2 : U == 2 ? 1 : 0;
                RS<Ac, U, 16>::run(dot, lane);
                const int u = (lane >> (5 - L)) & (U - 1);
                const int meta = __shfl_sync(0xffffffffu, lmeta, (e + u) & 31);
                if ((lane & ((1 << (5 - L)) - 1)) == 0 && e + u < n && ((meta >> 5) & 1)) {
                    const int64_t slot = (uint32_t)meta >> 7;
                    reinterpret_cast<Ac*>(a.part)[(int64_t)chunk * a.n_out * K + slot] = dot[0];
                }
            }
        }
    }
    if (active) store_from_acc<Ac, VEC>(reinterpret_cast<Ac*>(a.gx) + (int64_t)row * a.ldgx + col, acc);
}

// ---------------------------------------------------------------------------------------------
// Fast fp32 path.  Once per step (after the softmax) every occurrence is baked into a 32-byte record
//   { element offset of the other operand's row (-1: not read), element offset of its grad_y row,
//     p * c_self * s, p * c3 * s,                                   (s: the fused GroupSum's grad scale)
//     and, for the slot's owner occurrence only, the gate seen from the own operand (c0, cs, co, c3) * s,
//     zero otherwise }
// and its slot id (-1 when not the owner), so the walk does no decoding, no division, no table lookup and
// no branch per occurrence: a warp stages 32 records in shared memory (padded with zero records) and reads
// each as a broadcast, issues the two row gathers of 4 occurrences, then
//   grad_x[i] += (p c_self + p c3 x_other) * grad_y,   d loss / d p partial += grad_y * f(x_i, x_other)
// with the 4 partials reduced by a butterfly and stored by the owner's lanes.
// ---------------------------------------------------------------------------------------------
__global__ void bake_kernel(const int2* __restrict__ recs, const int32_t* __restrict__ n_valid, int64_t total,
                            const float* __restrict__ probs, int K, int64_t group, int64_t ldx, int use_gs,
                            int64_t gs_size, int64_t ldg, float scale, int4* __restrict__ baked,
                            int* __restrict__ owner_slot) {
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    // the record array has room for 2 n_out K occurrences; only the first starts[in_features] are filled
    if (e >= total || e >= (int64_t)*n_valid) return;
    const int2 rec = recs[e];
    const int meta = rec.y;
    const int64_t slot = (uint32_t)meta >> 7;
    const int64_t j = slot / K, k = slot - j * K;
    const float p = probs[(group == 1 ? j : j / group) * K + k];
    const GatePoly gp = gate_poly(meta & 15);
    const bool side_b = (meta >> 4) & 1, owner = (meta >> 5) & 1, zero = (meta >> 6) & 1, absent = rec.x < 0;
    const float cs = zero ? 0.f : (side_b ? gp.c2 : gp.c1);
    const float co = absent ? 0.f : (side_b ? gp.c1 : gp.c2);
    const float c3 = (zero || absent) ? 0.f : gp.c3;
    baked[2 * e] = make_int4(absent ? -1 : (int)((int64_t)rec.x * ldx), (int)((use_gs ? j / gs_size : j) * ldg),
                             __float_as_int(p * cs * scale), __float_as_int(p * c3 * scale));
    const float d = owner ? scale : 0.f;
    baked[2 * e + 1] = make_int4(__float_as_int(gp.c0 * d), __float_as_int(cs * d), __float_as_int(co * d),
                                 __float_as_int(c3 * d));
    owner_slot[e] = owner ? (int)slot : -1;
}

// Broadcast read of a staged 16-byte record as one 128-bit, two 64-bit or four 32-bit shared loads.
template <int LDW>
__device__ __forceinline__ int4 lds_rec(const int4* p) {
    const unsigned a = (unsigned)__cvta_generic_to_shared(p);
    int4 r;
    if constexpr (LDW == 2) {  // inline PTX so the two halves are not fused into one 128-bit load
        asm volatile("ld.shared.v2.s32 {%0, %1}, [%2];" : "=r"(r.x), "=r"(r.y) : "r"(a));
        asm volatile("ld.shared.v2.s32 {%0, %1}, [%2];" : "=r"(r.z), "=r"(r.w) : "r"(a + 8));
    } else if constexpr (LDW == 4) {
        asm volatile("ld.shared.s32 %0, [%1];" : "=r"(r.x) : "r"(a));
        asm volatile("ld.shared.s32 %0, [%1];" : "=r"(r.y) : "r"(a + 4));
        asm volatile("ld.shared.s32 %0, [%1];" : "=r"(r.z) : "r"(a + 8));
        asm volatile("ld.shared.s32 %0, [%1];" : "=r"(r.w) : "r"(a + 12));
    } else {
        r = *p;
    }
    return r;
}

template <typename T, int kU2, int MINB, int LDW = 1>  // activation type, occurrences in flight per warp step, CTAs per SM, record read width
__global__ void __launch_bounds__(kThreads, MINB) logic_backward_gather2_kernel(
    const GatherArgs a, const int4* __restrict__ baked, const int* __restrict__ owner_slot) {
    __shared__ int4 srec[kWarps][2 * 32];
    __shared__ int sslot[kWarps][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int row = blockIdx.x * kWarps + warp;
    if (row >= (int)a.in_features) return;
    const int chunk = blockIdx.y;
    const int col = chunk * 128 + lane * 4;
    const bool active = col < (int)a.ncols;
    const int lcol = active ? col : 0;  // inactive lanes read column 0; their results are dropped
    const T* __restrict__ x = reinterpret_cast<const T*>(a.x);
    const float* __restrict__ gsrc = reinterpret_cast<const float*>(a.gs_grad != nullptr ? a.gs_grad : a.gy);
    const int rowoff = row * (int)a.ldx;
    float* part = reinterpret_cast<float*>(a.part);
    const int64_t pbase = (int64_t)chunk * a.n_out * a.K;
    float xs[4];
    load_acc<T, 4>(x + rowoff + lcol, xs);
#pragma unroll
    for (int i = 0; i < 4; ++i) xs[i] = active ? xs[i] : 0.f;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    const int beg = a.starts[row], end = a.starts[row + 1];
    for (int base = beg; base < end; base += 32) {
        const int n = min(32, end - base);
        __syncwarp();
        const int my_slot = lane < n ? owner_slot[base + lane] : -1;
        if (lane < n) {
            srec[warp][2 * lane] = baked[2 * (base + lane)];
            srec[warp][2 * lane + 1] = baked[2 * (base + lane) + 1];
        } else {  // zero records: own row, coefficient 0, no owner
            srec[warp][2 * lane] = make_int4(-1, 0, 0, 0);
            srec[warp][2 * lane + 1] = make_int4(0, 0, 0, 0);
        }
        sslot[warp][lane] = my_slot;
        // The index lists a row's owner occurrences first, so the owners of this batch are a prefix of it:
        // only they need the gate value, the d loss / d p reduction and its store.  The rest (the second
        // operand of two-operand slots) take the light loop below.  Not a prefix: the whole batch is full.
        const unsigned om = __ballot_sync(0xffffffffu, my_slot >= 0);
        const int nown = __popc(om);
        const int split = part == nullptr ? 0
                          : a.split && om == (nown == 32 ? 0xffffffffu : (1u << nown) - 1u) ? min(n, (nown + kU2 - 1) / kU2 * kU2)
                                                                                  : n;
        __syncwarp();
        for (int e = 0; e < split; e += kU2) {
            float xo[kU2][4];
            float4 g[kU2];
            int4 r[kU2];
#pragma unroll
            for (int u = 0; u < kU2; ++u) {
                r[u] = lds_rec<LDW>(&srec[warp][2 * ((e + u) & 31)]);
                if (!std::is_same<T, float>::value) {  // 16-bit rows: the unconditional load measured faster
                    load_acc<T, 4>(x + (r[u].x >= 0 ? r[u].x : rowoff) + lcol, xo[u]);
                } else if (r[u].x >= 0) {  // warp-uniform: absent other operands (zero coefficients) issue no load
                    load_acc<T, 4>(x + r[u].x + lcol, xo[u]);
                } else {
#pragma unroll
                    for (int i = 0; i < 4; ++i) xo[u][i] = 0.f;
                }
                g[u] = *reinterpret_cast<const float4*>(gsrc + r[u].y + lcol);
            }
            float dot[kU2];
#pragma unroll
            for (int u = 0; u < kU2; ++u) {
                const int4 cd = lds_rec<LDW>(&srec[warp][2 * ((e + u) & 31) + 1]);
                const float pcs = __int_as_float(r[u].z), pc3 = __int_as_float(r[u].w);
                const float c0 = __int_as_float(cd.x), cs = __int_as_float(cd.y), co = __int_as_float(cd.z),
                            c3 = __int_as_float(cd.w);
                const float* o = xo[u];
                const float gg[4] = {g[u].x, g[u].y, g[u].z, g[u].w};
                float d = 0.f;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    acc[i] = fmaf(fmaf(pc3, o[i], pcs), gg[i], acc[i]);
                    d = fmaf(gg[i], fmaf(fmaf(c3, xs[i], co), o[i], fmaf(cs, xs[i], c0)), d);
                }
                dot[u] = active ? d : 0.f;
            }
            if (part != nullptr) {
                RS<float, kU2, 16>::run(dot, lane);
                constexpr int SH = kU2 == 8 ? 2 : kU2 == 4 ? 3 : 4;  // log2(lanes per reduced value) = 5 - log2(kU2)
                const int slot = sslot[warp][(e + ((lane >> SH) & (kU2 - 1))) & 31];
                if ((lane & ((1 << SH) - 1)) == 0 && slot >= 0) part[pbase + slot] = dot[0];
            }
        }
        // light loop: grad_x only (records past n are zero records)
        for (int e = split; e < n; e += kU2) {
            float xo[kU2][4];
            float4 g[kU2];
            int4 r[kU2];
#pragma unroll
            for (int u = 0; u < kU2; ++u) {
                r[u] = lds_rec<LDW>(&srec[warp][2 * ((e + u) & 31)]);
                if (!std::is_same<T, float>::value) {  // 16-bit rows: the unconditional load measured faster
                    load_acc<T, 4>(x + (r[u].x >= 0 ? r[u].x : rowoff) + lcol, xo[u]);
                } else if (r[u].x >= 0) {  // warp-uniform: absent other operands (zero coefficients) issue no load
                    load_acc<T, 4>(x + r[u].x + lcol, xo[u]);
                } else {
#pragma unroll
                    for (int i = 0; i < 4; ++i) xo[u][i] = 0.f;
                }
                g[u] = *reinterpret_cast<const float4*>(gsrc + r[u].y + lcol);
            }
#pragma unroll
            for (int u = 0; u < kU2; ++u) {
                const float pcs = __int_as_float(r[u].z), pc3 = __int_as_float(r[u].w);
                const float gg[4] = {g[u].x, g[u].y, g[u].z, g[u].w};
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[i] = fmaf(fmaf(pc3, xo[u][i], pcs), gg[i], acc[i]);
            }
        }
    }
    if (active) *reinterpret_cast<float4*>(reinterpret_cast<float*>(a.gx) + (int64_t)row * a.ldgx + col) =
        make_float4(acc[0], acc[1], acc[2], acc[3]);
}

// The 4 pieces (columns p + 32 m .. p + 32 m + 3, m = 0..3) of a gather4 lane's share of a row.
template <typename T>
__device__ __forceinline__ void load_pieces(const T* __restrict__ p, float (&out)[16]) {
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        float v[4];
        load_acc<T, 4>(p + 32 * m, v);
#pragma unroll
        for (int i = 0; i < 4; ++i) out[4 * m + i] = v[i];
    }
}

// Variant of logic_backward_gather2_kernel with 8 lanes per occurrence: lane (q, c) = (lane / 8, lane % 8)
// owns columns 32 m + 4 c .. 32 m + 4 c + 3 (m = 0..3) of the 128-column chunk, so each 4-column load of
// a quarter-warp is one contiguous 128-byte piece of a row, and works on occurrence e + q, so one warp step
// covers 4 occurrences.  A 128-bit shared-memory read then fetches 4 different records (one per
// quarter-warp) instead of broadcasting one record to all 32 lanes (several wavefronts for one record),
// the gate-value dot product is reduced over 8 lanes (3 shuffles per 4 occurrences instead of a 6-shuffle
// butterfly), and the 4 partial grad_x rows are summed once per row by a 2-step reduce-scatter at the
// end.  Row gathers stay 512 bytes per occurrence (8 lanes x 4 pieces of 16 bytes).  Needs ncols % 128 == 0.
template <typename T, int MINB>
__global__ void __launch_bounds__(kThreads, MINB) logic_backward_gather4_kernel(
    const GatherArgs a, const int4* __restrict__ baked, const int* __restrict__ owner_slot) {
    constexpr int C = 16;  // columns per lane
    __shared__ int4 srec[kWarps][2 * 32];
    __shared__ int sslot[kWarps][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int q = lane >> 3, cg = lane & 7;
    const int row = blockIdx.x * kWarps + warp;
    if (row >= (int)a.in_features) return;
    const int chunk = blockIdx.y;
    const int lcol = chunk * 128 + cg * 4;  // + 32 m for piece m; every column is < ncols
    const T* __restrict__ x = reinterpret_cast<const T*>(a.x);
    const float* __restrict__ gsrc = reinterpret_cast<const float*>(a.gs_grad != nullptr ? a.gs_grad : a.gy);
    const int rowoff = row * (int)a.ldx;
    float* part = reinterpret_cast<float*>(a.part);
    const int64_t pbase = (int64_t)chunk * a.n_out * a.K;
    float xs[C];
    load_pieces<T>(x + rowoff + lcol, xs);
    float acc[C];
#pragma unroll
    for (int i = 0; i < C; ++i) acc[i] = 0.f;
    const int beg = a.starts[row], end = a.starts[row + 1];
    for (int base = beg; base < end; base += 32) {
        const int n = min(32, end - base);
        __syncwarp();
        const int my_slot = lane < n ? owner_slot[base + lane] : -1;
        if (lane < n) {
            srec[warp][2 * lane] = baked[2 * (base + lane)];
            srec[warp][2 * lane + 1] = baked[2 * (base + lane) + 1];
        } else {  // zero records: own row, coefficient 0, no owner
            srec[warp][2 * lane] = make_int4(-1, 0, 0, 0);
            srec[warp][2 * lane + 1] = make_int4(0, 0, 0, 0);
        }
        sslot[warp][lane] = my_slot;
        // owners first (see gather2): they need the gate value and its reduction, the rest only grad_x
        const unsigned om = __ballot_sync(0xffffffffu, my_slot >= 0);
        const int nown = __popc(om);
        const int split = part == nullptr ? 0
                          : a.split && om == (nown == 32 ? 0xffffffffu : (1u << nown) - 1u)
                              ? min(n, (nown + 3) & ~3)
                              : n;
        __syncwarp();
        for (int e = 0; e < split; e += 4) {
            const int o = (e + q) & 31;
            const int4 r = srec[warp][2 * o];
            float xo[C], g[C];
            if (r.x >= 0) {
                load_pieces<T>(x + r.x + lcol, xo);
            } else {
#pragma unroll
                for (int i = 0; i < C; ++i) xo[i] = 0.f;
            }
            load_pieces<float>(gsrc + r.y + lcol, g);
            const int4 cd = srec[warp][2 * o + 1];
            const float pcs = __int_as_float(r.z), pc3 = __int_as_float(r.w);
            const float c0 = __int_as_float(cd.x), cs = __int_as_float(cd.y), co = __int_as_float(cd.z),
                        c3 = __int_as_float(cd.w);
            float d = 0.f;
#pragma unroll
            for (int i = 0; i < C; ++i) {
                acc[i] = fmaf(fmaf(pc3, xo[i], pcs), g[i], acc[i]);
                d = fmaf(g[i], fmaf(fmaf(c3, xs[i], co), xo[i], fmaf(cs, xs[i], c0)), d);
            }
            d += __shfl_xor_sync(0xffffffffu, d, 4);
            d += __shfl_xor_sync(0xffffffffu, d, 2);
            d += __shfl_xor_sync(0xffffffffu, d, 1);
            if (part != nullptr && cg == 0) {
                const int slot = sslot[warp][o];
                if (slot >= 0) part[pbase + slot] = d;
            }
        }
        for (int e = split; e < n; e += 4) {  // non-owners: grad_x only (records past n are zero records)
            const int4 r = srec[warp][2 * ((e + q) & 31)];
            float xo[C], g[C];
            if (r.x >= 0) {
                load_pieces<T>(x + r.x + lcol, xo);
            } else {
#pragma unroll
                for (int i = 0; i < C; ++i) xo[i] = 0.f;
            }
            load_pieces<float>(gsrc + r.y + lcol, g);
            const float pcs = __int_as_float(r.z), pc3 = __int_as_float(r.w);
#pragma unroll
            for (int i = 0; i < C; ++i) acc[i] = fmaf(fmaf(pc3, xo[i], pcs), g[i], acc[i]);
        }
    }
    // sum the 4 occurrence groups' rows: after the two steps lane (q, c) holds the total of piece m = q
    {
        const bool up = (lane & 16) != 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float send = up ? acc[i] : acc[i + 8];
            const float keep = up ? acc[i + 8] : acc[i];
            acc[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
        }
        const bool up2 = (lane & 8) != 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float send = up2 ? acc[i] : acc[i + 4];
            const float keep = up2 ? acc[i + 4] : acc[i];
            acc[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
        }
    }
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(a.gx) + (int64_t)row * a.ldgx + lcol + 32 * q) =
        make_float4(acc[0], acc[1], acc[2], acc[3]);
}

// The fast (baked) path applies to fp32 / bf16 / fp16 activations with whole 4-column vectors and every element offset below 2^31.
bool fast_ok(const GatherArgs& a) {
    static const bool enabled = [] {
        const char* e = getenv("CLB_GATHER_FAST");
        return !(e && e[0] == '0');
    }();
    const int64_t lim = int64_t(1) << 31;
    const int64_t gext = a.gs_grad ? (a.n_out / a.gs_size + 1) * a.ld_gs : a.n_out * a.ldgy;
    return enabled && a.in_features * a.ldx < lim && gext < lim && a.ncols < lim && a.ldgx * a.in_features < lim;
}

template <typename T> constexpr int gvec() { return 16 / (int)sizeof(T) > 4 ? 4 : 16 / (int)sizeof(T); }

inline bool al(const void* p, int bytes) { return p == nullptr || ((uintptr_t)p % bytes) == 0; }

// Vector width of the gather backward for these pointers / strides (1 if any breaks alignment).
template <typename T>
int gather_vec(const GatherArgs& a) {
    using Ac = typename Acc<T>::type;
    constexpr int V = gvec<T>();
    const bool ok = a.ncols % V == 0 && a.ldx % V == 0 && a.ldgx % V == 0 &&
                    (a.gy == nullptr || a.ldgy % V == 0) && (a.gs_grad == nullptr || a.ld_gs % V == 0) &&
                    al(a.x, (int)(sizeof(T) * V)) && al(a.gx, (int)(sizeof(Ac) * V > 16 ? 16 : sizeof(Ac) * V)) &&
                    al(a.gy, (int)(sizeof(Ac) * V > 16 ? 16 : sizeof(Ac) * V)) &&
                    al(a.gs_grad, (int)(sizeof(Ac) * V > 16 ? 16 : sizeof(Ac) * V));
    return ok ? V : 1;
}

// Occurrences in flight per warp step.  With the column chunk's x and grad_y slabs resident in L2, 4
// (3 CTAs per SM) issues fewer instructions per byte; when they spill to HBM, 2 (4 CTAs per SM, more
// warps to cover DRAM latency) measured faster.  CLB_GATHER_U overrides.
int gather_unroll(size_t slab_bytes) {
    static const int forced = [] {
        const char* e = getenv("CLB_GATHER_U");
        const int v = e ? atoi(e) : 0;
        return (v == 2 || v == 4 || v == 8) ? v : 0;
    }();
    if (forced) return forced;
    return slab_bytes > (size_t(96) << 20) ? 2 : 4;
}

template <typename T, int VEC, typename I>
cudaError_t gather_launch_vi(const GatherArgs& a, dim3 grid, cudaStream_t s) {
    using Ac = typename Acc<T>::type;
    const size_t slab = (size_t)(32 * VEC) * ((size_t)a.in_features * sizeof(T) + (size_t)a.n_out * sizeof(Ac));
    switch (gather_unroll(slab)) {
        case 2: logic_backward_gather_kernel<T, VEC, 2, I><<<grid, kThreads, 0, s>>>(a); break;
        case 8: logic_backward_gather_kernel<T, VEC, 8, I><<<grid, kThreads, 0, s>>>(a); break;
        default: logic_backward_gather_kernel<T, VEC, 4, I><<<grid, kThreads, 0, s>>>(a); break;
    }
    return cudaGetLastError();
}

template <typename T, int VEC>
cudaError_t gather_launch_v(const GatherArgs& a, cudaStream_t s) {
    dim3 grid((unsigned)ceil_div64(a.in_features, kWarps), (unsigned)ceil_div64(a.ncols, 32 * VEC));
    if (grid.x == 0 || grid.y == 0) return cudaSuccess;
    const int64_t lim = int64_t(1) << 31;
    const int64_t gext = a.gs_grad ? (a.n_out / a.gs_size + 1) * a.ld_gs : a.n_out * a.ldgy;
    const bool small = a.in_features * a.ldx < lim && gext < lim && a.in_features < lim;
    return small ? gather_launch_vi<T, VEC, int>(a, grid, s) : gather_launch_vi<T, VEC, int64_t>(a, grid, s);
}

template <typename T>
int64_t gather_chunks_t(const GatherArgs& a) {
    return ceil_div64(a.ncols, 32 * gather_vec<T>(a));
}

template <typename T>
cudaError_t gather_t(const GatherArgs& a, int mode, const void* weights, cudaStream_t s) {
    using Ac = typename Acc<T>::type;
    const int64_t rows = a.n_out / a.group;
    if (rows > 0) {
        softmax_rows_kernel<Ac><<<(unsigned)ceil_div64(rows, 256), 256, 0, s>>>(
            reinterpret_cast<const Ac*>(weights), rows, a.K, mode, reinterpret_cast<Ac*>(const_cast<void*>(a.probs)));
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    if constexpr (!std::is_same<T, double>::value) if (gather_vec<T>(a) == 4 && fast_ok(a)) {
        const int64_t total = a.starts == nullptr ? 0 : 2 * a.n_out * a.K;
        if (total > 0) {
            bake_kernel<<<(unsigned)ceil_div64(total, 256), 256, 0, s>>>(
                a.recs, a.starts + a.in_features, total, reinterpret_cast<const float*>(a.probs), a.K, a.group, a.ldx, a.gs_grad != nullptr,
                a.gs_size, a.gs_grad ? a.ld_gs : a.ldgy, (float)(a.gs_grad ? a.gs_scale : 1.0), a.baked,
                reinterpret_cast<int*>(a.tmp));
            cudaError_t e = cudaGetLastError();
            if (e != cudaSuccess) return e;
        }
        dim3 grid((unsigned)ceil_div64(a.in_features, kWarps), (unsigned)ceil_div64(a.ncols, 128));
        if (grid.x == 0 || grid.y == 0) return cudaSuccess;
        // CLB_GATHER2: occurrences in flight x resident CTAs per SM (tuning; 44 = 4 x 4, the default), with the
        // staged records read as four 32-bit broadcasts (one shared wavefront each; a 128-bit broadcast costs
        // several: c2 gather 1.082 -> 1.069 ms); 441 / 442 read them as one 128-bit / two 64-bit loads
        static const int cfg = [] {
            const char* e = getenv("CLB_GATHER2");
            const int v = e ? atoi(e) : 44;
            return (v == 43 || v == 25 || v == 26 || v == 441 || v == 442) ? v : 44;
        }();
        int* owner = reinterpret_cast<int*>(a.tmp);
        static const int split = [] {
            const char* e = getenv("CLB_GATHER_SPLIT");
            return (e && e[0] == '0') ? 0 : 1;
        }();
        GatherArgs as = a;
        as.split = split;
        // CLB_GATHER4: 0 = gather2, 3 / 2 = the 8-lanes-per-occurrence kernel with 3 / 2 resident CTAs per SM;
        // unset = gather4 (3) for fp32 layers averaging >= 64 occurrences per input row, where its per-row
        // reduce-scatter is amortised (measured: c3 dense layer 0.87 -> 0.79 ms; c2, 32 per row, 1.08 ->
        // 1.24 ms, and bf16 rows, whose 8-byte pieces half-fill a quarter-warp's 128 bytes, slower)
        static const int g4env = [] {
            const char* e = getenv("CLB_GATHER4");
            return e ? atoi(e) : -1;
        }();
        const bool dense_rows = std::is_same<T, float>::value && 2 * a.n_out * a.K >= 64 * a.in_features;
        const int g4 = g4env >= 0 ? g4env : (dense_rows ? 3 : 0);
        if (g4 != 0 && a.ncols % 128 == 0) {
            if (g4 == 2) logic_backward_gather4_kernel<T, 2><<<grid, kThreads, 0, s>>>(as, a.baked, owner);
            else logic_backward_gather4_kernel<T, 3><<<grid, kThreads, 0, s>>>(as, a.baked, owner);
            return cudaGetLastError();
        }
        switch (cfg) {
            case 43: logic_backward_gather2_kernel<T, 4, 3><<<grid, kThreads, 0, s>>>(as, a.baked, owner); break;
            case 25: logic_backward_gather2_kernel<T, 2, 5><<<grid, kThreads, 0, s>>>(as, a.baked, owner); break;
            case 26: logic_backward_gather2_kernel<T, 2, 6><<<grid, kThreads, 0, s>>>(as, a.baked, owner); break;
            case 441: logic_backward_gather2_kernel<T, 4, 4, 1><<<grid, kThreads, 0, s>>>(as, a.baked, owner); break;
            case 442: logic_backward_gather2_kernel<T, 4, 4, 2><<<grid, kThreads, 0, s>>>(as, a.baked, owner); break;
            default: logic_backward_gather2_kernel<T, 4, 4, 4><<<grid, kThreads, 0, s>>>(as, a.baked, owner); break;
        }
        return cudaGetLastError();
    }
    if (gather_vec<T>(a) == gvec<T>()) return gather_launch_v<T, gvec<T>()>(a, s);
    return gather_launch_v<T, 1>(a, s);
}

GatherArgs make_args(const void* x, int64_t ldx, int64_t ncols, const void* gy, int64_t ldgy, const void* gs_grad,
                     int64_t gs_size, int64_t ld_gs, double gs_scale, void* gx, int64_t ldgx, void* part,
                     const void* probs, const IndexParts& ip, int64_t in_features, int64_t n_out, int K,
                     int64_t group) {
    GatherArgs a{};
    a.x = x;
    a.ldx = ldx;
    a.ncols = ncols;
    a.gy = gs_grad ? nullptr : gy;
    a.ldgy = ldgy;
    a.gs_grad = gs_grad;
    a.gs_size = gs_size;
    a.ld_gs = ld_gs;
    a.gs_scale = gs_scale;
    a.gx = gx;
    a.ldgx = ldgx;
    a.part = part;
    a.probs = probs;
    a.starts = ip.starts;
    a.recs = ip.recs;
    a.baked = ip.baked;
    a.tmp = ip.tmp;
    a.in_features = in_features;
    a.n_out = n_out;
    a.K = K;
    a.group = group;
    return a;
}

int64_t chunks_for(int dtype, const GatherArgs& a) {
    switch (dtype) {
        case CLB_F32: return gather_chunks_t<float>(a);
        case CLB_F64: return gather_chunks_t<double>(a);
        case CLB_BF16: return gather_chunks_t<__nv_bfloat16>(a);
        case CLB_F16: return gather_chunks_t<__half>(a);
    }
    return -1;
}

bool dtype_ok(int d) { return d == CLB_F32 || d == CLB_F64 || d == CLB_BF16 || d == CLB_F16; }

int cuda_fail(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return CLB_OK;
    return set_error(CLB_ERR_CUDA, what);
}

}  // namespace

}  // namespace clb

using namespace clb;

extern "C" int64_t clb_logic_index_bytes(int64_t n_out, int64_t K, int64_t in_features) {
    if (n_out < 0 || K < 1 || in_features < 1 || n_out * K > kMaxSlots) return -1;
    return (int64_t)index_parts(nullptr, n_out, K, in_features).bytes;
}

extern "C" int clb_logic_index_build(const int32_t* slots, int64_t n_out, int64_t K, int64_t group,
                                     const uint8_t* gates, int64_t in_features, void* index, int64_t index_bytes,
                                     clb_stream_t stream) {
    const int64_t need = clb_logic_index_bytes(n_out, K, in_features);
    if (need < 0)
        return set_error(CLB_ERR_INVALID, "index_build: need 1 <= K, 1 <= in_features, n_out*K <= 2^24");
    if (group < 1 || n_out % group) return set_error(CLB_ERR_INVALID, "index_build: n_out not a multiple of group");
    if (index_bytes < need) return set_error(CLB_ERR_WORKSPACE, "index_build: index buffer too small");
    if (!index || (n_out > 0 && (!slots || !gates))) return set_error(CLB_ERR_INVALID, "index_build: null pointer");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const IndexParts ip = index_parts(index, n_out, K, in_features);
    // counts live in the starts array's first in_features entries until the scan rewrites them
    cudaError_t e = cudaMemsetAsync(ip.cursor, 0, sizeof(int32_t) * (size_t)in_features, s);
    if (e != cudaSuccess) return cuda_fail(e, "index_build: memset");
    const int64_t slots_n = n_out * K;
    const unsigned nb = (unsigned)ceil_div64(slots_n, 256);
    const int2* sl = reinterpret_cast<const int2*>(slots);
    if (nb) index_count_kernel<<<nb, 256, 0, s>>>(sl, gates, n_out, (int)K, group, in_features, ip.cursor);
    // scan counts (in cursor) into starts; the scan also resets cursor to the row starts
    index_scan_kernel<<<1, 1024, 0, s>>>(ip.cursor, in_features, ip.starts, ip.cursor);
    if (nb) index_fill_kernel<<<nb, 256, 0, s>>>(sl, gates, n_out, (int)K, group, in_features, ip.cursor, ip.tmp);
    index_sort_kernel<<<(unsigned)ceil_div64(in_features, kWarps), kThreads, 0, s>>>(ip.starts, in_features, ip.tmp,
                                                                                    ip.recs);
    count_launches(nb ? 4 : 2);
    return cuda_fail(cudaGetLastError(), "index_build: launch");
}

extern "C" int64_t clb_logic_backward_gather_chunks(int dtype, const void* x, int64_t ldx, int64_t ncols,
                                                    const void* grad_y, int64_t ldgy, const void* gs_grad,
                                                    int64_t ld_gs, const void* grad_x, int64_t ldgx) {
    if (!dtype_ok(dtype)) return -1;
    IndexParts ip{};
    const GatherArgs a = make_args(x, ldx, ncols, grad_y, ldgy, gs_grad, 1, ld_gs, 1.0, const_cast<void*>(grad_x), ldgx,
                                   nullptr, nullptr, ip, 1, 0, 1, 1);
    return chunks_for(dtype, a);
}

extern "C" int clb_logic_backward_gather(int dtype, const void* x, int64_t ldx, int64_t ncols, int64_t in_features,
                                         int64_t n_out, int64_t K, int64_t group, int weight_mode,
                                         const void* weights, const void* index, const void* grad_y, int64_t ldgy,
                                         const void* gs_grad, int64_t gs_k, int64_t gs_size, int64_t ld_gs,
                                         double gs_scale, void* grad_x, int64_t ldgx, void* probs, void* partials,
                                         int64_t partials_chunks, clb_stream_t stream) {
    if (!dtype_ok(dtype)) return set_error(CLB_ERR_DTYPE, "backward_gather: dtype");
    if (clb_logic_index_bytes(n_out, K, in_features) < 0 || group < 1 || n_out % group)
        return set_error(CLB_ERR_INVALID, "backward_gather: bad layer sizes");
    if (weight_mode != CLB_W_LOGITS && weight_mode != CLB_W_PROBS)
        return set_error(CLB_ERR_INVALID, "backward_gather: weight mode must be logits or probabilities");
    if (ncols < 0 || ldx < ncols || ldgx < ncols) return set_error(CLB_ERR_INVALID, "backward_gather: ld < ncols");
    if (ncols == 0 || in_features == 0) return CLB_OK;  // nothing to write (an empty grad_x may have no address)
    if (!grad_x || !index || !probs || !weights || !x)
        return set_error(CLB_ERR_INVALID, "backward_gather: null pointer");
    if (gs_grad) {
        if (gs_k < 1 || gs_size < 1 || ld_gs < ncols || gs_k * gs_size < n_out)
            return set_error(CLB_ERR_INVALID, "backward_gather: bad GroupSum geometry");
    } else if (n_out > 0 && (!grad_y || ldgy < ncols)) {
        return set_error(CLB_ERR_INVALID, "backward_gather: null grad_y or ldgy < ncols");
    }
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const IndexParts ip = index_parts(const_cast<void*>(index), n_out, K, in_features);
    const GatherArgs a = make_args(x, ldx, ncols, grad_y, ldgy, gs_grad, gs_size, ld_gs, gs_scale, grad_x, ldgx,
                                   partials, probs, ip, in_features, n_out, (int)K, group);
    if (partials && chunks_for(dtype, a) != partials_chunks)
        return set_error(CLB_ERR_INVALID, "backward_gather: partials sized for another column split");
    cudaError_t e = cudaErrorInvalidValue;
    switch (dtype) {
        case CLB_F32: e = gather_t<float>(a, weight_mode, weights, s); break;
        case CLB_F64: e = gather_t<double>(a, weight_mode, weights, s); break;
        case CLB_BF16: e = gather_t<__nv_bfloat16>(a, weight_mode, weights, s); break;
        case CLB_F16: e = gather_t<__half>(a, weight_mode, weights, s); break;
    }
    count_launches(2);
    return cuda_fail(e, "backward_gather: launch");
}
