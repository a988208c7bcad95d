// Soft-mode and select-mode logic-layer kernels (dense and convolutional).
//
// One kernel family serves both layer kinds.  A layer is a table of "slots": output neuron j owns
// K candidate gates, slot (j, k) reads input features (a, b) = slots[j, k] and applies gate
// gates[r, k] weighted by prob p[r, k], where r = j / group is the parameter row.  Dense layers
// (compactlogic/compactlogic.py:83-118) have group 1 and slots copied from `indices`; conv layers
// (compactlogic/compactlogic.py:598-626) have one row per output channel shared by its
// h_out*w_out positions, and slots computed from the receptive-field offsets with -1 marking
// zero padding.
//
// Work decomposition (both passes): a CTA owns TN consecutive neurons and one chunk of 32*VEC batch
// columns; each warp walks TN/8 of the neurons with its lanes on consecutive columns, so every
// gather of an input row is one coalesced 128..512-byte segment.  The chunk index is the slow grid
// dimension, so resident CTAs share one column chunk and its input slab stays in L2 while ~2K
// gathers per neuron hit it.  The per-neuron softmax over the K logits and the gate polynomial
// coefficients are computed once per CTA into shared memory and read back as broadcasts.
#include <cuda_runtime.h>
#include <float.h>
#include <stdlib.h>

#include <type_traits>

#include "common.cuh"
#include "gates.cuh"
#include "kernels.h"

namespace clb {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

template <typename A> struct A4 { A x, y, z, w; };

// Shared-memory slot stage for TN neurons.
// Forward: each neuron's entries are compacted, two-operand gates first (ns of them: ab, p*c1, p*c2,
// p*c3), then one-operand gates (n1 of them: the used operand in ab.x and its coefficient p*c1 or p*c2
// in cf.x); constant gates only contribute to c0.  Backward: entry k is slot k (ns = K).
template <typename A> struct Stage {
    A4<A>* cf;   // [TN*K] forward: see above ; backward: c0, c1, c2, c3 (raw)
    int2* ab;    // [TN*K]
    A* p;        // [TN*K] backward only
    A* c0;       // [TN]   forward: sum_k p*c0
    int* ns;     // [TN]   forward: two-operand entries; backward: slots
    int* n1;     // [TN]   forward: one-operand entries
};

template <typename A>
__host__ __device__ inline size_t stage_bytes(int TN, int K, bool backward) {
    size_t b = (size_t)TN * K * (sizeof(A4<A>) + sizeof(int2)) + (size_t)TN * (sizeof(A) + 2 * sizeof(int));
    if (backward) b += (size_t)TN * K * sizeof(A);
    return b;
}

template <typename A>
__device__ __forceinline__ Stage<A> carve(unsigned char* smem, int TN, int K, bool backward) {
    Stage<A> s;
    s.cf = reinterpret_cast<A4<A>*>(smem);
    s.ab = reinterpret_cast<int2*>(s.cf + (size_t)TN * K);
    A* after = reinterpret_cast<A*>(s.ab + (size_t)TN * K);
    s.p = after;
    if (backward) after += (size_t)TN * K;
    s.c0 = after;
    s.ns = reinterpret_cast<int*>(s.c0 + TN);
    s.n1 = s.ns + TN;
    return s;
}

// Operands a gate does not depend on are marked -1, so neither the forward gather nor the backward
// gather / scatter touches them: constant gates (0, 15) read nothing, gates A, B, not A, not B
// (3, 5, 12, 10) read one operand.  Exact: the dropped terms have zero coefficients.
__device__ __forceinline__ int2 used_operands(int2 s, const GatePoly& gp) {
    if (gp.c1 == 0.f && gp.c3 == 0.f) s.x = -1;
    if (gp.c2 == 0.f && gp.c3 == 0.f) s.y = -1;
    return s;
}

// Forward entry of one slot: 2 = two-operand gate, 1 = one-operand gate (operand moved to .x),
// 0 = constant gate (contributes p*c0 only).
template <typename A>
__device__ __forceinline__ int fwd_entry(int2 s, const GatePoly& gp, A p, int2& ab, A4<A>& cf) {
    const bool ua = gp.c1 != 0.f || gp.c3 != 0.f, ub = gp.c2 != 0.f || gp.c3 != 0.f;
    if (ua && ub) {
        ab = s;
        cf = A4<A>{p * (A)gp.c1, p * (A)gp.c2, p * (A)gp.c3, (A)0};
        return 2;
    }
    ab = make_int2(ua ? s.x : s.y, -1);
    cf = A4<A>{p * (A)(ua ? gp.c1 : gp.c2), (A)0, (A)0, (A)0};
    return (ua || ub) ? 1 : 0;
}

__device__ __forceinline__ float exp_acc(float v) { return expf(v); }
__device__ __forceinline__ double exp_acc(double v) { return exp(v); }

template <typename A> __device__ __forceinline__ A seg_max(A v, int K) {
    for (int o = K >> 1; o > 0; o >>= 1) {
        const A other = __shfl_xor_sync(0xffffffffu, v, o);
        v = other > v ? other : v;
    }
    return v;
}
template <typename A> __device__ __forceinline__ A seg_sum(A v, int K) {
    for (int o = K >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Fill the stage for neurons [j0, j0+TN).
// K a power of two <= 32 (the usual 4 / 8 / 16): one thread per slot, the K slots of a neuron in K
// adjacent lanes, softmax max/sum and the constant term by segmented warp reductions, so all
// threads of the CTA share the staging work.  Otherwise, and in select mode: one thread per neuron.
template <typename A, bool BACKWARD>
__device__ void fill_stage(const LayerArgs& a, int64_t j0, int TN, Stage<A> st) {
    const int K = a.K;
    const A* w = reinterpret_cast<const A*>(a.weights);
    const int2* slots = reinterpret_cast<const int2*>(a.slots);
    if (a.mode != CLB_W_SELECT && K <= 32 && (K & (K - 1)) == 0) {
        const int total = TN * K;
        const int rounds = (total + blockDim.x - 1) / blockDim.x;
        for (int it = 0; it < rounds; ++it) {
            const int e = it * blockDim.x + threadIdx.x;  // warp-uniform trip count keeps the shuffles legal
            const int t = e / K, k = e - t * K;
            const int64_t j = j0 + t;
            const bool valid = e < total && j < a.n_out;
            const int64_t r = valid ? j / a.group : 0;
            A p = 0;
            if (a.mode == CLB_W_LOGITS) {
                const A wv = valid ? w[r * K + k] : -(A)FLT_MAX;
                const A m = seg_max(wv, K);
                const A ex = valid ? exp_acc(wv - m) : (A)0;
                const A sum = seg_sum(ex, K);
                p = valid ? ex / sum : (A)0;
            } else if (valid && w != nullptr) {
                p = w[r * K + k];
            }
            GatePoly gp{0.f, 0.f, 0.f, 0.f};
            if (valid) gp = gate_poly(a.gates[r * K + k] & 15);
            if (BACKWARD) {
                if (valid) {
                    st.ab[e] = used_operands(slots[j * K + k], gp);
                    st.cf[e] = A4<A>{(A)gp.c0, (A)gp.c1, (A)gp.c2, (A)gp.c3};
                    st.p[e] = p;
                }
                if (e < total && k == 0) st.ns[t] = valid ? K : 0;
            } else {
                int2 ab;
                A4<A> cf;
                const int cls = valid ? fwd_entry(slots[j * K + k], gp, p, ab, cf) : 0;
                // compact the K lanes of this neuron: two-operand entries first, then one-operand ones
                const unsigned pm = __ballot_sync(0xffffffffu, cls == 2), om = __ballot_sync(0xffffffffu, cls == 1);
                const int lane = threadIdx.x & 31;
                const unsigned seg = K == 32 ? 0xffffffffu : (((1u << K) - 1u) << (lane & ~(K - 1)));
                const unsigned below = seg & ((1u << lane) - 1u);
                const int np = __popc(pm & seg), n1 = __popc(om & seg);
                if (cls != 0) {
                    const int pos = cls == 2 ? __popc(pm & below) : np + __popc(om & below);
                    st.ab[t * K + pos] = ab;
                    st.cf[t * K + pos] = cf;
                }
                const A c0sum = seg_sum(p * (A)gp.c0, K);
                if (e < total && k == 0) {
                    st.ns[t] = valid ? np : 0;
                    st.n1[t] = valid ? n1 : 0;
                    st.c0[t] = c0sum;
                }
            }
        }
        return;
    }
    for (int t = threadIdx.x; t < TN; t += blockDim.x) {
        const int64_t j = j0 + t;
        int ns = 0, n1 = 0;
        A c0sum = 0;
        if (j < a.n_out) {
            const int64_t r = j / a.group;
            const uint8_t* g = a.gates + r * K;
            if (a.mode == CLB_W_SELECT) {
                const int k = a.select[r];
                if (k < K) {
                    const GatePoly gp = gate_poly(g[k] & 15);
                    if (BACKWARD) {
                        st.ab[t * K] = used_operands(slots[j * K + k], gp);
                        st.cf[t * K] = A4<A>{(A)gp.c0, (A)gp.c1, (A)gp.c2, (A)gp.c3};
                        st.p[t * K] = (A)1;
                        ns = 1;
                    } else {
                        const int cls = fwd_entry(slots[j * K + k], gp, (A)1, st.ab[t * K], st.cf[t * K]);
                        ns = cls == 2 ? 1 : 0;
                        n1 = cls == 1 ? 1 : 0;
                        c0sum = (A)gp.c0;
                    }
                }
            } else {
                const A* wr = w != nullptr ? w + r * K : nullptr;
                A m = (A)0, sum = (A)1;
                if (a.mode == CLB_W_LOGITS) {
                    m = wr[0];
                    for (int k = 1; k < K; ++k) m = wr[k] > m ? wr[k] : m;
                    sum = 0;
                    for (int k = 0; k < K; ++k) sum += exp_acc(wr[k] - m);
                }
                if (BACKWARD) {
                    for (int k = 0; k < K; ++k) {
                        const A p = a.mode == CLB_W_LOGITS ? exp_acc(wr[k] - m) / sum : (w != nullptr ? wr[k] : (A)0);
                        const GatePoly gp = gate_poly(g[k] & 15);
                        st.ab[t * K + k] = used_operands(slots[j * K + k], gp);
                        st.cf[t * K + k] = A4<A>{(A)gp.c0, (A)gp.c1, (A)gp.c2, (A)gp.c3};
                        st.p[t * K + k] = p;
                    }
                    ns = K;
                } else {
                    for (int k = 0; k < K; ++k) {
                        const GatePoly gp = gate_poly(g[k] & 15);
                        ns += (gp.c1 != 0.f || gp.c3 != 0.f) && (gp.c2 != 0.f || gp.c3 != 0.f);
                    }
                    int ip = 0, io = ns;
                    for (int k = 0; k < K; ++k) {
                        const A p = a.mode == CLB_W_LOGITS ? exp_acc(wr[k] - m) / sum : (w != nullptr ? wr[k] : (A)0);
                        const GatePoly gp = gate_poly(g[k] & 15);
                        int2 ab;
                        A4<A> cf;
                        const int cls = fwd_entry(slots[j * K + k], gp, p, ab, cf);
                        if (cls != 0) {
                            const int pos = cls == 2 ? ip++ : io++;
                            st.ab[t * K + pos] = ab;
                            st.cf[t * K + pos] = cf;
                        }
                        c0sum += p * (A)gp.c0;
                    }
                    n1 = io - ns;
                }
            }
        }
        st.ns[t] = ns;
        if (!BACKWARD) {
            st.n1[t] = n1;
            st.c0[t] = c0sum;
        }
    }
}

template <typename T, int VEC>
__device__ __forceinline__ void gather(const T* __restrict__ x, int idx, int64_t ldx, int64_t col,
                                       typename Acc<T>::type (&v)[VEC]) {
    if (idx >= 0) {
        load_acc<T, VEC>(x + (int64_t)idx * ldx + col, v);
    } else {
#pragma unroll
        for (int i = 0; i < VEC; ++i) v[i] = 0;
    }
}

#ifndef CLB_FWD_GROUP
#define CLB_FWD_GROUP 2
#endif
constexpr int kFwdGroup = CLB_FWD_GROUP;  // two-operand slots whose gathers the forward issues together

// Offset mode (OFF): the stage holds element offsets idx * ldx instead of row ids (-1 stays -1), so a
// gather is one multiply-add from the lane's column pointer instead of 64-bit row * stride arithmetic.
// Used when in_features * ldx < 2^31 (and, for the backward's scatter, ldgx == ldx).
__device__ __forceinline__ void scale_stage(int2* ab, int n, int64_t ld) {
    __syncthreads();
    for (int e = threadIdx.x; e < n; e += blockDim.x) {
        int2 v = ab[e];
        // unused compacted entries hold stale values: unsigned arithmetic keeps their scaling defined
        v.x = v.x >= 0 ? (int)((unsigned)v.x * (unsigned)ld) : -1;
        v.y = v.y >= 0 ? (int)((unsigned)v.y * (unsigned)ld) : -1;
        ab[e] = v;
    }
}

// All-zero bytes: the gather source of an absent operand (-1), up to 64 bytes per lane, so offset-mode
// gathers need no branch and the compiler can issue the loads of several slots back to back.
__device__ __align__(16) unsigned char g_zero_cols[32 * 64];

template <typename T, int VEC>
__device__ __forceinline__ void gather_off(const T* __restrict__ xc, int off, typename Acc<T>::type (&v)[VEC]) {
    static_assert(sizeof(T) * VEC <= 64, "zero row holds 64 bytes per lane");
    const T* p = off >= 0 ? xc + off : reinterpret_cast<const T*>(g_zero_cols) + (threadIdx.x & 31) * VEC;
    load_acc<T, VEC>(p, v);
}

// Forward stage baked once per call: the softmax, the compaction into two- / one-operand entries and
// (offset mode) the row-offset scaling depend only on the neuron, yet the stage is otherwise rebuilt by
// every CTA of every column chunk.  fwd_bake_kernel writes it once to global memory ([nb, K] entries,
// nb = n_out rounded up to TN), and the forward CTAs copy their TN neurons' part into shared memory.
template <typename A> struct FwdBake {
    A4<A>* cf;
    int2* ab;
    A* c0;
    int* ns;
    int* n1;
};

inline size_t r256(size_t v) { return (v + 255) & ~size_t(255); }

template <typename A>
size_t bake_bytes(int64_t nb, int K) {
    return r256((size_t)nb * K * sizeof(A4<A>)) + r256((size_t)nb * K * sizeof(int2)) + r256((size_t)nb * sizeof(A)) +
           2 * r256((size_t)nb * sizeof(int));
}

template <typename A>
FwdBake<A> carve_bake(void* base, int64_t nb, int K) {
    unsigned char* b = reinterpret_cast<unsigned char*>(base);
    FwdBake<A> f;
    f.cf = reinterpret_cast<A4<A>*>(b);
    b += r256((size_t)nb * K * sizeof(A4<A>));
    f.ab = reinterpret_cast<int2*>(b);
    b += r256((size_t)nb * K * sizeof(int2));
    f.c0 = reinterpret_cast<A*>(b);
    b += r256((size_t)nb * sizeof(A));
    f.ns = reinterpret_cast<int*>(b);
    b += r256((size_t)nb * sizeof(int));
    f.n1 = reinterpret_cast<int*>(b);
    return f;
}

template <typename A, bool OFF>
__global__ void __launch_bounds__(kThreads) fwd_bake_kernel(const LayerArgs a, const int TN, const FwdBake<A> f) {
    const int K = a.K;
    const int64_t j0 = (int64_t)blockIdx.x * TN;
    Stage<A> st;
    st.cf = f.cf + j0 * K;
    st.ab = f.ab + j0 * K;
    st.p = nullptr;
    st.c0 = f.c0 + j0;
    st.ns = f.ns + j0;
    st.n1 = f.n1 + j0;
    fill_stage<A, false>(a, j0, TN, st);
    if (OFF) scale_stage(st.ab, TN * K, a.ldx);
}

// ---------------------------------------------------------------------------------------------
// Forward: y[j, n] = sum_k p[r,k] * f_{g[r,k]}(x[a_jk, n], x[b_jk, n])   (difflogic_kernel.cu:39-78)
// Select mode (float eval, difflogic_kernel.cu:341-369): only the chosen slot, p = 1.
// With GroupSum fused (compactlogic.py:460-465), y is never written; per-class column sums are
// accumulated into gs.acc instead.
// ---------------------------------------------------------------------------------------------
template <typename T, int VEC, bool PEERS, bool OFF, bool BAKED = false>
__global__ void __launch_bounds__(kThreads)
logic_forward_kernel(const LayerArgs a, T* __restrict__ y, const int64_t ldy, const GroupSumArgs gs,
                     const bool use_gs, const int TN, const PeerArgs pa, const FwdBake<typename Acc<T>::type> fb) {
    using A = typename Acc<T>::type;
    extern __shared__ __align__(16) unsigned char smem[];
    const int K = a.K;
    Stage<A> st = carve<A>(smem, TN, K, false);
    const int64_t j0 = (int64_t)blockIdx.x * TN;
    if (BAKED) {  // copy this CTA's part of the baked stage (entries past ns + n1 are never read)
        const int nk = TN * K;
        const A4<A>* __restrict__ gcf = fb.cf + j0 * K;
        const int2* __restrict__ gab = fb.ab + j0 * K;
        for (int e = threadIdx.x; e < nk; e += blockDim.x) {
            st.cf[e] = gcf[e];
            st.ab[e] = gab[e];
        }
        for (int t = threadIdx.x; t < TN; t += blockDim.x) {
            st.c0[t] = fb.c0[j0 + t];
            st.ns[t] = fb.ns[j0 + t];
            st.n1[t] = fb.n1[j0 + t];
        }
    } else {
        fill_stage<A, false>(a, j0, TN, st);
        if (OFF) scale_stage(st.ab, TN * K, a.ldx);
    }
    __syncthreads();

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t col = (int64_t)blockIdx.y * (32 * VEC) + lane * VEC;
    const bool active = col < a.ncols;
    const T* __restrict__ x = reinterpret_cast<const T*>(a.x);
    const T* __restrict__ xc = x + (active ? col : 0);

    A gacc[VEC];
#pragma unroll
    for (int i = 0; i < VEC; ++i) gacc[i] = 0;
    int64_t gcls = -1;

    for (int t = warp; t < TN; t += kWarps) {
        const int64_t j = j0 + t;
        if (j >= a.n_out) break;
        A acc[VEC];
        const A c0 = st.c0[t];
#pragma unroll
        for (int i = 0; i < VEC; ++i) acc[i] = c0;
        if (active) {
            const int ns = st.ns[t], n1 = st.n1[t];
            const int2* ab = st.ab + t * K;
            const A4<A>* cf = st.cf + t * K;
            int s0 = 0;
            if (OFF && kFwdGroup > 1) {  // the gathers of kFwdGroup slots issued before their arithmetic
                for (; s0 + kFwdGroup <= ns; s0 += kFwdGroup) {
                    A vas[kFwdGroup][VEC], vbs[kFwdGroup][VEC];
#pragma unroll
                    for (int u = 0; u < kFwdGroup; ++u) {
                        const int2 pr = ab[s0 + u];
                        gather_off<T, VEC>(xc, pr.x, vas[u]);
                        gather_off<T, VEC>(xc, pr.y, vbs[u]);
                    }
#pragma unroll
                    for (int u = 0; u < kFwdGroup; ++u) {
                        const A4<A> c = cf[s0 + u];
#pragma unroll
                        for (int i = 0; i < VEC; ++i) {
                            const A w = fma(c.z, vas[u][i], c.y);  // p*(c2 + c3 a)
                            acc[i] = fma(c.x, vas[u][i], acc[i]);
                            acc[i] = fma(w, vbs[u][i], acc[i]);
                        }
                    }
                }
            }
#pragma unroll 4
            for (int s = s0; s < ns; ++s) {
                const int2 pr = ab[s];
                const A4<A> c = cf[s];
                A va[VEC], vb[VEC];
                if (OFF) {
                    gather_off<T, VEC>(xc, pr.x, va);
                    gather_off<T, VEC>(xc, pr.y, vb);
                } else {
                    gather<T, VEC>(x, pr.x, a.ldx, col, va);
                    gather<T, VEC>(x, pr.y, a.ldx, col, vb);
                }
#pragma unroll
                for (int i = 0; i < VEC; ++i) {
                    const A u = fma(c.z, va[i], c.y);  // p*(c2 + c3 a)
                    acc[i] = fma(c.x, va[i], acc[i]);
                    acc[i] = fma(u, vb[i], acc[i]);
                }
            }
#pragma unroll 4
            for (int s = ns; s < ns + n1; ++s) {  // one-operand gates: acc += p*c * operand
                const int idx = ab[s].x;
                const A c = cf[s].x;
                A va[VEC];
                if (OFF)
                    gather_off<T, VEC>(xc, idx, va);
                else
                    gather<T, VEC>(x, idx, a.ldx, col, va);
#pragma unroll
                for (int i = 0; i < VEC; ++i) acc[i] = fma(c, va[i], acc[i]);
            }
        }
        if (!use_gs) {
            if (active) {
                if (!PEERS) {
                    store_from_acc<T, VEC>(y + j * ldy + col, acc);
                } else {
                    for (int p = 0; p < pa.n; ++p)
                        store_from_acc<T, VEC>(reinterpret_cast<T*>(pa.p[p]) + j * ldy + col, acc);
                }
            }
        } else {
            const int64_t cls = j / gs.size;
            if (cls != gcls) {
                if (gcls >= 0 && active) red_add<VEC>(reinterpret_cast<A*>(gs.acc) + gcls * gs.ld + col, gacc);
#pragma unroll
                for (int i = 0; i < VEC; ++i) gacc[i] = 0;
                gcls = cls;
            }
#pragma unroll
            for (int i = 0; i < VEC; ++i) gacc[i] += acc[i];
        }
    }
    if (use_gs && gcls >= 0 && active) red_add<VEC>(reinterpret_cast<A*>(gs.acc) + gcls * gs.ld + col, gacc);
    if (PEERS) __threadfence_system();  // peer stores complete before the host-side barrier that follows
}

// Butterfly reduce-scatter of N per-lane values over the warp: afterwards lane l holds the warp sum
// of value index (l >> (5 - log2 N)) & (N - 1).  N + N/2 + ... shuffles instead of 5 N.
template <typename A, int N, int OFF> struct ReduceScatter {
    static __device__ __forceinline__ void run(A* v, int lane) {
        const bool up = (lane & OFF) != 0;
#pragma unroll
        for (int i = 0; i < N / 2; ++i) {
            const A send = up ? v[i] : v[i + N / 2];
            const A keep = up ? v[i + N / 2] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, OFF);
        }
        ReduceScatter<A, N / 2, OFF / 2>::run(v, lane);
    }
};
template <typename A, int OFF> struct ReduceScatter<A, 1, OFF> {
    static __device__ __forceinline__ void run(A* v, int lane) {
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], OFF);
        ReduceScatter<A, 1, OFF / 2>::run(v, lane);
    }
};
template <typename A> struct ReduceScatter<A, 1, 0> {
    static __device__ __forceinline__ void run(A*, int) {}
};

#ifndef CLB_BWD_GROUP
#define CLB_BWD_GROUP 2
#endif
constexpr int kBwdGroup = CLB_BWD_GROUP;  // slots whose gathers the backward issues together

constexpr int log2c(int n) { return n <= 1 ? 0 : 1 + log2c(n / 2); }

// ---------------------------------------------------------------------------------------------
// Fused backward.  Per slot and column it reads x[a], x[b] once and produces
//   d loss/d p[r,k] partial  = sum_n gy[j,n] * f(a,b)                  (difflogic_kernel.cu:82-137)
//   grad_x[a,n] += p * (c1 + c3 b) * gy[j,n],  grad_x[b,n] += p * (c2 + c3 a) * gy[j,n]
//                                                                     (difflogic_kernel.cu:574-610)
// The scatter uses fire-and-forget vector reductions into L2; the partials are per column chunk
// ([nchunks, n_out, K], deterministic) and folded by the finalize kernel.
// KT > 0: K is a compile-time constant and the K partial sums live in registers.
// ---------------------------------------------------------------------------------------------
template <typename T, int VEC, int KT, bool PEERS, bool OFF, bool GX>
__global__ void __launch_bounds__(kThreads)
logic_backward_kernel(const LayerArgs a, const typename Acc<T>::type* __restrict__ gy, const int64_t ldgy,
                      const GroupSumArgs gs, const bool use_gs, typename Acc<T>::type* __restrict__ gx,
                      const int64_t ldgx, typename Acc<T>::type* __restrict__ part, const int TN, const PeerArgs pa) {
    using A = typename Acc<T>::type;
    extern __shared__ __align__(16) unsigned char smem[];
    const int K = KT > 0 ? KT : a.K;
    Stage<A> st = carve<A>(smem, TN, K, true);
    const int64_t j0 = (int64_t)blockIdx.x * TN;
    fill_stage<A, true>(a, j0, TN, st);
    if (OFF) scale_stage(st.ab, TN * K, a.ldx);
    __syncthreads();

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t chunk = blockIdx.y;
    const int64_t col = chunk * (32 * VEC) + lane * VEC;
    const bool active = col < a.ncols;
    const T* __restrict__ x = reinterpret_cast<const T*>(a.x);
    const T* __restrict__ xc = x + (active ? col : 0);
    A* __restrict__ gxc = gx != nullptr ? gx + (active ? col : 0) : nullptr;
    const A* gsg = reinterpret_cast<const A*>(gs.grad);

    for (int t = warp; t < TN; t += kWarps) {
        const int64_t j = j0 + t;
        if (j >= a.n_out) break;
        A g[VEC];
        if (active) {
            if (use_gs) {
                load_acc<A, VEC>(gsg + (j / gs.size) * gs.ld + col, g);
#pragma unroll
                for (int i = 0; i < VEC; ++i) g[i] *= (A)gs.scale;
            } else if (!PEERS) {
                load_acc<A, VEC>(gy + j * ldgy + col, g);
            } else {
                load_acc<A, VEC>(reinterpret_cast<const A*>(pa.p[0]) + j * ldgy + col, g);
                for (int p = 1; p < pa.n; ++p) {
                    A h[VEC];
                    load_acc<A, VEC>(reinterpret_cast<const A*>(pa.p[p]) + j * ldgy + col, h);
#pragma unroll
                    for (int i = 0; i < VEC; ++i) g[i] += h[i];
                }
            }
        } else {
#pragma unroll
            for (int i = 0; i < VEC; ++i) g[i] = 0;
        }
        const int2* ab = st.ab + t * K;
        const A4<A>* cf = st.cf + t * K;
        const A* pp = st.p + t * K;
        A pk[KT > 0 ? KT : 1];

        // Offset mode with a compile-time K: the gathers of G slots are issued before their arithmetic
        // (branch-free, inactive lanes read column 0, which lane 0 reads as well).
        constexpr int G = (OFF && KT > 0) ? (KT < kBwdGroup ? KT : kBwdGroup) : 1;
#pragma unroll(KT > 0 ? KT / G : 4)
        for (int s0 = 0; s0 < K; s0 += G) {
            int2 prs[G];
            A vas[G][VEC], vbs[G][VEC];
#pragma unroll
            for (int u = 0; u < G; ++u) {
                prs[u] = ab[s0 + u];
                if (OFF && KT > 0) {
                    gather_off<T, VEC>(xc, prs[u].x, vas[u]);
                    gather_off<T, VEC>(xc, prs[u].y, vbs[u]);
                } else if (active) {
                    if (OFF) {
                        gather_off<T, VEC>(xc, prs[u].x, vas[u]);
                        gather_off<T, VEC>(xc, prs[u].y, vbs[u]);
                    } else {
                        gather<T, VEC>(x, prs[u].x, a.ldx, col, vas[u]);
                        gather<T, VEC>(x, prs[u].y, a.ldx, col, vbs[u]);
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < VEC; ++i) vas[u][i] = vbs[u][i] = 0;
                }
            }
#pragma unroll
            for (int u = 0; u < G; ++u) {
            const int s = s0 + u;
            const int2 pr = prs[u];
            const A4<A> c = cf[s];
            const A* va = vas[u];
            const A* vb = vbs[u];
            A dot = 0;
            if (!GX) {  // no activation gradient wanted (a network's first layer): f only
#pragma unroll
                for (int i = 0; i < VEC; ++i)
                    dot = fma(g[i], fma(fma(c.w, va[i], c.z), vb[i], fma(c.y, va[i], c.x)), dot);
            }
            A da[VEC], db[VEC];
            const A pw = GX ? pp[s] : (A)0;
#pragma unroll
            for (int i = 0; i < VEC && GX; ++i) {
                const A dfdb = fma(c.w, va[i], c.z);  // c2 + c3 a
                const A dfda = fma(c.w, vb[i], c.y);  // c1 + c3 b
                const A f = fma(dfdb, vb[i], fma(c.y, va[i], c.x));
                dot = fma(g[i], f, dot);
                const A pg = pw * g[i];
                da[i] = dfda * pg;
                db[i] = dfdb * pg;
            }
            if (GX && gx != nullptr && active) {
                if (OFF) {
                    if (pr.x >= 0) red_add<VEC>(gxc + pr.x, da);
                    if (pr.y >= 0) red_add<VEC>(gxc + pr.y, db);
                } else {
                    if (pr.x >= 0) red_add<VEC>(gx + (int64_t)pr.x * ldgx + col, da);
                    if (pr.y >= 0) red_add<VEC>(gx + (int64_t)pr.y * ldgx + col, db);
                }
            }
            if (KT > 0) {
                pk[KT > 0 ? s : 0] = dot;
            } else if (part != nullptr) {
                dot = warp_sum(dot);
                if (lane == 0) part[(chunk * a.n_out + j) * K + s] = dot;
            }
            }
        }
        if (KT > 0 && part != nullptr) {
            constexpr int L = log2c(KT > 0 ? KT : 1);
            ReduceScatter<A, (KT > 0 ? KT : 1), 16>::run(pk, lane);
            constexpr int SH = 5 - L;
            if ((lane & ((1 << SH) - 1)) == 0) part[(chunk * a.n_out + j) * K + ((lane >> SH) & (K - 1))] = pk[0];
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Narrow-chunk variants for very wide inputs.  With 32*VEC columns per chunk, the slab of x (and of
// grad_x) that one column chunk touches is in_features * 32*VEC elements — 1.5 GB for a 1M-wide layer —
// so the gathers and scatter reductions of a chunk miss L2.  Here LPN lanes share a neuron (32/LPN
// neurons per warp step) and a chunk is LPN*VEC columns, chosen on the host so the slab fits L2.
// Each gather is still a whole 32-byte sector per lane group; the stage is read per lane group.
// ---------------------------------------------------------------------------------------------
template <typename T, int VEC, int LPN>
__global__ void __launch_bounds__(kThreads)
logic_forward_narrow_kernel(const LayerArgs a, T* __restrict__ y, const int64_t ldy, const GroupSumArgs gs,
                            const bool use_gs, const int TN) {
    using A = typename Acc<T>::type;
    constexpr int G = 32 / LPN;
    extern __shared__ __align__(16) unsigned char smem[];
    const int K = a.K;
    Stage<A> st = carve<A>(smem, TN, K, false);
    const int64_t j0 = (int64_t)blockIdx.x * TN;
    fill_stage<A, false>(a, j0, TN, st);
    __syncthreads();

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int lc = lane % LPN, sub = lane / LPN;
    const int64_t col = (int64_t)blockIdx.y * (LPN * VEC) + lc * VEC;
    const bool active = col < a.ncols;
    const T* __restrict__ x = reinterpret_cast<const T*>(a.x);
    A gacc[VEC];
#pragma unroll
    for (int i = 0; i < VEC; ++i) gacc[i] = 0;
    int64_t gcls = -1;
    for (int t0 = warp * G; t0 < TN; t0 += kWarps * G) {
        const int t = t0 + sub;
        const int64_t j = j0 + t;
        if (t >= TN || j >= a.n_out) continue;
        A acc[VEC];
        const A c0 = st.c0[t];
#pragma unroll
        for (int i = 0; i < VEC; ++i) acc[i] = c0;
        if (active) {
            const int ns = st.ns[t], n1 = st.n1[t];
            const int2* ab = st.ab + t * K;
            const A4<A>* cf = st.cf + t * K;
#pragma unroll 4
            for (int s = 0; s < ns; ++s) {
                const int2 pr = ab[s];
                const A4<A> c = cf[s];
                A va[VEC], vb[VEC];
                gather<T, VEC>(x, pr.x, a.ldx, col, va);
                gather<T, VEC>(x, pr.y, a.ldx, col, vb);
#pragma unroll
                for (int i = 0; i < VEC; ++i) {
                    const A u = fma(c.z, va[i], c.y);
                    acc[i] = fma(c.x, va[i], acc[i]);
                    acc[i] = fma(u, vb[i], acc[i]);
                }
            }
#pragma unroll 4
            for (int s = ns; s < ns + n1; ++s) {  // one-operand gates: acc += p*c * operand
                const int idx = ab[s].x;
                const A c = cf[s].x;
                A va[VEC];
                gather<T, VEC>(x, idx, a.ldx, col, va);
#pragma unroll
                for (int i = 0; i < VEC; ++i) acc[i] = fma(c, va[i], acc[i]);
            }
        }
        if (!use_gs) {
            if (active) store_from_acc<T, VEC>(y + j * ldy + col, acc);
        } else {
            const int64_t cls = j / gs.size;
            if (cls != gcls) {
                if (gcls >= 0 && active) red_add<VEC>(reinterpret_cast<A*>(gs.acc) + gcls * gs.ld + col, gacc);
#pragma unroll
                for (int i = 0; i < VEC; ++i) gacc[i] = 0;
                gcls = cls;
            }
#pragma unroll
            for (int i = 0; i < VEC; ++i) gacc[i] += acc[i];
        }
    }
    if (use_gs && gcls >= 0 && active) red_add<VEC>(reinterpret_cast<A*>(gs.acc) + gcls * gs.ld + col, gacc);
}

template <typename T, int VEC, int LPN, int KT>
__global__ void __launch_bounds__(kThreads)
logic_backward_narrow_kernel(const LayerArgs a, const typename Acc<T>::type* __restrict__ gy, const int64_t ldgy,
                             const GroupSumArgs gs, const bool use_gs, typename Acc<T>::type* __restrict__ gx,
                             const int64_t ldgx, typename Acc<T>::type* __restrict__ part, const int TN) {
    using A = typename Acc<T>::type;
    constexpr int G = 32 / LPN;
    extern __shared__ __align__(16) unsigned char smem[];
    const int K = KT > 0 ? KT : a.K;
    Stage<A> st = carve<A>(smem, TN, K, true);
    const int64_t j0 = (int64_t)blockIdx.x * TN;
    fill_stage<A, true>(a, j0, TN, st);
    __syncthreads();

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int lc = lane % LPN, sub = lane / LPN;
    const int64_t chunk = blockIdx.y;
    const int64_t col = chunk * (LPN * VEC) + lc * VEC;
    const bool active = col < a.ncols;
    const T* __restrict__ x = reinterpret_cast<const T*>(a.x);
    const A* gsg = reinterpret_cast<const A*>(gs.grad);
    for (int t0 = warp * G; t0 < TN; t0 += kWarps * G) {  // warp-uniform trip count (segment shuffles)
        const int t = t0 + sub;
        const int64_t j = j0 + t;
        const bool valid = t < TN && j < a.n_out;
        const bool live = valid && active;
        const int ts = valid ? t : 0;
        A g[VEC];
        if (live) {
            if (use_gs) {
                load_acc<A, VEC>(gsg + (j / gs.size) * gs.ld + col, g);
#pragma unroll
                for (int i = 0; i < VEC; ++i) g[i] *= (A)gs.scale;
            } else {
                load_acc<A, VEC>(gy + j * ldgy + col, g);
            }
        } else {
#pragma unroll
            for (int i = 0; i < VEC; ++i) g[i] = 0;
        }
        const int2* ab = st.ab + ts * K;
        const A4<A>* cf = st.cf + ts * K;
        const A* pp = st.p + ts * K;
        A pk[KT > 0 ? KT : 1];
#pragma unroll(KT > 0 ? KT : 4)
        for (int s = 0; s < K; ++s) {
            const int2 pr = live ? ab[s] : make_int2(-1, -1);
            const A4<A> c = cf[s];
            A va[VEC], vb[VEC];
            gather<T, VEC>(x, pr.x, a.ldx, col, va);
            gather<T, VEC>(x, pr.y, a.ldx, col, vb);
            A dot = 0;
            A da[VEC], db[VEC];
            const A pw = pp[s];
#pragma unroll
            for (int i = 0; i < VEC; ++i) {
                const A dfdb = fma(c.w, va[i], c.z);
                const A dfda = fma(c.w, vb[i], c.y);
                const A f = fma(dfdb, vb[i], fma(c.y, va[i], c.x));
                dot = fma(g[i], f, dot);
                const A pg = pw * g[i];
                da[i] = dfda * pg;
                db[i] = dfdb * pg;
            }
            if (gx != nullptr) {
                if (pr.x >= 0) red_add<VEC>(gx + (int64_t)pr.x * ldgx + col, da);
                if (pr.y >= 0) red_add<VEC>(gx + (int64_t)pr.y * ldgx + col, db);
            }
            if (KT > 0) {
                pk[KT > 0 ? s : 0] = dot;
            } else if (part != nullptr) {
                dot = seg_sum(dot, LPN);
                if (lc == 0 && valid) part[(chunk * a.n_out + j) * K + s] = dot;
            }
        }
        if (KT > 0 && part != nullptr) {
#pragma unroll
            for (int s = 0; s < (KT > 0 ? KT : 1); ++s) {
                const A v = seg_sum(pk[s], LPN);
                if (lc == 0 && valid) part[(chunk * a.n_out + j) * K + s] = v;
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Finalize: sum partials over chunks (and over the group of neurons sharing a parameter row), then
// for logits apply the softmax backward  dL/dw_k = p_k (g_k - sum_i p_i g_i)  (torch softmax
// backward, compactlogic.py:108 + autograd).
// Row-per-warp variant for group == 1 and K <= 32.
// ---------------------------------------------------------------------------------------------
template <typename A>
__global__ void grad_finalize_warp_kernel(const LayerArgs a, const A* __restrict__ part, const int64_t nchunks,
                                          A* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int64_t R = a.n_out;  // group == 1
    if (r >= R) return;
    const int K = a.K;
    A g = 0;
    if (lane < K) {
        for (int64_t c = 0; c < nchunks; ++c) g += part[(c * a.n_out + r) * K + lane];
    }
    if (a.mode == CLB_W_LOGITS) {
        const A* w = reinterpret_cast<const A*>(a.weights) + r * K;
        A wv = lane < K ? w[lane] : -(A)FLT_MAX;
        A m = wv;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const A other = __shfl_xor_sync(0xffffffffu, m, o);
            m = other > m ? other : m;
        }
        const A e = lane < K ? exp_acc(wv - m) : (A)0;
        const A sum = warp_sum(e);
        const A p = e / sum;
        const A sp = warp_sum(p * g);
        if (lane < K) out[r * K + lane] = p * (g - sp);
    } else {
        if (lane < K) out[r * K + lane] = g;
    }
}

// Block-per-row variant (any group, K <= 256).
template <typename A>
__global__ void grad_finalize_block_kernel(const LayerArgs a, const A* __restrict__ part, const int64_t nchunks,
                                           A* __restrict__ out) {
    __shared__ A s_g[256];
    __shared__ A s_stat[3];
    const int K = a.K;
    const int64_t r = blockIdx.x;
    const int64_t G = a.group;
    for (int k = threadIdx.x; k < K; k += blockDim.x) s_g[k] = 0;
    __syncthreads();
    const int lanes_per_k = blockDim.x / K;  // >= 1
    if ((int)threadIdx.x < lanes_per_k * K) {
        const int k = threadIdx.x % K;
        const int q = threadIdx.x / K;
        A acc = 0;
        const int64_t total = nchunks * G;
        for (int64_t idx = q; idx < total; idx += lanes_per_k) {
            const int64_t c = idx / G, jj = idx - c * G;
            acc += part[(c * a.n_out + r * G + jj) * K + k];
        }
        atomicAdd(&s_g[k], acc);
    }
    __syncthreads();
    if (a.mode == CLB_W_LOGITS) {
        const A* w = reinterpret_cast<const A*>(a.weights) + r * K;
        if (threadIdx.x == 0) {
            A m = w[0];
            for (int k = 1; k < K; ++k) m = w[k] > m ? w[k] : m;
            A sum = 0, sp = 0;
            for (int k = 0; k < K; ++k) sum += exp_acc(w[k] - m);
            for (int k = 0; k < K; ++k) sp += exp_acc(w[k] - m) / sum * s_g[k];
            s_stat[0] = m;
            s_stat[1] = sum;
            s_stat[2] = sp;
        }
        __syncthreads();
        for (int k = threadIdx.x; k < K; k += blockDim.x) {
            const A p = exp_acc(w[k] - s_stat[0]) / s_stat[1];
            out[r * K + k] = p * (s_g[k] - s_stat[2]);
        }
    } else {
        for (int k = threadIdx.x; k < K; k += blockDim.x) out[r * K + k] = s_g[k];
    }
}

// ---------------------------------------------------------------------------------------------
// grad_x by gathering over the inverse connection index (difflogic_kernel.cu:140-194): a warp owns
// one input feature and a column chunk and walks every (neuron, slot, side) that reads it.
// ---------------------------------------------------------------------------------------------
template <typename T, int VEC>
__global__ void __launch_bounds__(kThreads)
backward_x_csr_kernel(const LayerArgs a, const typename Acc<T>::type* __restrict__ gy, const int64_t ldgy,
                      const int64_t in_dim, const int64_t* __restrict__ starts, const int64_t* __restrict__ ys,
                      const int8_t* __restrict__ codes, typename Acc<T>::type* __restrict__ gx, const int64_t ldgx) {
    using A = typename Acc<T>::type;
    const int lane = threadIdx.x & 31;
    const int64_t i = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
    const int64_t col = (int64_t)blockIdx.y * (32 * VEC) + lane * VEC;
    if (i >= in_dim || col >= a.ncols) return;
    const T* __restrict__ x = reinterpret_cast<const T*>(a.x);
    const A* w = reinterpret_cast<const A*>(a.weights);
    const int2* slots = reinterpret_cast<const int2*>(a.slots);
    const int K = a.K;
    A acc[VEC];
#pragma unroll
    for (int v = 0; v < VEC; ++v) acc[v] = 0;
    const int64_t e = starts[i + 1];
    for (int64_t o = starts[i]; o < e; ++o) {
        const int64_t j = ys[o];
        const int code = codes[o];
        const bool side_a = code >= 0;
        const int k = side_a ? code : -code - 1;
        const int2 pr = slots[j * K + k];
        const int64_t r = j / a.group;
        const GatePoly gp = gate_poly(a.gates[r * K + k] & 15);
        const A pw = w[r * K + k];
        A ov[VEC], gv[VEC];
        gather<T, VEC>(x, side_a ? pr.y : pr.x, a.ldx, col, ov);
        load_acc<A, VEC>(gy + j * ldgy + col, gv);
        const A c_const = side_a ? (A)gp.c1 : (A)gp.c2;
#pragma unroll
        for (int v = 0; v < VEC; ++v) acc[v] += pw * fma((A)gp.c3, ov[v], c_const) * gv[v];
    }
    store_from_acc<A, VEC>(gx + i * ldgx + col, acc);
}

// ---------------------------------------------------------------------------------------------
// Slot tables.
// ---------------------------------------------------------------------------------------------
__global__ void slots_dense_kernel(const int64_t* __restrict__ ia, const int64_t* __restrict__ ib, const int64_t n,
                                   const int64_t in_dim, int2* __restrict__ slots, int32_t* __restrict__ err) {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t va = ia[e], vb = ib[e];
        const bool oka = va >= 0 && va < in_dim, okb = vb >= 0 && vb < in_dim;
        if ((!oka || !okb) && err != nullptr) atomicOr(err, 1);
        slots[e] = make_int2(oka ? (int)va : -1, okb ? (int)vb : -1);
    }
}

// Conv slot (c, oy, ox, k): operand at (ch, oy*stride + dh, ox*stride + dw); offsets are already
// shifted by -padding (compactlogic.py:690-691), so out-of-frame coordinates are zero padding
// (convlogic_kernel.cu:110-137).
__global__ void slots_conv_kernel(const int32_t* __restrict__ och, const int8_t* __restrict__ oh,
                                  const int8_t* __restrict__ ow, const int64_t c_out, const int64_t K,
                                  const int64_t c_in, const int64_t h_in, const int64_t w_in, const int64_t h_out,
                                  const int64_t w_out, const int stride, int2* __restrict__ slots,
                                  int32_t* __restrict__ err) {
    const int64_t hw = h_out * w_out;
    const int64_t n = c_out * hw * K;
    const int64_t plane = c_out * K;  // offsets are [2, c_out, K]
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t k = e % K;
        const int64_t j = e / K;
        const int64_t c = j / hw;
        const int64_t pos = j - c * hw;
        const int64_t oy = pos / w_out, ox = pos - oy * w_out;
        int idx[2];
#pragma unroll
        for (int side = 0; side < 2; ++side) {
            const int64_t o = side * plane + c * K + k;
            const int64_t ch = och[o];
            const int64_t yy = oy * stride + oh[o];
            const int64_t xx = ox * stride + ow[o];
            if (ch < 0 || ch >= c_in) {
                if (err != nullptr) atomicOr(err, 1);
                idx[side] = -1;
            } else if (yy < 0 || yy >= h_in || xx < 0 || xx >= w_in) {
                idx[side] = -1;
            } else {
                idx[side] = (int)((ch * h_in + yy) * w_in + xx);
            }
        }
        slots[e] = make_int2(idx[0], idx[1]);
    }
}

template <typename T>
__global__ void transpose_kernel(const T* __restrict__ src, int64_t rows, int64_t cols, int64_t ld_src,
                                 T* __restrict__ dst, int64_t ld_dst) {
    __shared__ T tile[32][33];
    const int64_t r0 = (int64_t)blockIdx.y * 32, c0 = (int64_t)blockIdx.x * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int64_t r = r0 + i, c = c0 + threadIdx.x;
        if (r < rows && c < cols) tile[i][threadIdx.x] = src[r * ld_src + c];
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int64_t c = c0 + i, r = r0 + threadIdx.x;
        if (r < rows && c < cols) dst[c * ld_dst + r] = tile[threadIdx.x][i];
    }
}

template <typename S, typename D>
__global__ void cast_kernel(const S* __restrict__ src, D* __restrict__ dst, int64_t n) {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x)
        dst[e] = from_acc<D>(to_acc(src[e]));
}

int env_int(const char* name, int dflt) {
    const char* v = getenv(name);
    return v != nullptr ? atoi(v) : dflt;
}

// Tuning override (read once): CLB_TN neurons per CTA (32 / 64 / 128; default 64).
int tn_max() {
    static const int v = env_int("CLB_TN", 64);
    return (v == 32 || v == 128) ? v : 64;
}

// Column-chunk width: LPN lanes per neuron (32 = one neuron per warp step, 32*VEC columns per chunk).
// CLB_FWD_LPN / CLB_BWD_LPN force the lanes per neuron (tuning; 32 = always the full-warp chunk).
int forced_lpn(bool backward) {
    static const int f = env_int("CLB_FWD_LPN", 0);
    static const int b = env_int("CLB_BWD_LPN", 0);
    const int v = backward ? b : f;
    return (v == 2 || v == 4 || v == 8 || v == 16 || v == 32) ? v : 0;
}

int pick_lpn(int64_t in_features, int V, size_t bytes, bool backward) {
    // Measured on B200 (c5: 1M-wide inputs, bf16): narrow chunks keep the slab in L2 but cost 4-16x
    // more LSU wavefronts per byte and were slower at every width tried, so the full-warp chunk is
    // the default and the narrow kernels are opt-in.
    (void)in_features;
    (void)V;
    (void)bytes;
    return forced_lpn(backward) ? forced_lpn(backward) : 32;
}

int choose_tn(size_t bytes_per_neuron) {
    int tn = tn_max();
    while (tn > 8 && bytes_per_neuron * tn > 96 * 1024) tn >>= 1;
    return tn;
}

template <typename T> constexpr int vmax() { return 16 / (int)sizeof(T); }

// fp32 vector width of the forward / backward column split (4 = 128 columns per CTA; 2 = 64, 8 = 256);
// the environment variables CLB_FWD_VEC / CLB_BWD_VEC override it for tuning, read once per process.
int env_vec(const char* name) {
    const char* v = getenv(name);
    const int n = v != nullptr ? atoi(v) : 4;
    return (n == 2 || n == 8) ? n : 4;
}
// Offset mode of the main kernels (see scale_stage): the layer's rows must be known and every element
// offset idx * ldx must fit an int; the backward scatters with the same offsets, so ldgx must equal ldx.
// CLB_OFF32=0 disables it.
bool off32_ok(const LayerArgs& a, const void* gx, int64_t ldgx) {
    static const bool enabled = [] {
        const char* e = getenv("CLB_OFF32");
        return !(e && e[0] == '0');
    }();
    return enabled && a.in_features > 0 && a.in_features * a.ldx < (int64_t(1) << 31) &&
           (gx == nullptr || ldgx == a.ldx);
}

int fwd_vec_f32() {
    static const int v = env_vec("CLB_FWD_VEC");
    return v;
}
int bwd_vec_f32() {
    static const int v = env_vec("CLB_BWD_VEC");
    return v;
}

inline bool aligned(const void* p, int bytes) { return p == nullptr || ((uintptr_t)p % bytes) == 0; }

template <typename T>
bool can_vec(int64_t ncols, std::initializer_list<int64_t> lds, std::initializer_list<const void*> ptrs) {
    constexpr int V = vmax<T>();
    if (ncols % V) return false;
    for (int64_t ld : lds)
        if (ld % V) return false;
    for (const void* p : ptrs)
        if (!aligned(p, 16)) return false;
    return true;
}

template <typename T, int LPN>
cudaError_t fwd_narrow_l(const LayerArgs& a, void* y, int64_t ldy, const GroupSumArgs* gs, cudaStream_t s) {
    using A = typename Acc<T>::type;
    constexpr int V = vmax<T>();
    const int TN = kWarps * (32 / LPN);
    const size_t smem = stage_bytes<A>(TN, a.K, false);
    GroupSumArgs g{};
    if (gs) g = *gs;
    dim3 grid((unsigned)ceil_div64(a.n_out, TN), (unsigned)ceil_div64(a.ncols, LPN * V));
    if (grid.x == 0 || grid.y == 0) return cudaSuccess;
    auto k = logic_forward_narrow_kernel<T, V, LPN>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k<<<grid, kThreads, smem, s>>>(a, reinterpret_cast<T*>(y), ldy, g, gs != nullptr, TN);
    return cudaGetLastError();
}

template <typename T>
cudaError_t fwd_narrow(const LayerArgs& a, void* y, int64_t ldy, const GroupSumArgs* gs, int lpn, cudaStream_t s) {
    switch (lpn) {
        case 16: return fwd_narrow_l<T, 16>(a, y, ldy, gs, s);
        case 8: return fwd_narrow_l<T, 8>(a, y, ldy, gs, s);
        case 4: return fwd_narrow_l<T, 4>(a, y, ldy, gs, s);
        default: return fwd_narrow_l<T, 2>(a, y, ldy, gs, s);
    }
}

template <typename T, int LPN, int KT>
cudaError_t bwd_narrow_k(const LayerArgs& a, const void* gy, int64_t ldgy, const GroupSumArgs& g, bool use_gs, void* gx,
                         int64_t ldgx, void* part, cudaStream_t s) {
    using A = typename Acc<T>::type;
    constexpr int V = vmax<T>();
    const int TN = kWarps * (32 / LPN);
    const size_t smem = stage_bytes<A>(TN, a.K, true);
    dim3 grid((unsigned)ceil_div64(a.n_out, TN), (unsigned)ceil_div64(a.ncols, LPN * V));
    if (grid.x == 0 || grid.y == 0) return cudaSuccess;
    auto k = logic_backward_narrow_kernel<T, V, LPN, KT>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k<<<grid, kThreads, smem, s>>>(a, reinterpret_cast<const A*>(gy), ldgy, g, use_gs, reinterpret_cast<A*>(gx), ldgx,
                                   reinterpret_cast<A*>(part), TN);
    return cudaGetLastError();
}

template <typename T, int LPN>
cudaError_t bwd_narrow_l(const LayerArgs& a, const void* gy, int64_t ldgy, const GroupSumArgs& g, bool use_gs, void* gx,
                         int64_t ldgx, void* part, cudaStream_t s) {
    switch (a.K) {
        case 4: return bwd_narrow_k<T, LPN, 4>(a, gy, ldgy, g, use_gs, gx, ldgx, part, s);
        case 8: return bwd_narrow_k<T, LPN, 8>(a, gy, ldgy, g, use_gs, gx, ldgx, part, s);
        case 16: return bwd_narrow_k<T, LPN, 16>(a, gy, ldgy, g, use_gs, gx, ldgx, part, s);
        default: return bwd_narrow_k<T, LPN, 0>(a, gy, ldgy, g, use_gs, gx, ldgx, part, s);
    }
}

template <typename T>
cudaError_t bwd_narrow(const LayerArgs& a, const void* gy, int64_t ldgy, const GroupSumArgs& g, bool use_gs, void* gx,
                       int64_t ldgx, void* part, int lpn, cudaStream_t s) {
    switch (lpn) {
        case 16: return bwd_narrow_l<T, 16>(a, gy, ldgy, g, use_gs, gx, ldgx, part, s);
        case 8: return bwd_narrow_l<T, 8>(a, gy, ldgy, g, use_gs, gx, ldgx, part, s);
        case 4: return bwd_narrow_l<T, 4>(a, gy, ldgy, g, use_gs, gx, ldgx, part, s);
        default: return bwd_narrow_l<T, 2>(a, gy, ldgy, g, use_gs, gx, ldgx, part, s);
    }
}

template <typename T>
int bwd_lpn(const LayerArgs& a, bool vec, int V, const void* gx, bool peers) {
    using A = typename Acc<T>::type;
    if (!vec || V != vmax<T>() || std::is_same<T, double>::value || peers) return 32;
    return pick_lpn(a.in_features, V, sizeof(T) + (gx != nullptr ? sizeof(A) : 0), true);
}

template <typename T, int VEC>
void fwd_launch(const LayerArgs& a, void* y, int64_t ldy, const GroupSumArgs& g, bool use_gs, dim3 grid, size_t smem,
                int TN, cudaStream_t s, const PeerArgs& pa, void* stage) {
    using A = typename Acc<T>::type;
    const bool off = off32_ok(a, nullptr, 0);
    FwdBake<A> fb{};
    if (stage != nullptr && pa.n == 0) {
        fb = carve_bake<A>(stage, (int64_t)grid.x * TN, a.K);
        if (off) fwd_bake_kernel<A, true><<<grid.x, kThreads, 0, s>>>(a, TN, fb);
        else fwd_bake_kernel<A, false><<<grid.x, kThreads, 0, s>>>(a, TN, fb);
        auto k = off ? logic_forward_kernel<T, VEC, false, true, true> : logic_forward_kernel<T, VEC, false, false, true>;
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        k<<<grid, kThreads, smem, s>>>(a, reinterpret_cast<T*>(y), ldy, g, use_gs, TN, pa, fb);
        return;
    }
    // the peer-store epilogue is a separate instantiation so the single-GPU kernel keeps its registers
    auto k = pa.n ? logic_forward_kernel<T, VEC, true, false>
                  : off ? logic_forward_kernel<T, VEC, false, true>
                        : logic_forward_kernel<T, VEC, false, false>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k<<<grid, kThreads, smem, s>>>(a, reinterpret_cast<T*>(y), ldy, g, use_gs, TN, pa, fb);
}

// Bytes of the baked forward stage of a layer (0 when the layer's forward does not use one).
template <typename T>
size_t fwd_stage_bytes_t(int64_t n_out, int K) {
    using A = typename Acc<T>::type;
    const int TN = choose_tn(stage_bytes<A>(1, K, false));
    return bake_bytes<A>(ceil_div64(n_out, TN) * TN, K);
}

template <typename T>
cudaError_t fwd_t(const LayerArgs& a, void* y, int64_t ldy, const GroupSumArgs* gs, cudaStream_t s,
                  const PeerArgs& pa, void* stage) {
    using A = typename Acc<T>::type;
    const int K = a.K;
    const int TN = choose_tn(stage_bytes<A>(1, K, false));
    const size_t smem = stage_bytes<A>(TN, K, false);
    GroupSumArgs g{};
    if (gs) g = *gs;
    const bool vec = can_vec<T>(a.ncols, {a.ldx, gs ? gs->ld : ldy}, {a.x, y, gs ? gs->acc : nullptr}) &&
                     (gs == nullptr || (gs->ld % vmax<T>() == 0));
    const int fv = std::is_same<T, float>::value ? fwd_vec_f32() : vmax<T>();
    const bool wide = vec && fv == 8 && a.ncols % 8 == 0 && a.ldx % 8 == 0 && (gs ? gs->ld : ldy) % 8 == 0;
    const bool half = vec && fv == 2;
    const int V = vec ? (half ? 2 : wide ? 8 : vmax<T>()) : 1;
    dim3 grid((unsigned)ceil_div64(a.n_out, TN), (unsigned)ceil_div64(a.ncols, 32 * V));
    if (grid.x == 0 || grid.y == 0) return cudaSuccess;
    const int lpn = (vec && !wide && !half && !std::is_same<T, double>::value && pa.n == 0) ? pick_lpn(a.in_features, V, sizeof(T), false)
                                                                                  : 32;
    if (lpn < 32) return fwd_narrow<T>(a, y, ldy, gs, lpn, s);
    if (wide) {
        fwd_launch<T, 8>(a, y, ldy, g, gs != nullptr, grid, smem, TN, s, pa, stage);
    } else if (half) {
        fwd_launch<T, 2>(a, y, ldy, g, gs != nullptr, grid, smem, TN, s, pa, stage);
    } else if (vec) {
        fwd_launch<T, vmax<T>()>(a, y, ldy, g, gs != nullptr, grid, smem, TN, s, pa, stage);
    } else {
        fwd_launch<T, 1>(a, y, ldy, g, gs != nullptr, grid, smem, TN, s, pa, stage);
    }
    return cudaGetLastError();
}

template <typename T, int VEC, int KT>
cudaError_t bwd_launch(const LayerArgs& a, const void* gy, int64_t ldgy, const GroupSumArgs& g, bool use_gs,
                       void* gx, int64_t ldgx, void* part, dim3 grid, size_t smem, int TN, cudaStream_t s,
                       const PeerArgs& pa) {
    using A = typename Acc<T>::type;
    // GX = false (no grad_x) only in offset mode; the other variants check gx at run time
    auto k = pa.n ? logic_backward_kernel<T, VEC, KT, true, false, true>
                  : !off32_ok(a, gx, ldgx) ? logic_backward_kernel<T, VEC, KT, false, false, true>
                  : gx != nullptr          ? logic_backward_kernel<T, VEC, KT, false, true, true>
                                           : logic_backward_kernel<T, VEC, KT, false, true, false>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k<<<grid, kThreads, smem, s>>>(a, reinterpret_cast<const A*>(gy), ldgy, g, use_gs, reinterpret_cast<A*>(gx), ldgx,
                                   reinterpret_cast<A*>(part), TN, pa);
    return cudaGetLastError();
}

template <typename T, int VEC>
cudaError_t bwd_k(const LayerArgs& a, const void* gy, int64_t ldgy, const GroupSumArgs& g, bool use_gs, void* gx,
                  int64_t ldgx, void* part, dim3 grid, size_t smem, int TN, cudaStream_t s, const PeerArgs& pa) {
    switch (a.K) {
        case 4: return bwd_launch<T, VEC, 4>(a, gy, ldgy, g, use_gs, gx, ldgx, part, grid, smem, TN, s, pa);
        case 8: return bwd_launch<T, VEC, 8>(a, gy, ldgy, g, use_gs, gx, ldgx, part, grid, smem, TN, s, pa);
        case 16: return bwd_launch<T, VEC, 16>(a, gy, ldgy, g, use_gs, gx, ldgx, part, grid, smem, TN, s, pa);
        default: return bwd_launch<T, VEC, 0>(a, gy, ldgy, g, use_gs, gx, ldgx, part, grid, smem, TN, s, pa);
    }
}

template <typename T>
bool bwd_vec(const LayerArgs& a, const void* gy, int64_t ldgy, const GroupSumArgs* gs, const void* gx,
             int64_t ldgx) {
    using A = typename Acc<T>::type;
    constexpr int V = vmax<T>();
    // gradients are in the arithmetic type: V elements of A must also be whole vectors
    if (!can_vec<T>(a.ncols, {a.ldx, ldgx}, {a.x, gx})) return false;
    if (gy != nullptr && (ldgy % V || !aligned(gy, (int)(sizeof(A) * V > 16 ? 16 : sizeof(A) * V)))) return false;
    if (gs != nullptr && (gs->ld % V || !aligned(gs->grad, 16))) return false;
    return true;
}

inline bool bwd_wide_ok(const LayerArgs& a, int64_t ldgy, const GroupSumArgs* gs, int64_t ldgx) {
    return a.ncols % 8 == 0 && a.ldx % 8 == 0 && ldgx % 8 == 0 && (gs ? gs->ld : ldgy) % 8 == 0;
}

template <typename T>
cudaError_t bwd_t(const LayerArgs& a, const void* gy, int64_t ldgy, const GroupSumArgs* gs, void* gx, int64_t ldgx,
                  void* part, int64_t part_chunks, cudaStream_t s, const PeerArgs& pa) {
    using A = typename Acc<T>::type;
    const int K = a.K;
    const int TN = choose_tn(stage_bytes<A>(1, K, true));
    const size_t smem = stage_bytes<A>(TN, K, true);
    GroupSumArgs g{};
    if (gs) g = *gs;
    const bool vec = bwd_vec<T>(a, gy, ldgy, gs, gx, ldgx);
    const int bv = std::is_same<T, float>::value ? bwd_vec_f32() : vmax<T>();
    const bool wide = vec && bv == 8 && bwd_wide_ok(a, ldgy, gs, ldgx);
    const bool half = vec && bv == 2;
    const int V = vec ? (half ? 2 : wide ? 8 : vmax<T>()) : 1;
    const int lpn = bwd_lpn<T>(a, vec, V, gx, pa.n != 0);
    if (lpn < 32) {
        if (part != nullptr && ceil_div64(a.ncols, lpn * V) != part_chunks) return cudaErrorInvalidValue;
        return bwd_narrow<T>(a, gy, ldgy, g, gs != nullptr, gx, ldgx, part, lpn, s);
    }
    dim3 grid((unsigned)ceil_div64(a.n_out, TN), (unsigned)ceil_div64(a.ncols, 32 * V));
    if (part != nullptr && (int64_t)grid.y != part_chunks) return cudaErrorInvalidValue;  // scratch sized for another split
    if (grid.x == 0 || grid.y == 0) return cudaSuccess;
    if (half) return bwd_k<T, 2>(a, gy, ldgy, g, gs != nullptr, gx, ldgx, part, grid, smem, TN, s, pa);
    if (wide) return bwd_k<T, 8>(a, gy, ldgy, g, gs != nullptr, gx, ldgx, part, grid, smem, TN, s, pa);
    if (vec) return bwd_k<T, vmax<T>()>(a, gy, ldgy, g, gs != nullptr, gx, ldgx, part, grid, smem, TN, s, pa);
    return bwd_k<T, 1>(a, gy, ldgy, g, gs != nullptr, gx, ldgx, part, grid, smem, TN, s, pa);
}

template <typename T>
cudaError_t csr_t(const LayerArgs& a, const void* gy, int64_t ldgy, int64_t in_dim, const int64_t* starts,
                  const int64_t* ys, const int8_t* codes, void* gx, int64_t ldgx, cudaStream_t s) {
    using A = typename Acc<T>::type;
    const bool vec = bwd_vec<T>(a, gy, ldgy, nullptr, gx, ldgx);
    const int V = vec ? vmax<T>() : 1;
    dim3 grid((unsigned)ceil_div64(in_dim, kWarps), (unsigned)ceil_div64(a.ncols, 32 * V));
    if (grid.x == 0 || grid.y == 0) return cudaSuccess;
    if (vec)
        backward_x_csr_kernel<T, vmax<T>()><<<grid, kThreads, 0, s>>>(a, reinterpret_cast<const A*>(gy), ldgy, in_dim,
                                                                    starts, ys, codes, reinterpret_cast<A*>(gx), ldgx);
    else
        backward_x_csr_kernel<T, 1><<<grid, kThreads, 0, s>>>(a, reinterpret_cast<const A*>(gy), ldgy, in_dim, starts,
                                                              ys, codes, reinterpret_cast<A*>(gx), ldgx);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_logic_forward(const LayerArgs& a, void* y, int64_t ldy, const GroupSumArgs* gs, cudaStream_t s,
                                 const PeerArgs* peers, void* stage) {
    const PeerArgs pa = peers ? *peers : PeerArgs{};
    switch (a.dtype) {
        case CLB_F32: return fwd_t<float>(a, y, ldy, gs, s, pa, stage);
        case CLB_F64: return fwd_t<double>(a, y, ldy, gs, s, pa, stage);
        case CLB_BF16: return fwd_t<__nv_bfloat16>(a, y, ldy, gs, s, pa, stage);
        case CLB_F16: return fwd_t<__half>(a, y, ldy, gs, s, pa, stage);
    }
    return cudaErrorInvalidValue;
}

size_t logic_forward_stage_bytes(int dtype, int64_t n_out, int64_t K) {
    switch (dtype) {
        case CLB_F32: return fwd_stage_bytes_t<float>(n_out, (int)K);
        case CLB_F64: return fwd_stage_bytes_t<double>(n_out, (int)K);
        case CLB_BF16: return fwd_stage_bytes_t<__nv_bfloat16>(n_out, (int)K);
        case CLB_F16: return fwd_stage_bytes_t<__half>(n_out, (int)K);
    }
    return 0;
}

cudaError_t launch_logic_backward(const LayerArgs& a, const void* gy, int64_t ldgy, const GroupSumArgs* gs, void* gx,
                                  int64_t ldgx, void* partials, int64_t part_chunks, cudaStream_t s,
                                  const PeerArgs* peers) {
    const PeerArgs pa = peers ? *peers : PeerArgs{};
    switch (a.dtype) {
        case CLB_F32: return bwd_t<float>(a, gy, ldgy, gs, gx, ldgx, partials, part_chunks, s, pa);
        case CLB_F64: return bwd_t<double>(a, gy, ldgy, gs, gx, ldgx, partials, part_chunks, s, pa);
        case CLB_BF16: return bwd_t<__nv_bfloat16>(a, gy, ldgy, gs, gx, ldgx, partials, part_chunks, s, pa);
        case CLB_F16: return bwd_t<__half>(a, gy, ldgy, gs, gx, ldgx, partials, part_chunks, s, pa);
    }
    return cudaErrorInvalidValue;
}

int64_t logic_backward_chunks(int dtype, int64_t ncols, int64_t ldx, const void* x, int64_t ldgy, const void* gy,
                              int64_t ld_gs, const void* gs_grad, int64_t ldgx, const void* gx, int64_t in_features) {
    GroupSumArgs g{};
    g.grad = gs_grad;
    g.ld = ld_gs;
    const GroupSumArgs* gs = gs_grad != nullptr ? &g : nullptr;
    if (gs != nullptr) gy = nullptr;
    LayerArgs a{};
    a.dtype = dtype;
    a.ncols = ncols;
    a.ldx = ldx;
    a.x = x;
    a.in_features = in_features;
    bool vec = false;
    int v = 1, lpn = 32;
    switch (dtype) {
        case CLB_F32: {
            vec = bwd_vec<float>(a, gy, ldgy, gs, gx, ldgx);
            const int bv = bwd_vec_f32();
            const bool wide = vec && bv == 8 && bwd_wide_ok(a, gs ? 0 : ldgy, gs, ldgx);
            v = vec ? (bv == 2 ? 2 : wide ? 8 : 4) : 1;
            lpn = bwd_lpn<float>(a, vec, v, gx, false);
            break;
        }
        case CLB_F64:
            vec = bwd_vec<double>(a, gy, ldgy, gs, gx, ldgx);
            v = vec ? vmax<double>() : 1;
            break;
        case CLB_BF16:
            vec = bwd_vec<__nv_bfloat16>(a, gy, ldgy, gs, gx, ldgx);
            v = vec ? vmax<__nv_bfloat16>() : 1;
            lpn = bwd_lpn<__nv_bfloat16>(a, vec, v, gx, false);
            break;
        case CLB_F16:
            vec = bwd_vec<__half>(a, gy, ldgy, gs, gx, ldgx);
            v = vec ? vmax<__half>() : 1;
            lpn = bwd_lpn<__half>(a, vec, v, gx, false);
            break;
        default: return -1;
    }
    return ceil_div64(ncols, lpn * v);
}

cudaError_t launch_grad_finalize(const LayerArgs& a, const void* partials, int64_t nchunks, void* out, int out_dtype,
                                 cudaStream_t s) {
    (void)out_dtype;
    const int64_t R = a.n_out / a.group;
    if (R == 0) return cudaSuccess;
    if (a.dtype == CLB_F64) {
        if (a.group == 1 && a.K <= 32)
            grad_finalize_warp_kernel<double><<<(unsigned)ceil_div64(R, 8), 256, 0, s>>>(
                a, reinterpret_cast<const double*>(partials), nchunks, reinterpret_cast<double*>(out));
        else
            grad_finalize_block_kernel<double><<<(unsigned)R, 256, 0, s>>>(a, reinterpret_cast<const double*>(partials),
                                                                          nchunks, reinterpret_cast<double*>(out));
    } else {
        if (a.group == 1 && a.K <= 32)
            grad_finalize_warp_kernel<float><<<(unsigned)ceil_div64(R, 8), 256, 0, s>>>(
                a, reinterpret_cast<const float*>(partials), nchunks, reinterpret_cast<float*>(out));
        else
            grad_finalize_block_kernel<float><<<(unsigned)R, 256, 0, s>>>(a, reinterpret_cast<const float*>(partials),
                                                                         nchunks, reinterpret_cast<float*>(out));
    }
    return cudaGetLastError();
}

cudaError_t launch_backward_x_csr(const LayerArgs& a, const void* gy, int64_t ldgy, int64_t in_dim,
                                  const int64_t* starts, const int64_t* ys, const int8_t* codes, void* gx,
                                  int64_t ldgx, cudaStream_t s) {
    switch (a.dtype) {
        case CLB_F32: return csr_t<float>(a, gy, ldgy, in_dim, starts, ys, codes, gx, ldgx, s);
        case CLB_F64: return csr_t<double>(a, gy, ldgy, in_dim, starts, ys, codes, gx, ldgx, s);
        case CLB_BF16: return csr_t<__nv_bfloat16>(a, gy, ldgy, in_dim, starts, ys, codes, gx, ldgx, s);
        case CLB_F16: return csr_t<__half>(a, gy, ldgy, in_dim, starts, ys, codes, gx, ldgx, s);
    }
    return cudaErrorInvalidValue;
}

cudaError_t launch_slots_dense(const int64_t* a, const int64_t* b, int64_t n_out, int64_t K, int64_t in_dim,
                               int32_t* slots, int32_t* err, cudaStream_t s) {
    const int64_t n = n_out * K;
    if (n == 0) return cudaSuccess;
    const unsigned blocks = (unsigned)std::min<int64_t>(ceil_div64(n, 256), 148 * 16);
    slots_dense_kernel<<<blocks, 256, 0, s>>>(a, b, n, in_dim, reinterpret_cast<int2*>(slots), err);
    return cudaGetLastError();
}

cudaError_t launch_slots_conv(const int32_t* och, const int8_t* oh, const int8_t* ow, int64_t c_out, int64_t K,
                              int64_t c_in, int64_t h_in, int64_t w_in, int64_t h_out, int64_t w_out, int stride,
                              int32_t* slots, int32_t* err, cudaStream_t s) {
    const int64_t n = c_out * h_out * w_out * K;
    if (n == 0) return cudaSuccess;
    const unsigned blocks = (unsigned)std::min<int64_t>(ceil_div64(n, 256), 148 * 16);
    slots_conv_kernel<<<blocks, 256, 0, s>>>(och, oh, ow, c_out, K, c_in, h_in, w_in, h_out, w_out, stride,
                                             reinterpret_cast<int2*>(slots), err);
    return cudaGetLastError();
}

cudaError_t launch_transpose(int elem_bytes, const void* src, int64_t rows, int64_t cols, int64_t ld_src, void* dst,
                             int64_t ld_dst, cudaStream_t s) {
    if (rows == 0 || cols == 0) return cudaSuccess;
    dim3 grid((unsigned)ceil_div64(cols, 32), (unsigned)ceil_div64(rows, 32));
    dim3 block(32, 8);
    switch (elem_bytes) {
        case 1: transpose_kernel<uint8_t><<<grid, block, 0, s>>>((const uint8_t*)src, rows, cols, ld_src, (uint8_t*)dst, ld_dst); break;
        case 2: transpose_kernel<uint16_t><<<grid, block, 0, s>>>((const uint16_t*)src, rows, cols, ld_src, (uint16_t*)dst, ld_dst); break;
        case 4: transpose_kernel<uint32_t><<<grid, block, 0, s>>>((const uint32_t*)src, rows, cols, ld_src, (uint32_t*)dst, ld_dst); break;
        case 8: transpose_kernel<uint64_t><<<grid, block, 0, s>>>((const uint64_t*)src, rows, cols, ld_src, (uint64_t*)dst, ld_dst); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_cast(int src_dtype, const void* src, int dst_dtype, void* dst, int64_t n, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    const unsigned blocks = (unsigned)std::min<int64_t>(ceil_div64(n, 256), 148 * 16);
    if (src_dtype == CLB_F32 && dst_dtype == CLB_BF16)
        cast_kernel<float, __nv_bfloat16><<<blocks, 256, 0, s>>>((const float*)src, (__nv_bfloat16*)dst, n);
    else if (src_dtype == CLB_BF16 && dst_dtype == CLB_F32)
        cast_kernel<__nv_bfloat16, float><<<blocks, 256, 0, s>>>((const __nv_bfloat16*)src, (float*)dst, n);
    else if (src_dtype == CLB_F32 && dst_dtype == CLB_F16)
        cast_kernel<float, __half><<<blocks, 256, 0, s>>>((const float*)src, (__half*)dst, n);
    else if (src_dtype == CLB_F16 && dst_dtype == CLB_F32)
        cast_kernel<__half, float><<<blocks, 256, 0, s>>>((const __half*)src, (float*)dst, n);
    else
        return cudaErrorInvalidValue;
    return cudaGetLastError();
}

}  // namespace clb
