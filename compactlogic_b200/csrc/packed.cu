// Bit-packed discrete inference: 64 samples per uint64 word, one argmax gate per neuron.
//
// Activations are [features, words] with bit i of word w holding sample 64*w + i (LSB first), the
// bit order of the reference's tensor_packbits_cuda (compactlogic/cuda/difflogic_kernel.cu:434-449).
// Because that order is little-endian, a row packed into 8/16/32/64-bit words has the same bytes
// for every width; only the row length is rounded to the word width.
//
// A layer evaluates one gate per neuron on whole words (gates.cuh gate_word, a branch-free
// multiplexer over the truth-table bits), so one 8-byte load per operand yields 64 gate-evals.
// GroupSum on packed words (groupbitsum, difflogic_kernel.cu:500-533) is a per-bit-position
// ("vertical") population count over the neurons of a class; it is computed with a Harley-Seal
// carry-save adder tree over 16 words at a time (about 4 logic ops per word instead of 64 bit
// tests), and the final layer can be fused with it so its outputs are never stored.
#include <cuda_runtime.h>
#include <utility>

#include <stdlib.h>

#include <algorithm>

#include "common.cuh"
#include "gates.cuh"
#include "kernels.h"

namespace clb {

namespace {

// ------------------------------------------------------------------------------------------
// Harley-Seal vertical counter: 64 independent counters, one per bit position.
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void csa(uint64_t& h, uint64_t& l, uint64_t a, uint64_t b, uint64_t c) {
    const uint64_t u = a ^ b;
    h = (a & b) | (u & c);
    l = u ^ c;
}

// 64 bit-sliced counters of 8 bits (counts up to 255): ones/twos/fours/eights are the Harley-Seal
// state, hi[0..3] count the 16s.  A thread adds at most kMaxWords words.
struct VCounter {
    static constexpr int kMaxWords = 240;
    uint64_t ones = 0, twos = 0, fours = 0, eights = 0;
    uint64_t hi[4] = {0, 0, 0, 0};
    // Add 16 words.
    __device__ __forceinline__ void add16(const uint64_t (&d)[16]) {
        uint64_t twosA, twosB, foursA, foursB, eightsA, eightsB, sixteens;
        csa(twosA, ones, ones, d[0], d[1]);
        csa(twosB, ones, ones, d[2], d[3]);
        csa(foursA, twos, twos, twosA, twosB);
        csa(twosA, ones, ones, d[4], d[5]);
        csa(twosB, ones, ones, d[6], d[7]);
        csa(foursB, twos, twos, twosA, twosB);
        csa(eightsA, fours, fours, foursA, foursB);
        csa(twosA, ones, ones, d[8], d[9]);
        csa(twosB, ones, ones, d[10], d[11]);
        csa(foursA, twos, twos, twosA, twosB);
        csa(twosA, ones, ones, d[12], d[13]);
        csa(twosB, ones, ones, d[14], d[15]);
        csa(foursB, twos, twos, twosA, twosB);
        csa(eightsB, fours, fours, foursA, foursB);
        csa(sixteens, eights, eights, eightsA, eightsB);
        uint64_t carry = sixteens;
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            const uint64_t t = hi[p] & carry;
            hi[p] ^= carry;
            carry = t;
        }
    }
    // Add 8 words (the carry out of the 8s plane is a half-adder step).
    __device__ __forceinline__ void add8(const uint64_t (&d)[8]) {
        uint64_t twosA, twosB, foursA, foursB, eightsA;
        csa(twosA, ones, ones, d[0], d[1]);
        csa(twosB, ones, ones, d[2], d[3]);
        csa(foursA, twos, twos, twosA, twosB);
        csa(twosA, ones, ones, d[4], d[5]);
        csa(twosB, ones, ones, d[6], d[7]);
        csa(foursB, twos, twos, twosA, twosB);
        csa(eightsA, fours, fours, foursA, foursB);
        uint64_t carry = eights & eightsA;
        eights ^= eightsA;
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            const uint64_t t = hi[p] & carry;
            hi[p] ^= carry;
            carry = t;
        }
    }
    // 8x8 bit-matrix transpose: in byte r / bit c -> out byte c / bit r.
    static __device__ __forceinline__ uint64_t transpose8x8(uint64_t x) {
        uint64_t t;
        t = (x ^ (x >> 7)) & 0x00AA00AA00AA00AAull;
        x = x ^ t ^ (t << 7);
        t = (x ^ (x >> 14)) & 0x0000CCCC0000CCCCull;
        x = x ^ t ^ (t << 14);
        t = (x ^ (x >> 28)) & 0x00000000F0F0F0F0ull;
        x = x ^ t ^ (t << 28);
        return x;
    }
    // Counts of positions 8m .. 8m+7 as the 8 bytes of one word: byte q of the gathered word is byte m
    // of plane q; after the transpose byte r holds the 8-bit count of position 8m + r.
    __device__ __forceinline__ uint64_t counts8(int m) const {
        const int sh = 8 * m;
        const uint64_t x = ((ones >> sh) & 0xff) | (((twos >> sh) & 0xff) << 8) | (((fours >> sh) & 0xff) << 16) |
                           (((eights >> sh) & 0xff) << 24) | (((hi[0] >> sh) & 0xff) << 32) |
                           (((hi[1] >> sh) & 0xff) << 40) | (((hi[2] >> sh) & 0xff) << 48) |
                           (((hi[3] >> sh) & 0xff) << 56);
        return transpose8x8(x);
    }
};

// Load 8 bytes of a packed row at byte offset `off`, zero beyond `row_bytes`.
__device__ __forceinline__ uint64_t load_word_bytes(const uint8_t* __restrict__ row, int64_t off, int64_t row_bytes,
                                                    bool aligned8) {
    if (aligned8 && off + 8 <= row_bytes) return *reinterpret_cast<const uint64_t*>(row + off);
    uint64_t v = 0;
    for (int b = 0; b < 8; ++b)
        if (off + b < row_bytes) v |= (uint64_t)row[off + b] << (8 * b);
    return v;
}

// ------------------------------------------------------------------------------------------
// tensor_packbits: bool [rows, cols] -> little-endian packed rows of `row_bytes` bytes.
// One warp per 32 samples of one row: the ballot of the 32 bools is the 4 packed bytes.
// ------------------------------------------------------------------------------------------
__global__ void packbits_kernel(const uint8_t* __restrict__ t, int64_t rows, int64_t cols, int64_t ld_t,
                                uint8_t* __restrict__ out, int64_t row_bytes) {
    const int lane = threadIdx.x & 31;
    const int64_t nblk = (row_bytes + 3) / 4;
    const int64_t total = rows * nblk;
    for (int64_t e = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; e < total;
         e += ((int64_t)gridDim.x * blockDim.x) >> 5) {
        const int64_t r = e / nblk, blk = e - r * nblk;
        const int64_t c = blk * 32 + lane;
        const bool bit = c < cols && t[r * ld_t + c] != 0;
        const uint32_t word = __ballot_sync(0xffffffffu, bit);
        if (lane < 4) {
            const int64_t byte = blk * 4 + lane;
            if (byte < row_bytes) out[r * row_bytes + byte] = (uint8_t)(word >> (8 * lane));
        }
    }
}

// pack_inputs: x [batch, features] (sample-major, values in {0,1}; bit = x > 0.5)
//           -> out [features, ldw] uint64, bit i of word w = sample 64 w + i.
template <typename T>
__global__ void pack_inputs_kernel(const T* __restrict__ x, int64_t batch, int64_t features, int64_t ldx,
                                   uint64_t* __restrict__ out, int64_t ldw) {
    __shared__ uint8_t tile[64][33];
    const int64_t s0 = (int64_t)blockIdx.y * 64, f0 = (int64_t)blockIdx.x * 32;
    for (int i = threadIdx.y; i < 64; i += blockDim.y) {
        const int64_t s = s0 + i, f = f0 + threadIdx.x;
        uint8_t b = 0;
        if (s < batch && f < features) b = to_acc(x[s * ldx + f]) > 0.5f;
        tile[i][threadIdx.x] = b;
    }
    __syncthreads();
    if (threadIdx.y < 2) {
        const int64_t f = f0 + threadIdx.x;
        uint32_t half = 0;
        for (int i = 0; i < 32; ++i) half |= (uint32_t)tile[threadIdx.y * 32 + i][threadIdx.x] << i;
        if (f < features) reinterpret_cast<uint32_t*>(out + f * ldw + blockIdx.y)[threadIdx.y] = half;
    }
}

// pack_thresholds: raw inputs x [batch, C*HW] -> nthr*C*HW packed features, feature t*C*HW + f having
// bit = x[s, f] > (t+1)/(nthr+1) (the reference's CIFAR binarisation, experiments/experiment_script.py:92,
// threshold-major channel order).  Each raw value is read once for all thresholds.
template <typename T>
__global__ void pack_thresholds_kernel(const T* __restrict__ x, int64_t batch, int64_t features, int64_t ldx,
                                       int nthr, uint64_t* __restrict__ out, int64_t ldw) {
    __shared__ float tile[64][33];
    const int64_t s0 = (int64_t)blockIdx.y * 64, f0 = (int64_t)blockIdx.x * 32;
    for (int i = threadIdx.y; i < 64; i += blockDim.y) {
        const int64_t s = s0 + i, f = f0 + threadIdx.x;
        tile[i][threadIdx.x] = (s < batch && f < features) ? (float)to_acc(x[s * ldx + f]) : -1.0f;
    }
    __syncthreads();
    const int64_t f = f0 + threadIdx.x;
    for (int t = threadIdx.y; t < 2 * nthr; t += blockDim.y) {  // (threshold, 32-sample half) pairs
        const int thr = t >> 1, half = t & 1;
        const float level = (float)((thr + 1.0) / (nthr + 1.0));
        uint32_t bits = 0;
        for (int i = 0; i < 32; ++i) bits |= (uint32_t)(tile[half * 32 + i][threadIdx.x] > level) << i;
        if (f < features) reinterpret_cast<uint32_t*>(out + ((int64_t)thr * features + f) * ldw + blockIdx.y)[half] = bits;
    }
}

__global__ void packed_select_kernel(const int2* __restrict__ slots, const uint8_t* __restrict__ gates,
                                     const uint8_t* __restrict__ select, int64_t n_out, int K, int64_t group,
                                     int2* __restrict__ sel_ab, uint8_t* __restrict__ sel_gate) {
    for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n_out; j += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = j / group;
        const int k = select[r];
        if (k < K) {
            // drop the operands the gate ignores (constant / single-input gates) so no load is issued
            const int g = gates[r * K + k] & 15;
            const GatePoly gp = gate_poly(g);
            int2 s = slots[j * K + k];
            if (gp.c1 == 0.f && gp.c3 == 0.f) s.x = -1;
            if (gp.c2 == 0.f && gp.c3 == 0.f) s.y = -1;
            sel_ab[j] = s;
            sel_gate[j] = (uint8_t)g;
        } else {  // invalid selection: constant-0 gate
            sel_ab[j] = make_int2(-1, -1);
            sel_gate[j] = 0;
        }
    }
}

__device__ __forceinline__ uint64_t word_or_zero(const uint64_t* __restrict__ x, int idx, int64_t ldx, int64_t w) {
    return idx >= 0 ? __ldg(x + (int64_t)idx * ldx + w) : 0ull;
}

// Programmatic dependent launch: a kernel of the packed chain lets the next one be scheduled as soon as
// all its CTAs have started (launch_dependents), and waits for its predecessor's completion and memory
// (wait) only after the prologue that reads nothing the predecessor writes.  Both are no-ops when the
// kernel was not launched with the programmatic-serialization attribute.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// One packed layer.  Each lane owns V consecutive word columns (V = 2: one 16-byte load per operand),
// TW lanes span TW*V columns, 32/TW neurons share a warp row, and each thread handles R neurons
// spaced 32/TW apart so that 2R independent loads are in flight per thread.
template <int R, int V, int MINB = 1>
__global__ void __launch_bounds__(256, MINB)
packed_layer_kernel(const uint64_t* __restrict__ x, int64_t ldx, int64_t nwords, const int2* __restrict__ sel_ab,
                    const uint8_t* __restrict__ sel_gate, int64_t n_out, uint64_t* __restrict__ y, int64_t ldy,
                    int tw_log2) {
    using Vw = Vec<uint64_t, V>;
    const int TW = 1 << tw_log2;
    const int lane = threadIdx.x & 31;
    const int64_t w = ((int64_t)blockIdx.x * TW + (lane & (TW - 1))) * V;
    const int64_t npw = 32 >> tw_log2;  // neurons per warp row
    const int64_t warp_global = ((int64_t)blockIdx.y * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.y * blockDim.x) >> 5;
    if (w >= nwords) return;
    for (int64_t base = warp_global * npw * R; base < n_out; base += nwarps * npw * R) {
        int2 ab[R];
        int g[R];
#pragma unroll
        for (int q = 0; q < R; ++q) {
            const int64_t j = base + q * npw + (lane >> tw_log2);
            ab[q] = j < n_out ? sel_ab[j] : make_int2(-1, -1);
            g[q] = j < n_out ? sel_gate[j] : 0;
        }
        Vw va[R], vb[R];
#pragma unroll
        for (int q = 0; q < R; ++q) {
#pragma unroll
            for (int i = 0; i < V; ++i) va[q].v[i] = vb[q].v[i] = 0;
            if (ab[q].x >= 0) va[q] = *reinterpret_cast<const Vw*>(x + (int64_t)ab[q].x * ldx + w);
            if (ab[q].y >= 0) vb[q] = *reinterpret_cast<const Vw*>(x + (int64_t)ab[q].y * ldx + w);
        }
#pragma unroll
        for (int q = 0; q < R; ++q) {
            const int64_t j = base + q * npw + (lane >> tw_log2);
            if (j < n_out) {
                Vw o;
#pragma unroll
                for (int i = 0; i < V; ++i) o.v[i] = gate_word<uint64_t>(g[q], va[q].v[i], vb[q].v[i]);
                *reinterpret_cast<Vw*>(y + j * ldy + w) = o;
            }
        }
    }
}

// Stores of a packed layer's output words.  ST = 0: plain store.  ST = 1: store under an L2 evict-first
// cache policy, so the 262 MB of freshly written output (read again only by the next launch) displaces
// less of the operand slab that this launch is still gathering from.
template <int ST, int V>
__device__ __forceinline__ void store_words(uint64_t* p, const Vec<uint64_t, V>& o, uint64_t policy) {
    if constexpr (ST == 1 && V == 2) {
        asm volatile("st.global.L2::cache_hint.v2.u64 [%0], {%1, %2}, %3;" ::"l"(p), "l"(o.v[0]), "l"(o.v[1]),
                     "l"(policy)
                     : "memory");
    } else if constexpr (ST == 1) {
#pragma unroll
        for (int i = 0; i < V; ++i)
            asm volatile("st.global.L2::cache_hint.u64 [%0], %1, %2;" ::"l"(p + i), "l"(o.v[i]), "l"(policy) : "memory");
    } else {
        *reinterpret_cast<Vec<uint64_t, V>*>(p) = o;
    }
}

__device__ __forceinline__ uint64_t evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// Persistent variant: a grid of about one wave strides over the neuron tiles, and each warp loads the
// tables of its next tile while the operand words of the current one are in flight, so a tile costs one
// memory round trip instead of two (tables, then operands) plus a CTA launch.
template <int R, int V, int MINB = 1, int ST = 0>
__global__ void __launch_bounds__(256, MINB)
packed_layer_pipe_kernel(const uint64_t* __restrict__ x, int64_t ldx, int64_t nwords, const int2* __restrict__ sel_ab,
                         const uint8_t* __restrict__ sel_gate, int64_t n_out, uint64_t* __restrict__ y, int64_t ldy,
                         int tw_log2) {
    using Vw = Vec<uint64_t, V>;
    const int TW = 1 << tw_log2;
    const int lane = threadIdx.x & 31;
    const int64_t w = ((int64_t)blockIdx.x * TW + (lane & (TW - 1))) * V;
    const int64_t npw = 32 >> tw_log2;
    const int64_t warp_global = ((int64_t)blockIdx.y * blockDim.x + threadIdx.x) >> 5;
    const int64_t stride = (((int64_t)gridDim.y * blockDim.x) >> 5) * npw * R;
    pdl_trigger();
    if (w >= nwords) return;
    const uint64_t policy = ST ? evict_first_policy() : 0ull;
    const int64_t sub = lane >> tw_log2;
    int64_t base = warp_global * npw * R;
    int2 ab[R];
    int g[R];
#pragma unroll
    for (int q = 0; q < R; ++q) {
        const int64_t j = base + q * npw + sub;
        ab[q] = j < n_out ? sel_ab[j] : make_int2(-1, -1);
        g[q] = j < n_out ? sel_gate[j] : 0;
    }
    pdl_wait();  // the operand rows are the previous layer's output
    for (; base < n_out; base += stride) {
        Vw va[R], vb[R];
#pragma unroll
        for (int q = 0; q < R; ++q) {
#pragma unroll
            for (int i = 0; i < V; ++i) va[q].v[i] = vb[q].v[i] = 0;
            if (ab[q].x >= 0) va[q] = *reinterpret_cast<const Vw*>(x + (int64_t)ab[q].x * ldx + w);
            if (ab[q].y >= 0) vb[q] = *reinterpret_cast<const Vw*>(x + (int64_t)ab[q].y * ldx + w);
        }
        int gc[R];
#pragma unroll
        for (int q = 0; q < R; ++q) {
            gc[q] = g[q];
            const int64_t j = base + stride + q * npw + sub;
            ab[q] = j < n_out ? sel_ab[j] : make_int2(-1, -1);
            g[q] = j < n_out ? sel_gate[j] : 0;
        }
#pragma unroll
        for (int q = 0; q < R; ++q) {
            const int64_t j = base + q * npw + sub;
            if (j < n_out) {
                Vw o;
#pragma unroll
                for (int i = 0; i < V; ++i) o.v[i] = gate_word<uint64_t>(gc[q], va[q].v[i], vb[q].v[i]);
                store_words<ST, V>(y + j * ldy + w, o, policy);
            }
        }
    }
}

int sm_count() {
    int dev = 0, n = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

// ------------------------------------------------------------------------------------------
// Packed GroupSum: counts[(sample0 + 64 w + i) * k + c] += #{rows r of class c : bit i of word(r, w)}.
// A CTA owns one class, a tile of TW word columns and S = 256/TW row segments of up to 240 rows:
// thread (segment, column) runs a vertical counter over its rows, the CTA folds the S counters in
// shared memory (four 16-bit counts per 64-bit shared atomic), then adds each nonzero
// (column, position) total to global memory once.  `Src` yields word(r, w): a stored packed row
// (groupbitsum) or, for the fused last layer, the gate output computed on the fly.
// ------------------------------------------------------------------------------------------
struct RowWords {
    const uint8_t* words;
    int64_t row_bytes;
    bool al8;
    // rows r .. r+15 (zero at and beyond r1)
    __device__ __forceinline__ void load16(int64_t r, int64_t r1, int64_t w, uint64_t (&d)[16]) const {
#pragma unroll
        for (int q = 0; q < 16; ++q)
            d[q] = (r + q < r1) ? load_word_bytes(words + (r + q) * row_bytes, 8 * w, row_bytes, al8) : 0ull;
    }
};

struct GateWords {
    const uint64_t* x;
    int64_t ldx;
    const int2* ab;
    const uint8_t* gate;
    // neurons j .. j+15 (zero at and beyond j1): all table loads first, then the gathers 8 at a time,
    // so the dependent loads of 8 neurons are in flight together
    __device__ __forceinline__ void load16(int64_t j, int64_t j1, int64_t w, uint64_t (&d)[16]) const {
        int2 p[16];
        int g[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) {
            const int64_t jj = j + q < j1 ? j + q : j1 - 1;
            p[q] = ab[jj];
            g[q] = gate[jj];
        }
#pragma unroll
        for (int h = 0; h < 16; h += 8) {
            uint64_t va[8], vb[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                va[q] = word_or_zero(x, p[h + q].x, ldx, w);
                vb[q] = word_or_zero(x, p[h + q].y, ldx, w);
            }
#pragma unroll
            for (int q = 0; q < 8; ++q) d[h + q] = (j + h + q < j1) ? gate_word<uint64_t>(g[h + q], va[q], vb[q]) : 0ull;
        }
    }
};

struct CountPlan {
    int tw_log2;      // columns per CTA = 1 << tw_log2
    int64_t seg_len;  // rows per thread (multiple of 16, <= 240)
    int64_t nseg;     // segments per class
    int64_t groups;   // CTAs per (class, column tile) = ceil(nseg / S)
};

// CTA fold of the per-thread counters: each thread's 64 counts go to shared memory as four 16-bit lanes
// per word, the S segments of each (column, 4-position group) are summed (packed 16-bit adds cannot
// overflow: at most 256 * 240 < 65536 per lane), and each total goes to global memory once.
// partial != null: instead of atomics into counts, the CTA stores its totals (zeros included) to
// partial[blockIdx.y][64 * w + pos] (row length 64 * gridDim.x * TW) and sum_partials folds them.
__device__ __forceinline__ void count_fold(const VCounter& vc, unsigned long long* s_cnt, const int TW, const int S,
                                           const int64_t nwords, const int64_t k, const int64_t c,
                                           int32_t* __restrict__ counts, const int64_t sample0, const int64_t samples,
                                           int32_t* __restrict__ partial) {
#pragma unroll
    for (int m = 0; m < 8; ++m) {
        const uint64_t v8 = vc.counts8(m);
        unsigned long long lo = 0, hi = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            lo |= ((v8 >> (8 * q)) & 0xffull) << (16 * q);
            hi |= ((v8 >> (8 * q + 32)) & 0xffull) << (16 * q);
        }
        // slot index rotated by the thread id so the 16 stores of a warp spread over the banks
        s_cnt[threadIdx.x * 16 + ((2 * m + threadIdx.x) & 15)] = lo;
        s_cnt[threadIdx.x * 16 + ((2 * m + 1 + threadIdx.x) & 15)] = hi;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < TW * 16; e += blockDim.x) {
        const int col = e >> 4, grp = e & 15;
        unsigned long long acc = 0;
        for (int t2 = 0; t2 < S; ++t2) {
            const int tid = t2 * TW + col;
            acc += s_cnt[tid * 16 + ((grp + tid) & 15)];
        }
        const int64_t ww = (int64_t)blockIdx.x * TW + col;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int pos = grp * 4 + q;
            const int v = (int)((acc >> (16 * q)) & 0xffff);
            const int64_t n = 64 * ww + pos;
            if (partial != nullptr)
                partial[(int64_t)blockIdx.y * (64 * (int64_t)gridDim.x * TW) + n] = v;
            else if (v && ww < nwords && n < samples)
                atomicAdd(counts + (sample0 + n) * k + c, v);
        }
    }
}

template <class Src>
__global__ void __launch_bounds__(256)
count_kernel(const Src src, const int64_t rows, const int64_t nwords, const int64_t k, const int64_t class_size,
             const CountPlan plan, int32_t* __restrict__ counts, const int64_t sample0, const int64_t samples,
             int32_t* __restrict__ partial) {
    __shared__ unsigned long long s_cnt[256 * 16];  // [thread][position / 4]
    const int TW = 1 << plan.tw_log2;
    const int S = 256 >> plan.tw_log2;
    const int wl = threadIdx.x & (TW - 1), sl = threadIdx.x >> plan.tw_log2;
    const int64_t c = blockIdx.y / plan.groups;
    const int64_t seg = (blockIdx.y - c * plan.groups) * S + sl;
    const int64_t w = (int64_t)blockIdx.x * TW + wl;
    pdl_trigger();
    pdl_wait();
    VCounter vc;
    if (w < nwords && seg < plan.nseg) {
        const int64_t r0 = c * class_size + seg * plan.seg_len;
        const int64_t r1 = min(min(r0 + plan.seg_len, (c + 1) * class_size), rows);
        for (int64_t r = r0; r < r1; r += 16) {
            uint64_t d[16];
            src.load16(r, r1, w, d);
            vc.add16(d);
        }
    }
    count_fold(vc, s_cnt, TW, S, nwords, k, c, counts, sample0, samples, partial);
}

// The fused last layer as a software pipeline over groups of 8 neurons: the tables (operand rows, gate)
// of the next group are loaded while the 16 operand words of the current group are in flight, so a
// group costs one memory round trip instead of two (tables, then operands), with about half the
// registers of count_kernel<GateWords> (more resident warps).  The tables do not depend on the
// previous layer, so the first group's are loaded before the programmatic-launch wait.
template <int MINB>
__global__ void __launch_bounds__(256, MINB)
count_gate_pipe_kernel(const GateWords src, const int64_t rows, const int64_t nwords, const int64_t k,
                       const int64_t class_size, const CountPlan plan, int32_t* __restrict__ counts,
                       const int64_t sample0, const int64_t samples, int32_t* __restrict__ partial) {
    __shared__ unsigned long long s_cnt[256 * 16];
    const int TW = 1 << plan.tw_log2;
    const int S = 256 >> plan.tw_log2;
    const int wl = threadIdx.x & (TW - 1), sl = threadIdx.x >> plan.tw_log2;
    const int64_t c = blockIdx.y / plan.groups;
    const int64_t seg = (blockIdx.y - c * plan.groups) * S + sl;
    const int64_t w = (int64_t)blockIdx.x * TW + wl;
    pdl_trigger();
    VCounter vc;
    const bool active = w < nwords && seg < plan.nseg;
    int64_t r0 = 0, r1 = 0;
    int2 p[8];
    int g[8];
    if (active) {
        r0 = c * class_size + seg * plan.seg_len;
        r1 = min(min(r0 + plan.seg_len, (c + 1) * class_size), rows);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const int64_t jj = min(r0 + q, r1 - 1);
            p[q] = src.ab[jj];
            g[q] = src.gate[jj];
        }
    }
    pdl_wait();  // the operand rows are the previous layer's output
    if (active) {
        const uint64_t* __restrict__ xw = src.x + w;
        const int64_t ldx = src.ldx;
        // one group: gather the 16 operand words of the staged tables, load the next group's tables
        // (rows from `nx`, clamped below `r1` only near the end), evaluate the 8 gates
        auto group = [&](int64_t nx, bool clamp, int64_t valid, uint64_t (&d)[8]) {
            uint64_t va[8], vb[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                va[q] = p[q].x >= 0 ? __ldg(xw + (int64_t)p[q].x * ldx) : 0ull;
                vb[q] = p[q].y >= 0 ? __ldg(xw + (int64_t)p[q].y * ldx) : 0ull;
            }
            int gc[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                gc[q] = g[q];
                const int64_t jj = clamp ? min(nx + q, r1 - 1) : nx + q;
                p[q] = src.ab[jj];
                g[q] = src.gate[jj];
            }
#pragma unroll
            for (int q = 0; q < 8; ++q) d[q] = q < valid ? gate_word<uint64_t>(gc[q], va[q], vb[q]) : 0ull;
        };
        int64_t r = r0;
        // full 16-row steps whose next tables are in range: no clamping, no masking, one carry chain
        for (; r + 24 <= r1; r += 16) {
            uint64_t d[16];
            group(r + 8, false, 8, *reinterpret_cast<uint64_t(*)[8]>(d));
            group(r + 16, false, 8, *reinterpret_cast<uint64_t(*)[8]>(d + 8));
            vc.add16(d);
        }
        for (; r < r1; r += 8) {
            uint64_t d[8];
            group(r + 8, true, r1 - r, d);
            vc.add8(d);
        }
    }
    count_fold(vc, s_cnt, TW, S, nwords, k, c, counts, sample0, samples, partial);
}

// counts[(sample0 + n) * k + c] += sum_g partial[c * groups + g][n]   (one writer per element)
__global__ void sum_partials_kernel(const int32_t* __restrict__ partial, int64_t row, int64_t groups, int64_t k,
                                    int32_t* __restrict__ counts, int64_t sample0, int64_t samples) {
    pdl_trigger();
    pdl_wait();
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < samples * k; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t c = e / samples, n = e - c * samples;
        int32_t v = 0;
        for (int64_t g = 0; g < groups; ++g) v += partial[(c * groups + g) * row + n];
        counts[(sample0 + n) * k + c] += v;
    }
}

// Launch with the programmatic-serialization attribute when CLB_PACKED_PDL is on (default) so consecutive
// kernels of a packed pass overlap launch latency and ramp-up with their predecessor's tail.
bool pdl_enabled() {
    static const bool on = [] {
        const char* e = getenv("CLB_PACKED_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}

template <typename... Exp, typename... Act>
void launch_chain(void (*kern)(Exp...), dim3 grid, dim3 block, cudaStream_t s, Act&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    cudaLaunchKernelEx(&cfg, kern, std::forward<Act>(args)...);
}

unsigned grid_for(int64_t threads) {
    return (unsigned)std::max<int64_t>(1, std::min<int64_t>(ceil_div64(threads, 256), (int64_t)148 * 32));
}

// Segments as long as possible (fewer flushes) while keeping ~150 K threads; every thread keeps 16-32
// independent loads in flight, so this hides the L2 latency.
CountPlan plan_count(int64_t k, int64_t class_size, int64_t W, bool to_partial) {
    CountPlan p{};
    p.tw_log2 = 0;
    while ((1 << p.tw_log2) < W && p.tw_log2 < 5) ++p.tw_log2;
    // with atomics every CTA of a class hits the same counters, so fewer, longer segments pay off;
    // with the partials there is no contention and more threads hide the gather latency better
    const int64_t target = to_partial ? 148 * 2048 : 148 * 1024;
    int64_t len = ceil_div64(std::max<int64_t>(1, class_size * k * W), target);
    len = std::min<int64_t>(VCounter::kMaxWords, std::max<int64_t>(16, ceil_div64(len, 16) * 16));
    for (;;) {
        p.seg_len = len;
        p.nseg = ceil_div64(class_size, len);
        p.groups = ceil_div64(p.nseg, 256 >> p.tw_log2);
        if (k * p.groups <= 65535 || len >= VCounter::kMaxWords) break;
        len = std::min<int64_t>(VCounter::kMaxWords, len + 16);
    }
    return p;
}

template <class Src>
void launch_count_kernel(const Src& src, dim3 grid, cudaStream_t s, int64_t rows, int64_t nwords, int64_t k,
                         int64_t class_size, const CountPlan& p, int32_t* counts, int64_t sample0, int64_t samples,
                         int32_t* partial) {
    launch_chain(count_kernel<Src>, grid, dim3(256), s, src, rows, nwords, k, class_size, p, counts, sample0, samples,
                 partial);
}

// The fused last layer: the pipelined kernel by default; CLB_COUNT_PIPE=0 selects count_kernel<GateWords>,
// CLB_COUNT_PIPE=2 the pipelined kernel with its registers capped for 3 resident CTAs per SM.
void launch_count_kernel(const GateWords& src, dim3 grid, cudaStream_t s, int64_t rows, int64_t nwords, int64_t k,
                         int64_t class_size, const CountPlan& p, int32_t* counts, int64_t sample0, int64_t samples,
                         int32_t* partial) {
    static const int mode = [] {
        const char* e = getenv("CLB_COUNT_PIPE");
        return e != nullptr ? atoi(e) : 1;
    }();
    if (mode == 0)
        launch_chain(count_kernel<GateWords>, grid, dim3(256), s, src, rows, nwords, k, class_size, p, counts, sample0,
                     samples, partial);
    else if (mode == 2)
        launch_chain(count_gate_pipe_kernel<3>, grid, dim3(256), s, src, rows, nwords, k, class_size, p, counts,
                     sample0, samples, partial);
    else
        launch_chain(count_gate_pipe_kernel<2>, grid, dim3(256), s, src, rows, nwords, k, class_size, p, counts,
                     sample0, samples, partial);
}

template <class Src>
cudaError_t launch_count(const Src& src, int64_t rows, int64_t nwords, int64_t k, int64_t class_size,
                         int32_t* counts, int64_t sample0, int64_t samples, void* ws, size_t ws_bytes,
                         cudaStream_t s) {
    CountPlan p = plan_count(k, class_size, nwords, ws != nullptr);
    const int64_t tiles = ceil_div64(nwords, 1 << p.tw_log2);
    const int64_t row = 64 * tiles * (1 << p.tw_log2);
    int32_t* partial = nullptr;
    if (ws != nullptr) {
        if ((size_t)(k * p.groups * row) * sizeof(int32_t) > ws_bytes) {
            p = plan_count(k, class_size, nwords, false);  // workspace too small: atomics
        } else {
            partial = reinterpret_cast<int32_t*>(ws);
        }
    }
    if (k * p.groups > 65535) return cudaErrorInvalidConfiguration;
    dim3 grid((unsigned)tiles, (unsigned)(k * p.groups));
    launch_count_kernel(src, grid, s, rows, nwords, k, class_size, p, counts, sample0, samples, partial);
    if (partial != nullptr) {
        launch_chain(sum_partials_kernel, dim3(grid_for(samples * k)), dim3(256), s, (const int32_t*)partial, row,
                     p.groups, k, counts, sample0, samples);
    }
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_packbits(const uint8_t* t, int64_t rows, int64_t cols, int64_t ld_t, int bits, uint8_t* out,
                            int64_t row_bytes, cudaStream_t s) {
    (void)bits;
    if (rows == 0 || row_bytes == 0) return cudaSuccess;
    const int64_t warps = rows * ((row_bytes + 3) / 4);
    packbits_kernel<<<grid_for(warps * 32), 256, 0, s>>>(t, rows, cols, ld_t, out, row_bytes);
    return cudaGetLastError();
}

cudaError_t launch_groupbitsum(const uint8_t* words, int64_t rows, int64_t row_bytes, int64_t samples, int64_t k,
                               int64_t class_size, int32_t* counts, bool accumulate, int64_t sample0,
                               cudaStream_t s) {
    if (!accumulate) {
        cudaError_t e = cudaMemsetAsync(counts + sample0 * k, 0, sizeof(int32_t) * samples * k, s);
        if (e != cudaSuccess) return e;
    }
    if (rows == 0 || samples == 0 || k == 0) return cudaSuccess;
    const RowWords src{words, row_bytes, (row_bytes % 8) == 0 && ((uintptr_t)words % 8) == 0};
    return launch_count(src, rows, (row_bytes + 7) / 8, k, class_size, counts, sample0, samples, nullptr, 0, s);
}

cudaError_t launch_pack_inputs(int dtype, const void* x, int64_t batch, int64_t features, int64_t ldx,
                               uint64_t* out, int64_t ldw, cudaStream_t s) {
    if (batch == 0 || features == 0) return cudaSuccess;
    dim3 grid((unsigned)ceil_div64(features, 32), (unsigned)ceil_div64(batch, 64));
    dim3 block(32, 8);
    switch (dtype) {
        case CLB_F32: pack_inputs_kernel<float><<<grid, block, 0, s>>>((const float*)x, batch, features, ldx, out, ldw); break;
        case CLB_F64: pack_inputs_kernel<double><<<grid, block, 0, s>>>((const double*)x, batch, features, ldx, out, ldw); break;
        case CLB_BF16: pack_inputs_kernel<__nv_bfloat16><<<grid, block, 0, s>>>((const __nv_bfloat16*)x, batch, features, ldx, out, ldw); break;
        case CLB_F16: pack_inputs_kernel<__half><<<grid, block, 0, s>>>((const __half*)x, batch, features, ldx, out, ldw); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_pack_thresholds(int dtype, const void* x, int64_t batch, int64_t features, int64_t ldx, int nthr,
                                   uint64_t* out, int64_t ldw, cudaStream_t s) {
    if (batch == 0 || features == 0) return cudaSuccess;
    dim3 grid((unsigned)ceil_div64(features, 32), (unsigned)ceil_div64(batch, 64));
    dim3 block(32, 8);
    switch (dtype) {
        case CLB_F32: pack_thresholds_kernel<float><<<grid, block, 0, s>>>((const float*)x, batch, features, ldx, nthr, out, ldw); break;
        case CLB_F64: pack_thresholds_kernel<double><<<grid, block, 0, s>>>((const double*)x, batch, features, ldx, nthr, out, ldw); break;
        case CLB_BF16: pack_thresholds_kernel<__nv_bfloat16><<<grid, block, 0, s>>>((const __nv_bfloat16*)x, batch, features, ldx, nthr, out, ldw); break;
        case CLB_F16: pack_thresholds_kernel<__half><<<grid, block, 0, s>>>((const __half*)x, batch, features, ldx, nthr, out, ldw); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_packed_select(const int32_t* slots, const uint8_t* gates, const uint8_t* select, int64_t n_out,
                                 int K, int64_t group, int32_t* sel_ab, uint8_t* sel_gate, cudaStream_t s) {
    if (n_out == 0) return cudaSuccess;
    packed_select_kernel<<<grid_for(n_out), 256, 0, s>>>(reinterpret_cast<const int2*>(slots), gates, select, n_out, K,
                                                         group, reinterpret_cast<int2*>(sel_ab), sel_gate);
    return cudaGetLastError();
}

// Tuning overrides (read once): CLB_PACKED_R neurons per thread (2/4/8), CLB_PACKED_MINB registers capped for 4
// (default) or 1 resident CTAs per SM (measured: 437 vs 459-558 ms per c4 pass at 128-word chunks).
int packed_env(const char* name, int dflt) {
    const char* v = getenv(name);
    return v != nullptr ? atoi(v) : dflt;
}

template <int R, int V>
void packed_layer_go(dim3 grid, cudaStream_t s, int minb, const uint64_t* x, int64_t ldx, int64_t nwords, const int2* ab,
                     const uint8_t* g, int64_t n_out, uint64_t* y, int64_t ldy, int tw_log2) {
    static const int pipe = packed_env("CLB_PACKED_PIPE", 1);
    if (pipe > 0) {
        // about `pipe` waves of resident CTAs, striding over the tiles
        const int64_t cap = std::max<int64_t>(1, (int64_t)sm_count() * (minb == 4 ? 4 : 2) * pipe / grid.x);
        grid.y = (unsigned)std::min<int64_t>(grid.y, cap);
        static const int st = packed_env("CLB_PACKED_ST", 1);  // evict-first stores (measured 400.6 -> 398.2 ms per c4 pass)
        if (minb == 4 && st == 1)
            launch_chain(packed_layer_pipe_kernel<R, V, 4, 1>, grid, dim3(256), s, x, ldx, nwords, ab, g, n_out, y,
                         ldy, tw_log2);
        else if (minb == 4)
            launch_chain(packed_layer_pipe_kernel<R, V, 4>, grid, dim3(256), s, x, ldx, nwords, ab, g, n_out, y, ldy,
                         tw_log2);
        else
            launch_chain(packed_layer_pipe_kernel<R, V, 1>, grid, dim3(256), s, x, ldx, nwords, ab, g, n_out, y, ldy,
                         tw_log2);
        return;
    }
    if (minb == 4)
        packed_layer_kernel<R, V, 4><<<grid, 256, 0, s>>>(x, ldx, nwords, ab, g, n_out, y, ldy, tw_log2);
    else
        packed_layer_kernel<R, V, 1><<<grid, 256, 0, s>>>(x, ldx, nwords, ab, g, n_out, y, ldy, tw_log2);
}

cudaError_t launch_packed_layer(const uint64_t* x, int64_t ldx, int64_t nwords, const int32_t* sel_ab,
                                const uint8_t* sel_gate, int64_t n_out, uint64_t* y, int64_t ldy, cudaStream_t s) {
    if (n_out == 0 || nwords == 0) return cudaSuccess;
    // default: the persistent table-prefetching kernel with 2 neurons per thread (measured best: c4 pass
    // 406.8 ms vs 438.2 ms for the one-shot kernel with 4); CLB_PACKED_PIPE=0 selects the one-shot kernel
    static const int R = packed_env("CLB_PACKED_R", packed_env("CLB_PACKED_PIPE", 1) > 0 ? 2 : 4);
    static const int minb = packed_env("CLB_PACKED_MINB", 4);
    const bool v2 = nwords % 2 == 0 && ldx % 2 == 0 && ldy % 2 == 0 && (uintptr_t)x % 16 == 0 && (uintptr_t)y % 16 == 0;
    const int V = v2 ? 2 : 1;
    const int64_t cols = nwords / V;  // lane-owned column groups
    int tw_log2 = 0;
    while ((1 << tw_log2) < cols && tw_log2 < 5) ++tw_log2;
    const int64_t TW = 1 << tw_log2;
    const int64_t npw = 32 / TW;
    const int r = (R == 2 || R == 8) ? R : 4;
    const int64_t warps_needed = ceil_div64(n_out, npw * r);
    const int64_t by = std::min<int64_t>(ceil_div64(warps_needed, 8), 65535);
    dim3 grid((unsigned)ceil_div64(cols, TW), (unsigned)by);
    const int2* ab = reinterpret_cast<const int2*>(sel_ab);
    if (v2) {
        if (r == 2) packed_layer_go<2, 2>(grid, s, minb, x, ldx, nwords, ab, sel_gate, n_out, y, ldy, tw_log2);
        else if (r == 8) packed_layer_go<8, 2>(grid, s, minb, x, ldx, nwords, ab, sel_gate, n_out, y, ldy, tw_log2);
        else packed_layer_go<4, 2>(grid, s, minb, x, ldx, nwords, ab, sel_gate, n_out, y, ldy, tw_log2);
    } else {
        packed_layer_go<4, 1>(grid, s, 1, x, ldx, nwords, ab, sel_gate, n_out, y, ldy, tw_log2);
    }
    return cudaGetLastError();
}

cudaError_t launch_packed_layer_count(const uint64_t* x, int64_t ldx, int64_t nwords, const int32_t* sel_ab,
                                      const uint8_t* sel_gate, int64_t n_out, int64_t k, int64_t class_size,
                                      int32_t* counts, int64_t sample0, int64_t nsamples, void* ws, size_t ws_bytes,
                                      cudaStream_t s) {
    if (n_out == 0 || nwords == 0 || k == 0) return cudaSuccess;
    const GateWords src{x, ldx, reinterpret_cast<const int2*>(sel_ab), sel_gate};
    return launch_count(src, n_out, nwords, k, class_size, counts, sample0, nsamples, ws, ws_bytes, s);
}

size_t packed_count_workspace_bytes(int64_t k, int64_t class_size, int64_t nwords) {
    const CountPlan p = plan_count(k, class_size, nwords, true);
    const int64_t row = 64 * ceil_div64(nwords, 1 << p.tw_log2) * (1 << p.tw_log2);
    return (size_t)(k * p.groups * row) * sizeof(int32_t);
}

}  // namespace clb
