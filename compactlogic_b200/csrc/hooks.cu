// Device side of the training hooks that watch the gate distributions.
//
// EntropyRowResampler.step (compactlogic/compactlogic.py:1113-1150) runs, per layer and iteration,
// weights_entropy (log_softmax, exp, product, row sum, division; compactlogic.py:370-385), an EMA update,
// a patience counter update and a nonzero() on the counters.  This kernel does all of it for one layer
// in one pass over the logits: one warp per row, the K logits in the lanes.
#include <cuda_runtime.h>
#include <float.h>

#include "common.cuh"
#include "kernels.h"

namespace clb {

namespace {

__global__ void entropy_monitor_kernel(const float* __restrict__ logits, int64_t rows, int K, float inv_log_k,
                                       float* __restrict__ ema, int32_t* __restrict__ counter, int first, float decay,
                                       float eps, int patience, uint8_t* __restrict__ converged,
                                       int32_t* __restrict__ n_converged) {
    const int lane = threadIdx.x & 31;
    const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (r >= rows) return;
    const float* w = logits + r * K;
    // log-sum-exp over the K logits (strided over lanes for K > 32)
    float m = -FLT_MAX;
    for (int k = lane; k < K; k += 32) m = fmaxf(m, w[k]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float s = 0.f;
    for (int k = lane; k < K; k += 32) s += expf(w[k] - m);
    s = warp_sum(s);
    const float lse = m + logf(s);
    float h = 0.f;
    for (int k = lane; k < K; k += 32) {
        const float lp = w[k] - lse;  // log_softmax
        h -= expf(lp) * lp;
    }
    h = warp_sum(h) * inv_log_k;
    if (lane != 0) return;
    int flag = 0;
    if (first) {
        ema[r] = h;
        counter[r] = 0;
    } else {
        const float old = ema[r];
        ema[r] = decay * old + (1.0f - decay) * h;
        const int c = fabsf(h - old) < eps ? counter[r] + 1 : 0;
        counter[r] = c;
        flag = c >= patience;
    }
    converged[r] = (uint8_t)flag;
    if (flag) atomicAdd(n_converged, 1);
}


// Row resampling of LogicLayer.resample_connections (compactlogic/compactlogic.py:282-368) for the rows the
// monitor flagged, from pre-drawn random tensors (so no host needs the row counts): one warp per row, the
// K <= 32 slots in the lanes.  Per picked row, with p = softmax(logits) and (pmax, kmax) its first maximum:
//   weak   (pmax < low):  logits <- randn draws, gate ids <- gate draws (update_gate), both inputs of every
//                         slot <- index draws;
//   strong (pmax > high): logits <- 0 except the winner's, log(p (K-1) / (1-p)) with p clamped to
//                         [1e-6, 1-1e-6] (or log(9 (K-1)) without keep_strong), the other slots get gate
//                         draws (update_gate) and index draws.
// Weak is applied before strong, both from the row's original distribution, as the host code does.  Rows
// that changed get their Adam moments zeroed (reset_adam_state_for_mask, compactlogic.py:1152-1180) and
// changed[r] = 1; every picked row's patience counter restarts at 0.
__global__ void resample_rows_kernel(float* __restrict__ logits, uint8_t* __restrict__ gates,
                                     int64_t* __restrict__ idx_a, int64_t* __restrict__ idx_b, int64_t rows, int K,
                                     const uint8_t* __restrict__ picked, float high, float low, int keep_strong,
                                     int update_gate, const float* __restrict__ d_logits,
                                     const uint8_t* __restrict__ d_gates, const int64_t* __restrict__ d_a,
                                     const int64_t* __restrict__ d_b, uint8_t* __restrict__ changed,
                                     float* __restrict__ m1, float* __restrict__ m2, int32_t* __restrict__ counter) {
    const int lane = threadIdx.x & 31;
    const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (r >= rows) return;
    if (!picked[r]) {
        if (lane == 0) changed[r] = 0;
        return;
    }
    const int64_t e = r * K + lane;
    const bool live = lane < K;
    const float w = live ? logits[e] : -FLT_MAX;
    float m = w;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float ex = live ? expf(w - m) : 0.f;
    const float sum = warp_sum(ex);
    // first maximum of the probabilities = first maximum of the logits
    const unsigned at_max = __ballot_sync(0xffffffffu, live && w == m);
    const int kmax = __ffs(at_max) - 1;
    const float pmax = 1.0f / sum;  // exp(m - m) / sum
    const bool strong = pmax > high, weak = pmax < low;
    if (live && weak) {
        logits[e] = d_logits[e];
        if (update_gate) gates[e] = d_gates[e];
        idx_a[e] = d_a[e];
        idx_b[e] = d_b[e];
    }
    if (live && strong) {
        if (lane == kmax) {
            const float pc = fminf(fmaxf(pmax, 1e-6f), 1.0f - 1e-6f);
            logits[e] = keep_strong ? logf(pc * (float)(K - 1) / (1.0f - pc)) : logf(9.0f * (float)(K - 1));
        } else {
            logits[e] = 0.0f;
            if (update_gate) gates[e] = d_gates[e];
            idx_a[e] = d_a[e];
            idx_b[e] = d_b[e];
        }
    }
    if (live && (weak || strong)) {
        if (m1 != nullptr) m1[e] = 0.f;
        if (m2 != nullptr) m2[e] = 0.f;
    }
    if (lane == 0) {
        changed[r] = (uint8_t)(weak || strong);
        if (counter != nullptr) counter[r] = 0;
    }
}

}  // namespace

cudaError_t launch_entropy_monitor(const float* logits, int64_t rows, int K, float inv_log_k, float* ema,
                                   int32_t* counter, int first, float decay, float eps, int patience,
                                   uint8_t* converged, int32_t* n_converged, cudaStream_t s) {
    if (rows == 0) return cudaSuccess;
    const int64_t threads = rows * 32;
    entropy_monitor_kernel<<<(unsigned)ceil_div64(threads, 256), 256, 0, s>>>(logits, rows, K, inv_log_k, ema, counter,
                                                                             first, decay, eps, patience, converged,
                                                                             n_converged);
    return cudaGetLastError();
}

cudaError_t launch_resample_rows(float* logits, uint8_t* gates, int64_t* idx_a, int64_t* idx_b, int64_t rows, int K,
                                 const uint8_t* picked, float high, float low, int keep_strong, int update_gate,
                                 const float* d_logits, const uint8_t* d_gates, const int64_t* d_a,
                                 const int64_t* d_b, uint8_t* changed, float* m1, float* m2, int32_t* counter,
                                 cudaStream_t s) {
    if (rows == 0) return cudaSuccess;
    resample_rows_kernel<<<(unsigned)ceil_div64(rows * 32, 256), 256, 0, s>>>(
        logits, gates, idx_a, idx_b, rows, K, picked, high, low, keep_strong, update_gate, d_logits, d_gates, d_a, d_b,
        changed, m1, m2, counter);
    return cudaGetLastError();
}

}  // namespace clb
