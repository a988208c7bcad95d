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

}  // namespace clb
