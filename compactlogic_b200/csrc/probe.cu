// Memory-system probe used by the benchmark to measure the ceiling of the soft kernels' access
// pattern on the GPU it runs on.
//
// The soft logic-layer kernels gather whole 512-byte activation rows (128 fp32 batch columns) at
// random feature indices and, in the backward, add 512-byte rows of grad_x at random indices with
// red.global.add.v4.f32.  Both slabs of one column chunk (rows x 512 bytes) stay resident in L2, so
// the kernels are bound by L2 gather / reduction throughput rather than by HBM.  This probe issues
// exactly that pattern with no arithmetic: per warp step, two row gathers and (mode 1) two row
// reductions at hashed rows, over slabs the caller sizes like the kernel's.  Bytes moved per warp
// step: 1024 (mode 0) or 2048 (mode 1).  Row indices come from a two-instruction linear congruential
// sequence masked to a power-of-two slab, so address generation costs almost no issue slots.
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"

namespace clb {
namespace {

template <bool RED>
__global__ void __launch_bounds__(256) l2_probe_kernel(const float* __restrict__ src, float* __restrict__ dst,
                                                       const uint32_t mask, const int iters, float* __restrict__ sink) {
    const int lane = threadIdx.x & 31;
    const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    uint32_t h = warp * 0x9e3779b9u + 0x7f4a7c15u;  // warp-uniform linear congruential row sequence
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    const float* s0 = src + lane * 4;
    float* d0 = dst + lane * 4;
#pragma unroll 2
    for (int it = 0; it < iters; ++it) {
        const uint32_t h1 = h * 1664525u + 1013904223u;
        const uint32_t h2 = h1 * 1664525u + 1013904223u;
        h = h2;
        const float4 a = *reinterpret_cast<const float4*>(s0 + (size_t)((h1 >> 8) & mask) * 128);
        const float4 b = *reinterpret_cast<const float4*>(s0 + (size_t)((h2 >> 8) & mask) * 128);
        if (RED) {
            const float da[4] = {a.x, a.y, a.z, a.w}, db[4] = {b.x, b.y, b.z, b.w};
            red_add<4>(d0 + (size_t)((h1 >> 12) & mask) * 128, da);
            red_add<4>(d0 + (size_t)((h2 >> 12) & mask) * 128, db);
        } else {
            acc.x += a.x + b.x;
            acc.y += a.y + b.y;
            acc.z += a.z + b.z;
            acc.w += a.w + b.w;
        }
    }
    if (!RED && acc.x + acc.y + acc.z + acc.w == 1234.5f) sink[0] = acc.x;  // keeps the loads live
}

}  // namespace
}  // namespace clb

using namespace clb;

/* Probe of L2 row-gather (mode 0) or row-gather + row-reduction (mode 1) throughput: `ctas` CTAs of
 * 256 threads, each warp doing `iters` steps over src / dst slabs of `rows` 512-byte rows. */
extern "C" int clb_l2_probe(int mode, const float* src, float* dst, int64_t rows, int iters, int ctas, float* sink,
                            clb_stream_t stream) {
    if (rows < 1 || rows > (int64_t(1) << 24) || (rows & (rows - 1)) || iters < 1 || ctas < 1 || !src || !sink ||
        (mode == 1 && !dst))
        return set_error(CLB_ERR_INVALID, "l2_probe: rows must be a power of two <= 2^24");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (mode == 1)
        l2_probe_kernel<true><<<ctas, 256, 0, s>>>(src, dst, (uint32_t)(rows - 1), iters, sink);
    else
        l2_probe_kernel<false><<<ctas, 256, 0, s>>>(src, dst, (uint32_t)(rows - 1), iters, sink);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(CLB_ERR_CUDA, cudaGetErrorString(e));
    count_launches(1);
    return CLB_OK;
}
