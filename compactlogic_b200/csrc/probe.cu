// Memory-system probe used by the benchmark to measure the ceiling of the soft kernels' access
// pattern on the GPU it runs on.
//
// The soft logic-layer kernels gather whole 512-byte activation rows (128 fp32 batch columns) at
// random feature indices and, in the backward, add 512-byte rows of grad_x at random indices with
// red.global.add.v4.f32.  Both slabs of one column chunk (rows x 512 bytes) stay resident in L2, so
// the kernels are bound by L2 gather / reduction throughput rather than by HBM.  This probe issues
// exactly that pattern with no arithmetic: per warp step, two row gathers and (mode 1) two row
// reductions at hashed rows, over slabs the caller sizes like the kernel's.  Bytes moved per warp
// step: 1024 (mode 0) or 2048 (mode 1).
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"

namespace clb {
namespace {

__device__ __forceinline__ uint32_t mix32(uint32_t v) {
    v ^= v >> 16;
    v *= 0x7feb352du;
    v ^= v >> 15;
    v *= 0x846ca68bu;
    v ^= v >> 16;
    return v;
}

template <bool RED>
__global__ void __launch_bounds__(256) l2_probe_kernel(const float* __restrict__ src, float* __restrict__ dst,
                                                       const uint32_t rows, const int iters, float* __restrict__ sink) {
    const int lane = threadIdx.x & 31;
    const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    uint32_t h = mix32(warp * 0x9e3779b9u + 1u);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int it = 0; it < iters; ++it) {
        const uint32_t h1 = mix32(h + 1u), h2 = mix32(h + 2u);
        h = mix32(h + 3u);
        const uint32_t r1 = h1 % rows, r2 = h2 % rows;
        const float4 a = *reinterpret_cast<const float4*>(src + (size_t)r1 * 128 + lane * 4);
        const float4 b = *reinterpret_cast<const float4*>(src + (size_t)r2 * 128 + lane * 4);
        if (RED) {
            const float da[4] = {a.x, a.y, a.z, a.w}, db[4] = {b.x, b.y, b.z, b.w};
            red_add<4>(dst + (size_t)(mix32(h1) % rows) * 128 + lane * 4, da);
            red_add<4>(dst + (size_t)(mix32(h2) % rows) * 128 + lane * 4, db);
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
    if (rows < 1 || rows > 0x7fffffff || iters < 1 || ctas < 1 || !src || !sink || (mode == 1 && !dst))
        return set_error(CLB_ERR_INVALID, "l2_probe: bad arguments");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (mode == 1)
        l2_probe_kernel<true><<<ctas, 256, 0, s>>>(src, dst, (uint32_t)rows, iters, sink);
    else
        l2_probe_kernel<false><<<ctas, 256, 0, s>>>(src, dst, (uint32_t)rows, iters, sink);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(CLB_ERR_CUDA, cudaGetErrorString(e));
    count_launches(1);
    return CLB_OK;
}
