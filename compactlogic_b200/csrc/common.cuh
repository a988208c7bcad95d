// Shared device helpers for the CompactLogic B200 kernels.
//
// Activations are stored feature-major, [features, batch] with the batch contiguous, the layout the
// reference dense kernels use (compactlogic/cuda/difflogic_kernel.cu:8-12).  A warp always spans
// consecutive batch columns, so every gathered activation row is one coalesced 128..512-byte
// segment, whatever the connection pattern.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/compactlogic_b200.h"

namespace clb {

// ---------------------------------------------------------------------------------------------
// Element types.  `Acc<T>` is the arithmetic type: fp32 for fp32/bf16 activations, fp64 for fp64.
// Gradients (grad_y, grad_x, logit grads) are always stored in the arithmetic type.
// ---------------------------------------------------------------------------------------------
template <typename T> struct Acc { using type = float; };
template <> struct Acc<double> { using type = double; };

__device__ __forceinline__ float to_acc(float v) { return v; }
__device__ __forceinline__ double to_acc(double v) { return v; }
__device__ __forceinline__ float to_acc(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_acc(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_acc(float v);
template <> __device__ __forceinline__ float from_acc<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_acc<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half from_acc<__half>(float v) { return __float2half_rn(v); }
template <typename T> __device__ __forceinline__ T from_acc(double v) { return (T)v; }

// VEC consecutive elements as one aligned vector of at most 16 bytes.
template <typename T, int VEC> struct alignas(sizeof(T) * VEC <= 16 ? sizeof(T) * VEC : 16) Vec { T v[VEC]; };

// Vectors wider than 16 bytes are moved as several 16-byte pieces (the pointers are only 16-byte aligned).
template <typename T, int VEC>
__device__ __forceinline__ void load_acc(const T* __restrict__ p, typename Acc<T>::type (&out)[VEC]) {
    constexpr int P = (int)(sizeof(T) * VEC <= 16 ? VEC : 16 / sizeof(T));
#pragma unroll
    for (int o = 0; o < VEC; o += P) {
        Vec<T, P> r = *reinterpret_cast<const Vec<T, P>*>(p + o);
#pragma unroll
        for (int i = 0; i < P; ++i) out[o + i] = to_acc(r.v[i]);
    }
}

template <typename T, int VEC>
__device__ __forceinline__ void store_from_acc(T* __restrict__ p, const typename Acc<T>::type (&in)[VEC]) {
    constexpr int P = (int)(sizeof(T) * VEC <= 16 ? VEC : 16 / sizeof(T));
#pragma unroll
    for (int o = 0; o < VEC; o += P) {
        Vec<T, P> r;
#pragma unroll
        for (int i = 0; i < P; ++i) r.v[i] = from_acc<T>(in[o + i]);
        *reinterpret_cast<Vec<T, P>*>(p + o) = r;
    }
}

// ---------------------------------------------------------------------------------------------
// Fire-and-forget global reductions (no return value).  fp32 uses the sm_90+ vector form so one
// instruction adds 2 or 4 consecutive columns; fp64 falls back to scalar atomics.
// ---------------------------------------------------------------------------------------------
template <int VEC> __device__ __forceinline__ void red_add(float* p, const float (&v)[VEC]);
template <> __device__ __forceinline__ void red_add<1>(float* p, const float (&v)[1]) {
    asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(v[0]) : "memory");
}
template <> __device__ __forceinline__ void red_add<2>(float* p, const float (&v)[2]) {
    asm volatile("red.global.add.v2.f32 [%0], {%1, %2};" ::"l"(p), "f"(v[0]), "f"(v[1]) : "memory");
}
template <> __device__ __forceinline__ void red_add<4>(float* p, const float (&v)[4]) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(v[0]), "f"(v[1]), "f"(v[2]),
                 "f"(v[3])
                 : "memory");
}
template <> __device__ __forceinline__ void red_add<8>(float* p, const float (&v)[8]) {
    red_add<4>(p, *reinterpret_cast<const float(*)[4]>(&v[0]));
    red_add<4>(p + 4, *reinterpret_cast<const float(*)[4]>(&v[4]));
}
template <int VEC> __device__ __forceinline__ void red_add(double* p, const double (&v)[VEC]) {
#pragma unroll
    for (int i = 0; i < VEC; ++i) atomicAdd(p + i, v[i]);
}

// ---------------------------------------------------------------------------------------------
// Warp reductions.
// ---------------------------------------------------------------------------------------------
template <typename A> __device__ __forceinline__ A warp_sum(A v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

inline int64_t ceil_div64(int64_t a, int64_t b) { return (a + b - 1) / b; }

}  // namespace clb
