// device_util.cuh — small device helpers shared by the kernel files.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

namespace lssm {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide sum; `red` must hold blockDim.x/32 floats. Result broadcast to all threads.
__device__ __forceinline__ float block_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    float t = (threadIdx.x < (unsigned)nw) ? red[threadIdx.x] : 0.0f;
    if (wid == 0) t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
    __syncthreads();
    float r = red[0];
    return r;
}

// SiLU / softplus as in shaders/common.metal:48-61 (expf / logf are CUDA's own).
__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float softplus(float x) { return (x > 20.0f) ? x : logf(1.0f + expf(x)); }

__device__ __forceinline__ float h2f(__half h) { return __half2float(h); }
__device__ __forceinline__ __half f2h(float f) { return __float2half_rn(f); }
__device__ __forceinline__ float hround(float f) { return __half2float(__float2half_rn(f)); }

// Load one element of a runtime-typed array (0 = f16, 1 = bf16, 2 = f32) as float.
__device__ __forceinline__ float load_any(const void* p, uint64_t i, uint32_t dt) {
    if (dt == 0) return __half2float(reinterpret_cast<const __half*>(p)[i]);
    if (dt == 1) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    return reinterpret_cast<const float*>(p)[i];
}
__device__ __forceinline__ void store_any(void* p, uint64_t i, uint32_t dt, float v) {
    if (dt == 0) reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
    else if (dt == 1) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
    else reinterpret_cast<float*>(p)[i] = v;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

}  // namespace lssm
