// k_elementwise.cu — RMSNorm, activations, residual add, xBC split, causal conv1d
// (prefill / rolling-state decode / state seeding). All memory-bound; each kernel
// reads and writes every element once with coalesced (and, where the layout
// allows, vectorised) accesses.
//
// Numerics follow the reference shaders: fp16 storage, fp32 arithmetic, one
// rounding to fp16 on store.
#include "device_util.cuh"
#include "lssm_internal.h"

namespace lssm {

// ---------------------------------------------------------------------------
//  RMSNorm — shaders/norm.metal:32-80. One CTA per row; y = half((x*w)*rrms).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_rmsnorm_f16(const __half* __restrict__ x, const __half* __restrict__ w,
                                                     __half* __restrict__ y, uint32_t dim, float eps, int vec) {
    __shared__ float red[32];
    const uint64_t row = blockIdx.x;
    const __half* xr = x + row * dim;
    __half* yr = y + row * dim;
    float ss = 0.0f;
    if (vec) {
        const uint32_t n2 = dim >> 1;
        const __half2* x2 = reinterpret_cast<const __half2*>(xr);
        for (uint32_t i = threadIdx.x; i < n2; i += blockDim.x) {
            float2 v = __half22float2(x2[i]);
            ss += v.x * v.x + v.y * v.y;
        }
    } else {
        for (uint32_t i = threadIdx.x; i < dim; i += blockDim.x) {
            float v = __half2float(xr[i]);
            ss += v * v;
        }
    }
    const float total = block_sum(ss, red);
    const float rrms = rsqrtf(total / (float)dim + eps);
    if (vec) {
        const uint32_t n2 = dim >> 1;
        const __half2* x2 = reinterpret_cast<const __half2*>(xr);
        const __half2* w2 = reinterpret_cast<const __half2*>(w);
        __half2* y2 = reinterpret_cast<__half2*>(yr);
        for (uint32_t i = threadIdx.x; i < n2; i += blockDim.x) {
            float2 v = __half22float2(x2[i]);
            float2 g = __half22float2(w2[i]);
            y2[i] = __floats2half2_rn(v.x * g.x * rrms, v.y * g.y * rrms);
        }
    } else {
        for (uint32_t i = threadIdx.x; i < dim; i += blockDim.x)
            yr[i] = __float2half_rn(__half2float(xr[i]) * __half2float(w[i]) * rrms);
    }
}

// 16-byte form: dim % 8 == 0, dim / 8 <= 4 * blockDim; each thread keeps its (<= 4) octets of the
// row in registers between the sum of squares and the scaling (one read of x, one write of y).
__global__ void __launch_bounds__(256) k_rmsnorm_f16_v8(const __half* __restrict__ x, const __half* __restrict__ w,
                                                        __half* __restrict__ y, uint32_t dim, float eps) {
    __shared__ float red[32];
    const uint64_t row = blockIdx.x;
    const uint4* xr = reinterpret_cast<const uint4*>(x + row * dim);
    uint4* yr = reinterpret_cast<uint4*>(y + row * dim);
    const uint32_t n8 = dim / 8;
    uint4 xv[4];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t q = threadIdx.x + i * blockDim.x;
        if (q < n8) xv[i] = xr[q];
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t q = threadIdx.x + i * blockDim.x;
        if (q >= n8) continue;
        const __half2* h2 = reinterpret_cast<const __half2*>(&xv[i]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 f = __half22float2(h2[j]);
            ss += f.x * f.x + f.y * f.y;
        }
    }
    const float rrms = rsqrtf(block_sum(ss, red) / (float)dim + eps);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t q = threadIdx.x + i * blockDim.x;
        if (q >= n8) continue;
        const uint4 wv = __ldg(reinterpret_cast<const uint4*>(w) + q);
        const __half* xh = reinterpret_cast<const __half*>(&xv[i]);
        const __half* wh = reinterpret_cast<const __half*>(&wv);
        uint4 o;
        __half* oh = reinterpret_cast<__half*>(&o);
#pragma unroll
        for (int j = 0; j < 8; ++j) oh[j] = __float2half_rn(__half2float(xh[j]) * __half2float(wh[j]) * rrms);
        yr[q] = o;
    }
}

cudaError_t launch_rmsnorm_f16(const void* x, const void* w, void* y, uint32_t rows, uint32_t dim, float eps,
                               cudaStream_t s) {
    if (rows == 0 || dim == 0) return cudaSuccess;
    if (dim % 8 == 0 && aligned(x, 16) && aligned(w, 16) && aligned(y, 16) && dim / 8 <= 4 * 256) {
        uint32_t threads = (dim / 8 + 3) / 4;                 // <= 4 octets per thread
        threads = (threads + 31) / 32 * 32;
        threads = threads < 64 ? (dim / 8 < 64 ? (dim / 8 + 31) / 32 * 32 : 64) : threads;
        k_rmsnorm_f16_v8<<<rows, threads, 0, s>>>(static_cast<const __half*>(x), static_cast<const __half*>(w),
                                                  static_cast<__half*>(y), dim, eps);
        return cudaGetLastError();
    }
    const int vec = aligned(x, 4) && aligned(w, 4) && aligned(y, 4) && (dim % 2 == 0);
    uint32_t threads = (dim / 2 + 31) / 32 * 32;
    threads = threads < 32 ? 32 : (threads > 256 ? 256 : threads);
    k_rmsnorm_f16<<<rows, threads, 0, s>>>(static_cast<const __half*>(x), static_cast<const __half*>(w),
                                           static_cast<__half*>(y), dim, eps, vec);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
//  Elementwise activations — shaders/activations.metal:12-87.
// ---------------------------------------------------------------------------
__global__ void k_silu_f16(const __half* __restrict__ x, __half* __restrict__ y, uint32_t n) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        y[i] = __float2half_rn(silu(__half2float(x[i])));
}

__global__ void k_add_inplace_f16(__half* y, const __half* __restrict__ x, uint32_t n) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        y[i] = __float2half_rn(__half2float(y[i]) + __half2float(x[i]));
}

// 8 elements per thread (16-byte accesses), the same rounding per element.
__global__ void k_add_inplace_f16x8(__half* y, const __half* __restrict__ x, uint32_t n8) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += gridDim.x * blockDim.x) {
        uint4 a = reinterpret_cast<const uint4*>(y)[i];
        const uint4 b = reinterpret_cast<const uint4*>(x)[i];
        __half* ah = reinterpret_cast<__half*>(&a);
        const __half* bh = reinterpret_cast<const __half*>(&b);
#pragma unroll
        for (int e = 0; e < 8; ++e) ah[e] = __float2half_rn(__half2float(ah[e]) + __half2float(bh[e]));
        reinterpret_cast<uint4*>(y)[i] = a;
    }
}

// gated = half(silu(z) * gate)  (kernel arg x = z, gate = SSD output; mamba2_block.cpp:231-234)
__global__ void k_silu_gated_f16(const __half* __restrict__ z, const __half* __restrict__ g,
                                 __half* __restrict__ y, uint32_t n) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        y[i] = __float2half_rn(silu(__half2float(z[i])) * __half2float(g[i]));
}

static inline unsigned grid_for(uint64_t n, unsigned threads) {
    uint64_t g = (n + threads - 1) / threads;
    if (g > 148u * 32u) g = 148u * 32u;
    return g == 0 ? 1u : (unsigned)g;
}

cudaError_t launch_silu_f16(const void* x, void* y, uint32_t n, cudaStream_t s) {
    if (!n) return cudaSuccess;
    k_silu_f16<<<grid_for(n, 256), 256, 0, s>>>(static_cast<const __half*>(x), static_cast<__half*>(y), n);
    return cudaGetLastError();
}
cudaError_t launch_add_inplace_f16(void* y, const void* x, uint32_t n, cudaStream_t s) {
    if (!n) return cudaSuccess;
    if (n % 8 == 0 && aligned(y, 16) && aligned(x, 16)) {
        k_add_inplace_f16x8<<<grid_for(n / 8, 256), 256, 0, s>>>(static_cast<__half*>(y), static_cast<const __half*>(x),
                                                                  n / 8);
        return cudaGetLastError();
    }
    k_add_inplace_f16<<<grid_for(n, 256), 256, 0, s>>>(static_cast<__half*>(y), static_cast<const __half*>(x), n);
    return cudaGetLastError();
}
cudaError_t launch_silu_gated_f16(const void* z, const void* g, void* y, uint32_t n, cudaStream_t s) {
    if (!n) return cudaSuccess;
    k_silu_gated_f16<<<grid_for(n, 256), 256, 0, s>>>(static_cast<const __half*>(z), static_cast<const __half*>(g),
                                                      static_cast<__half*>(y), n);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
//  SiLU + split of the conv output — shaders/activations.metal:49-73.
// ---------------------------------------------------------------------------
__global__ void k_split_silu(const __half* __restrict__ xbc, __half* __restrict__ xo, __half* __restrict__ bo,
                             __half* __restrict__ co, uint32_t L, uint32_t d_inner, uint32_t GN) {
    const uint32_t D = d_inner + 2 * GN;
    const uint64_t total = (uint64_t)L * D;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t t = (uint32_t)(i / D), f = (uint32_t)(i % D);
        const __half v = __float2half_rn(silu(__half2float(xbc[i])));
        if (f < d_inner) xo[(uint64_t)t * d_inner + f] = v;
        else if (f < d_inner + GN) bo[(uint64_t)t * GN + (f - d_inner)] = v;
        else co[(uint64_t)t * GN + (f - d_inner - GN)] = v;
    }
}

cudaError_t launch_split_silu_xBC_f16(const void* xBC, void* xo, void* Bo, void* Co, uint32_t L, uint32_t d_inner,
                                      uint32_t d_state, uint32_t n_groups, cudaStream_t s) {
    const uint64_t n = (uint64_t)L * (d_inner + 2ull * n_groups * d_state);
    if (!n) return cudaSuccess;
    k_split_silu<<<grid_for(n, 256), 256, 0, s>>>(static_cast<const __half*>(xBC), static_cast<__half*>(xo),
                                                  static_cast<__half*>(Bo), static_cast<__half*>(Co), L, d_inner,
                                                  n_groups * d_state);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
//  Causal depthwise conv1d, prefill — shaders/conv1d.metal:63-93.
//  Each thread owns one channel and a run of CONV_T consecutive time steps,
//  keeping the K-1 previous inputs in registers (one read per input instead of K).
// ---------------------------------------------------------------------------
constexpr int CONV_T = 16;
constexpr int CONV_KMAX = 8;

__global__ void k_causal_conv1d(const __half* __restrict__ x, const __half* __restrict__ w,
                                const __half* __restrict__ bias, __half* __restrict__ y, uint32_t L, uint32_t D,
                                uint32_t K) {
    const uint32_t d = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t t0 = blockIdx.y * CONV_T;
    const uint32_t b = blockIdx.z;
    if (d >= D) return;
    const __half* xb = x + (uint64_t)b * L * D;
    __half* yb = y + (uint64_t)b * L * D;
    float wk[CONV_KMAX], win[CONV_KMAX];
    for (uint32_t k = 0; k < K; ++k) wk[k] = __half2float(w[(uint64_t)d * K + k]);
    const float bv = bias ? __half2float(bias[d]) : 0.0f;
    // window[k] holds x[t - (K-1) + k]; prime with the K-1 samples before t0.
    for (uint32_t k = 0; k + 1 < K; ++k) {
        const int src = (int)t0 - (int)(K - 1) + (int)k;
        win[k] = src >= 0 ? __half2float(xb[(uint64_t)src * D + d]) : 0.0f;
    }
    const uint32_t tend = min(t0 + CONV_T, L);
    for (uint32_t t = t0; t < tend; ++t) {
        win[K - 1] = __half2float(xb[(uint64_t)t * D + d]);
        float acc = bv;
        for (uint32_t k = 0; k < K; ++k) acc += wk[k] * win[k];
        yb[(uint64_t)t * D + d] = __float2half_rn(acc);
        for (uint32_t k = 0; k + 1 < K; ++k) win[k] = win[k + 1];
    }
}

cudaError_t launch_causal_conv1d_f16(const void* x, const void* w, const void* bias, void* y, uint32_t B,
                                     uint32_t L, uint32_t D, uint32_t K, cudaStream_t s) {
    if (!B || !L || !D) return cudaSuccess;
    if (K == 0 || K > (uint32_t)CONV_KMAX) return cudaErrorInvalidValue;
    dim3 grid((D + 127) / 128, (L + CONV_T - 1) / CONV_T, B);
    k_causal_conv1d<<<grid, 128, 0, s>>>(static_cast<const __half*>(x), static_cast<const __half*>(w),
                                         static_cast<const __half*>(bias), static_cast<__half*>(y), L, D, K);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
//  Causal conv1d decode update — shaders/conv1d.metal:108-137.
//  state (B, D, K) oldest first; shift left, append x_new, dot with w.
// ---------------------------------------------------------------------------
__global__ void k_conv1d_update(const __half* __restrict__ x_new, __half* __restrict__ state,
                                const __half* __restrict__ w, const __half* __restrict__ bias,
                                __half* __restrict__ y, uint32_t B, uint32_t D, uint32_t K) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (uint64_t)B * D) return;
    const uint32_t d = (uint32_t)(i % D);
    __half* sd = state + i * K;
    const __half* wd = w + (uint64_t)d * K;
    float acc = bias ? __half2float(bias[d]) : 0.0f;
    for (uint32_t k = 0; k + 1 < K; ++k) {
        const __half v = sd[k + 1];
        sd[k] = v;
        acc += __half2float(v) * __half2float(wd[k]);
    }
    const __half xn = x_new[i];
    sd[K - 1] = xn;
    acc += __half2float(xn) * __half2float(wd[K - 1]);
    y[i] = __float2half_rn(acc);
}

cudaError_t launch_causal_conv1d_update_f16(const void* x_new, void* state, const void* w, const void* bias,
                                            void* y, uint32_t B, uint32_t D, uint32_t K, cudaStream_t s) {
    const uint64_t n = (uint64_t)B * D;
    if (!n) return cudaSuccess;
    if (K == 0) return cudaErrorInvalidValue;
    k_conv1d_update<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(
        static_cast<const __half*>(x_new), static_cast<__half*>(state), static_cast<const __half*>(w),
        static_cast<const __half*>(bias), static_cast<__half*>(y), B, D, K);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
//  Conv-state seeding — shaders/conv1d.metal:35-51:
//  state[b, d, k] = xBC[b, L-K+k, d] (0 when L-K+k < 0).
// ---------------------------------------------------------------------------
__global__ void k_seed_conv_state(const __half* __restrict__ xbc, __half* __restrict__ state, uint32_t B,
                                  uint32_t L, uint32_t D, uint32_t K) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (uint64_t)B * D * K) return;
    const uint32_t k = (uint32_t)(i % K);
    const uint64_t bd = i / K;
    const uint32_t d = (uint32_t)(bd % D), b = (uint32_t)(bd / D);
    const int src = (int)L - (int)K + (int)k;
    state[i] = src >= 0 ? xbc[((uint64_t)b * L + (uint32_t)src) * D + d] : __float2half_rn(0.0f);
}

cudaError_t launch_seed_conv_state_batched(const void* xBC, void* state, uint32_t B, uint32_t L, uint32_t D,
                                           uint32_t K, cudaStream_t s) {
    const uint64_t n = (uint64_t)B * D * K;
    if (!n) return cudaSuccess;
    k_seed_conv_state<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(static_cast<const __half*>(xBC),
                                                                 static_cast<__half*>(state), B, L, D, K);
    return cudaGetLastError();
}

cudaError_t launch_seed_conv_state_f16(const void* xBC, void* state, uint32_t L, uint32_t D, uint32_t K,
                                       cudaStream_t s) {
    return launch_seed_conv_state_batched(xBC, state, 1, L, D, K, s);
}

// ---------------------------------------------------------------------------
//  Routing epilogue of the fused in_proj (shaders/fused.metal:122-164): from the fp32
//  matmul tile mm (L, proj): z and dt rounded to fp16, the pre-conv xBC copy, and the
//  causal conv over the fp32 values + bias -> SiLU -> x / B / C.
// ---------------------------------------------------------------------------
__global__ void k_inproj_route(const float* __restrict__ mm, const __half* __restrict__ wconv,
                               const __half* __restrict__ cbias, __half* __restrict__ z, __half* __restrict__ xs,
                               __half* __restrict__ Bs, __half* __restrict__ Cs, __half* __restrict__ dt,
                               __half* __restrict__ xbc_pre, uint32_t L, uint32_t d_inner, uint32_t GN, uint32_t H,
                               uint32_t K) {
    const uint32_t xd = d_inner + 2 * GN, proj = d_inner + xd + H;
    const uint64_t total = (uint64_t)L * proj;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t m = (uint32_t)(i / proj), c = (uint32_t)(i % proj);
        const float v = mm[i];
        if (c < d_inner) {
            z[(uint64_t)m * d_inner + c] = __float2half_rn(v);
        } else if (c < d_inner + xd) {
            const uint32_t f = c - d_inner;
            xbc_pre[(uint64_t)m * xd + f] = __float2half_rn(v);
            float sum = __half2float(cbias[f]);
            for (uint32_t kk = 0; kk < K; ++kk) {
                const int sm = (int)m - (int)(K - 1 - kk);
                if (sm >= 0) sum += __half2float(wconv[(uint64_t)f * K + kk]) * mm[(uint64_t)sm * proj + c];
            }
            const __half o = __float2half_rn(silu(sum));
            if (f < d_inner) xs[(uint64_t)m * d_inner + f] = o;
            else if (f < d_inner + GN) Bs[(uint64_t)m * GN + (f - d_inner)] = o;
            else Cs[(uint64_t)m * GN + (f - d_inner - GN)] = o;
        } else {
            dt[(uint64_t)m * H + (c - d_inner - xd)] = __float2half_rn(v);
        }
    }
}

cudaError_t launch_inproj_route(const float* mm, const void* wconv, const void* cbias, void* z, void* xs, void* Bs,
                                void* Cs, void* dt, void* xbc_pre, uint32_t L, uint32_t d_inner, uint32_t GN,
                                uint32_t H, uint32_t K, cudaStream_t s) {
    const uint64_t n = (uint64_t)L * (2ull * d_inner + 2ull * GN + H);
    if (!n) return cudaSuccess;
    k_inproj_route<<<grid_for(n, 256), 256, 0, s>>>(mm, static_cast<const __half*>(wconv),
                                                    static_cast<const __half*>(cbias), static_cast<__half*>(z),
                                                    static_cast<__half*>(xs), static_cast<__half*>(Bs),
                                                    static_cast<__half*>(Cs), static_cast<__half*>(dt),
                                                    static_cast<__half*>(xbc_pre), L, d_inner, GN, H, K);
    return cudaGetLastError();
}

}  // namespace lssm
