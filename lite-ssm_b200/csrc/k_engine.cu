// k_engine.cu — kernels the model driver needs around the ops, replacing the host
// work the reference does through unified memory:
//   * embedding gather         (Mamba2Model::embed CPU memcpy, mamba2_model.cpp:128-137)
//   * conv1d + SiLU + split     (conv1d.metal:63-137 + activations.metal:49-73, fused;
//                                reads the xBC columns of the packed in_proj output)
//   * mixer gate                (activations.metal:76-87 on strided z)
//   * seeded synthetic weights in the .ssm payload layout (INT4_B32 packing restating
//     tools/export_mamba2.py:68-103 bit for bit).
#include "device_util.cuh"
#include "lssm_internal.h"
#include "synth_rng.h"

namespace lssm {

// hidden[r, :] = embed[tokens[r], :]; out-of-range ids raise *err and gather row 0.
__global__ void k_embed_gather(const uint32_t* __restrict__ tokens, const __half* __restrict__ embed,
                               __half* __restrict__ hidden, uint32_t rows, uint32_t d_model, uint32_t vocab,
                               int* err) {
    const uint32_t r = blockIdx.x;
    if (r >= rows) return;
    uint32_t t = tokens[r];
    if (t >= vocab) {
        if (threadIdx.x == 0) atomicExch(err, 2);
        t = 0;
    }
    const __half* src = embed + (uint64_t)t * d_model;
    __half* dst = hidden + (uint64_t)r * d_model;
    for (uint32_t i = threadIdx.x; i < d_model; i += blockDim.x) dst[i] = src[i];
}

cudaError_t launch_embed_gather(const uint32_t* tokens, const void* embed, void* hidden, uint32_t rows,
                                uint32_t d_model, uint32_t vocab, int* err, cudaStream_t s) {
    if (!rows) return cudaSuccess;
    k_embed_gather<<<rows, 256, 0, s>>>(tokens, static_cast<const __half*>(embed), static_cast<__half*>(hidden), rows,
                                        d_model, vocab, err);
    return cudaGetLastError();
}

// Prefill conv over the xBC columns of proj (B, L, proj_stride) -> SiLU -> x/B/C.
// conv output rounded to fp16 (the reference's conv_out slot), then SiLU rounded again.
constexpr int CT = 16;
__global__ void k_conv_silu_split(const __half* __restrict__ xbc, uint64_t in_stride, const __half* __restrict__ w,
                                  const __half* __restrict__ bias, __half* __restrict__ xo, __half* __restrict__ bo,
                                  __half* __restrict__ co, uint32_t L, uint32_t d_inner, uint32_t GN, uint32_t K) {
    const uint32_t D = d_inner + 2 * GN;
    const uint32_t d = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t t0 = blockIdx.y * CT, b = blockIdx.z;
    if (d >= D) return;
    const __half* xb = xbc + (uint64_t)b * L * in_stride;
    float wk[8], win[8];
    for (uint32_t k = 0; k < K; ++k) wk[k] = __half2float(w[(uint64_t)d * K + k]);
    const float bv = __half2float(bias[d]);
    for (uint32_t k = 0; k + 1 < K; ++k) {
        const int src = (int)t0 - (int)(K - 1) + (int)k;
        win[k] = src >= 0 ? __half2float(xb[(uint64_t)src * in_stride + d]) : 0.0f;
    }
    const uint32_t tend = min(t0 + CT, L);
    for (uint32_t t = t0; t < tend; ++t) {
        win[K - 1] = __half2float(xb[(uint64_t)t * in_stride + d]);
        float acc = bv;
        for (uint32_t k = 0; k < K; ++k) acc += wk[k] * win[k];
        const __half o = __float2half_rn(silu(__half2float(__float2half_rn(acc))));
        const uint64_t row = (uint64_t)b * L + t;
        if (d < d_inner) xo[row * d_inner + d] = o;
        else if (d < d_inner + GN) bo[row * GN + (d - d_inner)] = o;
        else co[row * GN + (d - d_inner - GN)] = o;
        for (uint32_t k = 0; k + 1 < K; ++k) win[k] = win[k + 1];
    }
}

// Vectorised form (d_conv == 4, 8 channels per thread, 16-byte loads and stores): the
// same arithmetic per channel. Needs in_stride, d_inner and GN multiples of 8 and 16-byte
// aligned rows, so an octet never straddles the x / B / C boundaries.
constexpr uint32_t CT8 = 8;    // tokens per thread
constexpr uint32_t CU8 = 8;    // rows loaded together (independent loads in flight per thread)
__global__ void __launch_bounds__(128) k_conv4_silu_split8(const __half* __restrict__ xbc, uint64_t in_stride,
                                                           const __half* __restrict__ w,
                                                           const __half* __restrict__ bias, __half* __restrict__ xo,
                                                           __half* __restrict__ bo, __half* __restrict__ co, uint32_t L,
                                                           uint32_t d_inner, uint32_t GN) {
    const uint32_t D = d_inner + 2 * GN;
    const uint32_t d0 = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
    const uint32_t t0 = blockIdx.y * CT8, b = blockIdx.z;
    if (d0 >= D) return;
    const __half* xb = xbc + (uint64_t)b * L * in_stride + d0;
    float wk[8][4], bv[8], win[3][8];
    {
        const uint4* w4 = reinterpret_cast<const uint4*>(w + (uint64_t)d0 * 4);   // 8 channels x 4 taps
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint4 u = w4[q];
            const __half* h = reinterpret_cast<const __half*>(&u);
#pragma unroll
            for (int e = 0; e < 8; ++e) wk[q * 2 + e / 4][e % 4] = __half2float(h[e]);
        }
        const uint4 bu = *reinterpret_cast<const uint4*>(bias + d0);
        const __half* bh = reinterpret_cast<const __half*>(&bu);
#pragma unroll
        for (int e = 0; e < 8; ++e) bv[e] = __half2float(bh[e]);
    }
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const int src = (int)t0 - 3 + k;
        uint4 u = make_uint4(0, 0, 0, 0);
        if (src >= 0) u = *reinterpret_cast<const uint4*>(xb + (uint64_t)src * in_stride);
        const __half* h = reinterpret_cast<const __half*>(&u);
#pragma unroll
        for (int e = 0; e < 8; ++e) win[k][e] = __half2float(h[e]);
    }
    __half* dst;
    uint32_t ds;
    if (d0 < d_inner) { dst = xo + d0; ds = d_inner; }
    else if (d0 < d_inner + GN) { dst = bo + (d0 - d_inner); ds = GN; }
    else { dst = co + (d0 - d_inner - GN); ds = GN; }
    const uint32_t tend = min(t0 + CT8, L);
    for (uint32_t tc = t0; tc < tend; tc += CU8) {
        // the rows of CU8 tokens are loaded before any is used: the loads are in flight together
        uint4 rows[CU8];
#pragma unroll
        for (uint32_t i = 0; i < CU8; ++i)
            rows[i] = tc + i < tend ? *reinterpret_cast<const uint4*>(xb + (uint64_t)(tc + i) * in_stride)
                                    : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (uint32_t i = 0; i < CU8; ++i) {
            if (tc + i >= tend) break;
            const __half* h = reinterpret_cast<const __half*>(&rows[i]);
            uint4 o;
            __half* oh = reinterpret_cast<__half*>(&o);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float xn = __half2float(h[e]);
                float acc = bv[e];
                acc += wk[e][0] * win[0][e];
                acc += wk[e][1] * win[1][e];
                acc += wk[e][2] * win[2][e];
                acc += wk[e][3] * xn;
                oh[e] = __float2half_rn(silu(__half2float(__float2half_rn(acc))));
                win[0][e] = win[1][e];
                win[1][e] = win[2][e];
                win[2][e] = xn;
            }
            *reinterpret_cast<uint4*>(dst + ((uint64_t)b * L + tc + i) * ds) = o;
        }
    }
}

cudaError_t launch_conv_silu_split(const void* xbc, uint64_t in_stride, const void* w, const void* bias, void* xo,
                                   void* bo, void* co, uint32_t B, uint32_t L, uint32_t d_inner, uint32_t GN,
                                   uint32_t K, cudaStream_t s) {
    const uint32_t D = d_inner + 2 * GN;
    if (!B || !L || K == 0 || K > 8) return K > 8 ? cudaErrorInvalidValue : cudaSuccess;
    if (K == 4 && in_stride % 8 == 0 && d_inner % 8 == 0 && GN % 8 == 0 && aligned(xbc, 16) && aligned(w, 16) &&
        aligned(bias, 16) && aligned(xo, 16) && aligned(bo, 16) && aligned(co, 16)) {
        dim3 grid((D / 8 + 127) / 128, (L + CT8 - 1) / CT8, B);
        k_conv4_silu_split8<<<grid, 128, 0, s>>>(static_cast<const __half*>(xbc), in_stride,
                                                 static_cast<const __half*>(w), static_cast<const __half*>(bias),
                                                 static_cast<__half*>(xo), static_cast<__half*>(bo),
                                                 static_cast<__half*>(co), L, d_inner, GN);
        return cudaGetLastError();
    }
    dim3 grid((D + 127) / 128, (L + CT - 1) / CT, B);
    k_conv_silu_split<<<grid, 128, 0, s>>>(static_cast<const __half*>(xbc), in_stride, static_cast<const __half*>(w),
                                           static_cast<const __half*>(bias), static_cast<__half*>(xo),
                                           static_cast<__half*>(bo), static_cast<__half*>(co), L, d_inner, GN, K);
    return cudaGetLastError();
}

// Decode conv update + SiLU + split: state (B, D, K) rolled in place.
__global__ void k_conv_update_silu_split(const __half* __restrict__ xbc, uint64_t in_stride, __half* __restrict__ state,
                                         const __half* __restrict__ w, const __half* __restrict__ bias,
                                         __half* __restrict__ xo, __half* __restrict__ bo, __half* __restrict__ co,
                                         uint32_t B, uint32_t d_inner, uint32_t GN, uint32_t K) {
    const uint32_t D = d_inner + 2 * GN;
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (uint64_t)B * D) return;
    const uint32_t d = (uint32_t)(i % D), b = (uint32_t)(i / D);
    __half* sd = state + i * K;
    const __half* wd = w + (uint64_t)d * K;
    float acc = __half2float(bias[d]);
    for (uint32_t k = 0; k + 1 < K; ++k) {
        const __half v = sd[k + 1];
        sd[k] = v;
        acc += __half2float(v) * __half2float(wd[k]);
    }
    const __half xn = xbc[(uint64_t)b * in_stride + d];
    sd[K - 1] = xn;
    acc += __half2float(xn) * __half2float(wd[K - 1]);
    const __half o = __float2half_rn(silu(__half2float(__float2half_rn(acc))));
    if (d < d_inner) xo[(uint64_t)b * d_inner + d] = o;
    else if (d < d_inner + GN) bo[(uint64_t)b * GN + (d - d_inner)] = o;
    else co[(uint64_t)b * GN + (d - d_inner - GN)] = o;
}

cudaError_t launch_conv_update_silu_split(const void* xbc, uint64_t in_stride, void* state, const void* w,
                                          const void* bias, void* xo, void* bo, void* co, uint32_t B, uint32_t d_inner,
                                          uint32_t GN, uint32_t K, cudaStream_t s) {
    const uint64_t n = (uint64_t)B * (d_inner + 2 * GN);
    if (!n) return cudaSuccess;
    k_conv_update_silu_split<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(
        static_cast<const __half*>(xbc), in_stride, static_cast<__half*>(state), static_cast<const __half*>(w),
        static_cast<const __half*>(bias), static_cast<__half*>(xo), static_cast<__half*>(bo), static_cast<__half*>(co), B,
        d_inner, GN, K);
    return cudaGetLastError();
}

// Seed conv state (B, D, K) from the last K rows of each sequence's pre-conv xBC.
__global__ void k_seed_strided(const __half* __restrict__ xbc, uint64_t in_stride, __half* __restrict__ state,
                               uint32_t B, uint32_t L, uint32_t D, uint32_t K) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (uint64_t)B * D * K) return;
    const uint32_t k = (uint32_t)(i % K);
    const uint64_t bd = i / K;
    const uint32_t d = (uint32_t)(bd % D), b = (uint32_t)(bd / D);
    const int src = (int)L - (int)K + (int)k;
    state[i] = src >= 0 ? xbc[((uint64_t)b * L + (uint32_t)src) * in_stride + d] : __float2half_rn(0.0f);
}

cudaError_t launch_seed_strided(const void* xbc, uint64_t in_stride, void* state, uint32_t B, uint32_t L, uint32_t D,
                                uint32_t K, cudaStream_t s) {
    const uint64_t n = (uint64_t)B * D * K;
    if (!n) return cudaSuccess;
    k_seed_strided<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(static_cast<const __half*>(xbc), in_stride,
                                                              static_cast<__half*>(state), B, L, D, K);
    return cudaGetLastError();
}

// gated[r, c] = half(silu(z[r*z_stride + c]) * y[r*d + c])
__global__ void k_gate(const __half* __restrict__ z, uint64_t z_stride, const __half* y, __half* out, uint32_t rows,
                       uint32_t d) {
    const uint64_t total = (uint64_t)rows * d;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t r = i / d, c = i % d;
        out[i] = __float2half_rn(silu(__half2float(z[r * z_stride + c])) * __half2float(y[i]));
    }
}

// 8 elements per thread with 16-byte accesses (d, z_stride multiples of 8, aligned rows).
__global__ void k_gate8(const __half* __restrict__ z, uint64_t z_stride, const __half* y, __half* out, uint32_t rows,
                        uint32_t d) {
    const uint32_t d8 = d / 8;
    const uint64_t total = (uint64_t)rows * d8;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t r = i / d8, c = (i % d8) * 8;
        const uint4 zu = *reinterpret_cast<const uint4*>(z + r * z_stride + c);
        const uint4 yu = *reinterpret_cast<const uint4*>(y + r * d + c);
        const __half* zh = reinterpret_cast<const __half*>(&zu);
        const __half* yh = reinterpret_cast<const __half*>(&yu);
        uint4 o;
        __half* oh = reinterpret_cast<__half*>(&o);
#pragma unroll
        for (int e = 0; e < 8; ++e) oh[e] = __float2half_rn(silu(__half2float(zh[e])) * __half2float(yh[e]));
        *reinterpret_cast<uint4*>(out + r * d + c) = o;
    }
}

cudaError_t launch_gate(const void* z, uint64_t z_stride, const void* y, void* out, uint32_t rows, uint32_t d,
                        cudaStream_t s) {
    const uint64_t n = (uint64_t)rows * d;
    if (!n) return cudaSuccess;
    if (d % 8 == 0 && z_stride % 8 == 0 && aligned(z, 16) && aligned(y, 16) && aligned(out, 16)) {
        uint64_t g = (n / 8 + 255) / 256;
        if (g > 148 * 16) g = 148 * 16;
        k_gate8<<<(unsigned)g, 256, 0, s>>>(static_cast<const __half*>(z), z_stride, static_cast<const __half*>(y),
                                            static_cast<__half*>(out), rows, d);
        return cudaGetLastError();
    }
    uint64_t g = (n + 255) / 256;
    if (g > 148 * 32) g = 148 * 32;
    k_gate<<<(unsigned)g, 256, 0, s>>>(static_cast<const __half*>(z), z_stride, static_cast<const __half*>(y),
                                       static_cast<__half*>(out), rows, d);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
//  Seeded synthetic weights (see synth_rng.h for the value recipe).
// ---------------------------------------------------------------------------
// fp16 tensor of n values: out[i] = half(synth_uniform(seed, stream, i) * amp)
__global__ void k_synth_f16(__half* __restrict__ out, uint64_t n, uint64_t seed, uint64_t stream, float amp) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
        out[i] = __float2half_rn(synth_value(seed, stream, i, amp));
}

// INT4_B32 tensor (N, K): values as k_synth_f16 (then rounded to fp16 like the exporter's
// t.to(float16)), quantised per 32-block: packed nibbles at out, scales at out + N*K/2.
__global__ void k_synth_int4(uint8_t* __restrict__ out, uint32_t N, uint32_t K, uint64_t seed, uint64_t stream,
                             float amp) {
    const uint32_t nb = K / 32;
    const uint64_t total = (uint64_t)N * nb;
    __half* scales = reinterpret_cast<__half*>(out + (uint64_t)N * K / 2);
    for (uint64_t blk = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; blk < total;
         blk += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t row = blk / nb, b = blk % nb;
        float v[32];
        float absmax = 0.0f;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            v[j] = __half2float(__float2half_rn(synth_value(seed, stream, row * K + b * 32 + j, amp)));
            absmax = fmaxf(absmax, fabsf(v[j]));
        }
        absmax = fmaxf(absmax, 1e-12f);
        const float scale = __fdiv_rn(absmax, 7.0f);
        scales[blk] = __float2half_rn(scale);
        uint8_t* dst = out + row * (K / 2) + b * 16;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const float q0 = fminf(fmaxf(rintf(__fdiv_rn(v[2 * j], scale)), -8.0f), 7.0f);
            const float q1 = fminf(fmaxf(rintf(__fdiv_rn(v[2 * j + 1], scale)), -8.0f), 7.0f);
            dst[j] = (uint8_t)((((int)q1 & 0xF) << 4) | ((int)q0 & 0xF));
        }
    }
}

cudaError_t launch_synth_f16(void* out, uint64_t n, uint64_t seed, uint64_t stream, float amp, cudaStream_t s) {
    if (!n) return cudaSuccess;
    uint64_t g = (n + 255) / 256;
    if (g > 148 * 64) g = 148 * 64;
    k_synth_f16<<<(unsigned)g, 256, 0, s>>>(static_cast<__half*>(out), n, seed, stream, amp);
    return cudaGetLastError();
}

cudaError_t launch_synth_int4(void* out, uint32_t N, uint32_t K, uint64_t seed, uint64_t stream, float amp,
                              cudaStream_t s) {
    const uint64_t n = (uint64_t)N * (K / 32);
    if (!n) return cudaSuccess;
    uint64_t g = (n + 127) / 128;
    if (g > 148 * 64) g = 148 * 64;
    k_synth_int4<<<(unsigned)g, 128, 0, s>>>(static_cast<uint8_t*>(out), N, K, seed, stream, amp);
    return cudaGetLastError();
}

}  // namespace lssm
