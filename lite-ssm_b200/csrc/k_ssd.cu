// k_ssd.cu — Mamba-2 state-space duality (SSD) kernels.
//
//   ssd_step    (decode)  shaders/ssd_step.metal:33-77
//     S[b,h,p,n] = exp(A_h dt) S + dt B[n] x[p];  y[p] = sum_n C[n] S[p,n] + D_h x[p]
//     One warp per (b, h, p) state row: the 128 d_state floats of the row are read and
//     written once as float4 (lanes across N — coalesced, unlike the reference's one
//     thread per row walking N). Optionally fuses the mixer gate
//     gated = half(silu(z) * half(y)) (mamba2_block.cpp:231-234).
//
//   ssd_chunked (prefill) shaders/ssd_chunked.metal:82-297, general-shape kernel.
//     One CTA per (batch, head) walks the sequence in chunks of Q tokens, keeping the
//     (P x N) state in fp32 shared memory (the reference stages it in fp16; fp32 here
//     is strictly more accurate). Per chunk: dt -> softplus/clamp, inclusive cumsum of
//     A dt, M[t,j] = (C_t . B_j) exp(Lc_t - Lc_j) dt_j (j <= t), y = M X + exp(Lc_t)
//     C_t S + D x, S <- exp(Lc_end) S + sum_j exp(Lc_end - Lc_j) dt_j B_j (x) X_j.
#include "device_util.cuh"
#include "lssm_internal.h"

namespace lssm {

// ---------------------------------------------------------------------------
//  ssd_step
// ---------------------------------------------------------------------------


// Vector path: each warp owns STEP_R consecutive (b, h, p) state rows with N == 128
// (one float4 per lane per row). P % STEP_R == 0, so a warp's rows share one (b, h):
// the head's dt / decay are computed once per warp and the row -> (b, h, p) split once,
// in 32-bit arithmetic. All rows' state loads are issued before any arithmetic, so a
// warp keeps STEP_R * 512 B of state in flight.
constexpr int STEP_R = 8;

__global__ void __launch_bounds__(256) k_ssd_step_r4(StepArgs a) {
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rows = a.batch * a.H * a.P;
    const uint32_t row0 = (blockIdx.x * 8 + warp) * STEP_R;
    if (row0 >= rows) return;
    const uint32_t p0 = row0 % a.P, bh = row0 / a.P, h = bh % a.H, b = bh / a.H;
    const uint32_t g = h / max(1u, a.H / a.G);
    float4 s[STEP_R];
#pragma unroll
    for (int r = 0; r < STEP_R; ++r)
        s[r] = *reinterpret_cast<const float4*>(a.state + (uint64_t)(row0 + r) * 128 + lane * 4);
    const uint2 bu = *reinterpret_cast<const uint2*>(a.B + b * a.bc_bs + (uint64_t)g * 128 + lane * 4);
    const uint2 cu = *reinterpret_cast<const uint2*>(a.C + b * a.bc_bs + (uint64_t)g * 128 + lane * 4);
    const __half* xrow = a.x + b * a.x_bs + (uint64_t)h * a.P + p0;
    float xv[STEP_R];
#pragma unroll
    for (int r = 0; r < STEP_R; ++r) xv[r] = __half2float(xrow[r]);
    const float A = -expf(__half2float(a.A_log[h]));
    const float dt = fminf(fmaxf(softplus(__half2float(a.dt_raw[b * a.dt_bs + h]) + __half2float(a.dt_bias[h])),
                                 a.dt_min), a.dt_max);
    const float decay = expf(A * dt);
    const float Dh = a.has_D ? __half2float(a.D[h]) : 0.0f;
    const float2 b01 = __half22float2(*reinterpret_cast<const __half2*>(&bu.x));
    const float2 b23 = __half22float2(*reinterpret_cast<const __half2*>(&bu.y));
    const float2 c01 = __half22float2(*reinterpret_cast<const __half2*>(&cu.x));
    const float2 c23 = __half22float2(*reinterpret_cast<const __half2*>(&cu.y));
    float acc[STEP_R];
#pragma unroll
    for (int r = 0; r < STEP_R; ++r) {
        const float dtx = dt * xv[r];
        float4 v = s[r];
        v.x = decay * v.x + b01.x * dtx;
        v.y = decay * v.y + b01.y * dtx;
        v.z = decay * v.z + b23.x * dtx;
        v.w = decay * v.w + b23.y * dtx;
        s[r] = v;
        acc[r] = c01.x * v.x + c01.y * v.y + c23.x * v.z + c23.y * v.w;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int r = 0; r < STEP_R; ++r) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
#pragma unroll
    for (int r = 0; r < STEP_R; ++r)
        *reinterpret_cast<float4*>(a.state + (uint64_t)(row0 + r) * 128 + lane * 4) = s[r];
    // lane r writes row r's output (y, or the gated value half(silu(z) * half(y)))
    float mine = acc[0], xm = xv[0];
#pragma unroll
    for (int r = 1; r < STEP_R; ++r)
        if ((int)lane == r) { mine = acc[r]; xm = xv[r]; }
    if (lane < STEP_R) {
        const uint64_t o = (uint64_t)h * a.P + p0 + lane;
        const __half yh = __float2half_rn(mine + Dh * xm);
        if (a.z) a.y[b * a.y_bs + o] = __float2half_rn(silu(__half2float(a.z[b * a.z_bs + o])) * __half2float(yh));
        else a.y[b * a.y_bs + o] = yh;
    }
}

template <bool VEC4>
__global__ void __launch_bounds__(256) k_ssd_step(StepArgs a) {
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint64_t row = (uint64_t)blockIdx.x * 8 + warp;
    const uint64_t rows = (uint64_t)a.batch * a.H * a.P;
    if (row >= rows) return;
    const uint32_t p = (uint32_t)(row % a.P);
    const uint32_t h = (uint32_t)((row / a.P) % a.H);
    const uint32_t b = (uint32_t)(row / ((uint64_t)a.P * a.H));
    const uint32_t hpg = max(1u, a.H / a.G);
    const uint32_t g = h / hpg;
    const float A = -expf(__half2float(a.A_log[h]));
    const float dt = fminf(fmaxf(softplus(__half2float(a.dt_raw[b * a.dt_bs + h]) + __half2float(a.dt_bias[h])),
                                 a.dt_min), a.dt_max);
    const float decay = expf(A * dt);
    const float xv = __half2float(a.x[b * a.x_bs + (uint64_t)h * a.P + p]);
    const float dtx = dt * xv;
    float* S = a.state + row * a.N;
    const __half* Bg = a.B + b * a.bc_bs + (uint64_t)g * a.N;
    const __half* Cg = a.C + b * a.bc_bs + (uint64_t)g * a.N;
    float acc = 0.0f;
    if (VEC4) {
        for (uint32_t n = lane * 4; n < a.N; n += 128) {
            float4 s = *reinterpret_cast<const float4*>(S + n);
            const uint2 bu = *reinterpret_cast<const uint2*>(Bg + n);
            const uint2 cu = *reinterpret_cast<const uint2*>(Cg + n);
            const float2 b01 = __half22float2(*reinterpret_cast<const __half2*>(&bu.x));
            const float2 b23 = __half22float2(*reinterpret_cast<const __half2*>(&bu.y));
            const float2 c01 = __half22float2(*reinterpret_cast<const __half2*>(&cu.x));
            const float2 c23 = __half22float2(*reinterpret_cast<const __half2*>(&cu.y));
            s.x = decay * s.x + b01.x * dtx;
            s.y = decay * s.y + b01.y * dtx;
            s.z = decay * s.z + b23.x * dtx;
            s.w = decay * s.w + b23.y * dtx;
            *reinterpret_cast<float4*>(S + n) = s;
            acc += c01.x * s.x + c01.y * s.y + c23.x * s.z + c23.y * s.w;
        }
    } else {
        for (uint32_t n = lane; n < a.N; n += 32) {
            const float s = decay * S[n] + __half2float(Bg[n]) * dtx;
            S[n] = s;
            acc += __half2float(Cg[n]) * s;
        }
    }
    acc = warp_sum(acc);
    if (lane == 0) {
        const float Dh = a.has_D ? __half2float(a.D[h]) : 0.0f;
        const __half yh = __float2half_rn(acc + Dh * xv);
        const uint64_t o = (uint64_t)h * a.P + p;
        if (a.z) {
            const float zv = __half2float(a.z[b * a.z_bs + o]);
            a.y[b * a.y_bs + o] = __float2half_rn(silu(zv) * __half2float(yh));
        } else {
            a.y[b * a.y_bs + o] = yh;
        }
    }
}

cudaError_t launch_ssd_step_ex(const StepArgs& a, cudaStream_t s) {
    const uint64_t rows = (uint64_t)a.batch * a.H * a.P;
    if (!rows) return cudaSuccess;
    const bool vec = (a.N % 4 == 0) && aligned(a.state, 16) && aligned(a.B, 8) && aligned(a.C, 8) &&
                     (a.bc_bs % 4 == 0) && (a.G == 1 || a.N % 4 == 0);
    if (vec && a.N == 128 && a.P % STEP_R == 0 && rows < (1ull << 31)) {
        k_ssd_step_r4<<<(unsigned)((rows + 8 * STEP_R - 1) / (8 * STEP_R)), 256, 0, s>>>(a);
        return cudaGetLastError();
    }
    const unsigned grid = (unsigned)((rows + 7) / 8);
    if (vec) k_ssd_step<true><<<grid, 256, 0, s>>>(a);
    else k_ssd_step<false><<<grid, 256, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_ssd_step(const void* x, const void* B, const void* C, const void* dt_raw, const void* dt_bias,
                            const void* A_log, const void* D, float* state, void* y, uint32_t batch, uint32_t H,
                            uint32_t P, uint32_t N, uint32_t G, float dt_min, float dt_max, uint32_t has_D,
                            cudaStream_t s) {
    StepArgs a{};
    a.x = static_cast<const __half*>(x); a.B = static_cast<const __half*>(B); a.C = static_cast<const __half*>(C);
    a.dt_raw = static_cast<const __half*>(dt_raw); a.dt_bias = static_cast<const __half*>(dt_bias);
    a.A_log = static_cast<const __half*>(A_log); a.D = static_cast<const __half*>(D);
    a.state = state; a.y = static_cast<__half*>(y); a.z = nullptr;
    a.batch = batch; a.H = H; a.P = P; a.N = N; a.G = G ? G : 1;
    a.dt_min = dt_min; a.dt_max = dt_max; a.has_D = has_D;
    a.x_bs = (uint64_t)H * P; a.bc_bs = (uint64_t)a.G * N; a.dt_bs = H; a.y_bs = (uint64_t)H * P; a.z_bs = 0;
    return launch_ssd_step_ex(a, s);
}

// ---------------------------------------------------------------------------
//  ssd_chunked, general shapes (SIMT, fp32 state in shared memory)
// ---------------------------------------------------------------------------
constexpr int SSD_Q = 32;          // tokens per chunk in this kernel
constexpr int SSD_THREADS = 256;

__global__ void __launch_bounds__(SSD_THREADS) k_ssd_chunked_simt(SsdArgs a) {
    extern __shared__ float sm[];
    const uint32_t P = a.P, N = a.N, Q = SSD_Q;
    float* S = sm;                          // P*N
    float* Bs = S + (size_t)P * N;          // Q*N
    float* Cs = Bs + (size_t)Q * N;         // Q*N
    float* Xs = Cs + (size_t)Q * N;         // Q*P
    float* M = Xs + (size_t)Q * P;          // Q*Q
    float* DT = M + Q * Q;                  // Q
    float* Lc = DT + Q;                     // Q
    float* Wj = Lc + Q;                     // Q  (exp(Lend - Lc_j) * dt_j)

    const uint32_t bh = blockIdx.x;
    const uint32_t h = bh % a.H, b = bh / a.H;
    const uint32_t hpg = max(1u, a.H / a.G), g = h / hpg;
    const uint64_t xrs = a.x_row_stride ? a.x_row_stride : (uint64_t)a.H * P;
    const uint64_t bcrs = a.bc_row_stride ? a.bc_row_stride : (uint64_t)a.G * N;
    const uint64_t dtrs = a.dt_row_stride ? a.dt_row_stride : a.H;
    const uint64_t yrs = a.y_row_stride ? a.y_row_stride : (uint64_t)a.H * P;
    const uint64_t xb = (uint64_t)b * a.L * xrs, bcb = (uint64_t)b * a.L * bcrs, dtb = (uint64_t)b * a.L * dtrs,
                   yb = (uint64_t)b * a.L * yrs;
    const float A = -expf(load_any(a.A_log, h, a.param_dtype));
    const float dbias = load_any(a.dt_bias, h, a.param_dtype);
    const float Dh = a.has_D ? load_any(a.D, h, a.param_dtype) : 0.0f;
    float* Sg = a.state + ((uint64_t)b * a.H + h) * P * N;

    for (uint32_t i = threadIdx.x; i < P * N; i += blockDim.x) S[i] = Sg[i];

    for (uint32_t t0 = 0; t0 < a.L; t0 += Q) {
        const uint32_t tl = min(Q, a.L - t0);
        __syncthreads();
        for (uint32_t i = threadIdx.x; i < Q * N; i += blockDim.x) {
            const uint32_t t = i / N, n = i % N;
            float bv = 0.0f, cv = 0.0f;
            if (t < tl) {
                const uint64_t o = bcb + (uint64_t)(t0 + t) * bcrs + (uint64_t)g * N + n;
                bv = load_any(a.B, o, a.x_dtype);
                cv = load_any(a.C, o, a.x_dtype);
            }
            Bs[i] = bv;
            Cs[i] = cv;
        }
        for (uint32_t i = threadIdx.x; i < Q * P; i += blockDim.x) {
            const uint32_t t = i / P, p = i % P;
            Xs[i] = t < tl ? load_any(a.X, xb + (uint64_t)(t0 + t) * xrs + (uint64_t)h * P + p, a.x_dtype) : 0.0f;
        }
        if (threadIdx.x < 32) {
            const uint32_t t = threadIdx.x;
            float d = 0.0f;
            if (t < tl) {
                d = softplus(load_any(a.dt_raw, dtb + (uint64_t)(t0 + t) * dtrs + h, a.dt_dtype) + dbias);
                d = fminf(fmaxf(d, a.dt_min), a.dt_max);
            }
            float v = A * d;   // inclusive warp scan (Q == 32)
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float u = __shfl_up_sync(0xffffffffu, v, o);
                if ((int)t >= o) v += u;
            }
            DT[t] = d;
            Lc[t] = v;
            const float lend = __shfl_sync(0xffffffffu, v, tl - 1);
            Wj[t] = t < tl ? expf(lend - v) * d : 0.0f;
        }
        __syncthreads();
        // M[t, j] (causal, j <= t)
        for (uint32_t i = threadIdx.x; i < Q * Q; i += blockDim.x) {
            const uint32_t t = i / Q, j = i % Q;
            float m = 0.0f;
            if (j <= t && t < tl) {
                float cb = 0.0f;
                for (uint32_t n = 0; n < N; ++n) cb += Cs[t * N + n] * Bs[j * N + n];
                m = cb * expf(Lc[t] - Lc[j]) * DT[j];
            }
            M[i] = m;
        }
        __syncthreads();
        // Y
        for (uint32_t i = threadIdx.x; i < tl * P; i += blockDim.x) {
            const uint32_t t = i / P, p = i % P;
            float yi = 0.0f;
            for (uint32_t j = 0; j <= t; ++j) yi += M[t * Q + j] * Xs[j * P + p];
            float ye = 0.0f;
            for (uint32_t n = 0; n < N; ++n) ye += Cs[t * N + n] * S[p * N + n];
            const float y = yi + ye * expf(Lc[t]) + Dh * Xs[t * P + p];
            store_any(a.Y, yb + (uint64_t)(t0 + t) * yrs + (uint64_t)h * P + p, a.y_dtype, y);
        }
        __syncthreads();
        // State update
        const float dch = expf(Lc[tl - 1]);
        for (uint32_t i = threadIdx.x; i < P * N; i += blockDim.x) {
            const uint32_t p = i / N, n = i % N;
            float acc = dch * S[i];
            for (uint32_t j = 0; j < tl; ++j) acc += Wj[j] * Bs[j * N + n] * Xs[j * P + p];
            S[i] = acc;
        }
    }
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < P * N; i += blockDim.x) Sg[i] = S[i];
}

cudaError_t launch_ssd_chunked_tc(const SsdArgs& s, cudaStream_t st);

cudaError_t launch_ssd_chunked(const SsdArgs& a, cudaStream_t s) {
    if (!a.batch || !a.L || !a.H) return cudaSuccess;
    // P = 64, N = 128 (every Mamba-2 checkpoint shape) with 16-byte aligned rows takes the
    // chunk-parallel tensor-core kernel when scratch for its carried states is given (and the
    // heads pair up within groups), else the sequential tensor-core kernel; anything else
    // uses the general-shape kernel below.
    cudaError_t e = cudaErrorNotSupported;
    if (a.ws) e = launch_ssd_chunked_cp(a, a.ws, a.ws_bytes, a.sm_count ? a.sm_count : 148, s);
    if (e != cudaErrorNotSupported) return e;
    e = launch_ssd_chunked_tc(a, s);
    if (e != cudaErrorNotSupported) return e;
    const size_t smem = sizeof(float) * ((size_t)a.P * a.N + 2ull * SSD_Q * a.N + (size_t)SSD_Q * a.P +
                                         (size_t)SSD_Q * SSD_Q + 3 * SSD_Q);
    if (smem > 220 * 1024) return cudaErrorInvalidValue;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(k_ssd_chunked_simt, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
    }
    k_ssd_chunked_simt<<<a.batch * a.H, SSD_THREADS, smem, s>>>(a);
    e = cudaGetLastError();
    if (e != cudaSuccess || !a.z) return e;
    // the general-shape kernel writes y; gate it in place
    const uint64_t yrs = a.y_row_stride ? a.y_row_stride : (uint64_t)a.H * a.P;
    if (yrs != (uint64_t)a.H * a.P || a.y_dtype != 0) return cudaErrorInvalidValue;
    return launch_gate(a.z, a.z_row_stride, a.Y, a.Y, a.batch * a.L, a.H * a.P, s);
}

}  // namespace lssm
