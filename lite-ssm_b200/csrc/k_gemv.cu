// k_gemv.cu — decode-side matrix-vector products (M <= 8 activation rows):
//
//   * fp16 weights  (shaders/linear.metal:82-204: linear_f16_gemv, linear_silu_f16_gemv,
//     rmsnorm_linear_f16_gemv) — 16-byte weight loads, fp32 FMAs.
//   * INT4_B32 weights (shaders/linear.metal:440-474: linear_int4_gemv) — the decode
//     hot loop. The INT4 stream is the roofline (0.5625 B/weight), so the kernel keeps
//     the per-weight instruction count near one: nibbles are turned into exact fp16
//     integers with one lop3 + one HFMA2 per pair (magic-number conversion), the
//     products run on the tensor pipe with register-operand mma.sync (m16n8k16,
//     fp32 accumulate), and the per-block fp16 scale is applied to the fp32 block
//     partial. Register-only: nothing is staged through shared memory except the
//     (tiny) activation vector, so the dequantised weights never cost SMEM bandwidth.
//
// Both kernels share the optional fused prologue (RMSNorm of the input rows, the
// reference's rmsnorm_f16 on the same data, shaders/norm.metal:51-79) and epilogues
// (store / SiLU / residual add).
#include <algorithm>

#include "device_util.cuh"
#include "lssm_internal.h"
#include "mma_int4.cuh"

namespace lssm {

static int gemv_sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

enum : int { EPI_STORE = 0, EPI_SILU = 1, EPI_RESIDUAL = 2, EPI_F32 = 3 };

constexpr int GEMV_THREADS = 256;
constexpr int GEMV_WARPS = GEMV_THREADS / 32;
constexpr int GEMV_MMAX = 8;

// Per-row RMSNorm factor of the CTA's input rows (fused prologue); rr[m] = rsqrt(mean(x^2)+eps).
__device__ __forceinline__ void prenorm_factors(const __half* __restrict__ x, uint32_t M, uint32_t K, float eps,
                                                float* rr, float* red) {
    for (uint32_t m = 0; m < M; ++m) {
        float ss = 0.0f;
        const __half* xr = x + (uint64_t)m * K;
        for (uint32_t k = threadIdx.x; k < K; k += blockDim.x) {
            float v = __half2float(xr[k]);
            ss += v * v;
        }
        float t = block_sum(ss, red);
        if (threadIdx.x == 0) rr[m] = rsqrtf(t / (float)K + eps);
    }
    __syncthreads();
}

__device__ __forceinline__ float in_val(const __half* __restrict__ x, const __half* __restrict__ nw, const float* rr,
                                        uint32_t m, uint32_t K, uint32_t k) {
    float v = __half2float(x[(uint64_t)m * K + k]);
    if (nw) v = __half2float(__float2half_rn(v * __half2float(nw[k]) * rr[m]));
    return v;
}

// Vectorised staging of the CTA's input rows (K % 8 == 0, x 16-byte aligned): 16-byte
// loads of x and of the norm weight, rr from a block reduction, then each octet
// x[m][8q .. 8q+7] -> half(v * w * rr) (in_val's arithmetic) stored as one uint4 at
// dst + m * row_quads + q, either in the INT4 fragment permutation {0,4,1,5,2,6,3,7}
// (frag) or in natural order.
__device__ __forceinline__ void stage_x_vec(const __half* __restrict__ x, const __half* __restrict__ nw, uint32_t M,
                                            uint32_t K, float eps, bool frag, uint4* dst, uint32_t row_quads,
                                            float* rr, float* red) {
    const uint32_t nq = K / 8;
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    const uint4* wv = reinterpret_cast<const uint4*>(nw);
    if (nw) {
        for (uint32_t m = 0; m < M; ++m) {
            float ss = 0.0f;
            for (uint32_t q = threadIdx.x; q < nq; q += blockDim.x) {
                const uint4 u = xv[(uint64_t)m * nq + q];
                const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float2 f = __half22float2(h[j]);
                    ss += f.x * f.x + f.y * f.y;
                }
            }
            const float t = block_sum(ss, red);
            if (threadIdx.x == 0) rr[m] = rsqrtf(t / (float)K + eps);
        }
        __syncthreads();
    }
    for (uint32_t i = threadIdx.x; i < M * nq; i += blockDim.x) {
        const uint32_t m = i / nq, q = i - m * nq;
        uint4 u = xv[(uint64_t)m * nq + q];
        __half v[8];
        *reinterpret_cast<uint4*>(v) = u;
        if (nw) {
            const uint4 wu = wv[q];
            const __half* w8 = reinterpret_cast<const __half*>(&wu);
            const float r = rr[m];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = __float2half_rn(__half2float(v[j]) * __half2float(w8[j]) * r);
        }
        if (frag) {
            const __half2 o0 = __halves2half2(v[0], v[4]), o1 = __halves2half2(v[1], v[5]);
            const __half2 o2 = __halves2half2(v[2], v[6]), o3 = __halves2half2(v[3], v[7]);
            u.x = *reinterpret_cast<const uint32_t*>(&o0);
            u.y = *reinterpret_cast<const uint32_t*>(&o1);
            u.z = *reinterpret_cast<const uint32_t*>(&o2);
            u.w = *reinterpret_cast<const uint32_t*>(&o3);
        } else {
            u = *reinterpret_cast<const uint4*>(v);
        }
        dst[(uint64_t)m * row_quads + q] = u;
    }
}

// Staging for the bias-folded INT4 MMA (dequant_word_fold): one thread per (row m,
// 32-k block b) writes the block's four fragment quads and corr[b * cs + m] =
// fold_bias(sum of x at even k, sum at odd k) over the block, summed in a fixed order (deterministic). cs = 8: rows
// m in [M, 8) get corr 0 (multi-row MMA columns); cs = 1: one row. x values as in_val
// (RMS-normalised with rr when nw is given).
__device__ __forceinline__ void stage_x_fold(const __half* __restrict__ x, const __half* __restrict__ nw, uint32_t M,
                                             uint32_t K, float eps, uint4* xs, float* corr, uint32_t cs, float* rr,
                                             float* red) {
    const uint32_t nq = K / 8, nb = K / 32;
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    const uint4* wv = reinterpret_cast<const uint4*>(nw);
    if (nw) {
        for (uint32_t m = 0; m < M; ++m) {
            float ss = 0.0f;
            for (uint32_t q = threadIdx.x; q < nq; q += blockDim.x) {
                const uint4 u = xv[(uint64_t)m * nq + q];
                const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float2 f = __half22float2(h[j]);
                    ss += f.x * f.x + f.y * f.y;
                }
            }
            const float t = block_sum(ss, red);
            if (threadIdx.x == 0) rr[m] = rsqrtf(t / (float)K + eps);
        }
        __syncthreads();
    }
    const uint32_t rows_out = cs == 1 ? 1 : 8;
    for (uint32_t i = threadIdx.x; i < rows_out * nb; i += blockDim.x) {
        const uint32_t m = i / nb, b = i - m * nb;
        if (m >= M) {
            corr[b * cs + m] = 0.0f;
            continue;
        }
        float se = 0.0f, so = 0.0f;
#pragma unroll
        for (uint32_t o = 0; o < 4; ++o) {
            const uint32_t q = b * 4 + o;
            const uint4 u = xv[(uint64_t)m * nq + q];
            __half v[8];
            *reinterpret_cast<uint4*>(v) = u;
            if (nw) {
                const uint4 wu = wv[q];
                const __half* w8 = reinterpret_cast<const __half*>(&wu);
                const float r = rr[m];
#pragma unroll
                for (int j = 0; j < 8; ++j) v[j] = __float2half_rn(__half2float(v[j]) * __half2float(w8[j]) * r);
            }
#pragma unroll
            for (int j = 0; j < 8; j += 2) {
                se += __half2float(v[j]);
                so += __half2float(v[j + 1]);
            }
            const __half2 o0 = __halves2half2(v[0], v[4]), o1 = __halves2half2(v[1], v[5]);
            const __half2 o2 = __halves2half2(v[2], v[6]), o3 = __halves2half2(v[3], v[7]);
            uint4 f;
            f.x = *reinterpret_cast<const uint32_t*>(&o0);
            f.y = *reinterpret_cast<const uint32_t*>(&o1);
            f.z = *reinterpret_cast<const uint32_t*>(&o2);
            f.w = *reinterpret_cast<const uint32_t*>(&o3);
            xs[(uint64_t)m * nq + q] = f;
        }
        corr[b * cs + m] = fold_bias(se, so);
    }
}

template <int EPI>
__device__ __forceinline__ void gemv_store(__half* y, uint64_t idx, float acc) {
    if (EPI == EPI_STORE) {
        y[idx] = __float2half_rn(acc);
    } else if (EPI == EPI_SILU) {
        y[idx] = __float2half_rn(silu(acc));
    } else if (EPI == EPI_F32) {
        reinterpret_cast<float*>(y)[idx] = acc;
    } else {
        // block_out rounded to fp16, then hidden += block_out (mamba2_block.cpp:274-276)
        const float o = __half2float(__float2half_rn(acc));
        y[idx] = __float2half_rn(__half2float(y[idx]) + o);
    }
}

// ---------------------------------------------------------------------------
//  fp16 GEMV: one warp per output row, lanes stride K in 8-half (16 B) vectors.
//  x (M, K) staged to shared memory as fp32 (optionally RMS-normalised).
// ---------------------------------------------------------------------------
template <int EPI, int VEC>
__global__ void __launch_bounds__(GEMV_THREADS) k_gemv_f16(const __half* __restrict__ x, const __half* __restrict__ w,
                                                         __half* __restrict__ y, uint32_t M, uint32_t N, uint32_t K,
                                                         const __half* __restrict__ norm_w, float eps) {
    extern __shared__ float xs[];          // M * K floats
    __shared__ float red[32];
    __shared__ float rr[GEMV_MMAX];
    if (norm_w) prenorm_factors(x, M, K, eps, rr, red);
    for (uint32_t i = threadIdx.x; i < M * K; i += blockDim.x)
        xs[i] = in_val(x, norm_w, rr, i / K, K, i % K);
    __syncthreads();

    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t nvec = K / VEC;
    for (uint32_t row = blockIdx.x * GEMV_WARPS + warp; row < N; row += gridDim.x * GEMV_WARPS) {
        float acc[GEMV_MMAX];
#pragma unroll
        for (int m = 0; m < GEMV_MMAX; ++m) acc[m] = 0.0f;
        const __half* wr = w + (uint64_t)row * K;
#pragma unroll 4
        for (uint32_t v = lane; v < nvec; v += 32) {
            float wf[VEC];
            if (VEC == 8) {
                const uint4 u = __ldg(reinterpret_cast<const uint4*>(wr) + v);
                const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
                for (int j = 0; j < 4; ++j) { float2 f = __half22float2(h[j]); wf[2 * j] = f.x; wf[2 * j + 1] = f.y; }
            } else if (VEC == 4) {
                const uint2 u = __ldg(reinterpret_cast<const uint2*>(wr) + v);
                const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
                for (int j = 0; j < 2; ++j) { float2 f = __half22float2(h[j]); wf[2 * j] = f.x; wf[2 * j + 1] = f.y; }
            } else {
                wf[0] = __half2float(wr[v]);
            }
#pragma unroll
            for (int m = 0; m < GEMV_MMAX; ++m) {
                if (m < (int)M) {
                    const float* xr = xs + (uint64_t)m * K + (uint64_t)v * VEC;
#pragma unroll
                    for (int j = 0; j < VEC; ++j) acc[m] += wf[j] * xr[j];
                }
            }
        }
#pragma unroll
        for (int m = 0; m < GEMV_MMAX; ++m) {
            if (m < (int)M) {
                float t = warp_sum(acc[m]);
                if (lane == 0) gemv_store<EPI>(y, (uint64_t)m * N + row, t);
            }
        }
    }
}

// ---------------------------------------------------------------------------
//  fp16 GEMV on mma.sync for 2..8 activation rows (lm_head of batched / tensor-
//  parallel decode). One warp per 16-row tile, over the whole K: lane (g, c) loads
//  16 bytes of rows g and g + 8 at k = 32s + 8c (each row's 64-byte span read whole),
//  which is the A fragment of two m16n8k16 MMAs under the k-slot map
//  {2c, 2c+1, 2c+8, 2c+9} -> 32s + 8c + {0, 1, 2, 3} (and + 4 for the second MMA); the
//  B fragment is x[g][32s + 8c .. +7] in natural order from shared memory (rows padded
//  by 64 bytes: conflict-free). Batch rows are the MMA columns, fp32 accumulate; tiles
//  are grid-strided so the staged x is reused.
// ---------------------------------------------------------------------------
constexpr int F16MMA_UNROLL = 8;

template <int EPI>
__global__ void __launch_bounds__(GEMV_THREADS) k_gemv_f16_mma(const __half* __restrict__ x,
                                                             const __half* __restrict__ w, __half* __restrict__ y,
                                                             uint32_t M, uint32_t N, uint32_t K,
                                                             const __half* __restrict__ norm_w, float eps) {
    extern __shared__ __align__(16) uint4 xs_nat[];
    __shared__ float red[32];
    __shared__ float rr[GEMV_MMAX];
    const uint32_t rq = K / 8 + 4;   // padded row, in uint4
    stage_x_vec(x, norm_w, M, K, eps, false, xs_nat, rq, rr, red);
    __syncthreads();
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t g = lane >> 2, c = lane & 3;
    const uint32_t ntiles = (N + 15) / 16, nsteps = K / 32;
    const bool has_x = g < M;
    const uint4* xr = xs_nat + (uint64_t)(has_x ? g : 0) * rq + c;
    for (uint32_t t = blockIdx.x * GEMV_WARPS + warp; t < ntiles; t += gridDim.x * GEMV_WARPS) {
        const uint32_t ra = min(t * 16 + g, N - 1), rb = min(t * 16 + g + 8, N - 1);
        const uint4* wa = reinterpret_cast<const uint4*>(w + (uint64_t)ra * K) + c;
        const uint4* wb = reinterpret_cast<const uint4*>(w + (uint64_t)rb * K) + c;
        float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (uint32_t s0 = 0; s0 < nsteps; s0 += F16MMA_UNROLL) {
            uint4 A[F16MMA_UNROLL], Bv[F16MMA_UNROLL];
#pragma unroll
            for (int j = 0; j < F16MMA_UNROLL; ++j) {
                if (s0 + j < nsteps) {
                    A[j] = __ldcs(wa + (s0 + j) * 4);
                    Bv[j] = __ldcs(wb + (s0 + j) * 4);
                }
            }
#pragma unroll
            for (int j = 0; j < F16MMA_UNROLL; ++j) {
                if (s0 + j < nsteps) {
                    const uint4 xf = has_x ? xr[(s0 + j) * 4] : make_uint4(0, 0, 0, 0);
                    const uint32_t a1[4] = {A[j].x, Bv[j].x, A[j].y, Bv[j].y};
                    const uint32_t a2[4] = {A[j].z, Bv[j].z, A[j].w, Bv[j].w};
                    mma_16816(d, a1, xf.x, xf.y);
                    mma_16816(d, a2, xf.z, xf.w);
                }
            }
        }
        const uint32_t row_a = t * 16 + g, row_b = row_a + 8, m0 = 2 * c, m1 = 2 * c + 1;
        if (row_a < N) {
            if (m0 < M) gemv_store<EPI>(y, (uint64_t)m0 * N + row_a, d[0]);
            if (m1 < M) gemv_store<EPI>(y, (uint64_t)m1 * N + row_a, d[1]);
        }
        if (row_b < N) {
            if (m0 < M) gemv_store<EPI>(y, (uint64_t)m0 * N + row_b, d[2]);
            if (m1 < M) gemv_store<EPI>(y, (uint64_t)m1 * N + row_b, d[3]);
        }
    }
}

template <int EPI>
static cudaError_t gemv_f16_dispatch(const void* x, const void* w, void* y, uint32_t M, uint32_t N, uint32_t K,
                                     const void* norm_w, float eps, cudaStream_t s) {
    const size_t smem = (size_t)M * K * sizeof(float);
    unsigned grid = (N + GEMV_WARPS - 1) / GEMV_WARPS;
    if (grid > 148u * 8u) grid = 148u * 8u;   // rows are grid-strided; caps the per-CTA prologue cost
    const __half* xp = static_cast<const __half*>(x);
    const __half* wp = static_cast<const __half*>(w);
    const __half* np = static_cast<const __half*>(norm_w);
    __half* yp = static_cast<__half*>(y);
    if (M >= 2 && K % 32 == 0 && aligned(w, 16) && aligned(x, 16) && (!norm_w || aligned(norm_w, 16))) {
        const size_t smem2 = (size_t)M * (K * 2 + 64);
        auto k = k_gemv_f16_mma<EPI>;
        if (smem2 > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem2);
        int occ = 0;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k, GEMV_THREADS, smem2);
        const unsigned tiles_cta = (N + 16 * GEMV_WARPS - 1) / (16 * GEMV_WARPS);
        const unsigned g2 = std::min<unsigned>(tiles_cta, (unsigned)std::max(occ, 1) * gemv_sm_count());
        k<<<g2, GEMV_THREADS, smem2, s>>>(xp, wp, yp, M, N, K, np, eps);
    } else if (K % 8 == 0 && aligned(w, 16)) {
        auto k = k_gemv_f16<EPI, 8>;
        if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        k<<<grid, GEMV_THREADS, smem, s>>>(xp, wp, yp, M, N, K, np, eps);
    } else if (K % 4 == 0 && aligned(w, 8)) {
        auto k = k_gemv_f16<EPI, 4>;
        if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        k<<<grid, GEMV_THREADS, smem, s>>>(xp, wp, yp, M, N, K, np, eps);
    } else {
        auto k = k_gemv_f16<EPI, 1>;
        if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        k<<<grid, GEMV_THREADS, smem, s>>>(xp, wp, yp, M, N, K, np, eps);
    }
    return cudaGetLastError();
}

cudaError_t launch_gemv_f16(const void* x, const void* w, void* y, uint32_t M, uint32_t N, uint32_t K,
                            const void* norm_w, float eps, int epilogue, cudaStream_t s) {
    if (!M || !N || !K) return cudaSuccess;
    if (M > (uint32_t)GEMV_MMAX || (size_t)M * K * 4 > 200 * 1024) return cudaErrorInvalidValue;
    switch (epilogue) {
        case EPI_STORE: return gemv_f16_dispatch<EPI_STORE>(x, w, y, M, N, K, norm_w, eps, s);
        case EPI_SILU: return gemv_f16_dispatch<EPI_SILU>(x, w, y, M, N, K, norm_w, eps, s);
        case EPI_F32: return gemv_f16_dispatch<EPI_F32>(x, w, y, M, N, K, norm_w, eps, s);
        default: return gemv_f16_dispatch<EPI_RESIDUAL>(x, w, y, M, N, K, norm_w, eps, s);
    }
}

cudaError_t launch_gemv_f16_f32out(const void* x, const void* w, float* y, uint32_t M, uint32_t N, uint32_t K,
                                   cudaStream_t s) {
    return launch_gemv_f16(x, w, y, M, N, K, nullptr, 0.0f, EPI_F32, s);
}

// ---------------------------------------------------------------------------
//  INT4_B32 GEMV on register-operand mma.sync.
//
//  Tile: 16 weight rows per CTA; the CTA's 8 warps split the K/32 blocks.
//  Per block and lane (group g = lane/4, c = lane%4):
//    word  = packed[row0+g][blk*16 + 4c .. +3]   (8 nibbles: k = 32*blk + 8c + 0..7)
//    word8 = same for row0+g+8
//  The eight nibbles become four exact fp16 pairs (n0,n4) (n1,n5) (n2,n6) (n3,n7):
//    lop3 places (nib ^ 8) in the mantissa of 1024.0 (or 16*(nib ^ 8) for the high
//    nibble of each byte), one HSUB2/HFMA2 removes the bias -> q = nib<8 ? nib : nib-16
//    (the reference's two's-complement nibble, linear.metal:57-58), exactly.
//  Two m16n8k16 MMAs consume the block: A rows are weight rows (g, g+8), A columns are
//  a fixed permutation of the block's 32 k, the B operand is the activation vector in
//  the same permutation (batch rows are the 8 MMA columns), D is the block partial in
//  fp32, which is multiplied by the block scale and accumulated.
// ---------------------------------------------------------------------------
// Stage x (M rows, fp16, optionally RMS-normalised with rr) into shared memory in
// MMA-fragment order: for row m, block b, quad c the 8 halves x[32b+8c+{0,4,1,5,2,6,3,7}].
__device__ __forceinline__ void stage_x_frag(const __half* __restrict__ x, const __half* __restrict__ nw,
                                             const float* rr, uint32_t M, uint32_t K, uint4* xs) {
    const uint32_t nq = K / 8;   // quads per row
    for (uint32_t i = threadIdx.x; i < M * nq; i += blockDim.x) {
        const uint32_t m = i / nq, q = i % nq, k0 = q * 8;
        __half v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = __float2half_rn(in_val(x, nw, rr, m, K, k0 + j));
        __half2 o0 = __halves2half2(v[0], v[4]), o1 = __halves2half2(v[1], v[5]);
        __half2 o2 = __halves2half2(v[2], v[6]), o3 = __halves2half2(v[3], v[7]);
        uint4 u;
        u.x = *reinterpret_cast<uint32_t*>(&o0);
        u.y = *reinterpret_cast<uint32_t*>(&o1);
        u.z = *reinterpret_cast<uint32_t*>(&o2);
        u.w = *reinterpret_cast<uint32_t*>(&o3);
        xs[i] = u;
    }
}

constexpr int I4_ROWS = 16;
constexpr int I4_PREFETCH = 8;   // blocks loaded ahead per warp

template <int EPI>
__global__ void __launch_bounds__(GEMV_THREADS) k_gemv_int4_mma(const __half* __restrict__ x,
                                                              const uint8_t* __restrict__ packed,
                                                              const __half* __restrict__ scales,
                                                              __half* __restrict__ y, uint32_t M, uint32_t N,
                                                              uint32_t K, const __half* __restrict__ norm_w,
                                                              float eps) {
    extern __shared__ uint4 xs_frag[];            // M * K/8 fragment quads
    uint4* xs = xs_frag;
    __shared__ float red[32];
    __shared__ float rr[GEMV_MMAX];
    __shared__ float part[GEMV_WARPS][32][4];
    if (norm_w) prenorm_factors(x, M, K, eps, rr, red);
    stage_x_frag(x, norm_w, rr, M, K, xs);
    __syncthreads();

    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t g = lane >> 2, c = lane & 3;
    const uint32_t nb = K / 32;
    const uint32_t row0 = blockIdx.x * I4_ROWS;
    const uint32_t ra = min(row0 + g, N - 1), rb = min(row0 + g + 8, N - 1);
    const uint32_t* pa = reinterpret_cast<const uint32_t*>(packed + (uint64_t)ra * (K / 2)) + c;
    const uint32_t* pb = reinterpret_cast<const uint32_t*>(packed + (uint64_t)rb * (K / 2)) + c;
    const __half* sa = scales + (uint64_t)ra * nb;
    const __half* sb = scales + (uint64_t)rb * nb;
    const uint32_t b_begin = (uint32_t)(((uint64_t)nb * warp) / GEMV_WARPS);
    const uint32_t b_end = (uint32_t)(((uint64_t)nb * (warp + 1)) / GEMV_WARPS);
    const bool has_x = g < M;
    const uint4* xrow = xs + (uint64_t)(has_x ? g : 0) * (K / 8) + c;

    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (uint32_t b0 = b_begin; b0 < b_end; b0 += I4_PREFETCH) {
        uint32_t wa[I4_PREFETCH], wb[I4_PREFETCH];
        __half s_a[I4_PREFETCH], s_b[I4_PREFETCH];
#pragma unroll
        for (int j = 0; j < I4_PREFETCH; ++j) {
            const uint32_t b = b0 + j;
            if (b < b_end) {
                wa[j] = __ldg(pa + b * 4);
                wb[j] = __ldg(pb + b * 4);
                s_a[j] = sa[b];
                s_b[j] = sb[b];
            }
        }
#pragma unroll
        for (int j = 0; j < I4_PREFETCH; ++j) {
            const uint32_t b = b0 + j;
            if (b < b_end) {
                uint4 xf = has_x ? xrow[b * 4] : make_uint4(0, 0, 0, 0);
                uint32_t qa[4], qb[4];
                dequant_word(wa[j], qa);
                dequant_word(wb[j], qb);
                float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                const uint32_t a1[4] = {qa[0], qb[0], qa[1], qb[1]};
                const uint32_t a2[4] = {qa[2], qb[2], qa[3], qb[3]};
                mma_16816(d, a1, xf.x, xf.y);
                mma_16816(d, a2, xf.z, xf.w);
                const float fa = __half2float(s_a[j]), fb = __half2float(s_b[j]);
                acc[0] += d[0] * fa;
                acc[1] += d[1] * fa;
                acc[2] += d[2] * fb;
                acc[3] += d[3] * fb;
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) part[warp][lane][i] = acc[i];
    __syncthreads();
    if (threadIdx.x < 128) {
        const uint32_t l = threadIdx.x >> 2, i = threadIdx.x & 3;
        float t = 0.0f;
#pragma unroll
        for (int w2 = 0; w2 < GEMV_WARPS; ++w2) t += part[w2][l][i];
        const uint32_t row = row0 + (l >> 2) + ((i & 2) ? 8 : 0);
        const uint32_t m = (l & 3) * 2 + (i & 1);
        if (row < N && m < M) gemv_store<EPI>(y, (uint64_t)m * N + row, t);
    }
}

// ---------------------------------------------------------------------------
//  One-row INT4 MMA with one 32-k block per MMA column ("column blocks").
//
//  With a single activation row, 7 of the 8 MMA columns would carry zeros. Instead,
//  in a group of up to 8 consecutive blocks, block j feeds only column j: all lanes
//  load block j's weight words (16 rows x 32 k) as the A fragment, and only the lanes
//  of group g == j supply the activation fragment (the others give zeros), so after
//  the group D[row][j] is block j's dot product. The bias folding of
//  dequant_word_fold starts column j at corr[j] (fold_bias of the block's x), and the
//  per-block scales are applied once per group in the epilogue (lane (g, c) owns
//  columns 2c, 2c + 1): per block 2 shared loads of weight words, one predicated
//  fragment load, 10 dequant ops and 2 MMAs.
//  wa / wb: row g / g + 8 weight word of block b at wa[b * 4]; sa / sb: their scales;
//  xq: the fragment quads of this lane's c (block b at xq[b * 4]); corr[b] biases.
// ---------------------------------------------------------------------------
// One group of blocks gb .. gb + G - 1 (G <= 8); FULL = (G == 8) without predicates.
template <bool FULL>
__device__ __forceinline__ void group_m1(const uint32_t* __restrict__ wa, const uint32_t* __restrict__ wb,
                                         const __half* __restrict__ sa, const __half* __restrict__ sb,
                                         const uint4* __restrict__ xq, const float* __restrict__ corr, uint32_t gb,
                                         uint32_t G, uint32_t g, uint32_t c, float& acc_a, float& acc_b) {
    const uint32_t j0 = 2 * c, j1 = 2 * c + 1;
    uint32_t w0[8], w1[8];
    uint4 xf[8];
#pragma unroll
    for (uint32_t j = 0; j < 8; ++j) {
        if (FULL || j < G) {
            w0[j] = wa[(gb + j) * 4];
            w1[j] = wb[(gb + j) * 4];
            xf[j] = g == j ? xq[(gb + j) * 4] : make_uint4(0, 0, 0, 0);
        }
    }
    const float c0 = (FULL || j0 < G) ? corr[gb + j0] : 0.0f, c1 = (FULL || j1 < G) ? corr[gb + j1] : 0.0f;
    const float s0a = (FULL || j0 < G) ? __half2float(sa[gb + j0]) : 0.0f;
    const float s1a = (FULL || j1 < G) ? __half2float(sa[gb + j1]) : 0.0f;
    const float s0b = (FULL || j0 < G) ? __half2float(sb[gb + j0]) : 0.0f;
    const float s1b = (FULL || j1 < G) ? __half2float(sb[gb + j1]) : 0.0f;
    float d[4] = {c0, c1, c0, c1};
#pragma unroll
    for (uint32_t j = 0; j < 8; ++j) {
        if (FULL || j < G) {
            uint32_t qa[4], qb[4];
            dequant_word_fold(w0[j], qa);
            dequant_word_fold(w1[j], qb);
            const uint32_t a1[4] = {qa[0], qb[0], qa[1], qb[1]};
            const uint32_t a2[4] = {qa[2], qb[2], qa[3], qb[3]};
            mma_16816(d, a1, xf[j].x, xf[j].y);
            mma_16816(d, a2, xf[j].z, xf[j].w);
        }
    }
    acc_a += d[0] * s0a + d[1] * s1a;
    acc_b += d[2] * s0b + d[3] * s1b;
}

__device__ __forceinline__ void consume_m1(const uint32_t* __restrict__ wa, const uint32_t* __restrict__ wb,
                                           const __half* __restrict__ sa, const __half* __restrict__ sb,
                                           const uint4* __restrict__ xq, const float* __restrict__ corr,
                                           uint32_t b_begin, uint32_t b_end, uint32_t g, uint32_t c, float& acc_a,
                                           float& acc_b) {
    uint32_t gb = b_begin;
    for (; gb + 8 <= b_end; gb += 8) group_m1<true>(wa, wb, sa, sb, xq, corr, gb, 8, g, c, acc_a, acc_b);
    if (gb < b_end) group_m1<false>(wa, wb, sa, sb, xq, corr, gb, b_end - gb, g, c, acc_a, acc_b);
}

// ---------------------------------------------------------------------------
//  INT4_B32 GEMV with TMA bulk staging (the decode hot kernel).
//
//  One CTA per 16-row tile. Before anything else one thread issues cp.async.bulk
//  copies of the tile's 16 packed rows (K/2 bytes each, into rows padded by 16 B so
//  the fragment reads below are bank-conflict free) and of the tile's contiguous
//  scale block, all completing on one mbarrier. The whole tile (22.5 KB at K=2560)
//  is in flight from a single instruction stream while the CTA stages (and
//  optionally RMS-normalises) the activation vector; many resident CTAs per SM keep
//  >100 KB per SM in flight, enough to cover HBM latency. The math is the same
//  register-operand mma.sync dequant as k_gemv_int4_mma, reading words from shared
//  memory instead of global.
// ---------------------------------------------------------------------------
template <int EPI>
__global__ void __launch_bounds__(GEMV_THREADS) k_gemv_int4_tma(const __half* __restrict__ x,
                                                              const uint8_t* __restrict__ packed,
                                                              const __half* __restrict__ scales,
                                                              __half* __restrict__ y, uint32_t M, uint32_t N,
                                                              uint32_t K, const __half* __restrict__ norm_w,
                                                              float eps, int* __restrict__ err, bool vec_x) {
    extern __shared__ __align__(128) uint8_t smem_gemv[];
    __shared__ float red[32];
    __shared__ float rr[GEMV_MMAX];
    __shared__ float part[GEMV_WARPS][32][4];
    __shared__ __align__(8) uint64_t bar;
    const uint32_t nb = K / 32;
    const uint32_t row_bytes = K / 2, row_stride = K / 2 + 16;
    uint8_t* sW = smem_gemv;                                   // 16 rows, padded
    __half* sS = reinterpret_cast<__half*>(sW + I4_ROWS * row_stride);   // 16 x nb scales
    uint4* xs = reinterpret_cast<uint4*>(sS + I4_ROWS * nb);             // M x K/8 fragment quads
    float* corr = reinterpret_cast<float*>(xs + (size_t)M * (K / 8));    // one-row path: K/32 biases
    // column blocks pay off from two full 8-block groups per warp (K >= 4096: measured
    // 18.5 -> 14.7 us at 18560 x 4096); at K = 2560 the per-block path is faster
    const bool fold1 = M == 1 && vec_x && K / 32 / GEMV_WARPS >= 16;
    const uint32_t row0 = blockIdx.x * I4_ROWS;
    const uint32_t nrows = min((uint32_t)I4_ROWS, N - row0);
    const uint32_t bar_a = smem_u32(&bar);
    if (threadIdx.x == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar_a));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        const uint32_t total = nrows * row_bytes + nrows * nb * 2;
        asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}" ::"r"(bar_a),
                     "r"(total)
                     : "memory");
        for (uint32_t r = 0; r < nrows; ++r)
            bulk_g2s(smem_u32(sW + r * row_stride), packed + (uint64_t)(row0 + r) * row_bytes, row_bytes, bar_a);
        bulk_g2s(smem_u32(sS), scales + (uint64_t)row0 * nb, nrows * nb * 2, bar_a);
    }
    if (fold1) {
        stage_x_fold(x, norm_w, 1, K, eps, xs, corr, 1, rr, red);
    } else if (vec_x) {
        stage_x_vec(x, norm_w, M, K, eps, true, xs, K / 8, rr, red);
    } else {
        if (norm_w) prenorm_factors(x, M, K, eps, rr, red);
        stage_x_frag(x, norm_w, rr, M, K, xs);
    }
    __syncthreads();
    if (!bar_wait_bounded(bar_a, 0)) {
        if (threadIdx.x == 0) atomicExch(err, 1);
        return;
    }

    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t g = lane >> 2, c = lane & 3;
    const uint32_t ga = min(g, nrows - 1), gb = min(g + 8, nrows - 1);
    const uint32_t* wa_row = reinterpret_cast<const uint32_t*>(sW + ga * row_stride) + c;
    const uint32_t* wb_row = reinterpret_cast<const uint32_t*>(sW + gb * row_stride) + c;
    const __half* sa = sS + ga * nb;
    const __half* sb = sS + gb * nb;
    const uint32_t b_begin = (nb * warp) / GEMV_WARPS, b_end = (nb * (warp + 1)) / GEMV_WARPS;
    if (fold1) {
        float acc_a = 0.0f, acc_b = 0.0f;
        consume_m1(wa_row, wb_row, sa, sb, xs + c, corr, b_begin, b_end, g, c, acc_a, acc_b);
        acc_a += __shfl_xor_sync(0xffffffffu, acc_a, 1);
        acc_a += __shfl_xor_sync(0xffffffffu, acc_a, 2);
        acc_b += __shfl_xor_sync(0xffffffffu, acc_b, 1);
        acc_b += __shfl_xor_sync(0xffffffffu, acc_b, 2);
        if (c == 0) {
            part[warp][g][0] = acc_a;
            part[warp][g][1] = acc_b;
        }
        __syncthreads();
        if (threadIdx.x < 16) {
            const uint32_t r = threadIdx.x & 7, h = threadIdx.x >> 3;
            float t = 0.0f;
#pragma unroll
            for (int w2 = 0; w2 < GEMV_WARPS; ++w2) t += part[w2][r][h];
            const uint32_t row = row0 + r + 8 * h;
            if (row < N) gemv_store<EPI>(y, row, t);
        }
        return;
    }
    const bool has_x = g < M;
    const uint4* xrow = xs + (uint64_t)(has_x ? g : 0) * (K / 8) + c;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 4
    for (uint32_t b = b_begin; b < b_end; ++b) {
        const uint32_t wa = wa_row[b * 4], wb = wb_row[b * 4];
        const uint4 xf = has_x ? xrow[b * 4] : make_uint4(0, 0, 0, 0);
        uint32_t qa[4], qb[4];
        dequant_word(wa, qa);
        dequant_word(wb, qb);
        float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        const uint32_t a1[4] = {qa[0], qb[0], qa[1], qb[1]};
        const uint32_t a2[4] = {qa[2], qb[2], qa[3], qb[3]};
        mma_16816(d, a1, xf.x, xf.y);
        mma_16816(d, a2, xf.z, xf.w);
        const float fa = __half2float(sa[b]), fb = __half2float(sb[b]);
        acc[0] += d[0] * fa;
        acc[1] += d[1] * fa;
        acc[2] += d[2] * fb;
        acc[3] += d[3] * fb;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) part[warp][lane][i] = acc[i];
    __syncthreads();
    if (threadIdx.x < 128) {
        const uint32_t l = threadIdx.x >> 2, i = threadIdx.x & 3;
        float t = 0.0f;
#pragma unroll
        for (int w2 = 0; w2 < GEMV_WARPS; ++w2) t += part[w2][l][i];
        const uint32_t row = row0 + (l >> 2) + ((i & 2) ? 8 : 0);
        const uint32_t m = (l & 3) * 2 + (i & 1);
        if (row < N && m < M) gemv_store<EPI>(y, (uint64_t)m * N + row, t);
    }
}

int* tc_error_word();

// ---------------------------------------------------------------------------
//  Streaming INT4_B32 GEMV (1 CTA per SM; the multi-row decode linears).
//
//  Each CTA stages its (optionally RMS-normalised) input rows once, in the fragment
//  order of k_gemv_int4_tma, then streams its 16-row tiles (tile = blockIdx.x + i *
//  gridDim.x) through a ring of `nst` shared-memory stages. A stage is one K chunk
//  (KC = 256 * segl k) of one 32-row tile, brought by two tensor-map copies issued by
//  warp 15: the packed rows viewed as [K/256 lines][N rows][128 B] (box segl x 32 x
//  128 B, 128-byte swizzle, so smem line = s * 32 + r and the 8 rows an MMA fragment
//  reads fall in 8 different swizzle phases: conflict-free) and the scales viewed the
//  same way as [K/256 lines][N rows][8 scales] (box segl x 32 x 16 B: a row's scales of
//  one line are 16 B from the next row's, so the 8 rows' scale reads hit 8 bank groups).
//  Warps 0..14 split the stage's (16-row sub-tile, 32-k block) items, run the
//  bias-folded dequant (dequant_word_fold) + m16n8k16 MMAs, release the stage (empty
//  barrier, 15 arrivals) and at the end of a tile reduce their partials through a
//  double-buffered shared array (one named barrier per tile). Up to nst stages are in
//  flight per SM.
//  Every wait is bounded (2 s); a timeout raises *err, the consumers stop computing but
//  keep the tile barriers, and the producer waits (bounded) for its own copies before
//  the CTA exits.
// ---------------------------------------------------------------------------
constexpr int ST_MAX = 16;
constexpr int ST_CONS = 15;   // consumer warps; warp 15 issues the copies

__device__ __forceinline__ void st_mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void st_mbar_arrive(uint32_t bar) {
    asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void st_mbar_expect(uint32_t bar, uint32_t bytes) {
    asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}" ::"r"(bar),
                 "r"(bytes)
                 : "memory");
}

constexpr uint32_t ST_ROWS = 32;   // rows per tile (two 16-row MMA sub-tiles)

template <int EPI>
__global__ void __launch_bounds__(512, 1) k_gemv_int4_stream(const __grid_constant__ CUtensorMap wmap,
                                                            const __grid_constant__ CUtensorMap smap,
                                                            const __half* __restrict__ x, __half* __restrict__ y,
                                                            uint32_t M, uint32_t N, uint32_t K,
                                                            const __half* __restrict__ norm_w, float eps,
                                                            uint32_t segl, uint32_t nst, uint32_t stage_bytes,
                                                            int* __restrict__ err) {
    extern __shared__ __align__(128) uint8_t smem_st[];
    __shared__ __align__(8) uint64_t full[ST_MAX], empty[ST_MAX];
    __shared__ float part[2][2][ST_CONS][32][4];   // [tile parity][sub-tile][warp][lane][fragment]
    __shared__ float red[32];
    __shared__ float rr[GEMV_MMAX];
    __shared__ volatile int abort_flag;
    // ring first, 1024-aligned (128-byte swizzle atoms), then the staged x
    uint8_t* ring = smem_st + ((1024u - (smem_u32(smem_st) & 1023u)) & 1023u);
    uint4* xs = reinterpret_cast<uint4*>(ring + (size_t)nst * stage_bytes);
    float* corr = reinterpret_cast<float*>(xs + (size_t)M * (K / 8));   // [K/32][8]
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t ntiles = (N + ST_ROWS - 1) / ST_ROWS, KC = 256 * segl, nchunk = K / KC;
    const uint32_t wbytes = segl * ST_ROWS * 128, sbytes = segl * ST_ROWS * 16;
    const uint32_t my_tiles = blockIdx.x < ntiles ? (ntiles - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
    const uint32_t total = my_tiles * nchunk;
    if (threadIdx.x == 0) {
        for (uint32_t i = 0; i < nst; ++i) {
            st_mbar_init(smem_u32(&full[i]), 1);
            st_mbar_init(smem_u32(&empty[i]), ST_CONS);
        }
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    auto issue = [&](uint32_t q, uint64_t pol) {   // lane 0 of the producer warp: stage q = (tile, chunk)
        const uint32_t slot = q % nst;
        const uint32_t t = blockIdx.x + (q / nchunk) * gridDim.x, ch = q % nchunk;
        const uint32_t fb = smem_u32(&full[slot]);
        const uint32_t st = smem_u32(ring + (size_t)slot * stage_bytes);
        st_mbar_expect(fb, wbytes + sbytes);
        tma3(st, &wmap, 0, (int32_t)(t * ST_ROWS), (int32_t)(ch * segl), fb, pol);
        tma3(st + wbytes, &smap, 0, (int32_t)(t * ST_ROWS), (int32_t)(ch * segl), fb, pol);
    };
    uint32_t issued = 0;
    uint64_t pol = 0;
    if (warp == ST_CONS && lane == 0) {
        pol = evict_first_policy();
        for (; issued < total && issued < nst; ++issued) issue(issued, pol);
    }
    stage_x_fold(x, norm_w, M, K, eps, xs, corr, 8, rr, red);
    __syncthreads();

    if (warp == ST_CONS) {
        if (lane == 0) {
            bool ok = true;
            for (; issued < total && ok; ++issued) {
                const uint32_t slot = issued % nst;
                ok = bar_wait_bounded(smem_u32(&empty[slot]), ((issued / nst) - 1) & 1) && !abort_flag;
                if (ok) issue(issued, pol);
            }
            if (!ok) {
                abort_flag = 1;
                atomicExch(err, 1);
            }
            // the CTA may not exit with copies in flight: wait (bounded) for the last stages
            const uint32_t first = issued > nst ? issued - nst : 0;
            for (uint32_t q = first; q < issued; ++q)
                if (!bar_wait_bounded(smem_u32(&full[q % nst]), (q / nst) & 1)) break;
        }
        return;
    }

    const uint32_t g = lane >> 2, c = lane & 3;
    const uint32_t nbc = KC / 32, items = 2 * nbc;   // (sub-tile, block) pairs per stage
    const bool has_x = g < M;
    const uint4* xrow = xs + (uint64_t)(has_x ? g : 0) * (K / 8) + c;
    const float2* corr2 = reinterpret_cast<const float2*>(corr) + c;   // rows (2c, 2c + 1) of block b at [4b]
    uint32_t q = 0;
    for (uint32_t i = 0; i < my_tiles; ++i) {
        const uint32_t t = blockIdx.x + i * gridDim.x;
        const uint32_t row0 = t * ST_ROWS;
        float acc0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, acc1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (uint32_t ch = 0; ch < nchunk; ++ch, ++q) {
            const uint32_t slot = q % nst;
            bool live = !abort_flag;
            if (live && !bar_wait_bounded(smem_u32(&full[slot]), (q / nst) & 1)) {
                live = false;
                if (lane == 0) {
                    abort_flag = 1;
                    atomicExch(err, 1);
                }
            }
            if (live) {
                const uint8_t* st = ring + (size_t)slot * stage_bytes;
                // (sub-tile s, block b): rows s*16 + g (and + 8) on smem line (b / 8) * 32 + row,
                // 16-byte chunk (b % 8) ^ g; scales at [b / 8][row][b % 8]
                const uint8_t* w_base = st + g * 128 + 4 * c;
                const __half* s_base = reinterpret_cast<const __half*>(st + wbytes) + g * 8;
                const uint32_t gb0 = ch * nbc;
                const uint4* xc = xrow + (uint64_t)gb0 * 4;
                const float2* cc = corr2 + (uint64_t)gb0 * 4;
                // (sub-tile, block) items go round-robin over the consumer warps (balanced per tile)
                const uint32_t ifirst = (warp + ST_CONS - (ch * items) % ST_CONS) % ST_CONS;
#pragma unroll 4
                for (uint32_t it = ifirst; it < items; it += ST_CONS) {
                    const uint32_t sub = it >= nbc, b = it - sub * nbc;
                    const uint32_t line = (b >> 3) * 32 + sub * 16;
                    const uint32_t off = line * 128 + (((b & 7) ^ g) << 4);
                    const uint32_t wa = *reinterpret_cast<const uint32_t*>(w_base + off);
                    const uint32_t wb = *reinterpret_cast<const uint32_t*>(w_base + off + 8 * 128);
                    const uint4 xf = has_x ? xc[b * 4] : make_uint4(0, 0, 0, 0);
                    const float2 cr = cc[b * 4];
                    uint32_t qa[4], qb[4];
                    dequant_word_fold(wa, qa);
                    dequant_word_fold(wb, qb);
                    float d[4] = {cr.x, cr.y, cr.x, cr.y};
                    const uint32_t a1[4] = {qa[0], qb[0], qa[1], qb[1]};
                    const uint32_t a2[4] = {qa[2], qb[2], qa[3], qb[3]};
                    mma_16816(d, a1, xf.x, xf.y);
                    mma_16816(d, a2, xf.z, xf.w);
                    const uint32_t so = line * 8 + (b & 7);
                    const float fa = __half2float(s_base[so]), fb = __half2float(s_base[so + 64]);
                    if (sub) {
                        acc1[0] += d[0] * fa;
                        acc1[1] += d[1] * fa;
                        acc1[2] += d[2] * fb;
                        acc1[3] += d[3] * fb;
                    } else {
                        acc0[0] += d[0] * fa;
                        acc0[1] += d[1] * fa;
                        acc0[2] += d[2] * fb;
                        acc0[3] += d[3] * fb;
                    }
                }
                __syncwarp();
                if (lane == 0) st_mbar_arrive(smem_u32(&empty[slot]));
            }
        }
        const uint32_t pb = i & 1;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            part[pb][0][warp][lane][j] = acc0[j];
            part[pb][1][warp][lane][j] = acc1[j];
        }
        asm volatile("bar.sync 1, %0;" ::"n"(ST_CONS * 32) : "memory");
        if (threadIdx.x < 256 && !abort_flag) {
            const uint32_t sub = threadIdx.x >> 7, l = (threadIdx.x & 127) >> 2, j = threadIdx.x & 3;
            float tsum = 0.0f;
#pragma unroll
            for (int w2 = 0; w2 < ST_CONS; ++w2) tsum += part[pb][sub][w2][l][j];
            const uint32_t row = row0 + sub * 16 + (l >> 2) + ((j & 2) ? 8 : 0);
            const uint32_t m = (l & 3) * 2 + (j & 1);
            if (row < N && m < M) gemv_store<EPI>(y, (uint64_t)m * N + row, tsum);
        }
    }
}

// Tensor maps of one INT4_B32 matrix for k_gemv_int4_stream: packed rows as
// [K/256 lines][N rows][128 B] (box segl x 32 x 128, 128-byte swizzle) and scales as
// [K/256 lines][N rows][8 fp16] (box segl x 32 x 8).
static bool stream_maps(CUtensorMap* wm, CUtensorMap* sm, const void* packed, const void* scales, uint32_t N,
                        uint32_t K, uint32_t segl) {
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    cuuint64_t wd[3] = {128, N, K / 256};
    cuuint64_t ws[2] = {K / 2, 128};
    cuuint32_t wbox[3] = {128, ST_ROWS, segl};
    cuuint32_t one[3] = {1, 1, 1};
    if (enc(wm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(packed), wd, ws, wbox, one,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    cuuint64_t sd[3] = {8, N, K / 256};
    cuuint64_t ss[2] = {K / 32 * 2, 16};
    cuuint32_t sbox[3] = {8, ST_ROWS, segl};
    return enc(sm, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(scales), sd, ss, sbox, one,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int EPI>
static cudaError_t launch_int4_stream(const void* x, const void* packed, const void* scales, void* y, uint32_t M,
                                      uint32_t N, uint32_t K, const void* norm_w, float eps, cudaStream_t s) {
    const uint32_t lines = K / 256;
    uint32_t segl = 8;
    while (lines % segl) --segl;
    const uint32_t stage_bytes = (ST_ROWS * segl * 128 + ST_ROWS * segl * 16 + 1023) & ~1023u;
    const size_t xbytes = (size_t)M * K * 2 + (size_t)K;   // fragments + corr[K/32][8] floats
    const size_t budget = 188 * 1024;   // dynamic; the kernel's static shared memory is about 31 KB
    if (xbytes + 4 * (size_t)stage_bytes > budget) return cudaErrorNotSupported;
    const uint32_t nst = (uint32_t)std::min<size_t>(ST_MAX, (budget - xbytes) / stage_bytes);
    const size_t smem = 1024 + (size_t)nst * stage_bytes + xbytes;
    CUtensorMap wm, sm;
    if (!stream_maps(&wm, &sm, packed, scales, N, K, segl)) return cudaErrorNotSupported;
    auto k = k_gemv_int4_stream<EPI>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    const uint32_t ntiles = (N + ST_ROWS - 1) / ST_ROWS;
    const uint32_t grid = std::min<uint32_t>(ntiles, (uint32_t)gemv_sm_count());
    k<<<grid, (ST_CONS + 1) * 32, smem, s>>>(wm, sm, static_cast<const __half*>(x), static_cast<__half*>(y), M, N, K,
                              static_cast<const __half*>(norm_w), eps, segl, nst, stage_bytes, tc_error_word());
    return cudaGetLastError();
}

// Fallback for layouts the vector kernel cannot address (unaligned packed rows):
// one warp per row, lane = k within a block, like linear.metal:440-474.
template <int EPI>
__global__ void k_gemv_int4_scalar(const __half* __restrict__ x, const uint8_t* __restrict__ packed,
                                   const __half* __restrict__ scales, __half* __restrict__ y, uint32_t M, uint32_t N,
                                   uint32_t K, const __half* __restrict__ norm_w, float eps) {
    __shared__ float red[32];
    __shared__ float rr[GEMV_MMAX];
    if (norm_w) prenorm_factors(x, M, K, eps, rr, red);
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t nb = K / 32;
    for (uint32_t row = blockIdx.x * GEMV_WARPS + warp; row < N; row += gridDim.x * GEMV_WARPS) {
        float acc[GEMV_MMAX];
        for (int m = 0; m < GEMV_MMAX; ++m) acc[m] = 0.0f;
        for (uint32_t b = 0; b < nb; ++b) {
            const uint8_t byte = packed[(uint64_t)row * (K / 2) + b * 16 + (lane >> 1)];
            const uint32_t nib = (lane & 1) ? (byte >> 4) : (byte & 0xF);
            const int q = nib < 8 ? (int)nib : (int)nib - 16;
            const float wv = (float)q * __half2float(scales[(uint64_t)row * nb + b]);
            for (uint32_t m = 0; m < M; ++m) acc[m] += wv * in_val(x, norm_w, rr, m, K, b * 32 + lane);
        }
        for (uint32_t m = 0; m < M; ++m) {
            float t = warp_sum(acc[m]);
            if (lane == 0) gemv_store<EPI>(y, (uint64_t)m * N + row, t);
        }
    }
}

template <int EPI>
static cudaError_t gemv_int4_dispatch(const void* x, const void* packed, const void* scales, void* y, uint32_t M,
                                      uint32_t N, uint32_t K, const void* norm_w, float eps, cudaStream_t s) {
    const __half* xp = static_cast<const __half*>(x);
    const uint8_t* pp = static_cast<const uint8_t*>(packed);
    const __half* sp = static_cast<const __half*>(scales);
    const __half* np = static_cast<const __half*>(norm_w);
    __half* yp = static_cast<__half*>(y);
    const bool vec = aligned(x, 16) && (!norm_w || aligned(norm_w, 16));
    // several rows: the streaming kernel stages x once per SM; one row: the per-tile kernel
    // (column-block MMA) with many CTAs per SM
    if (M >= 2 && vec && aligned(packed, 16) && aligned(scales, 16) && K % 256 == 0 &&
        N >= ST_ROWS * (uint32_t)gemv_sm_count()) {
        const cudaError_t e = launch_int4_stream<EPI>(x, packed, scales, y, M, N, K, norm_w, eps, s);
        if (e != cudaErrorNotSupported) return e;
    }
    if (aligned(packed, 16) && aligned(scales, 16) && K % 256 == 0) {
        const size_t smem =
            (size_t)I4_ROWS * (K / 2 + 16) + (size_t)I4_ROWS * (K / 32) * 2 + (size_t)M * K * 2 + (size_t)K / 8;
        auto k = k_gemv_int4_tma<EPI>;
        if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        const bool vec_x = aligned(x, 16) && (!norm_w || aligned(norm_w, 16));
        k<<<(N + I4_ROWS - 1) / I4_ROWS, GEMV_THREADS, smem, s>>>(xp, pp, sp, yp, M, N, K, np, eps, tc_error_word(),
                                                                 vec_x);
    } else if (aligned(packed, 4) && aligned(scales, 2)) {
        const size_t smem = (size_t)M * K * 2;
        auto k = k_gemv_int4_mma<EPI>;
        if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        k<<<(N + I4_ROWS - 1) / I4_ROWS, GEMV_THREADS, smem, s>>>(xp, pp, sp, yp, M, N, K, np, eps);
    } else {
        k_gemv_int4_scalar<EPI><<<(N + GEMV_WARPS - 1) / GEMV_WARPS, GEMV_THREADS, 0, s>>>(xp, pp, sp, yp, M, N, K,
                                                                                           np, eps);
    }
    return cudaGetLastError();
}

cudaError_t launch_gemv_int4_ex(const void* x, const void* packed, const void* scales, void* y, uint32_t M,
                                uint32_t N, uint32_t K, const void* norm_w, float eps, int epilogue,
                                cudaStream_t s) {
    if (!M || !N || !K) return cudaSuccess;
    if (M > (uint32_t)GEMV_MMAX || K % 32 != 0 || (size_t)M * K * 2 > 200 * 1024) return cudaErrorInvalidValue;
    switch (epilogue) {
        case EPI_STORE: return gemv_int4_dispatch<EPI_STORE>(x, packed, scales, y, M, N, K, norm_w, eps, s);
        case EPI_SILU: return gemv_int4_dispatch<EPI_SILU>(x, packed, scales, y, M, N, K, norm_w, eps, s);
        case EPI_F32: return gemv_int4_dispatch<EPI_F32>(x, packed, scales, y, M, N, K, norm_w, eps, s);
        default: return gemv_int4_dispatch<EPI_RESIDUAL>(x, packed, scales, y, M, N, K, norm_w, eps, s);
    }
}

cudaError_t launch_gemv_int4(const void* x, const void* packed, const void* scales, void* y, uint32_t M, uint32_t N,
                             uint32_t K, cudaStream_t s) {
    return launch_gemv_int4_ex(x, packed, scales, y, M, N, K, nullptr, 0.0f, EPI_STORE, s);
}

// Loads the GEMV kernels and raises their dynamic shared-memory limit to the device's
// opt-in maximum, once per device, from context creation: a kernel first touched under
// stream capture could otherwise fail its attribute call.
void gemv_init() {
    static bool done[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || done[dev]) return;
    done[dev] = true;
    int optin = 0;
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    auto set = [&](const void* f) {
        cudaFuncAttributes a;
        if (cudaFuncGetAttributes(&a, f) == cudaSuccess)
            cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)a.sharedSizeBytes);
    };
    set((const void*)k_gemv_int4_stream<EPI_STORE>);
    set((const void*)k_gemv_int4_stream<EPI_SILU>);
    set((const void*)k_gemv_int4_stream<EPI_RESIDUAL>);
    set((const void*)k_gemv_int4_stream<EPI_F32>);
    set((const void*)k_gemv_int4_tma<EPI_STORE>);
    set((const void*)k_gemv_int4_tma<EPI_SILU>);
    set((const void*)k_gemv_int4_tma<EPI_RESIDUAL>);
    set((const void*)k_gemv_int4_tma<EPI_F32>);
    set((const void*)k_gemv_f16_mma<EPI_STORE>);
    set((const void*)k_gemv_f16_mma<EPI_SILU>);
    set((const void*)k_gemv_f16_mma<EPI_RESIDUAL>);
    set((const void*)k_gemv_f16_mma<EPI_F32>);
    cudaGetLastError();
}

}  // namespace lssm
