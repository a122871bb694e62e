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
#include "device_util.cuh"
#include "lssm_internal.h"
#include "mma_int4.cuh"

namespace lssm {

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
    if (K % 8 == 0 && aligned(w, 16)) {
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
                                                              float eps, int* __restrict__ err) {
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
    if (norm_w) prenorm_factors(x, M, K, eps, rr, red);
    stage_x_frag(x, norm_w, rr, M, K, xs);
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
    if (aligned(packed, 16) && aligned(scales, 16) && K % 256 == 0) {
        const size_t smem = (size_t)I4_ROWS * (K / 2 + 16) + (size_t)I4_ROWS * (K / 32) * 2 + (size_t)M * K * 2;
        auto k = k_gemv_int4_tma<EPI>;
        if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        k<<<(N + I4_ROWS - 1) / I4_ROWS, GEMV_THREADS, smem, s>>>(xp, pp, sp, yp, M, N, K, np, eps, tc_error_word());
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
        default: return gemv_int4_dispatch<EPI_RESIDUAL>(x, packed, scales, y, M, N, K, norm_w, eps, s);
    }
}

cudaError_t launch_gemv_int4(const void* x, const void* packed, const void* scales, void* y, uint32_t M, uint32_t N,
                             uint32_t K, cudaStream_t s) {
    return launch_gemv_int4_ex(x, packed, scales, y, M, N, K, nullptr, 0.0f, EPI_STORE, s);
}

}  // namespace lssm
