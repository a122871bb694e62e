// k_gemm.cu — prefill GEMM on the 5th-generation tensor cores.
//
//   Y[M,N] = X[M,K] . W[N,K]^T   (fp16 operands, fp32 accumulation, fp16 result)
//
// Replaces shaders/linear.metal:253-343 (linear_f16_gemm) and, with the INT4
// weights dequantised to fp16 first (rounded like linear.metal:538),
// linear.metal:492-574 (linear_int4_gemm).
//
// Design (one CTA per SM, persistent over output tiles):
//   warp 0        TMA producer: X and W tiles (128-byte swizzled, K-major) into a
//                 STAGES-deep shared-memory ring, one mbarrier per stage.
//   warp 1        TMEM owner + single-thread tcgen05.mma issuer (M=128, N=BN, K=16
//                 per instruction), tcgen05.commit frees ring stages / publishes a
//                 finished accumulator.
//   warps 2..5    epilogue: tcgen05.ld (32 lanes x 32 columns) -> fp16 -> global.
//   The fp32 accumulator is double buffered in TMEM (two BN-column buffers, each from a
//   32-column boundary; BN % 32 == 16 ends in a 16-column chunk), so the
//   epilogue of tile i overlaps the main loop of tile i+1.
// All waits are bounded (tc_common.cuh); a timeout raises the kernel's error word.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "device_util.cuh"
#include "lssm_internal.h"
#include "mma_int4.cuh"
#include "tc_common.cuh"

namespace lssm {

// ---------------------------------------------------------------------------
//  Tensor-map encoding through the driver entry point (no -lcuda link needed); shared
//  by every kernel file that builds tensor maps.
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 2-D row-major [rows, cols] 16-bit matrix, box = [box_rows, 64 cols], 128-byte swizzle.
bool make_tmap_2d_k64(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t row_stride_elems,
                      uint32_t box_rows, CUtensorMapDataType dt) {
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {row_stride_elems * 2};
    cuuint32_t box[2] = {64, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 64;
constexpr int GEMM_THREADS = 192;

template <int BN>
struct GemmCfg {
    static constexpr int A_BYTES = GEMM_BM * GEMM_BK * 2;
    static constexpr int B_BYTES = BN * GEMM_BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGES = (200 * 1024) / STAGE_BYTES > 6 ? 6 : (200 * 1024) / STAGE_BYTES;
    static constexpr int ACC = (BN + 31) / 32 * 32;   // TMEM columns per accumulator buffer (32-aligned starts)
    static constexpr int TMEM_COLS = (2 * ACC <= 256) ? 256 : 512;
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
};

template <int BN>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, __half* __restrict__ Y,
              uint32_t M, uint32_t N, uint32_t K, uint32_t ldy, int epilogue, int* __restrict__ err) {
    using Cfg = GemmCfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + Cfg::STAGES * Cfg::A_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::STAGES * Cfg::STAGE_BYTES);
    uint64_t* full = bars;
    uint64_t* empty = bars + Cfg::STAGES;
    uint64_t* tfull = bars + 2 * Cfg::STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* done = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t m_tiles = (M + GEMM_BM - 1) / GEMM_BM, n_tiles = (N + BN - 1) / BN;
    const uint32_t ntiles = m_tiles * n_tiles, nk = (K + GEMM_BK - 1) / GEMM_BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < Cfg::STAGES; ++s) {
            tc::mbar_init(smem_u32(&full[s]), 1);
            tc::mbar_init(smem_u32(&empty[s]), 1);
        }
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(smem_u32(&tfull[b]), 1);
            tc::mbar_init(smem_u32(&tempty[b]), 4);
        }
        tc::mbar_init(smem_u32(done), 1);
        *abort_flag = 0;
        tc::fence_barrier_init();
        tc::prefetch_tmap(&tmA);
        tc::prefetch_tmap(&tmB);
    }
    if (warp == 1) tc::tmem_alloc(smem_u32(tmem_slot), Cfg::TMEM_COLS);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            uint32_t stage = 0, phase = 0;
            int last_phase[Cfg::STAGES];
            for (int s = 0; s < Cfg::STAGES; ++s) last_phase[s] = -1;
            for (uint32_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
                const uint32_t mb = tile % m_tiles, nb = tile / m_tiles;
                for (uint32_t kb = 0; kb < nk; ++kb) {
                    if (!tc::mbar_wait(smem_u32(&empty[stage]), phase ^ 1, abort_flag)) goto producer_done;
                    const uint32_t fb = smem_u32(&full[stage]);
                    tc::mbar_arrive_expect_tx(fb, Cfg::STAGE_BYTES);
                    tc::tma_load_2d(smem_u32(sA + stage * Cfg::A_BYTES), &tmA, kb * GEMM_BK, mb * GEMM_BM, fb);
                    tc::tma_load_2d(smem_u32(sB + stage * Cfg::B_BYTES), &tmB, kb * GEMM_BK, nb * BN, fb);
                    last_phase[stage] = (int)phase;
                    if (++stage == (uint32_t)Cfg::STAGES) { stage = 0; phase ^= 1; }
                }
            }
        producer_done:
            // Every issued TMA load must land before the CTA may exit (bounded).
            for (int s = 0; s < Cfg::STAGES; ++s)
                if (last_phase[s] >= 0) tc::mbar_wait_drain(smem_u32(&full[s]), (uint32_t)last_phase[s]);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t IDESC = tc::idesc_f16(GEMM_BM, BN, 0);
            uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
            for (uint32_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
                if (!tc::mbar_wait(smem_u32(&tempty[acc]), acc_phase ^ 1, abort_flag)) break;
                tc::tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * Cfg::ACC;
                bool ok = true;
                for (uint32_t kb = 0; kb < nk; ++kb) {
                    if (!tc::mbar_wait(smem_u32(&full[stage]), phase, abort_flag)) { ok = false; break; }
                    tc::tc_fence_after();
                    const uint64_t da = tc::sw128_kmajor_desc(smem_u32(sA + stage * Cfg::A_BYTES));
                    const uint64_t db = tc::sw128_kmajor_desc(smem_u32(sB + stage * Cfg::B_BYTES));
#pragma unroll
                    for (uint32_t k = 0; k < GEMM_BK / 16; ++k)
                        tc::umma_f16(d_tmem, da + 2 * k, db + 2 * k, IDESC, (kb | k) != 0);
                    tc::umma_commit(smem_u32(&empty[stage]));
                    if (++stage == (uint32_t)Cfg::STAGES) { stage = 0; phase ^= 1; }
                }
                tc::umma_commit(smem_u32(&tfull[acc]));
                if (!ok) break;
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1;
            }
            // All issued MMAs complete before TMEM is released.
            tc::umma_commit(smem_u32(done));
            tc::mbar_wait_drain(smem_u32(done), 0);
        }
    } else {
        // Epilogue warps 2..5 own TMEM lane quarters (warp % 4).
        const uint32_t q = warp & 3;
        uint32_t acc = 0, acc_phase = 0;
        const bool vec = (ldy % 8 == 0) && ((reinterpret_cast<uintptr_t>(Y) & 15) == 0);
        for (uint32_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
            const uint32_t mb = tile % m_tiles, nb = tile / m_tiles;
            if (!tc::mbar_wait(smem_u32(&tfull[acc]), acc_phase, abort_flag)) break;
            tc::tc_fence_after();
            const uint32_t row = mb * GEMM_BM + q * 32 + lane;
            // 32-column chunks; with BN % 32 == 16 the last chunk is 16 columns wide
            constexpr uint32_t NCH = (BN + 31) / 32;
#pragma unroll 1
            for (uint32_t ch = 0; ch < NCH; ++ch) {
                const uint32_t cw = (BN % 32 != 0 && ch == NCH - 1) ? 16u : 32u;
                uint32_t v[32];
                if (cw == 32) tc::tmem_ld32(tmem_base + acc * Cfg::ACC + ch * 32 + ((q * 32) << 16), v);
                else tc::tmem_ld16(tmem_base + acc * Cfg::ACC + ch * 32 + ((q * 32) << 16), *reinterpret_cast<uint32_t(*)[16]>(v));
                tc::tmem_ld_wait();
                const uint32_t col0 = nb * BN + ch * 32;
                const bool full = vec && col0 + cw <= N;
                if (row < M && col0 < N && epilogue == 3) {
                    // fp32 output (partial sums that a collective adds before rounding)
                    float* yf = reinterpret_cast<float*>(Y) + (uint64_t)row * ldy + col0;
                    if (full && (ldy % 4 == 0)) {
                        for (uint32_t j = 0; j < cw / 4; ++j) reinterpret_cast<uint4*>(yf)[j] = reinterpret_cast<uint4*>(v)[j];
                    } else {
                        for (uint32_t j = 0; j < cw && col0 + j < N; ++j) yf[j] = __uint_as_float(v[j]);
                    }
                } else if (row < M && col0 < N) {
                    __half h[32];
                    __half* yr = Y + (uint64_t)row * ldy + col0;
                    if (epilogue == 2) {   // residual: y = half(y + half(acc)) (mamba2_block.cpp:274-276)
                        if (full) {
                            for (uint32_t j = 0; j < cw / 8; ++j) reinterpret_cast<uint4*>(h)[j] = reinterpret_cast<const uint4*>(yr)[j];
                        } else {
                            for (uint32_t j = 0; j < cw && col0 + j < N; ++j) h[j] = yr[j];
                        }
                    }
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        if ((uint32_t)j >= cw) break;
                        float f = __uint_as_float(v[j]);
                        if (epilogue == 1) f = silu(f);
                        if (epilogue == 2) f = __half2float(h[j]) + __half2float(__float2half_rn(f));
                        h[j] = __float2half_rn(f);
                    }
                    if (full) {
                        for (uint32_t j = 0; j < cw / 8; ++j) reinterpret_cast<uint4*>(yr)[j] = reinterpret_cast<uint4*>(h)[j];
                    } else {
                        for (uint32_t j = 0; j < cw && col0 + j < N; ++j) yr[j] = h[j];
                    }
                }
            }
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(smem_u32(&tempty[acc]));
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1;
        }
    }

    __syncthreads();
    if (threadIdx.x == 0 && *abort_flag) atomicExch(err, 1);
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
    }
}

// ---------------------------------------------------------------------------
//  SIMT fallback for operands the TMA path cannot address (K not a multiple of 8,
//  or bases not 16-byte aligned): 64x64 tiles, fp32 accumulation.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_gemm_simt(const __half* __restrict__ X, const __half* __restrict__ W,
                                                   __half* __restrict__ Y, uint32_t M, uint32_t N, uint32_t K,
                                                   int epilogue) {
    __shared__ float As[16][65];
    __shared__ float Bs[16][65];
    const uint32_t tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    const uint32_t m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
    float acc[4][4] = {};
    for (uint32_t k0 = 0; k0 < K; k0 += 16) {
        for (uint32_t i = threadIdx.x; i < 64 * 16; i += 256) {
            const uint32_t r = i / 16, kk = i % 16;
            As[kk][r] = (m0 + r < M && k0 + kk < K) ? __half2float(X[(uint64_t)(m0 + r) * K + k0 + kk]) : 0.0f;
            Bs[kk][r] = (n0 + r < N && k0 + kk < K) ? __half2float(W[(uint64_t)(n0 + r) * K + k0 + kk]) : 0.0f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 16; ++kk)
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] += As[kk][ty * 4 + i] * Bs[kk][tx * 4 + j];
        __syncthreads();
    }
    for (int i = 0; i < 4; ++i)
        for (int j = 0; j < 4; ++j) {
            const uint32_t r = m0 + ty * 4 + i, c = n0 + tx * 4 + j;
            if (r < M && c < N) {
                float f = acc[i][j];
                if (epilogue == 3) { reinterpret_cast<float*>(Y)[(uint64_t)r * N + c] = f; continue; }
                if (epilogue == 1) f = silu(f);
                if (epilogue == 2) f = __half2float(Y[(uint64_t)r * N + c]) + __half2float(__float2half_rn(f));
                Y[(uint64_t)r * N + c] = __float2half_rn(f);
            }
        }
}

// Device-wide error word for the tensor-core kernels' bounded waits.
static int* gemm_err_word() {
    static int* p = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        if (cudaMalloc(&p, sizeof(int)) == cudaSuccess) cudaMemset(p, 0, sizeof(int));
    });
    return p;
}

int* tc_error_word() { return gemm_err_word(); }

template <int BN>
static cudaError_t run_gemm_tc(const void* x, const void* w, void* y, uint32_t M, uint32_t N, uint32_t K,
                               int epilogue, int sms, cudaStream_t s) {
    using Cfg = GemmCfg<BN>;
    CUtensorMap ta, tb;
    if (!make_tmap_2d_k64(&ta, x, M, K, K, GEMM_BM, CU_TENSOR_MAP_DATA_TYPE_FLOAT16) ||
        !make_tmap_2d_k64(&tb, w, N, K, K, BN, CU_TENSOR_MAP_DATA_TYPE_FLOAT16))
        return cudaErrorInvalidValue;
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(k_gemm_tc<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    const uint32_t tiles = ((M + GEMM_BM - 1) / GEMM_BM) * ((N + BN - 1) / BN);
    const uint32_t grid = tiles < (uint32_t)sms ? tiles : (uint32_t)sms;
    k_gemm_tc<BN><<<grid, GEMM_THREADS, Cfg::SMEM, s>>>(ta, tb, static_cast<__half*>(y), M, N, K, N, epilogue,
                                                        gemm_err_word());
    return cudaGetLastError();
}

static int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

// N tile of the fp16 GEMM: the share of SM-slots the persistent waves fill, times a shared-memory
// factor. At M = 128 one K = 16 MMA reads 4 KB of A and 32 * BN bytes of B in ~0.52 * BN cycles, so
// narrow tiles need more operand bytes per cycle than shared memory sustains (~100 of the nominal
// 128 B / cycle): 128 -> 123, 144 -> 116, 160 -> 111, 192 -> 102, 240 -> 94, 256 -> 92 B / cycle.
int gemm_f16_tile_n(uint32_t M, uint32_t N, int sms) {
    const uint32_t mt = (M + GEMM_BM - 1) / GEMM_BM;
    double best = -1.0;
    int best_bn = 256;
    const int cands[6] = {256, 240, 192, 160, 144, 128};
    for (int c : cands) {
        const uint32_t tiles = mt * ((N + c - 1) / c);
        const uint32_t waves = (tiles + sms - 1) / sms;
        const double eff = (double)M * N / ((double)waves * sms * GEMM_BM * c);
        const double bpc = (4096.0 + 32.0 * c) / (0.52 * c);
        const double score = eff * (bpc > 100.0 ? 100.0 / bpc : 1.0);
        if (score > best + 1e-9) { best = score; best_bn = c; }
    }
    return best_bn;
}

cudaError_t launch_gemm_f16(const void* x, const void* w, void* y, uint32_t M, uint32_t N, uint32_t K, int epilogue,
                            cudaStream_t s) {
    if (!M || !N || !K) return cudaSuccess;
    const bool tma_ok = (K % 8 == 0) && aligned(x, 16) && aligned(w, 16);
    if (!tma_ok) {
        dim3 grid((N + 63) / 64, (M + 63) / 64);
        k_gemm_simt<<<grid, 256, 0, s>>>(static_cast<const __half*>(x), static_cast<const __half*>(w),
                                         static_cast<__half*>(y), M, N, K, epilogue);
        return cudaGetLastError();
    }
    const int sms = sm_count();
    const int best_bn = gemm_f16_tile_n(M, N, sms);
    if (best_bn == 256) return run_gemm_tc<256>(x, w, y, M, N, K, epilogue, sms, s);
    if (best_bn == 192) return run_gemm_tc<192>(x, w, y, M, N, K, epilogue, sms, s);
    if (best_bn == 240) return run_gemm_tc<240>(x, w, y, M, N, K, epilogue, sms, s);
    if (best_bn == 160) return run_gemm_tc<160>(x, w, y, M, N, K, epilogue, sms, s);
    if (best_bn == 144) return run_gemm_tc<144>(x, w, y, M, N, K, epilogue, sms, s);
    return run_gemm_tc<128>(x, w, y, M, N, K, epilogue, sms, s);
}

// ---------------------------------------------------------------------------
//  INT4_B32 -> fp16 dequantisation (shaders/linear.metal:38-61, rounded to fp16 like
//  the reference GEMM tile, linear.metal:538: half(float(q) * scale)). One thread per
//  packed 32-bit word (8 weights): a warp reads 128 contiguous bytes and writes 512
//  contiguous bytes (one 16-byte store per thread). The nibbles become exact fp16 q values
//  (dequant_word), and one HMUL2 by the block's scale gives half(q * s) rounded once, the
//  same value as the fp32 product rounded to fp16 (q * s is exact in fp32); a byte permute
//  restores the k order.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_int4_dequant(const uint32_t* __restrict__ packed,
                                                      const __half* __restrict__ scales, uint4* __restrict__ out,
                                                      uint64_t n_words, uint32_t words_per_row) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_words) return;
    const uint64_t row = i / words_per_row, wr = i % words_per_row;
    const uint32_t w = __ldcs(packed + i);   // rows are contiguous: word i of the matrix
    const __half2 s2 = __half2half2(scales[row * (words_per_row / 4) + wr / 4]);
    uint32_t q[4];   // exact fp16 q pairs (k0,k4) (k1,k5) (k2,k6) (k3,k7)
    dequant_word(w, q);
    uint32_t v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const __half2 h = __hmul2(*reinterpret_cast<const __half2*>(&q[e]), s2);
        v[e] = *reinterpret_cast<const uint32_t*>(&h);
    }
    out[i] = make_uint4(__byte_perm(v[0], v[1], 0x5410),    // k0 k1
                        __byte_perm(v[2], v[3], 0x5410),    // k2 k3
                        __byte_perm(v[0], v[1], 0x7632),    // k4 k5
                        __byte_perm(v[2], v[3], 0x7632));   // k6 k7
}

// Any alignment (a packed matrix at an odd offset of a .ssm payload): byte loads.
__global__ void k_int4_dequant_bytes(const uint8_t* __restrict__ packed, const __half* __restrict__ scales,
                                     __half* __restrict__ out, uint32_t N, uint32_t K) {
    const uint32_t nb = K / 32;
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (uint64_t)N * nb) return;
    const uint64_t row = i / nb, b = i % nb;
    const uint8_t* src = packed + row * (K / 2) + b * 16;
    const float s = __half2float(scales[i]);
    __half* dst = out + row * K + b * 32;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const uint8_t byte = src[j];
        const int lo = byte & 0xF, hi = byte >> 4;
        dst[2 * j] = __float2half_rn((float)(lo < 8 ? lo : lo - 16) * s);
        dst[2 * j + 1] = __float2half_rn((float)(hi < 8 ? hi : hi - 16) * s);
    }
}

cudaError_t launch_int4_dequant_f16(const void* packed, const void* scales, void* out, uint32_t N, uint32_t K,
                                    cudaStream_t s) {
    const uint64_t n = (uint64_t)N * (K / 32);
    if (!n) return cudaSuccess;
    // 4-byte loads and 16-byte stores: K % 32 == 0 keeps every word aligned once the bases are
    if ((reinterpret_cast<uintptr_t>(packed) & 3) | (reinterpret_cast<uintptr_t>(out) & 15)) {
        k_int4_dequant_bytes<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(static_cast<const uint8_t*>(packed),
                                                                      static_cast<const __half*>(scales),
                                                                      static_cast<__half*>(out), N, K);
        return cudaGetLastError();
    }
    const uint64_t n_words = (uint64_t)N * (K / 8);
    k_int4_dequant<<<(unsigned)((n_words + 255) / 256), 256, 0, s>>>(static_cast<const uint32_t*>(packed),
                                                                    static_cast<const __half*>(scales),
                                                                    static_cast<uint4*>(out), n_words, K / 8);
    return cudaGetLastError();
}

}  // namespace lssm

// The N tile the fp16 GEMM launcher picks for an M x N output on `sms` SMs (its own function).
extern "C" int lssm_plan_gemm_f16(uint32_t M, uint32_t N, int sms) { return lssm::gemm_f16_tile_n(M, N, sms); }
