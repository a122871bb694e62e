// k_gemm_i4.cu — INT4_B32 GEMM with the dequantisation fused into the tensor-core
// pipeline: Y[M, N] = X[M, K] · dequant(W)[N, K]^T (shaders/linear.metal:492-574).
//
// The reference dequantises a 32x32 weight tile into threadgroup memory, rounding each
// weight to fp16 (half(float(q) * scale), linear.metal:538), then runs an 8x8 simdgroup
// MMA. Here the packed nibbles never exist as an fp16 matrix in HBM:
//   * warp 0 (TMA producer) streams, per 64-wide K block, the activation tile (128 x 64
//     fp16, 128-byte swizzle) and the BN x 32-byte packed INT4 rows of the weight tile;
//   * BN / 32 dequant warps (one weight row per thread) unpack 8 nibbles per 32-bit word
//     (the lop3 magic-number conversion of mma_int4.cuh), restore natural k order with
//     byte permutes, multiply by the block scale in fp16 (the same single rounding as
//     linear.metal:538) and write the fp16 B tile in the 128-byte-swizzled K-major
//     layout the UMMA descriptor expects;
//   * warp 1 issues tcgen05.mma (M 128, N BN, K 16) into a double-buffered TMEM
//     accumulator; warps 2..5 drain TMEM to fp16 (SiLU, residual or fp32 epilogues) in
//     global memory.
// Scales are read by the dequant threads straight from global memory, 8 blocks
// (16 bytes) at a time, two loads ahead. Persistent CTAs walk (m, n, k-split) units:
// with M <= 128 the launcher may split K (on 256-wide scale groups) so the units fill the
// SMs; each split then writes fp32 partials and k_splitk_reduce sums them in split order
// and applies the epilogue.
// Every wait is bounded (2 s) and reports through the shared tensor-core error word.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "device_util.cuh"
#include "lssm_internal.h"
#include "mma_int4.cuh"
#include "tc_common.cuh"

namespace lssm {

bool make_tmap_2d_k64(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t row_stride_elems,
                      uint32_t box_rows, CUtensorMapDataType dt);
int* tc_error_word();

namespace {

constexpr int I4_BM = 128, I4_BK = 64;

template <int BN>
struct I4Cfg {
    static constexpr int A_BYTES = I4_BM * I4_BK * 2;
    static constexpr int B_BYTES = BN * I4_BK * 2;
    static constexpr int Q_BYTES = BN * (I4_BK / 2);
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + Q_BYTES;
    static constexpr int STAGES = (196 * 1024) / STAGE_BYTES > 6 ? 6 : (196 * 1024) / STAGE_BYTES;
    static constexpr int DQ_WARPS = BN / 32;
    static constexpr int THREADS = (6 + DQ_WARPS) * 32;
    static constexpr int TMEM_COLS = 2 * BN <= 128 ? 128 : (2 * BN <= 256 ? 256 : 512);
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
};

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// One packed word (8 consecutive k, low nibble = even k) -> four fp16 pairs in natural
// k order, each weight half(q * s).
__device__ __forceinline__ uint4 dequant_scaled(uint32_t w, __half2 s2) {
    uint32_t q[4];
    dequant_word(w, q);   // (k0,k4) (k1,k5) (k2,k6) (k3,k7)
    uint32_t o[4] = {prmt(q[0], q[1], 0x5410), prmt(q[2], q[3], 0x5410), prmt(q[0], q[1], 0x7632),
                     prmt(q[2], q[3], 0x7632)};
    uint4 r;
    __half2 h;
    h = __hmul2(*reinterpret_cast<__half2*>(&o[0]), s2); r.x = *reinterpret_cast<uint32_t*>(&h);
    h = __hmul2(*reinterpret_cast<__half2*>(&o[1]), s2); r.y = *reinterpret_cast<uint32_t*>(&h);
    h = __hmul2(*reinterpret_cast<__half2*>(&o[2]), s2); r.z = *reinterpret_cast<uint32_t*>(&h);
    h = __hmul2(*reinterpret_cast<__half2*>(&o[3]), s2); r.w = *reinterpret_cast<uint32_t*>(&h);
    return r;
}

// Work unit `tile` of m_tiles x n_tiles x splits: its (m, n) tile and K-block range. K is
// split on 256-wide scale groups (four K blocks), so every split starts on a group.
struct I4Unit {
    uint32_t mb, nb, ks, kb0, kb1;
};
__host__ __device__ __forceinline__ I4Unit i4_unit(uint32_t tile, uint32_t m_tiles, uint32_t n_tiles, uint32_t splits,
                                          uint32_t nk) {
    const uint32_t mn = m_tiles * n_tiles, ks = tile / mn, rem = tile - ks * mn, groups = nk / 4;
    return {rem % m_tiles, rem / m_tiles, ks, 4 * (ks * groups / splits), 4 * ((ks + 1) * groups / splits)};
}

template <int BN>
__global__ void __launch_bounds__(I4Cfg<BN>::THREADS, 1)
    k_gemm_i4(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmQ,
              const __half* __restrict__ scales, __half* __restrict__ Y, uint32_t M, uint32_t N, uint32_t K,
              int epilogue, uint32_t splits, float* __restrict__ ws, int* __restrict__ err) {
    using Cfg = I4Cfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = sA + Cfg::STAGES * Cfg::A_BYTES;
    uint8_t* sQ = sB + Cfg::STAGES * Cfg::B_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sQ + Cfg::STAGES * Cfg::Q_BYTES);
    uint64_t* full = bars;                       // A + packed W landed (TMA)
    uint64_t* bready = full + Cfg::STAGES;       // fp16 W tile written (dequant warps)
    uint64_t* empty = bready + Cfg::STAGES;      // MMAs of the stage done
    uint64_t* tfull = empty + Cfg::STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* done = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t m_tiles = (M + I4_BM - 1) / I4_BM, n_tiles = (N + BN - 1) / BN;
    const uint32_t ntiles = m_tiles * n_tiles * splits, nk = K / I4_BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < Cfg::STAGES; ++s) {
            tc::mbar_init(smem_u32(&full[s]), 1);
            tc::mbar_init(smem_u32(&bready[s]), Cfg::DQ_WARPS);
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
        tc::prefetch_tmap(&tmQ);
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
                const I4Unit u = i4_unit(tile, m_tiles, n_tiles, splits, nk);
                const uint32_t mb = u.mb, nb = u.nb;
                for (uint32_t kb = u.kb0; kb < u.kb1; ++kb) {
                    if (!tc::mbar_wait(smem_u32(&empty[stage]), phase ^ 1, abort_flag)) goto producer_done;
                    const uint32_t fb = smem_u32(&full[stage]);
                    tc::mbar_arrive_expect_tx(fb, Cfg::A_BYTES + Cfg::Q_BYTES);
                    tc::tma_load_2d(smem_u32(sA + stage * Cfg::A_BYTES), &tmA, kb * I4_BK, mb * I4_BM, fb);
                    tc::tma_load_2d(smem_u32(sQ + stage * Cfg::Q_BYTES), &tmQ, kb * (I4_BK / 2), nb * BN, fb);
                    last_phase[stage] = (int)phase;
                    if (++stage == (uint32_t)Cfg::STAGES) { stage = 0; phase ^= 1; }
                }
            }
        producer_done:
            for (int s = 0; s < Cfg::STAGES; ++s)
                if (last_phase[s] >= 0) tc::mbar_wait_drain(smem_u32(&full[s]), (uint32_t)last_phase[s]);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t IDESC = tc::idesc_f16(I4_BM, BN, 0);
            uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
            for (uint32_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
                if (!tc::mbar_wait(smem_u32(&tempty[acc]), acc_phase ^ 1, abort_flag)) break;
                tc::tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                const I4Unit u = i4_unit(tile, m_tiles, n_tiles, splits, nk);
                bool ok = true;
                for (uint32_t kb = u.kb0; kb < u.kb1; ++kb) {
                    if (!tc::mbar_wait(smem_u32(&full[stage]), phase, abort_flag) ||
                        !tc::mbar_wait(smem_u32(&bready[stage]), phase, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc::tc_fence_after();
                    const uint64_t da = tc::sw128_kmajor_desc(smem_u32(sA + stage * Cfg::A_BYTES));
                    const uint64_t db = tc::sw128_kmajor_desc(smem_u32(sB + stage * Cfg::B_BYTES));
#pragma unroll
                    for (uint32_t k = 0; k < I4_BK / 16; ++k)
                        tc::umma_f16(d_tmem, da + 2 * k, db + 2 * k, IDESC, (kb != u.kb0) || k != 0);
                    tc::umma_commit(smem_u32(&empty[stage]));
                    if (++stage == (uint32_t)Cfg::STAGES) { stage = 0; phase ^= 1; }
                }
                tc::umma_commit(smem_u32(&tfull[acc]));
                if (!ok) break;
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1;
            }
            tc::umma_commit(smem_u32(done));
            tc::mbar_wait_drain(smem_u32(done), 0);
        }
    } else if (warp < 6) {
        // Epilogue warps 2..5 own TMEM lane quarters (warp % 4).
        const uint32_t q = warp & 3;
        uint32_t acc = 0, acc_phase = 0;
        const bool vec = (N % 8 == 0) && ((reinterpret_cast<uintptr_t>(Y) & 15) == 0);
        // split K: fp32 partials of split ks to ws[ks][M][N] (16-byte aligned), summed afterwards
        const bool part = splits > 1;
        const bool vecf = (N % 4 == 0) && ((reinterpret_cast<uintptr_t>(part ? (void*)ws : (void*)Y) & 15) == 0);
        for (uint32_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
            const I4Unit u = i4_unit(tile, m_tiles, n_tiles, splits, nk);
            const uint32_t mb = u.mb, nb = u.nb;
            if (!tc::mbar_wait(smem_u32(&tfull[acc]), acc_phase, abort_flag)) break;
            tc::tc_fence_after();
            const uint32_t row = mb * I4_BM + q * 32 + lane;
#pragma unroll 1
            for (uint32_t ch = 0; ch < (uint32_t)BN / 32; ++ch) {
                uint32_t v[32];
                tc::tmem_ld32(tmem_base + acc * BN + ch * 32 + ((q * 32) << 16), v);
                tc::tmem_ld_wait();
                const uint32_t col0 = nb * BN + ch * 32;
                if (row < M && col0 < N && (epilogue == 3 || part)) {
                    // fp32 output (partial sums that a collective, or the split-K sum, adds before rounding)
                    float* yf = (part ? ws + (uint64_t)u.ks * M * N : reinterpret_cast<float*>(Y)) + (uint64_t)row * N + col0;
                    if (vecf && col0 + 32 <= N) {
#pragma unroll
                        for (int j = 0; j < 8; ++j) reinterpret_cast<uint4*>(yf)[j] = reinterpret_cast<uint4*>(v)[j];
                    } else {
                        for (uint32_t j = 0; j < 32 && col0 + j < N; ++j) yf[j] = __uint_as_float(v[j]);
                    }
                } else if (row < M && col0 < N) {
                    __half h[32];
                    __half* yr = Y + (uint64_t)row * N + col0;
                    if (epilogue == 2) {   // residual: y = half(y + half(acc)) (mamba2_block.cpp:274-276)
                        if (vec && col0 + 32 <= N) {
#pragma unroll
                            for (int j = 0; j < 4; ++j) reinterpret_cast<uint4*>(h)[j] = reinterpret_cast<const uint4*>(yr)[j];
                        } else {
                            for (uint32_t j = 0; j < 32 && col0 + j < N; ++j) h[j] = yr[j];
                        }
                    }
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        float f = __uint_as_float(v[j]);
                        if (epilogue == 1) f = silu(f);
                        if (epilogue == 2) f = __half2float(h[j]) + __half2float(__float2half_rn(f));
                        h[j] = __float2half_rn(f);
                    }
                    if (vec && col0 + 32 <= N) {
#pragma unroll
                        for (int j = 0; j < 4; ++j) reinterpret_cast<uint4*>(yr)[j] = reinterpret_cast<uint4*>(h)[j];
                    } else {
                        for (uint32_t j = 0; j < 32 && col0 + j < N; ++j) yr[j] = h[j];
                    }
                }
            }
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(smem_u32(&tempty[acc]));
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1;
        }
    } else {
        // Dequant warps: thread r owns weight row r of every tile.
        const uint32_t r = (warp - 6) * 32 + lane;
        const uint32_t sw = r & 7;
        uint32_t stage = 0, phase = 0;
        const uint32_t nsc = K / 256;   // 16-byte scale groups (8 blocks) per row
        for (uint32_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
            const I4Unit u = i4_unit(tile, m_tiles, n_tiles, splits, nk);
            const uint32_t nb = u.nb, n = nb * BN + r;
            const bool valid = n < N;
            const uint4* srow = reinterpret_cast<const uint4*>(scales + (uint64_t)(valid ? n : 0) * (K / 32));
            const uint4 zero4 = make_uint4(0, 0, 0, 0);
            const uint32_t g0 = u.kb0 >> 2;
            uint4 cur = valid ? __ldg(srow + g0) : zero4;
            uint4 nxt = (valid && g0 + 1 < nsc) ? __ldg(srow + g0 + 1) : zero4;
            bool ok = true;
            for (uint32_t kb = u.kb0; kb < u.kb1; ++kb) {
                if ((kb & 3) == 0 && kb != u.kb0) {
                    cur = nxt;
                    const uint32_t g = (kb >> 2) + 1;
                    nxt = (valid && g < nsc) ? __ldg(srow + g) : zero4;
                }
                if (!tc::mbar_wait(smem_u32(&full[stage]), phase, abort_flag)) { ok = false; break; }
                // scales of blocks 2kb, 2kb+1: halves (kb & 3) * 2, +1 of cur
                const uint32_t sel = (kb & 3) == 0 ? cur.x : (kb & 3) == 1 ? cur.y : (kb & 3) == 2 ? cur.z : cur.w;
                const __half2 sp = *reinterpret_cast<const __half2*>(&sel);
                const __half2 s0 = __half2half2(__low2half(sp)), s1 = __half2half2(__high2half(sp));
                const uint4* qrow = reinterpret_cast<const uint4*>(sQ + stage * Cfg::Q_BYTES + r * 32);
                const uint4 w0 = qrow[0], w1 = qrow[1];
                uint8_t* brow = sB + stage * Cfg::B_BYTES + r * 128;
                const uint32_t wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                for (uint32_t j = 0; j < 8; ++j)
                    *reinterpret_cast<uint4*>(brow + ((j ^ sw) << 4)) = dequant_scaled(wv[j], j < 4 ? s0 : s1);
                tc::fence_proxy_async_shared();   // generic-proxy writes -> tcgen05 reads
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(smem_u32(&bready[stage]));
                if (++stage == (uint32_t)Cfg::STAGES) { stage = 0; phase ^= 1; }
            }
            if (!ok) break;
        }
    }

    __syncthreads();
    if (threadIdx.x == 0 && *abort_flag) atomicExch(err, 1);
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
    }
}

// [N rows][K/2 bytes] packed nibbles; box = BN rows x 32 bytes (one 64-wide K block).
bool make_tmap_q(CUtensorMap* map, const void* base, uint32_t N, uint32_t K, uint32_t BN) {
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    cuuint64_t dims[2] = {K / 2, N};
    cuuint64_t strides[1] = {K / 2};
    cuuint32_t box[2] = {I4_BK / 2, BN};
    cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// y = epilogue(sum over the splits of the fp32 partials ws[split][M][N]), four columns per
// thread, splits added in order: the same epilogues as the GEMM's own (0 fp16, 1 SiLU,
// 2 residual y = half(y + half(acc)), 3 fp32).
__global__ void k_splitk_reduce(const float* __restrict__ ws, uint32_t splits, uint64_t mn, void* __restrict__ Y,
                                int epilogue) {
    const uint64_t i = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (i >= mn) return;
    float a[4] = {0.f, 0.f, 0.f, 0.f};
    const uint32_t nv = mn - i < 4 ? (uint32_t)(mn - i) : 4;
    if (nv == 4 && (mn & 3) == 0) {
        for (uint32_t k = 0; k < splits; ++k) {
            const float4 p = *reinterpret_cast<const float4*>(ws + k * mn + i);
            a[0] += p.x; a[1] += p.y; a[2] += p.z; a[3] += p.w;
        }
    } else {
        for (uint32_t k = 0; k < splits; ++k)
            for (uint32_t j = 0; j < nv; ++j) a[j] += ws[k * mn + i + j];
    }
    if (epilogue == 3) {
        for (uint32_t j = 0; j < nv; ++j) static_cast<float*>(Y)[i + j] = a[j];
        return;
    }
    __half* y = static_cast<__half*>(Y) + i;
    for (uint32_t j = 0; j < nv; ++j) {
        float f = a[j];
        if (epilogue == 1) f = silu(f);
        if (epilogue == 2) f = __half2float(y[j]) + __half2float(__float2half_rn(f));
        y[j] = __float2half_rn(f);
    }
}

template <int BN>
cudaError_t run_gemm_i4(const void* x, const void* packed, const void* scales, void* y, uint32_t M, uint32_t N,
                        uint32_t K, int epilogue, int sms, cudaStream_t s, uint32_t splits = 1, float* ws = nullptr) {
    using Cfg = I4Cfg<BN>;
    CUtensorMap ta, tq;
    if (!make_tmap_2d_k64(&ta, x, M, K, K, I4_BM, CU_TENSOR_MAP_DATA_TYPE_FLOAT16) ||
        !make_tmap_q(&tq, packed, N, K, BN))
        return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(k_gemm_i4<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
    if (e != cudaSuccess) return e;
    const uint32_t tiles = ((M + I4_BM - 1) / I4_BM) * ((N + BN - 1) / BN) * splits;
    const uint32_t grid = tiles < (uint32_t)sms ? tiles : (uint32_t)sms;
    k_gemm_i4<BN><<<grid, Cfg::THREADS, Cfg::SMEM, s>>>(ta, tq, static_cast<const __half*>(scales),
                                                         static_cast<__half*>(y), M, N, K, epilogue, splits, ws,
                                                         tc_error_word());
    if (splits > 1) {
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        const uint64_t mn = (uint64_t)M * N;
        const uint64_t threads = (mn + 3) / 4;
        k_splitk_reduce<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(ws, splits, mn, y, epilogue);
    }
    return cudaGetLastError();
}

// Launch plan of the fused INT4 GEMM (host only): the N tile (0 = not taken: the caller
// dequantises, then runs the fp16 GEMM) and the number of K splits.
struct GemmI4Plan {
    int bn;
    uint32_t splits;
};

GemmI4Plan plan_gemm_i4(uint32_t M, uint32_t N, uint32_t K, int sms, size_t ws_bytes) {
    if (!M || !N || !K || K % 256 || M > 512 || sms < 1) return {0, 1};
    const uint32_t mt = (M + I4_BM - 1) / I4_BM;
    const int cands[3] = {256, 128, 64};
    if (M <= 128 && ws_bytes) {
        // Decode-size M has few (m, n) tiles, and each walks all of K at ~0.4-0.75 us per
        // 64-wide K block (the 3-, 5- and 6-stage rings of BN 256 / 128 / 64): split K over
        // 256-wide groups so the tiles x splits fill the SMs, fp32 partials in ws, then one
        // summing pass (~2 us).
        const uint32_t groups = K / 256;
        double best = 1e30;
        int best_bn = 128;
        uint32_t best_s = 1;
        for (int c : cands) {
            const uint32_t base = mt * ((N + c - 1) / c);
            uint32_t sp = base >= (uint32_t)sms ? 1 : (uint32_t)sms / base;
            if (sp > groups) sp = groups;
            if (sp > 8) sp = 8;
            while (sp > 1 && (size_t)sp * M * N * 4 > ws_bytes) --sp;
            const uint32_t waves = (base * sp + sms - 1) / sms;
            const double tblk = c >= 256 ? 0.75 : (c >= 128 ? 0.45 : 0.4);
            const double cost = waves * ((groups + sp - 1) / sp) * 4 * tblk + (sp > 1 ? 2.0 : 0.0);
            if (cost < best - 1e-9) { best = cost; best_bn = c; best_s = sp; }
        }
        if (best_s > 1) return {best_bn, best_s};
    }
    // Each M tile re-dequantises its weights: beyond a few M tiles, dequantising once and
    // running the fp16 GEMM is cheaper (2048 x 10576 x 2560: 148 vs 166 us); and with too
    // few N tiles to fill half the SMs the per-tile K loop is exposed. Both go to the caller's
    // dequantise-then-GEMM path.
    if ((N + 63) / 64 < (uint32_t)sms / 2) return {0, 1};
    // N tile with the fewest idle SM-slots over the persistent waves (small M: more tiles)
    double best = -1.0;
    int best_bn = 128;
    for (int c : cands) {
        const uint32_t tiles = mt * ((N + c - 1) / c);
        const uint32_t waves = (tiles + sms - 1) / sms;
        const double eff = (double)M * N / ((double)waves * sms * I4_BM * c);
        if (eff > best + 1e-9) { best = eff; best_bn = c; }
    }
    return {best_bn, 1};
}

}  // namespace

// Fused INT4 GEMM for the small-M (batched decode) shapes where it beats dequantising
// once: returns cudaErrorNotSupported otherwise, or when the operands do not fit the TMA
// path (K % 256, 16-byte alignment of x / packed / scales); the caller then falls back
// to dequantise-then-GEMM. `ws` (`ws_bytes`, 16-byte aligned, may be null) lets M <= 128
// split K over CTAs; `launches` (may be null) receives the number of kernels launched.
cudaError_t launch_gemm_i4(const void* x, const void* packed, const void* scales, void* y, uint32_t M, uint32_t N,
                           uint32_t K, int epilogue, cudaStream_t s, float* ws, size_t ws_bytes, int* launches) {
    if (launches) *launches = 0;
    if (!M || !N || !K) return cudaSuccess;
    if (K % 256 || !aligned(x, 16) || !aligned(packed, 16) || !aligned(scales, 16)) return cudaErrorNotSupported;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const GemmI4Plan p = plan_gemm_i4(M, N, K, sms, (ws && aligned(ws, 16)) ? ws_bytes : 0);
    if (!p.bn) return cudaErrorNotSupported;
    float* const w = p.splits > 1 ? ws : nullptr;
    if (launches) *launches = p.splits > 1 ? 2 : 1;
    if (p.bn == 256) return run_gemm_i4<256>(x, packed, scales, y, M, N, K, epilogue, sms, s, p.splits, w);
    if (p.bn == 128) return run_gemm_i4<128>(x, packed, scales, y, M, N, K, epilogue, sms, s, p.splits, w);
    return run_gemm_i4<64>(x, packed, scales, y, M, N, K, epilogue, sms, s, p.splits, w);
}

}  // namespace lssm

extern "C" int lssm_plan_int4_gemm(uint32_t M, uint32_t N, uint32_t K, int sms, size_t ws_bytes, uint32_t* bn,
                                   uint32_t* splits) {
    const lssm::GemmI4Plan p = lssm::plan_gemm_i4(M, N, K, sms, ws_bytes);
    if (bn) *bn = (uint32_t)p.bn;
    if (splits) *splits = p.splits;
    return p.bn ? 1 : 0;
}

// The work unit the kernel assigns to CTA-tile `tile` (same function the device code calls):
// out = {m tile, n tile, split, first K block, end K block}.
extern "C" void lssm_int4_gemm_unit(uint32_t tile, uint32_t m_tiles, uint32_t n_tiles, uint32_t splits, uint32_t nk,
                                    uint32_t* out) {
    const lssm::I4Unit u = lssm::i4_unit(tile, m_tiles, n_tiles, splits, nk);
    out[0] = u.mb; out[1] = u.nb; out[2] = u.ks; out[3] = u.kb0; out[4] = u.kb1;
}
