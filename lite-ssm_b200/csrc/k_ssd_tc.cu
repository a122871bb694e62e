// k_ssd_tc.cu — SSD chunked scan on the 5th-generation tensor cores
// (shaders/ssd_chunked.metal:82-297 restated for P = 64, N = 128).
//
// One CTA (512 threads: four warps per TMEM lane quarter, splitting the columns) per
// (sequence b, head h) walks the sequence in chunks of
// Q = 128 tokens. The fp32 state S (N x P) lives in TMEM for the whole walk. Per chunk:
//   inputs   X_c (Q x P), B_c, C_c (Q x N) arrive by TMA (128-byte swizzled,
//            double buffered: chunk c+1 loads while chunk c computes);
//   scan     dt -> softplus + clamp, Lc = inclusive cumsum of A dt (one warp);
//   MMA 1    CB = C_c B_c^T                         (128x128x128, TMEM)
//   threads  M[t,j] = CB[t,j] exp(Lc_t - Lc_j) dt_j for j <= t, else 0 -> smem (K-major),
//            as CB * 2^(Lc_t log2 e - q_j) with q_j = Lc_j log2 e - log2 dt_j per column;
//            B~_j = exp(Lc_end - Lc_j) dt_j B_j (in place),
//            S_old -> 16-bit smem operand, S <- exp(Lc_end) S in TMEM
//   MMA 2    Y  = M X                               (128x64, K = 128)
//            CS = C S_old                           (128x64, K = 128)
//            S += B~^T X                            (128x64, K = 128)
//   epilogue y_t = Y_t + exp(Lc_t) CS_t + D x_t -> global (f16 / bf16 / f32).
// Pipelining: Y is double-buffered in TMEM and the per-chunk scalars (DT, Lc, W, EL) in
// shared memory, so while the tensor cores run chunk c's MMA 2, the threads write chunk
// c - 1's epilogue and warp 0 scans chunk c + 1's dt.
// Math: the same recurrence as the reference (exp of segment sums, softplus-inside,
// dt clamp); only the order of accumulation differs. M, C' and S_old are rounded to the
// input dtype as MMA operands (the reference stores M and S as fp16, ssd_chunked.metal:116/121).
#include <cuda.h>
#include <cudaTypedefs.h>

#include "device_util.cuh"
#include "lssm_internal.h"
#include "tc_common.cuh"

namespace lssm {

namespace {

constexpr int TQ = 128, TP = 64, TN = 128;
constexpr int THREADS = 512;   // 4 warps per TMEM lane quarter, each a quarter of the columns
// shared-memory map (offsets from a 1024-byte aligned base)
constexpr uint32_t X_BYTES = TQ * TP * 2;          // 16 KB
constexpr uint32_t BC_BYTES = TQ * TN * 2;         // 32 KB (two 64-column panels of 16 KB)
constexpr uint32_t PANEL = TQ * 128;               // 16 KB: 128 rows x 128 B
constexpr uint32_t OFF_X = 0;
constexpr uint32_t OFF_C = OFF_X + 2 * X_BYTES;
constexpr uint32_t OFF_B = OFF_C + 2 * BC_BYTES;
constexpr uint32_t OFF_M = OFF_B + 2 * BC_BYTES;
constexpr uint32_t OFF_S = OFF_M + BC_BYTES;
constexpr uint32_t OFF_F = OFF_S + TN * TP * 2;     // 2 chunks x {DT, Lc, W, EL} (128 floats each)
constexpr uint32_t OFF_BAR = OFF_F + 8 * TQ * 4;
constexpr uint32_t SMEM_TOTAL = OFF_BAR + 64 + 1024;
constexpr uint32_t STAGE_TX = X_BYTES + 2 * BC_BYTES;
// TMEM columns: CB, two Y = M X buffers and two CS = C S_old buffers (chunk parity), S
constexpr uint32_t T_CB = 0, T_Y = 128, T_CS = 256, T_S = 384, TMEM_COLS = 512;

struct TcArgs {
    const void* dt_raw; const void* dt_bias; const void* A_log; const void* D;
    void* Y; float* state;
    const __half* z; uint64_t z_rs;   // optional gate: Y = half(silu(z) * half(y))
    uint32_t batch, L, H, P, N, G;
    float dt_min, dt_max;
    uint32_t has_D;
    uint32_t dt_dtype, param_dtype, y_dtype;
    uint64_t dt_rs, y_rs;
    int* err;
};

// 16-B chunk address of element (row, col) in a 128-byte-swizzled tile of 64-col panels.
__device__ __forceinline__ uint32_t sw_off(uint32_t row, uint32_t col) {
    const uint32_t panel = col >> 6, c = col & 63;
    return panel * PANEL + row * 128 + ((((c >> 3) ^ (row & 7)) & 7) << 4) + (c & 7) * 2;
}

constexpr float LOG2E = 1.4426950408889634f;

// 2^x with the PTX ex2.approx instruction (the same approximation __expf rests on).
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
    if (BF16) {
        __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&v);
    }
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
}

template <bool BF16>
__device__ __forceinline__ float2 unpack2(uint32_t u) {
    if (BF16) return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&u));
    return __half22float2(*reinterpret_cast<__half2*>(&u));
}

// Scale the 32-element quarter `hq` (half a panel) of a row of a swizzled tile in place.
template <bool BF16>
__device__ __forceinline__ void scale_quarter_row(uint8_t* tile, uint32_t row, uint32_t hq, float s) {
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {
        const uint32_t c8 = ((hq & 1) * 4 + (uint32_t)ch) ^ (row & 7);
        uint4* p = reinterpret_cast<uint4*>(tile + (hq >> 1) * PANEL + row * 128 + c8 * 16);
        uint4 u = *p;
        uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float2 f = unpack2<BF16>(w[i]);
            w[i] = pack2<BF16>(f.x * s, f.y * s);
        }
        *p = u;
    }
}

template <bool BF16>
__global__ void __launch_bounds__(THREADS, 1)
    k_ssd_chunked_tc(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, TcArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);   // full[0], full[1], cb, y
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t q4 = warp & 3, hc = warp >> 2;          // TMEM lane quarter, column half
    const uint32_t t = q4 * 32 + lane;                      // chunk row / TMEM lane owned
    const uint32_t b = blockIdx.x / a.H, h = blockIdx.x % a.H;
    const uint32_t g = h / max(1u, a.H / a.G);
    const uint32_t nc = (a.L + TQ - 1) / TQ;
    const float A = -expf(load_any(a.A_log, h, a.param_dtype));
    const float dbias = load_any(a.dt_bias, h, a.param_dtype);
    const float Dh = a.has_D ? load_any(a.D, h, a.param_dtype) : 0.0f;
    float* Sg = a.state + ((uint64_t)b * a.H + h) * TP * TN;
    constexpr uint32_t ID_CB = tc::idesc_f16_major(128, 128, BF16 ? 1 : 0, 0, 0);
    constexpr uint32_t ID_Y = tc::idesc_f16_major(128, 64, BF16 ? 1 : 0, 0, 1);
    constexpr uint32_t ID_DS = tc::idesc_f16_major(128, 64, BF16 ? 1 : 0, 1, 1);
    const uint32_t bar_cb = smem_u32(&bars[2]), bar_y = smem_u32(&bars[3]);

    if (tid == 0) {
        for (int i = 0; i < 4; ++i) tc::mbar_init(smem_u32(&bars[i]), 1);
        *abort_flag = 0;
        tc::fence_barrier_init();
        tc::prefetch_tmap(&tmX);
        tc::prefetch_tmap(&tmB);
        tc::prefetch_tmap(&tmC);
    }
    if (warp == 0) tc::tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_base = (q4 * 32) << 16;

    auto issue_chunk = [&](uint32_t c) {
        const uint32_t buf = c & 1, fb = smem_u32(&bars[buf]);
        const int32_t t0 = (int32_t)(c * TQ);
        tc::mbar_arrive_expect_tx(fb, STAGE_TX);
        tc::tma_load_3d(smem_u32(sm + OFF_X + buf * X_BYTES), &tmX, (int32_t)(h * TP), t0, (int32_t)b, fb);
        for (int pnl = 0; pnl < 2; ++pnl) {
            tc::tma_load_3d(smem_u32(sm + OFF_C + buf * BC_BYTES + pnl * PANEL), &tmC, (int32_t)(g * TN + pnl * 64), t0,
                            (int32_t)b, fb);
            tc::tma_load_3d(smem_u32(sm + OFF_B + buf * BC_BYTES + pnl * PANEL), &tmB, (int32_t)(g * TN + pnl * 64), t0,
                            (int32_t)b, fb);
        }
    };
    auto issue_cb = [&](uint32_t c) {   // CB = C B^T for chunk c (its tiles must have landed)
        const uint32_t buf = c & 1;
        const uint32_t sCa = smem_u32(sm + OFF_C + buf * BC_BYTES), sBa = smem_u32(sm + OFF_B + buf * BC_BYTES);
        tc::tc_fence_after();
#pragma unroll
        for (uint32_t k = 0; k < 8; ++k) {
            const uint32_t koff = (k >> 2) * PANEL + (k & 3) * 32;
            tc::umma_f16(tmem + T_CB, tc::sw128_desc(sCa + koff, 16, 1024), tc::sw128_desc(sBa + koff, 16, 1024), ID_CB,
                         k > 0);
        }
        tc::umma_commit(bar_cb);
    };

    uint32_t last_issued = 0;   // thread 0: newest chunk whose TMA was issued
    bool ok = true;
    if (tid == 0) {
        issue_chunk(0);
        if (nc > 1) { issue_chunk(1); last_issued = 1; }
        if (tc::mbar_wait(smem_u32(&bars[0]), 0, abort_flag)) issue_cb(0);
    }
    // initial state S[p][n] -> TMEM lane n, columns T_S + p (this thread: p in [hc*32, hc*32+32))
    {
        uint32_t v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = __float_as_uint(Sg[(uint64_t)(hc * 16 + j) * TN + t]);
        tc::tmem_st16(tmem + lane_base + T_S + hc * 16, v);
        tc::tmem_st_wait();
    }
    // dt of chunk 0 (warp 0, 4 tokens per lane), software-pipelined one chunk ahead
    float dnext[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    auto load_dt = [&](uint32_t c, float (&d)[4]) {
        const uint32_t t0 = c * TQ, tl = min((uint32_t)TQ, a.L - t0);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t tt = lane * 4 + i;
            d[i] = tt < tl ? load_any(a.dt_raw, ((uint64_t)b * a.L + t0 + tt) * a.dt_rs + h, a.dt_dtype) : -1e30f;
        }
    };
    if (warp == 0) load_dt(0, dnext);

    // dt of chunk c -> softplus/clamp, cumulative log decay into scalar buffer c & 1 (warp 0)
    auto scan_dt = [&](uint32_t c) {
        float* F = reinterpret_cast<float*>(sm + OFF_F) + (c & 1) * 4 * TQ;
        float d[4], run = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float v = 0.0f;
            if (dnext[i] > -1e29f) v = fminf(fmaxf(softplus(dnext[i] + dbias), a.dt_min), a.dt_max);
            d[i] = v;
            run += A * v;
        }
        if (c + 1 < nc) load_dt(c + 1, dnext);
        float incl = run;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float u = __shfl_up_sync(0xffffffffu, incl, o);
            if ((int)lane >= o) incl += u;
        }
        float pre = incl - run;
        const float lend = __shfl_sync(0xffffffffu, incl, 31);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t tt = lane * 4 + i;
            pre += A * d[i];
            F[tt] = pre * LOG2E - __log2f(fmaxf(d[i], 1e-30f));   // q_j (padding rows: masked anyway)
            F[TQ + tt] = pre;
            F[2 * TQ + tt] = __expf(lend - pre) * d[i];
            F[3 * TQ + tt] = __expf(pre);
        }
    };
    // y_t = Y_t + exp(Lc_t) CS_t + D x_t for chunk c (columns hc*16 .. +16), Y and CS from
    // TMEM buffers c & 1; el = exp(Lc_t) of this thread's row
    auto epilogue = [&](uint32_t c, const uint32_t (&xr)[8], float el) {
        const uint32_t t0 = c * TQ, tl = min((uint32_t)TQ, a.L - t0);
        uint32_t v[16], w[16];
        tc::tmem_ld16(tmem + lane_base + T_Y + (c & 1) * 64 + hc * 16, v);
        tc::tmem_ld16(tmem + lane_base + T_CS + (c & 1) * 64 + hc * 16, w);
        tc::tmem_ld_wait();
        if (t < tl) {
            float y[16];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float2 xv = unpack2<BF16>(xr[e]);
                y[2 * e] = __uint_as_float(v[2 * e]) + el * __uint_as_float(w[2 * e]) + Dh * xv.x;
                y[2 * e + 1] = __uint_as_float(v[2 * e + 1]) + el * __uint_as_float(w[2 * e + 1]) + Dh * xv.y;
            }
            const uint64_t o = ((uint64_t)b * a.L + t0 + t) * a.y_rs + (uint64_t)h * TP + hc * 16;
            if (a.y_dtype == 2) {
                float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.Y) + o);
#pragma unroll
                for (int qq = 0; qq < 4; ++qq)
                    dst[qq] = make_float4(y[4 * qq], y[4 * qq + 1], y[4 * qq + 2], y[4 * qq + 3]);
            } else if (a.z) {   // gated: half(silu(z) * half(y)), fp16
                const uint4* zs = reinterpret_cast<const uint4*>(
                    a.z + ((uint64_t)b * a.L + t0 + t) * a.z_rs + (uint64_t)h * TP + hc * 16);
                uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.Y) + o);
#pragma unroll
                for (int qq = 0; qq < 2; ++qq) {
                    const uint4 zu = zs[qq];
                    const __half* zh = reinterpret_cast<const __half*>(&zu);
                    uint4 u;
                    __half* oh = reinterpret_cast<__half*>(&u);
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const float yv = __half2float(__float2half_rn(y[qq * 8 + e]));
                        oh[e] = __float2half_rn(silu(__half2float(zh[e])) * yv);
                    }
                    dst[qq] = u;
                }
            } else {
                uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.Y) + o);
#pragma unroll
                for (int qq = 0; qq < 2; ++qq) {
                    uint4 u;
                    uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        w[e] = (a.y_dtype == 1) ? pack2<true>(y[qq * 8 + 2 * e], y[qq * 8 + 2 * e + 1])
                                                : pack2<false>(y[qq * 8 + 2 * e], y[qq * 8 + 2 * e + 1]);
                    dst[qq] = u;
                }
            }
        }
    };
    if (warp == 0) scan_dt(0);
    uint32_t xprev[8];    // x rows of the chunk whose epilogue is pending
    float elprev = 0.0f;  // and its exp(Lc_t)
#pragma unroll
    for (int e = 0; e < 8; ++e) xprev[e] = 0;

    for (uint32_t c = 0; c < nc && ok; ++c) {
        const uint32_t buf = c & 1;
        uint8_t* sX = sm + OFF_X + buf * X_BYTES;
        uint8_t* sC = sm + OFF_C + buf * BC_BYTES;
        uint8_t* sB = sm + OFF_B + buf * BC_BYTES;
        const float* F = reinterpret_cast<const float*>(sm + OFF_F) + buf * 4 * TQ;
        const float* Qj = F;
        const float* Lc = F + TQ;
        const float* Wj = F + 2 * TQ;
        const float* EL = F + 3 * TQ;
        __syncthreads();   // scalars of chunk c visible
        // tiles of chunk c visible to every thread, and CB(c) done
        if (!tc::mbar_wait(smem_u32(&bars[buf]), (c >> 1) & 1, abort_flag)) { ok = false; break; }
        if (!tc::mbar_wait(bar_cb, c & 1, abort_flag)) { ok = false; break; }
        tc::tc_fence_after();
        const float lend = Lc[TQ - 1];
        uint32_t xreg[8];    // x_t[hc*16 .. +16] packed, kept for the epilogue
        const float elcur = EL[t];
        {
            const float lct2 = Lc[t] * LOG2E;
            uint8_t* sM = sm + OFF_M;
#pragma unroll 1
            for (uint32_t jc = 0; jc < 1; ++jc) {
                const uint32_t col0 = hc * 32;
                if (col0 > q4 * 32 + 31) {   // above the diagonal for every row of this warp: zeros
#pragma unroll
                    for (int qq = 0; qq < 4; ++qq)
                        *reinterpret_cast<uint4*>(sM + sw_off(t, col0 + qq * 8)) = make_uint4(0, 0, 0, 0);
                    continue;
                }
                uint32_t v[32];
                tc::tmem_ld32(tmem + lane_base + T_CB + col0, v);
                tc::tmem_ld_wait();
#pragma unroll
                for (int qq = 0; qq < 4; ++qq) {
                    uint4 u;
                    uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const uint32_t j0 = col0 + qq * 8 + e * 2;
                        float m0 = 0.0f, m1 = 0.0f;
                        if (j0 <= t) m0 = __uint_as_float(v[qq * 8 + e * 2]) * ex2_approx(lct2 - Qj[j0]);
                        if (j0 + 1 <= t) m1 = __uint_as_float(v[qq * 8 + e * 2 + 1]) * ex2_approx(lct2 - Qj[j0 + 1]);
                        w[e] = pack2<BF16>(m0, m1);
                    }
                    *reinterpret_cast<uint4*>(sM + sw_off(t, col0 + qq * 8)) = u;
                }
            }
#pragma unroll
            for (int qq = 0; qq < 2; ++qq) {
                const uint4 u = *reinterpret_cast<const uint4*>(sX + sw_off(t, hc * 16 + qq * 8));
                xreg[qq * 4 + 0] = u.x; xreg[qq * 4 + 1] = u.y; xreg[qq * 4 + 2] = u.z; xreg[qq * 4 + 3] = u.w;
            }
            scale_quarter_row<BF16>(sB, t, hc, Wj[t]);
            uint8_t* sS = sm + OFF_S;
            const float dch = __expf(lend);
            uint32_t v[16];
            tc::tmem_ld16(tmem + lane_base + T_S + hc * 16, v);
            tc::tmem_ld_wait();
#pragma unroll
            for (int qq = 0; qq < 2; ++qq) {
                uint4 u;
                uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    w[e] = pack2<BF16>(__uint_as_float(v[qq * 8 + e * 2]), __uint_as_float(v[qq * 8 + e * 2 + 1]));
                *reinterpret_cast<uint4*>(sS + sw_off(t, hc * 16 + qq * 8)) = u;
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) * dch);
            tc::tmem_st16(tmem + lane_base + T_S + hc * 16, v);
            tc::tmem_st_wait();
        }
        tc::fence_proxy_async_shared();
        tc::tc_fence_before();
        __syncthreads();
        // -- Y(c) = M X and CS(c) = C S_old into TMEM buffers c & 1 ; S += B~^T X ; then CB(c+1)
        if (tid == 0) {
            tc::tc_fence_after();
            const uint32_t sMa = smem_u32(sm + OFF_M), sXa = smem_u32(sX), sSa = smem_u32(sm + OFF_S);
            const uint32_t sCa = smem_u32(sC), sBa = smem_u32(sB);
            const uint32_t ty = tmem + T_Y + buf * 64, tcs = tmem + T_CS + buf * 64;
#pragma unroll
            for (uint32_t k = 0; k < 8; ++k)
                tc::umma_f16(ty, tc::sw128_desc(sMa + (k >> 2) * PANEL + (k & 3) * 32, 16, 1024),
                             tc::sw128_desc(sXa + k * 2048, PANEL, 1024), ID_Y, k > 0);
#pragma unroll
            for (uint32_t k = 0; k < 8; ++k)
                tc::umma_f16(tcs, tc::sw128_desc(sCa + (k >> 2) * PANEL + (k & 3) * 32, 16, 1024),
                             tc::sw128_desc(sSa + k * 2048, PANEL, 1024), ID_Y, k > 0);
#pragma unroll
            for (uint32_t k = 0; k < 8; ++k)
                tc::umma_f16(tmem + T_S, tc::sw128_desc(sBa + k * 2048, PANEL, 1024),
                             tc::sw128_desc(sXa + k * 2048, PANEL, 1024), ID_DS, 1);
            tc::umma_commit(bar_y);
            if (c + 1 < nc) {
                if (tc::mbar_wait(smem_u32(&bars[(c + 1) & 1]), ((c + 1) >> 1) & 1, abort_flag)) issue_cb(c + 1);
            }
        }
        // -- while MMA 2 (c) runs: chunk c+1's dt scan, chunk c-1's epilogue
        if (warp == 0 && c + 1 < nc) scan_dt(c + 1);
        if (c > 0) epilogue(c - 1, xprev, elprev);
#pragma unroll
        for (int e = 0; e < 8; ++e) xprev[e] = xreg[e];
        elprev = elcur;
        if (!tc::mbar_wait(bar_y, c & 1, abort_flag)) { ok = false; break; }
        tc::tc_fence_after();
        // this chunk's buffer is free now: prefetch chunk c + 2 into it
        if (tid == 0 && c + 2 < nc) {
            issue_chunk(c + 2);
            last_issued = c + 2;
        }
        tc::tc_fence_before();
    }
    if (ok && !*abort_flag && nc > 0) {
        tc::tc_fence_after();
        epilogue(nc - 1, xprev, elprev);
    }

    if (ok && !*abort_flag) {   // final state -> global
        tc::tc_fence_after();
        uint32_t v[16];
        tc::tmem_ld16(tmem + lane_base + T_S + hc * 16, v);
        tc::tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) Sg[(uint64_t)(hc * 16 + j) * TN + t] = __uint_as_float(v[j]);
    }
    // teardown: pending TMA and tensor-core work must finish before exit (bounded)
    if (tid == 0 && *abort_flag) {
        atomicExch(a.err, 1);
        tc::mbar_wait_drain(smem_u32(&bars[last_issued & 1]), (last_issued >> 1) & 1);
        tc::umma_commit(bar_y);
        tc::mbar_wait_drain(bar_y, 0);
        tc::mbar_wait_drain(bar_y, 1);
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, TMEM_COLS);
    }
}

// 3-D map over (cols, L, batch) of a 16-bit row-major activation with row stride `rs`.
bool make_map3(CUtensorMap* m, const void* base, uint64_t cols, uint64_t L, uint64_t batch, uint64_t rs, bool bf16) {
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    cuuint64_t dims[3] = {cols, L, batch};
    cuuint64_t strides[2] = {rs * 2, L * rs * 2};
    cuuint32_t box[3] = {64, (cuuint32_t)TQ, 1};
    cuuint32_t es[3] = {1, 1, 1};
    return enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base),
               dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

int* tc_error_word();

// Returns cudaErrorNotSupported when the shape / layout is not handled here (the
// caller then uses the general-shape kernel).
cudaError_t launch_ssd_chunked_tc(const SsdArgs& s, cudaStream_t st) {
    if (s.P != TP || s.N != TN || s.x_dtype > 1) return cudaErrorNotSupported;
    const uint64_t xrs = s.x_row_stride ? s.x_row_stride : (uint64_t)s.H * s.P;
    const uint64_t bcrs = s.bc_row_stride ? s.bc_row_stride : (uint64_t)s.G * s.N;
    const uint64_t dtrs = s.dt_row_stride ? s.dt_row_stride : s.H;
    const uint64_t yrs = s.y_row_stride ? s.y_row_stride : (uint64_t)s.H * s.P;
    if (xrs % 8 || bcrs % 8 || yrs % 8 || s.batch == 0 || s.L == 0) return cudaErrorNotSupported;
    if (!aligned(s.X, 16) || !aligned(s.B, 16) || !aligned(s.C, 16) || !aligned(s.Y, 16))
        return cudaErrorNotSupported;
    if (s.z && (s.y_dtype != 0 || s.z_row_stride % 8 || !aligned(s.z, 16))) return cudaErrorNotSupported;
    const bool bf16 = s.x_dtype == 1;
    CUtensorMap mx, mb, mc;
    if (!make_map3(&mx, s.X, xrs, s.L, s.batch, xrs, bf16) || !make_map3(&mb, s.B, bcrs, s.L, s.batch, bcrs, bf16) ||
        !make_map3(&mc, s.C, bcrs, s.L, s.batch, bcrs, bf16))
        return cudaErrorNotSupported;
    TcArgs a{};
    a.dt_raw = s.dt_raw; a.dt_bias = s.dt_bias; a.A_log = s.A_log; a.D = s.D; a.Y = s.Y; a.state = s.state;
    a.z = static_cast<const __half*>(s.z); a.z_rs = s.z_row_stride;
    a.batch = s.batch; a.L = s.L; a.H = s.H; a.P = s.P; a.N = s.N; a.G = s.G ? s.G : 1;
    a.dt_min = s.dt_min; a.dt_max = s.dt_max; a.has_D = s.has_D;
    a.dt_dtype = s.dt_dtype; a.param_dtype = s.param_dtype; a.y_dtype = s.y_dtype;
    a.dt_rs = dtrs; a.y_rs = yrs; a.err = tc_error_word();
    auto k = bf16 ? k_ssd_chunked_tc<true> : k_ssd_chunked_tc<false>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_TOTAL);
    if (e != cudaSuccess) return e;
    k<<<s.batch * s.H, THREADS, SMEM_TOTAL, st>>>(mx, mb, mc, a);
    return cudaGetLastError();
}

}  // namespace lssm
