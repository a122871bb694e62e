// k_ssd_cp.cu — SSD chunked scan, chunk-parallel (shaders/ssd_chunked.metal:82-297 restated
// for P = 64, N = 128).
//
// The sequential form walks a head's chunks one after another, so one (sequence, head) pair
// keeps one SM busy for the whole sequence and the per-chunk dependency chain is exposed.
// Here every chunk is a work item of its own. For chunk c of head h (Q = 128 tokens):
//   intra-chunk (independent of every other chunk):
//     DT, Lc        softplus + clamp of dt, Lc = inclusive cumsum of A DT
//     CB = C B^T    (tcgen05, 128x128x128, TMEM)
//     M[t,j]      = CB[t,j] exp(Lc_t - Lc_j) DT_j for j <= t          (threads -> smem)
//     Y_c = M X     (tcgen05, 128x64, K = 128)
//     S_c = B^T X~, X~_j = exp(Lc_end - Lc_j) DT_j X_j               (tcgen05, 128x64, K = 128)
//   carried state (the only link between chunks):
//     S_in(c)     = state entering chunk c: the caller's state for c = 0, else published
//                   by chunk c - 1; S_in(c + 1) = exp(Lc_end) S_in(c) + S_c is published
//                   (fp32) for chunk c + 1, or written back as the final state
//     CS = C S_in   (tcgen05, 128x64, K = 128; S_in rounded to the input dtype as operand)
//   epilogue        y_t = Y_t + exp(Lc_t) CS_t + D x_t   (optionally gated, as k_ssd_tc.cu)
// Only the carry waits on the previous chunk; everything else runs as soon as the item's
// tiles land. Work items (chunk, sequence, head pair) are taken in chunk-major order by a
// persistent cooperative grid (one CTA per SM, co-resident), so an item only ever waits for
// an item with a lower index, which some CTA is already running or has finished.
// Each CTA runs two heads of the same group at once (two groups of 8 warps): they share the
// B / C tiles and CB. The carried state goes through a two-slot ring per (sequence, head) in
// global memory (slot c & 1, small enough to stay in L2) with a per-(sequence, head) counter
// of published chunks; chunk c + 2 overwrites slot c & 1 only after chunk c + 1 has read it
// (it waits for chunk c + 1's publication, which follows that read). Every wait is bounded.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "device_util.cuh"
#include "lssm_internal.h"
#include "tc_common.cuh"

namespace lssm {

namespace {

constexpr int TQ = 128, TP = 64, TN = 128;
constexpr int THREADS = 512;                       // two head groups x 8 warps
constexpr uint32_t PANEL = TQ * 128;               // 16 KB: 128 rows x 128 B (64 x 16-bit columns)
constexpr uint32_t X_BYTES = TQ * TP * 2;          // 16 KB
constexpr uint32_t BC_BYTES = TQ * TN * 2;         // 32 KB (two panels)
// shared-memory map (offsets from a 1024-byte aligned base)
constexpr uint32_t OFF_B = 0;
constexpr uint32_t OFF_C = OFF_B + BC_BYTES;
constexpr uint32_t OFF_G = OFF_C + BC_BYTES;       // per group: X, X~, M (M reused for the S_in operand)
constexpr uint32_t G_X = 0, G_XT = X_BYTES, G_M = 2 * X_BYTES, G_BYTES = 2 * X_BYTES + BC_BYTES;
// per group and item parity: Qj, W, EL, Lc (128 floats each), Lc_end, D
constexpr uint32_t OFF_F = OFF_G + 2 * G_BYTES;
constexpr uint32_t F_FLOATS = 4 * TQ + 4;
constexpr uint32_t OFF_BAR = OFF_F + 4 * F_FLOATS * 4;
constexpr uint32_t SMEM_TOTAL = OFF_BAR + 128 + 1024;
constexpr uint32_t STAGE_TX = 2 * BC_BYTES + 2 * X_BYTES;
// TMEM columns: CB (later CS of group g at 64 g), Y of group g at 128 + 64 g, S_c at 256 + 64 g
constexpr uint32_t T_CB = 0, T_Y = 128, T_SC = 256, TMEM_COLS = 512;

struct CpArgs {
    const void* dt_raw; const void* dt_bias; const void* A_log; const void* D;
    void* Y; float* state;
    const __half* z; uint64_t z_rs;
    uint32_t batch, L, H, G;
    float dt_min, dt_max;
    uint32_t has_D;
    uint32_t dt_dtype, param_dtype, y_dtype;
    uint64_t dt_rs, y_rs;
    float* ring;        // [2][batch][H][N][P] fp32 carried states
    uint32_t* count;    // [batch][H] chunks published (zeroed before the launch)
    int* err;
};

__device__ __forceinline__ uint32_t sw_off(uint32_t row, uint32_t col) {
    const uint32_t panel = col >> 6, c = col & 63;
    return panel * PANEL + row * 128 + ((((c >> 3) ^ (row & 7)) & 7) << 4) + (c & 7) * 2;
}

constexpr float LOG2E = 1.4426950408889634f;

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

__device__ __forceinline__ void group_sync(uint32_t g) {
    asm volatile("bar.sync %0, 256;" ::"r"(1 + g) : "memory");
}

// TMA tensor store shared -> global (3-D box) and untiled bulk store, both in the thread's
// bulk async-group; commit closes the group; wait_read: the groups' shared-memory reads are
// done (the buffer may be rewritten); wait_all: their global writes are complete.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int32_t c0, int32_t c1, int32_t c2) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(src), "r"(c0), "r"(c1), "r"(c2)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

template <bool BF16>
__global__ void __launch_bounds__(THREADS, 1)
    k_ssd_chunked_cp(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmY, CpArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);   // full, cb, mma[2], cs[2], drain[2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t g = warp >> 3;                      // head group (head 2 hp + g)
    const uint32_t q4 = warp & 3, hc = (warp >> 2) & 1;  // TMEM lane quarter, column half
    const uint32_t t = q4 * 32 + lane;                 // chunk row / TMEM lane
    const uint32_t gtid = tid & 255;                   // thread within the group
    const uint32_t nc = (a.L + TQ - 1) / TQ, HP = a.H / 2;
    const uint32_t nitems = nc * a.batch * HP;
    const uint32_t hpg = a.H / a.G;
    uint8_t* sB = sm + OFF_B;
    uint8_t* sC = sm + OFF_C;
    uint8_t* gX = sm + OFF_G + g * G_BYTES + G_X;
    uint8_t* gXT = sm + OFF_G + g * G_BYTES + G_XT;
    uint8_t* gM = sm + OFF_G + g * G_BYTES + G_M;
    float* F0 = reinterpret_cast<float*>(sm + OFF_F) + g * 2 * F_FLOATS;   // two parities: Qj, W, EL, Lc, Lc_end, D
    constexpr uint32_t ID_CB = tc::idesc_f16_major(128, 128, BF16 ? 1 : 0, 0, 0);
    constexpr uint32_t ID_Y = tc::idesc_f16_major(128, 64, BF16 ? 1 : 0, 0, 1);
    constexpr uint32_t ID_DS = tc::idesc_f16_major(128, 64, BF16 ? 1 : 0, 1, 1);
    const uint32_t bar_full = smem_u32(&bars[0]), bar_cb = smem_u32(&bars[1]);
    const uint32_t bar_mma = smem_u32(&bars[2 + g]), bar_cs = smem_u32(&bars[4 + g]);

    if (tid == 0) {
        for (int i = 0; i < 8; ++i) tc::mbar_init(smem_u32(&bars[i]), 1);
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

    // item -> (chunk, sequence, head pair): chunk-major
    auto decode = [&](uint32_t it, uint32_t& c, uint32_t& b, uint32_t& hp) {
        c = it / (a.batch * HP);
        const uint32_t r = it - c * (a.batch * HP);
        b = r / HP;
        hp = r - b * HP;
    };
    auto issue_tma = [&](uint32_t it) {
        uint32_t c, b, hp;
        decode(it, c, b, hp);
        const uint32_t h0 = 2 * hp, gg = h0 / hpg;
        const int32_t t0 = (int32_t)(c * TQ);
        tc::mbar_arrive_expect_tx(bar_full, STAGE_TX);
        for (int pnl = 0; pnl < 2; ++pnl) {
            tc::tma_load_3d(smem_u32(sC + pnl * PANEL), &tmC, (int32_t)(gg * TN + pnl * 64), t0, (int32_t)b, bar_full);
            tc::tma_load_3d(smem_u32(sB + pnl * PANEL), &tmB, (int32_t)(gg * TN + pnl * 64), t0, (int32_t)b, bar_full);
        }
        for (uint32_t gi = 0; gi < 2; ++gi)
            tc::tma_load_3d(smem_u32(sm + OFF_G + gi * G_BYTES + G_X), &tmX, (int32_t)((h0 + gi) * TP), t0, (int32_t)b,
                            bar_full);
    };

    // dt scan of one item's head (a group's first warp): inputs loaded ahead into registers
    // (raw dt of 4 tokens per lane, dt_bias, A_log, D), scalars -> Fd
    struct ScanIn {
        float raw[4], dbias, alog, dsk;
        uint32_t tl;
    };
    auto scan_load = [&](uint32_t item, ScanIn& in) {
        uint32_t c, b, hp;
        decode(item, c, b, hp);
        const uint32_t h = 2 * hp + g, t0 = c * TQ;
        in.tl = min((uint32_t)TQ, a.L - t0);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t tt = lane * 4 + i;
            in.raw[i] = tt < in.tl ? load_any(a.dt_raw, ((uint64_t)b * a.L + t0 + tt) * a.dt_rs + h, a.dt_dtype) : 0.0f;
        }
        in.dbias = load_any(a.dt_bias, h, a.param_dtype);
        in.alog = load_any(a.A_log, h, a.param_dtype);
        in.dsk = a.has_D ? load_any(a.D, h, a.param_dtype) : 0.0f;
    };
    auto scan = [&](const ScanIn& in, float* Fd) {
        const float A = -expf(in.alog);
        float d[4], run = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t tt = lane * 4 + i;
            d[i] = tt < in.tl ? fminf(fmaxf(softplus(in.raw[i] + in.dbias), a.dt_min), a.dt_max) : 0.0f;
            run += A * d[i];
        }
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
            Fd[tt] = pre * LOG2E - __log2f(fmaxf(d[i], 1e-30f));   // q_j (rows past L: masked / zero)
            Fd[TQ + tt] = __expf(lend - pre) * d[i];               // W_j (0 past L)
            Fd[2 * TQ + tt] = __expf(pre);                         // EL_t = exp(Lc_t)
            Fd[3 * TQ + tt] = pre;                                 // Lc_t
        }
        if (lane == 0) { Fd[4 * TQ] = lend; Fd[4 * TQ + 1] = in.dsk; }
    };
    ScanIn snext;
    if ((warp & 7) == 0 && blockIdx.x < nitems) {
        scan_load(blockIdx.x, snext);
        scan(snext, F0);
    }

    uint32_t it = blockIdx.x, iter = 0;
    bool tma_pending = false;   // thread 0: a load whose barrier phase `pend_par` was not waited for
    uint32_t pend_par = 0;
    if (tid == 0 && it < nitems) { issue_tma(it); tma_pending = true; pend_par = 0; }
    for (; it < nitems; it += gridDim.x, ++iter) {
        uint32_t c, b, hp;
        decode(it, c, b, hp);
        const uint32_t h = 2 * hp + g;
        const uint32_t ph = iter & 1;
        const uint32_t t0 = c * TQ, tl = min((uint32_t)TQ, a.L - t0);
        float* F = F0 + (iter & 1) * F_FLOATS;   // this item's scalars (scanned during the previous item)
        // the next item's scan inputs, loaded now and consumed at the end of this item
        if ((warp & 7) == 0 && it + gridDim.x < nitems) scan_load(it + gridDim.x, snext);
        // ---- tiles landed -> CB = C B^T
        if (tid == 0) {
            tc::mbar_wait(bar_full, ph, abort_flag);
            tma_pending = false;
            tc::tc_fence_after();
            const uint32_t sCa = smem_u32(sC), sBa = smem_u32(sB);
#pragma unroll
            for (uint32_t k = 0; k < 8; ++k) {
                const uint32_t koff = (k >> 2) * PANEL + (k & 3) * 32;
                tc::umma_f16(tmem + T_CB, tc::sw128_desc(sCa + koff, 16, 1024), tc::sw128_desc(sBa + koff, 16, 1024),
                             ID_CB, k > 0);
            }
            tc::umma_commit(bar_cb);
        }
        __syncthreads();   // scalars written
        tc::mbar_wait(bar_full, ph, abort_flag);
        tc::mbar_wait(bar_cb, ph, abort_flag);
        tc::tc_fence_after();
        // ---- M (row t, columns hc*64 .. +64) and X~ rows; x kept for the epilogue
        const float lct2 = F[3 * TQ + t] * LOG2E;
        {
#pragma unroll
            for (uint32_t half = 0; half < 2; ++half) {
                const uint32_t col0 = hc * 64 + half * 32;
                if (col0 > q4 * 32 + 31) {   // above the diagonal for every row of this warp
#pragma unroll
                    for (int qq = 0; qq < 4; ++qq)
                        *reinterpret_cast<uint4*>(gM + sw_off(t, col0 + qq * 8)) = make_uint4(0, 0, 0, 0);
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
                        if (j0 <= t) m0 = __uint_as_float(v[qq * 8 + e * 2]) * ex2_approx(lct2 - F[j0]);
                        if (j0 + 1 <= t) m1 = __uint_as_float(v[qq * 8 + e * 2 + 1]) * ex2_approx(lct2 - F[j0 + 1]);
                        w[e] = pack2<BF16>(m0, m1);
                    }
                    *reinterpret_cast<uint4*>(gM + sw_off(t, col0 + qq * 8)) = u;
                }
            }
        }
        uint32_t xreg[16];   // x_t[hc*32 .. +32] (packed 16-bit pairs)
        {
            const float wj = F[TQ + t];
#pragma unroll
            for (int qq = 0; qq < 4; ++qq) {
                const uint32_t off = sw_off(t, hc * 32 + qq * 8);
                const uint4 u = *reinterpret_cast<const uint4*>(gX + off);
                xreg[qq * 4 + 0] = u.x; xreg[qq * 4 + 1] = u.y; xreg[qq * 4 + 2] = u.z; xreg[qq * 4 + 3] = u.w;
                uint4 s;
                const uint32_t* ui = reinterpret_cast<const uint32_t*>(&u);
                uint32_t* so = reinterpret_cast<uint32_t*>(&s);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = unpack2<BF16>(ui[e]);
                    so[e] = pack2<BF16>(f.x * wj, f.y * wj);
                }
                *reinterpret_cast<uint4*>(gXT + off) = s;
            }
        }
        tc::fence_proxy_async_shared();
        tc::tc_fence_before();
        group_sync(g);
        // ---- Y = M X, S_c = B^T X~ (this group's thread 0)
        if (gtid == 0) {
            tc::tc_fence_after();
            const uint32_t sMa = smem_u32(gM), sXa = smem_u32(gX), sXTa = smem_u32(gXT), sBa = smem_u32(sB);
#pragma unroll
            for (uint32_t k = 0; k < 8; ++k)
                tc::umma_f16(tmem + T_Y + 64 * g, tc::sw128_desc(sMa + (k >> 2) * PANEL + (k & 3) * 32, 16, 1024),
                             tc::sw128_desc(sXa + k * 2048, PANEL, 1024), ID_Y, k > 0);
#pragma unroll
            for (uint32_t k = 0; k < 8; ++k)
                tc::umma_f16(tmem + T_SC + 64 * g, tc::sw128_desc(sBa + k * 2048, PANEL, 1024),
                             tc::sw128_desc(sXTa + k * 2048, PANEL, 1024), ID_DS, k > 0);
            tc::umma_commit(bar_mma);
        }
        tc::tc_fence_before();
        __syncthreads();   // both groups done reading CB: its columns may take CS
        tc::tc_fence_after();
        // ---- carried state entering this chunk
        float sin[32];
        if (c == 0) {
            const float* Sg = a.state + ((uint64_t)b * a.H + h) * TP * TN;
#pragma unroll
            for (int j = 0; j < 32; ++j) sin[j] = Sg[(uint64_t)(hc * 32 + j) * TN + t];
        } else {
            const uint32_t* cnt = a.count + (uint64_t)b * a.H + h;
            if (gtid == 0) {   // chunk c - 1 published (bounded wait)
                uint64_t t0w = 0;
                for (uint32_t k = 1;; ++k) {
                    if ((int32_t)(ld_acquire(cnt) - c) >= 0) break;
                    if ((k & 15) == 0) {
                        if (*abort_flag) break;
                        if (*reinterpret_cast<volatile int*>(a.err)) { *abort_flag = 1; break; }
                        const uint64_t tn = tc::globaltimer();
                        if (!t0w) t0w = tn;
                        else if (tn - t0w > tc::WAIT_LIMIT_NS) { *abort_flag = 1; break; }
                    }
                    __nanosleep(128);
                }
            }
            group_sync(g);
            // ring slot layout [16 p-quads][128 n][4]: lane-consecutive 16-byte pieces
            const float4* src = reinterpret_cast<const float4*>(
                                    a.ring + (((uint64_t)((c - 1) & 1) * a.batch + b) * a.H + h) * TN * TP) +
                                hc * 8 * TN + t;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float4 v = __ldcg(src + j * TN);
                sin[4 * j] = v.x; sin[4 * j + 1] = v.y; sin[4 * j + 2] = v.z; sin[4 * j + 3] = v.w;
            }
        }
        // ---- S_out = exp(Lc_end) S_in + S_c -> next chunk (ring) or final state; S_in -> operand
        tc::mbar_wait(bar_mma, ph, abort_flag);
        tc::tc_fence_after();
        {
            const float dch = __expf(F[4 * TQ]);
            uint32_t v[32];
            tc::tmem_ld32(tmem + lane_base + T_SC + 64 * g + hc * 32, v);
            tc::tmem_ld_wait();
            if (c + 1 < nc) {
                // stored straight from registers into ring slot c & 1 ([16 p-quads][128 n][4]:
                // a warp's 32 lanes write 512 contiguous bytes per store); published below
                float4* dst = reinterpret_cast<float4*>(
                                  a.ring + (((uint64_t)(c & 1) * a.batch + b) * a.H + h) * TN * TP) +
                              hc * 8 * TN + t;
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    dst[j * TN] = make_float4(dch * sin[4 * j] + __uint_as_float(v[4 * j]),
                                              dch * sin[4 * j + 1] + __uint_as_float(v[4 * j + 1]),
                                              dch * sin[4 * j + 2] + __uint_as_float(v[4 * j + 2]),
                                              dch * sin[4 * j + 3] + __uint_as_float(v[4 * j + 3]));
            } else {
                float* Sg = a.state + ((uint64_t)b * a.H + h) * TP * TN;
#pragma unroll
                for (int j = 0; j < 32; ++j) Sg[(uint64_t)(hc * 32 + j) * TN + t] = dch * sin[j] + __uint_as_float(v[j]);
            }
            // S_in[n = t][p] as the 16-bit operand of C S_in (M's buffer is free: Y / S_c are done)
#pragma unroll
            for (int qq = 0; qq < 4; ++qq) {
                uint4 u;
                uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
                for (int e = 0; e < 4; ++e) w[e] = pack2<BF16>(sin[qq * 8 + 2 * e], sin[qq * 8 + 2 * e + 1]);
                *reinterpret_cast<uint4*>(gM + sw_off(t, hc * 32 + qq * 8)) = u;
            }
        }
        tc::fence_proxy_async_shared();
        tc::tc_fence_before();
        group_sync(g);
        if (gtid == 0) {
            // CS = C S_in into this group's half of the CB columns (it needs S_in only)
            tc::tc_fence_after();
            const uint32_t sCa = smem_u32(sC), sSa = smem_u32(gM);
#pragma unroll
            for (uint32_t k = 0; k < 8; ++k)
                tc::umma_f16(tmem + T_CB + 64 * g, tc::sw128_desc(sCa + (k >> 2) * PANEL + (k & 3) * 32, 16, 1024),
                             tc::sw128_desc(sSa + k * 2048, PANEL, 1024), ID_Y, k > 0);
            tc::umma_commit(bar_cs);
            // publish S_out of chunk c while CS runs: the group's stores (ordered before this
            // thread by the group barrier) are released by one gpu-scope fence, then the counter
            if (c + 1 < nc) {
                asm volatile("fence.acq_rel.gpu;" ::: "memory");
                asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(a.count + (uint64_t)b * a.H + h), "r"(c + 1)
                             : "memory");
            }
        }
        tc::mbar_wait(bar_cs, ph, abort_flag);
        tc::tc_fence_before();
        __syncthreads();   // both groups' MMAs done: every tile buffer is free
        tc::tc_fence_after();
        if (tid == 0 && it + gridDim.x < nitems && !*abort_flag) {
            issue_tma(it + gridDim.x);
            tma_pending = true;
            pend_par = (iter + 1) & 1;
        }
        // ---- epilogue: y_t = Y_t + exp(Lc_t) CS_t + D x_t (columns hc*32 .. +32, two halves of
        // 16), staged 128-byte swizzled in the group's M buffer (free: CS is done) and written by
        // TMA tensor stores, which drop the rows past L
        {
            const float el = F[2 * TQ + t], Dh = F[4 * TQ + 1];
            const bool f32 = a.y_dtype == 2;
#pragma unroll
            for (uint32_t half = 0; half < 2; ++half) {
                uint32_t v[16], w[16];
                tc::tmem_ld16(tmem + lane_base + T_Y + 64 * g + hc * 32 + half * 16, v);
                tc::tmem_ld16(tmem + lane_base + T_CB + 64 * g + hc * 32 + half * 16, w);
                tc::tmem_ld_wait();
                float y[16];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const float2 xv = unpack2<BF16>(xreg[half * 8 + e]);
                    y[2 * e] = __uint_as_float(v[2 * e]) + el * __uint_as_float(w[2 * e]) + Dh * xv.x;
                    y[2 * e + 1] = __uint_as_float(v[2 * e + 1]) + el * __uint_as_float(w[2 * e + 1]) + Dh * xv.y;
                }
                if (f32) {   // box hc: [128 rows][32 floats]; this half is chunks 4 half .. +3
                    uint8_t* row = gM + hc * PANEL + t * 128;
#pragma unroll
                    for (int qq = 0; qq < 4; ++qq)
                        *reinterpret_cast<float4*>(row + ((((uint32_t)half * 4 + qq) ^ (t & 7)) << 4)) =
                            make_float4(y[4 * qq], y[4 * qq + 1], y[4 * qq + 2], y[4 * qq + 3]);
                } else {     // one box: [128 rows][64 x 16-bit]; this half is chunks 4 hc + 2 half .. +1
                    uint8_t* row = gM + t * 128;
                    uint4 u[2];
                    if (a.z) {   // gated: half(silu(z) * half(y)), fp16
                        const uint4* zs = reinterpret_cast<const uint4*>(
                            a.z + ((uint64_t)b * a.L + t0 + min(t, tl - 1)) * a.z_rs + (uint64_t)h * TP + hc * 32 +
                            half * 16);
#pragma unroll
                        for (int qq = 0; qq < 2; ++qq) {
                            const uint4 zu = zs[qq];
                            const __half* zh = reinterpret_cast<const __half*>(&zu);
                            __half* oh = reinterpret_cast<__half*>(&u[qq]);
#pragma unroll
                            for (int e = 0; e < 8; ++e) {
                                const float yv = __half2float(__float2half_rn(y[qq * 8 + e]));
                                oh[e] = __float2half_rn(silu(__half2float(zh[e])) * yv);
                            }
                        }
                    } else {
#pragma unroll
                        for (int qq = 0; qq < 2; ++qq) {
                            uint32_t* w2 = reinterpret_cast<uint32_t*>(&u[qq]);
#pragma unroll
                            for (int e = 0; e < 4; ++e)
                                w2[e] = (a.y_dtype == 1) ? pack2<true>(y[qq * 8 + 2 * e], y[qq * 8 + 2 * e + 1])
                                                         : pack2<false>(y[qq * 8 + 2 * e], y[qq * 8 + 2 * e + 1]);
                        }
                    }
#pragma unroll
                    for (int qq = 0; qq < 2; ++qq)
                        *reinterpret_cast<uint4*>(row + (((hc * 4 + half * 2 + qq) ^ (t & 7)) << 4)) = u[qq];
                }
            }
            tc::fence_proxy_async_shared();
            group_sync(g);
            if (gtid == 0) {
                if (f32) {
                    for (uint32_t bx = 0; bx < 2; ++bx)
                        tma_store_3d(&tmY, smem_u32(gM + bx * PANEL), (int32_t)(h * TP + bx * 32), (int32_t)t0,
                                     (int32_t)b);
                } else {
                    tma_store_3d(&tmY, smem_u32(gM), (int32_t)(h * TP), (int32_t)t0, (int32_t)b);
                }
                bulk_commit();
                bulk_wait_read();   // the next item rebuilds M here
            }
        }
        if ((warp & 7) == 0 && it + gridDim.x < nitems) scan(snext, F0 + ((iter + 1) & 1) * F_FLOATS);
        tc::tc_fence_before();
        if (__syncthreads_or(*abort_flag)) break;   // every thread leaves together
        tc::tc_fence_after();
    }
    // teardown: a prefetch still in flight must land, pending tensor-core work must finish
    // (the two MMA-issuing threads each commit their own earlier MMAs to a drain barrier)
    if (tid == 0) {
        if (*abort_flag) atomicExch(a.err, 1);
        if (tma_pending) tc::mbar_wait_drain(bar_full, pend_par);
    }
    if (gtid == 0) {
        bulk_wait_all();   // every bulk / tensor store of the group done
        tc::umma_commit(smem_u32(&bars[6 + g]));
        tc::mbar_wait_drain(smem_u32(&bars[6 + g]), 0);
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, TMEM_COLS);
    }
}

// Y: 3-D map over (y_rs columns, L, batch), element fp32 (box 32 x 128: two per head) or
// 16-bit (box 64 x 128), 128-byte swizzle.
bool make_map_y(CUtensorMap* m, void* base, uint64_t rs, uint64_t L, uint64_t batch, uint32_t y_dtype) {
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    const uint64_t es = y_dtype == 2 ? 4 : 2;
    cuuint64_t dims[3] = {rs, L, batch};
    cuuint64_t strides[2] = {rs * es, L * rs * es};
    cuuint32_t box[3] = {(cuuint32_t)(128 / es), (cuuint32_t)TQ, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    const CUtensorMapDataType dt = y_dtype == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                                : (y_dtype == 1 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                : CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
    return enc(m, dt, 3, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

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

size_t ssd_chunked_cp_scratch(uint32_t batch, uint32_t H) {
    return 2ull * batch * H * TN * TP * 4 + (size_t)batch * H * 4 + 256;
}

// Chunk-parallel scan for P = 64, N = 128, an even number of heads per group and 16-byte
// aligned operands; `ws` (ws_bytes >= ssd_chunked_cp_scratch) holds the carried-state ring
// and the publication counters. cudaErrorNotSupported otherwise (the caller then runs the
// sequential tensor-core kernel).
cudaError_t launch_ssd_chunked_cp(const SsdArgs& s, void* ws, size_t ws_bytes, int sm_count, cudaStream_t st) {
    if (s.P != TP || s.N != TN || s.x_dtype > 1) return cudaErrorNotSupported;
    const uint32_t G = s.G ? s.G : 1;
    if (s.H % G || (s.H / G) % 2 || !ws || ws_bytes < ssd_chunked_cp_scratch(s.batch, s.H) || !aligned(ws, 256))
        return cudaErrorNotSupported;
    const uint64_t xrs = s.x_row_stride ? s.x_row_stride : (uint64_t)s.H * s.P;
    const uint64_t bcrs = s.bc_row_stride ? s.bc_row_stride : (uint64_t)G * s.N;
    const uint64_t dtrs = s.dt_row_stride ? s.dt_row_stride : s.H;
    const uint64_t yrs = s.y_row_stride ? s.y_row_stride : (uint64_t)s.H * s.P;
    if (xrs % 8 || bcrs % 8 || yrs % 8 || s.batch == 0 || s.L == 0 || s.y_dtype > 2) return cudaErrorNotSupported;
    if (!aligned(s.X, 16) || !aligned(s.B, 16) || !aligned(s.C, 16) || !aligned(s.Y, 16))
        return cudaErrorNotSupported;
    if (s.z && (s.y_dtype != 0 || s.z_row_stride % 8 || !aligned(s.z, 16))) return cudaErrorNotSupported;
    const bool bf16 = s.x_dtype == 1;
    CUtensorMap mx, mb, mc, my;
    if (!make_map3(&mx, s.X, xrs, s.L, s.batch, xrs, bf16) || !make_map3(&mb, s.B, bcrs, s.L, s.batch, bcrs, bf16) ||
        !make_map3(&mc, s.C, bcrs, s.L, s.batch, bcrs, bf16) || !make_map_y(&my, s.Y, yrs, s.L, s.batch, s.y_dtype))
        return cudaErrorNotSupported;
    CpArgs a{};
    a.dt_raw = s.dt_raw; a.dt_bias = s.dt_bias; a.A_log = s.A_log; a.D = s.D; a.Y = s.Y; a.state = s.state;
    a.z = static_cast<const __half*>(s.z); a.z_rs = s.z_row_stride;
    a.batch = s.batch; a.L = s.L; a.H = s.H; a.G = G;
    a.dt_min = s.dt_min; a.dt_max = s.dt_max; a.has_D = s.has_D;
    a.dt_dtype = s.dt_dtype; a.param_dtype = s.param_dtype; a.y_dtype = s.y_dtype;
    a.dt_rs = dtrs; a.y_rs = yrs; a.err = tc_error_word();
    a.ring = static_cast<float*>(ws);
    a.count = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(ws) + 2ull * s.batch * s.H * TN * TP * 4);
    cudaError_t e = cudaMemsetAsync(a.count, 0, (size_t)s.batch * s.H * 4, st);
    if (e != cudaSuccess) return e;
    const void* k = bf16 ? (const void*)k_ssd_chunked_cp<true> : (const void*)k_ssd_chunked_cp<false>;
    e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_TOTAL);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, THREADS, SMEM_TOTAL);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorNotSupported;
    const uint32_t nitems = ((s.L + TQ - 1) / TQ) * s.batch * (s.H / 2);
    const uint64_t cap = (uint64_t)sm_count * per_sm;
    const uint32_t grid = (uint32_t)(cap < nitems ? cap : nitems);
    // cooperative: all CTAs co-resident (or the launch fails), so the counter waits end
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = SMEM_TOTAL;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (bf16) return cudaLaunchKernelEx(&cfg, k_ssd_chunked_cp<true>, mx, mb, mc, my, a);
    return cudaLaunchKernelEx(&cfg, k_ssd_chunked_cp<false>, mx, mb, mc, my, a);
}

}  // namespace lssm
