// k_decode_persist.cu — the whole greedy decode loop (all layers, lm_head, argmax,
// next-token embedding) as ONE persistent cooperative kernel: one CTA per SM,
// `n_steps` tokens per launch. Restates the decode half of the reference's
// generate() loop (src/runtime/inference.cpp:55-67: embed -> forward_step ->
// compute_logits -> sample_greedy) for batch <= 2 with INT4_B32 in/out_proj and an
// fp16 lm_head, the 2.7B-shaped headline workload.
//
// Why one kernel: a batch-1 decode token streams 2.05 GB of weights and state in
// ~0.32 ms at HBM speed, while a kernel-per-op step has ~260 launches whose ramp-up,
// tail and launch gaps cost several times that. Here:
//   * warp 10 is the TMA producer: it walks this CTA's weight chunks for every layer
//     and token in order and streams each chunk (16 rows x seg * 128 bytes, plus the
//     INT4 scales) with ONE tensor-map copy (128-byte swizzle, L2 evict-first) into
//     an 11-stage shared-memory ring, and bulk-copies this CTA's rows of the layer's
//     ssd state into a separate buffer. Weights do not depend on activations, so it
//     runs ahead across phase boundaries and grid barriers: HBM stays busy while the
//     consumers synchronise.
//   * warps 0..9 consume. Each warp releases a ring slot as soon as it has read it;
//     tiles / units are accumulated in registers in groups of up to 5 and reduced
//     across warps once per group. Per layer:
//       A  residual (hidden += half(sum of out_proj slots); every SM keeps the whole
//          hidden vector in shared memory) + RMSNorm, staged in MMA-fragment order;
//          in_proj INT4 GEMV tiles (16 rows x all of K) on register-operand mma.sync in
//          column mode (each MMA column one 32-wide block); the SM owns whole channel
//          units (8 z rows + 8 x rows per tile), so the x / z of its ssd rows stay in
//          shared memory; the B / C / dt tiles run first on the SMs with fewer units and
//          are published as {value, epoch} exchange words. Epilogue: xBC rows ->
//          conv-state roll + conv + SiLU.
//       -- no grid barrier: B / C / dt are polled from the exchange words --
//       B  ssd_step + gate on the SM's state rows (already in shared memory):
//          S = e^{A dt} S + dt B x, y = C.S + D x, gated = half(silu(z) * half(y)); the
//          updated rows are stored back by bulk copies
//       -- grid barrier --
//       C  RMSNorm(gated) staged; out_proj work cut into (16-row tile, K chunk) units
//          dealt round-robin over the SMs (every SM gets the same number +-1); each
//          unit's fp32 partial sums go to their own slot, and the next RMSNorm adds
//          the slots in a fixed order (deterministic, no atomics)
//       -- grid barrier --
//     then residual + norm_f + lm_head (fp16 weights, mma.sync), per-CTA first-max
//     argmax partials, a grid barrier, and every CTA reduces the partials to the
//     same next token (no host round-trip; the next token's embedding row is read
//     directly).
// The row -> SM assignments are the same in every layer and step, so each conv-state
// and ssd-state row is only ever written by its owner SM.
// Grid barriers are a monotonically increasing global counter (release add, acquire
// spin) with a 2 s %globaltimer bound; every mbarrier wait and exchange-word poll is
// bounded too. A timeout sets the error word; the consumer warps of a CTA decide to leave
// together (a barrier that ORs the abort flag), and every CTA drains its in-flight copies.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <vector>

#include "device_util.cuh"
#include "lssm_internal.h"
#include "mma_int4.cuh"

namespace lssm {

namespace {

// 10 consumer warps + 1 producer warp (352 threads). With 3 warps on some SM sub-partitions
// (16384 registers each) a thread may use at most 168 registers. An INT4 ring
// stage holds 16 rows x 5 segments of 256 k. The consumer warps form two halves that take
// alternate ring stages; warp w of a half reads segment w of a stage (eight 32-wide blocks),
// so one half releases each stage and two stages are consumed at a time.
constexpr int CONS_WARPS = 10, CONS = CONS_WARPS * 32, THREADS = CONS + 32;
constexpr uint32_t HALF_WARPS = CONS_WARPS / 2;
static_assert(HALF_WARPS == 5, "one consumer warp per segment of a stage");
constexpr int RING = 11;
constexpr uint32_t STAGE = 12288;                         // 1024-aligned (128-byte swizzle atoms)
constexpr uint32_t NOCT = 2;                              // staged octets (or residual quads) per thread
constexpr uint32_t SEG_MAX = 5;                           // 16 x 5 x 128 B + INT4 scales <= STAGE
constexpr uint32_t TG = 5;                                // tiles per register-accumulated group
constexpr uint32_t XBUF = 20480;                          // staged activation (<= 2 x 5120 halves)
constexpr uint32_t PART = TG * CONS_WARPS * 8 * 4 * 4;    // per-warp partial sums of one group ([ti][warp][g][4])
constexpr uint32_t XSUM = 2 * 5120 / 32 * 8;              // per-block {even, odd} sums of the staged activation
constexpr uint32_t SBUF = 40960;                          // this CTA's ssd state rows (<= 80 x 128 fp32)
constexpr uint32_t SROWS = SBUF / 512;
constexpr uint32_t HBUF = 10240;                          // hidden vector(s) (B x d_model fp16)
constexpr uint32_t BSLOTS = 4;                            // (seq, group) B / C vector slots in phase B
constexpr uint32_t NCH_MAX = 4;                           // out_proj K chunks (partial slots)
constexpr uint32_t LT_MAX = 64;                           // layers whose table entries fit in smem
constexpr uint32_t OFF_RING = 0;
constexpr uint32_t OFF_X = OFF_RING + RING * STAGE;
constexpr uint32_t OFF_XSUM = OFF_X + XBUF;
constexpr uint32_t OFF_PART = OFF_XSUM + XSUM;
constexpr uint32_t OFF_S = OFF_PART + PART;
constexpr uint32_t OFF_H = OFF_S + SBUF;
constexpr uint32_t OFF_BC = OFF_H + HBUF;                 // BSLOTS x {B, C} x 128 halves
constexpr uint32_t OFF_ROWV = OFF_BC + BSLOTS * 512;      // SROWS x 6 words: 5 per-layer floats + row info
constexpr uint32_t OFF_RSLOT = OFF_ROWV + SROWS * 6 * 4;  // SROWS slot ids + BSLOTS (seq, group) keys
constexpr uint32_t OFF_LT = OFF_RSLOT + 128;              // layer table
constexpr uint32_t OFF_BAR = OFF_LT + LT_MAX * sizeof(PLayer);
constexpr uint32_t N_BARS = 2 * RING + 2;
constexpr uint32_t OFF_MISC = OFF_BAR + N_BARS * 8;       // red[32], tok[2], abort, slots, arg v[32] / i[32]
constexpr uint32_t OFF_ZERO = OFF_MISC + 512;             // 16 zero bytes (masked MMA fragments)
// The in_proj epilogue: thread t < EPI_T owns output (tile t / (16 B), row (t / B) % 16, seq t % B).
constexpr uint32_t EPI_T = 160;
constexpr uint32_t OFF_CONV = OFF_ZERO + 16;              // per owning thread: its conv row's inputs (16 B)
constexpr uint32_t OFF_EPI = OFF_CONV + EPI_T * 16;       // per owning thread: packed output mapping
constexpr uint32_t SMEM_BYTES = OFF_EPI + EPI_T * 4;
// packed mapping word: in_proj row (bits 0..19) | owns an output | conv row | B / C / dt row | local state row << 24
constexpr uint32_t EPI_OWN = 1u << 20, EPI_CONV = 1u << 21, EPI_SPEC = 1u << 22;
constexpr uint64_t SPIN_NS = 2000000000ull;
static_assert(SMEM_BYTES <= 232448, "persistent decode kernel exceeds 227 KB of shared memory");
static_assert(sizeof(PLayer) % 8 == 0 && OFF_BAR % 8 == 0, "layer table / barriers misaligned");
static_assert(SEG_MAX * 16 * (128 + 16) <= STAGE, "INT4 chunk does not fit a stage");

__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void cons_sync() { asm volatile("bar.sync 1, %0;" ::"n"(CONS) : "memory"); }
__device__ __forceinline__ void mbar_init1(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_arrive1(uint32_t bar) {
    asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect(uint32_t bar, uint32_t bytes) {
    asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}" ::"r"(bar),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Phase wait: the common case (already complete) costs one try_wait; the clock is
// read only once the wait actually blocks. Gives up on the CTA abort flag or after 2 s.
__device__ __forceinline__ bool mbar_wait_ab(uint32_t bar, uint32_t parity, volatile int* abort) {
    if (mbar_try(bar, parity)) return true;
    const uint64_t t0 = gtimer();
    while (true) {
        if (mbar_try(bar, parity)) return true;
        if (*abort) return false;
        if (gtimer() - t0 > SPIN_NS) { *abort = 1; return false; }
    }
}

// Barrier over the consumer threads that also ORs `c` across them: every consumer gets the
// same answer, so decisions to leave (a bounded wait gave up somewhere) never diverge
// between warps that must meet at the next barrier.
__device__ __forceinline__ bool cons_any(bool c) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, %2, p;\n selp.u32 %0, 1, 0, q;\n}"
        : "=r"(r)
        : "r"((uint32_t)c), "n"(CONS)
        : "memory");
    return r != 0;
}

// Grid barrier over the consumer threads of every CTA (the producer warp never joins).
__device__ __forceinline__ bool grid_sync(const PParams& p, uint32_t& gen, volatile int* abort) {
    cons_sync();
    if (threadIdx.x == 0) {
        gen += 1;
        asm volatile("fence.acq_rel.gpu;\n red.relaxed.gpu.global.add.u32 [%0], 1;" ::"l"(p.bar) : "memory");
        const uint32_t target = gen * gridDim.x;
        uint64_t t0 = 0;
        for (uint32_t it = 1;; ++it) {
            uint32_t v;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p.bar) : "memory");
            if ((int32_t)(v - target) >= 0) break;
            if ((it & 31) == 0) {
                if (*abort) break;
                if (*reinterpret_cast<volatile int*>(p.err)) { *abort = 1; break; }   // another CTA gave up
                const uint64_t t = gtimer();
                if (!t0) t0 = t;
                else if (t - t0 > SPIN_NS) { *abort = 1; atomicExch(p.err, 1); break; }
            }
        }
    }
    return !cons_any(*abort != 0);
}

// ---- exchange words: {32-bit payload, 32-bit epoch} stored as one 64-bit word, so a reader
// that sees the epoch also sees the payload (no fence, no flag). Relaxed gpu-scope accesses
// (L2, never a stale L1 line).
__device__ __forceinline__ uint64_t mb_word(uint32_t payload, uint32_t tag) {
    return ((uint64_t)tag << 32) | payload;
}
__device__ __forceinline__ void mb_put(uint64_t* a, uint64_t w) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(a), "l"(w) : "memory");
}
__device__ __forceinline__ uint64_t mb_ld(const uint64_t* a) {
    uint64_t v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
    return v;
}
__device__ __forceinline__ void mb_ld2(const uint64_t* a, uint64_t& x, uint64_t& y) {
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(x), "=l"(y) : "l"(a) : "memory");
}
__device__ __forceinline__ bool mb_ok(uint64_t w, uint32_t tag) { return (uint32_t)(w >> 32) == tag; }
// Slow path: re-reads one word until it carries `tag`. Gives up (returns a word whose tag is
// wrong) on the CTA abort flag, on the device error word (another CTA gave up) or after 2 s,
// setting both flags.
__device__ __forceinline__ uint64_t mb_spin(const uint64_t* a, uint32_t tag, volatile int* abort, int* err) {
    uint64_t t0 = 0;
    for (uint32_t it = 1;; ++it) {
        const uint64_t w = mb_ld(a);
        if (mb_ok(w, tag)) return w;
        if ((it & 15) == 0) {
            if (*abort) return w;
            if (*reinterpret_cast<volatile int*>(err)) { *abort = 1; return w; }
            const uint64_t t = gtimer();
            if (!t0) t0 = t;
            else if (t - t0 > SPIN_NS) { *abort = 1; atomicExch(err, 1); return w; }
        }
        __nanosleep(it < 8 ? 64 : 256);
    }
}
__device__ __forceinline__ void mb_need(const uint64_t* a, uint32_t tag, uint64_t& w, volatile int* abort, int* err) {
    if (!mb_ok(w, tag)) w = mb_spin(a, tag, abort, err);
}

// Swizzled shared-memory offset of 16-byte chunk `j` (0..7) of 128-byte segment `s` of
// tile row `r` (rows of seg segments): the tensor map's 128-byte swizzle XORs the chunk
// index with the row's 128-byte line index mod 8. With an odd seg the 8 rows an MMA
// fragment reads land on 8 different chunk positions (no bank conflicts).
__device__ __forceinline__ uint32_t swz(uint32_t r, uint32_t seg, uint32_t s, uint32_t j) {
    const uint32_t line = r * seg + s;
    return line * 128 + ((j ^ (line & 7)) << 4);
}

// Accumulator start of a block from its {even, odd} activation sums (dequant_word_fold's bias).
__device__ __forceinline__ float fold_bias(float2 s) { return lssm::fold_bias(s.x, s.y); }

// Two k16 MMAs of one 32-wide block j of a segment line (rows g and g + 8), the B fragment
// (bx, by | bz, bw) supplied by the caller.
__device__ __forceinline__ void mma_block(const uint8_t* ra, uint32_t rb8, uint32_t off, uint32_t bx, uint32_t by,
                                          uint32_t bz, uint32_t bw, float da[4], float db[4]) {
    const uint32_t wa = *reinterpret_cast<const uint32_t*>(ra + off);
    const uint32_t wb = *reinterpret_cast<const uint32_t*>(ra + rb8 + off);
    uint32_t qa[4], qb[4];
    dequant_word_fold(wa, qa);
    dequant_word_fold(wb, qb);
    const uint32_t a1[4] = {qa[0], qb[0], qa[1], qb[1]};
    const uint32_t a2[4] = {qa[2], qb[2], qa[3], qb[3]};
    mma_16816(da, a1, bx, by);
    mma_16816(db, a2, bz, bw);
}

// INT4 chunk (16 rows x seg*256 k) in column mode: warp w of a consumer half takes the
// whole segment s = w % HALF_WARPS (eight 32-wide blocks); warps s >= seg have no work.
// Each of the MMA's 8 columns carries one (block, sequence) pair: with one sequence,
// column j is block 8s + j; with two, the segment runs as two passes h of four blocks and
// column 2j + m is block 8s + 4h + j of sequence m. Only the lanes of a column's group
// supply that block's activation fragment (the others zero), so column n ends up holding
// sum_k W[row][k] x_n[k] of its block alone and the scales are applied once per column.
// The weights use the bias-folded dequantisation (dequant_word_fold); the folded bias of each
// block is cancelled by starting the accumulator at fold_bias of its activation sums.
// acc: rows g / g + 8 (one sequence: acc[0] / acc[2]; two: acc[0..1] / acc[2..3] per m).
__device__ __forceinline__ void consume_int4(const uint8_t* stage, uint32_t seg, uint32_t chunk, const uint4* xs,
                                             const float* xsum, uint32_t K8, uint32_t K32, uint32_t M,
                                             uint32_t zaddr, float acc[4]) {
    const uint32_t lane = threadIdx.x & 31, sgi = (threadIdx.x >> 5) % HALF_WARPS;
    if (sgi >= seg) return;
    const uint32_t g = lane >> 2, c = lane & 3;
    const uint32_t rowb = seg * 128;
    const uint32_t line = g * seg + sgi;                 // 128-byte line of row g, segment sgi
    const uint32_t sw = line & 7;                        // swizzle of the line's 16-byte chunks (one per block)
    const uint8_t* ra = stage + line * 128 + 4 * c;
    const uint32_t rb8 = 8 * rowb;
    const uint32_t blk0 = chunk * seg * 8 + sgi * 8;     // first block of the segment (whole-K index)
    const __half* sc = reinterpret_cast<const __half*>(stage + 16 * rowb) + g * seg * 8 + sgi * 8;
    if (M == 1) {
        // column g = block g; the lane's accumulator columns 2c, 2c + 1 = blocks 2c, 2c + 1.
        // The B fragment of block j is this lane's activation quad when g == j, else 16 zero
        // bytes: one shared load from a selected address (no per-register masking).
        const uint32_t xa = smem_u32(xs + (blk0 + g) * 4 + c);
        const float4 xsv = *reinterpret_cast<const float4*>(xsum + 2 * (blk0 + 2 * c));
        const float i0 = fold_bias(make_float2(xsv.x, xsv.y)), i1 = fold_bias(make_float2(xsv.z, xsv.w));
        // column 2c (an even block) accumulates in da / db, column 2c + 1 in ea / eb
        float da[4] = {i0, 0.0f, i0, 0.0f}, db[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        float ea[4] = {0.0f, i1, 0.0f, i1}, eb[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (uint32_t j = 0; j < 8; ++j) {
            uint32_t bx, by, bz, bw;
            asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(bx), "=r"(by), "=r"(bz), "=r"(bw)
                         : "r"(g == j ? xa : zaddr));
            // even and odd blocks accumulate into separate pairs: two chains of four MMAs each
            if (j & 1) mma_block(ra, rb8, (j ^ sw) << 4, bx, by, bz, bw, ea, eb);
            else mma_block(ra, rb8, (j ^ sw) << 4, bx, by, bz, bw, da, db);
        }
        const float d0 = (da[0] + db[0]) + (ea[0] + eb[0]), d1 = (da[1] + db[1]) + (ea[1] + eb[1]);
        const float d2 = (da[2] + db[2]) + (ea[2] + eb[2]), d3 = (da[3] + db[3]) + (ea[3] + eb[3]);
        const float2 sa = __half22float2(*reinterpret_cast<const __half2*>(sc + 2 * c));
        const float2 sb = __half22float2(*reinterpret_cast<const __half2*>(sc + 8 * seg * 8 + 2 * c));
        acc[0] += d0 * sa.x + d1 * sa.y;
        acc[2] += d2 * sb.x + d3 * sb.y;
        return;
    }
    // two sequences: lane column (block myj of the pass, sequence mym)
    const uint32_t myj = g >> 1, mym = g & 1;
#pragma unroll
    for (uint32_t h = 0; h < 2; ++h) {
        const uint4 xg = xs[(uint64_t)mym * K8 + (uint64_t)(blk0 + 4 * h + myj) * 4 + c];
        // accumulator start: the folded bias of the lane's columns 2c, 2c + 1 = block 4h + c of sequences 0, 1
        const float2* xs2 = reinterpret_cast<const float2*>(xsum);
        const float i0 = fold_bias(xs2[blk0 + 4 * h + c]), i1 = fold_bias(xs2[K32 + blk0 + 4 * h + c]);
        float da[4] = {i0, i1, i0, i1}, db[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (uint32_t j = 0; j < 4; ++j) {
            const bool mine = myj == j;
            const uint32_t bx = mine ? xg.x : 0u, by = mine ? xg.y : 0u, bz = mine ? xg.z : 0u, bw = mine ? xg.w : 0u;
            mma_block(ra, rb8, ((4 * h + j) ^ sw) << 4, bx, by, bz, bw, da, db);
        }
        const float sa = __half2float(sc[4 * h + c]), sb = __half2float(sc[8 * seg * 8 + 4 * h + c]);
        acc[0] += (da[0] + db[0]) * sa;
        acc[1] += (da[1] + db[1]) * sa;
        acc[2] += (da[2] + db[2]) * sb;
        acc[3] += (da[3] + db[3]) * sb;
    }
}

// fp16 chunk (lm_head, 16 rows x seg*64 k): this warp's share (within its consumer half) of
// the 16-wide k steps.
__device__ __forceinline__ void consume_f16(const uint8_t* stage, uint32_t seg, uint32_t chunk, const __half* xh,
                                            uint32_t K, uint32_t M, float acc[4]) {
    const uint32_t lane = threadIdx.x & 31, warp = (threadIdx.x >> 5) % HALF_WARPS;
    const uint32_t g = lane >> 2, c = lane & 3;
    const uint32_t nks = seg * 4;
    const bool has_x = g < M;
    const __half* xr = xh + (uint64_t)(has_x ? g : 0) * K + (uint64_t)chunk * seg * 64;
    const uint32_t k0 = (nks * warp) / HALF_WARPS, k1 = (nks * (warp + 1)) / HALF_WARPS;
    constexpr uint32_t MAXK = (SEG_MAX * 4 + HALF_WARPS - 1) / HALF_WARPS;
#pragma unroll
    for (uint32_t i = 0; i < MAXK; ++i) {
        // predicated like consume_int4: past-the-end steps re-read step k0 with a zero activation
        const bool live = k0 + i < k1;
        const uint32_t ks = live ? k0 + i : k0;
        const uint32_t s = ks >> 2, j = (ks & 3) * 2;
        const uint32_t a[4] = {*reinterpret_cast<const uint32_t*>(stage + swz(g, seg, s, j) + 4 * c),
                               *reinterpret_cast<const uint32_t*>(stage + swz(g + 8, seg, s, j) + 4 * c),
                               *reinterpret_cast<const uint32_t*>(stage + swz(g, seg, s, j + 1) + 4 * c),
                               *reinterpret_cast<const uint32_t*>(stage + swz(g + 8, seg, s, j + 1) + 4 * c)};
        const bool xv = has_x && live;
        const uint32_t xb0 = xv ? *reinterpret_cast<const uint32_t*>(xr + ks * 16 + 2 * c) : 0u;
        const uint32_t xb1 = xv ? *reinterpret_cast<const uint32_t*>(xr + ks * 16 + 2 * c + 8) : 0u;
        mma_16816(acc, a, xb0, xb1);
    }
}

// One staged octet q of sequence m: half(x * w * rr) (rmsnorm_f16 arithmetic) -> xbuf, in
// the INT4 MMA fragment order {x0,x4} {x1,x5} {x2,x6} {x3,x7} when frag; with frag also the
// fp32 sums of its 32-wide block's staged values at even and at odd positions within the
// octets -> xsum[m][q / 4] = {even, odd} (the four octets of a block belong to four
// consecutive threads: a quad shuffle). Every consumer thread calls it; `valid` = q < nq
// (uniform over each quad, as nq % 4 == 0).
__device__ __forceinline__ void stage_octet(uint4 xv, uint4 wv, float rr, bool frag, bool valid, uint32_t m,
                                            uint32_t q, uint32_t nq, uint8_t* xbuf, float* xsum) {
    float se = 0.0f, so = 0.0f;
    if (valid) {
        const __half* xh8 = reinterpret_cast<const __half*>(&xv);
        const __half* wh8 = reinterpret_cast<const __half*>(&wv);
        __half v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = __float2half_rn(__half2float(xh8[j]) * __half2float(wh8[j]) * rr);
        uint4 u;
        if (frag) {
            __half2 o0 = __halves2half2(v[0], v[4]), o1 = __halves2half2(v[1], v[5]);
            __half2 o2 = __halves2half2(v[2], v[6]), o3 = __halves2half2(v[3], v[7]);
            u.x = *reinterpret_cast<uint32_t*>(&o0);
            u.y = *reinterpret_cast<uint32_t*>(&o1);
            u.z = *reinterpret_cast<uint32_t*>(&o2);
            u.w = *reinterpret_cast<uint32_t*>(&o3);
#pragma unroll
            for (int j = 0; j < 8; j += 2) {
                se += __half2float(v[j]);
                so += __half2float(v[j + 1]);
            }
        } else {
            u = *reinterpret_cast<uint4*>(v);
        }
        reinterpret_cast<uint4*>(xbuf)[(uint64_t)m * nq + q] = u;
    }
    if (frag) {
        se += __shfl_xor_sync(0xffffffffu, se, 1);
        so += __shfl_xor_sync(0xffffffffu, so, 1);
        se += __shfl_xor_sync(0xffffffffu, se, 2);
        so += __shfl_xor_sync(0xffffffffu, so, 2);
        if (valid && (q & 3) == 0)
            reinterpret_cast<float2*>(xsum)[m * (nq >> 2) + (q >> 2)] = make_float2(se, so);
    }
}

// RMSNorm of M <= 2 rows of `src` (length K, K % 8 == 0, K / 8 <= NOCT * CONS) with weight
// w -> staged fp16 values (rmsnorm_f16 arithmetic, shaders/norm.metal:51-79); `frag`
// selects the INT4 MMA fragment permutation (quads x[8q + {0,4,1,5,2,6,3,7}]). Each
// thread owns up to NOCT octets of each row, loaded once (with the weights) as 16-byte
// vectors through L2 (other CTAs wrote the rows); both rows' loads are issued before
// either reduction.
__device__ void stage_norm(const __half* src, uint64_t src_stride, const uint32_t* tok, const __half* embed,
                           const __half* w, uint32_t M, uint32_t K, bool frag, uint8_t* xbuf, float* xsum, float* red) {
    const uint32_t tid = threadIdx.x, nq = K / 8;
    uint4 xv[2][NOCT], wv[NOCT];
#pragma unroll
    for (int i = 0; i < (int)NOCT; ++i) {
        const uint32_t q = tid + i * CONS;
        if (q < nq) wv[i] = __ldg(reinterpret_cast<const uint4*>(w) + q);
    }
#pragma unroll
    for (uint32_t m = 0; m < 2; ++m) {
        if (m >= M) break;
        const __half* xr = tok ? embed + (uint64_t)tok[m] * K : src + (uint64_t)m * src_stride;
#pragma unroll
        for (int i = 0; i < (int)NOCT; ++i) {
            const uint32_t q = tid + i * CONS;
            if (q < nq) xv[m][i] = __ldcg(reinterpret_cast<const uint4*>(xr) + q);
        }
    }
#pragma unroll
    for (uint32_t m = 0; m < 2; ++m) {
        if (m >= M) break;
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < (int)NOCT; ++i) {
            if (tid + i * CONS < nq) {
                const __half2* h2 = reinterpret_cast<const __half2*>(&xv[m][i]);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float2 f = __half22float2(h2[j]);
                    ss += f.x * f.x + f.y * f.y;
                }
            }
        }
        ss = warp_sum(ss);
        if ((tid & 31) == 0) red[m * 16 + (tid >> 5)] = ss;
    }
    cons_sync();
#pragma unroll
    for (uint32_t m = 0; m < 2; ++m) {
        if (m >= M) break;
        float tot = 0.0f;
#pragma unroll
        for (int i = 0; i < CONS_WARPS; ++i) tot += red[m * 16 + i];
        const float rr = rsqrtf(tot / (float)K + 1e-5f);
#pragma unroll
        for (int i = 0; i < (int)NOCT; ++i) {
            const uint32_t q = tid + i * CONS;
            stage_octet(q < nq ? xv[m][i] : make_uint4(0, 0, 0, 0), wv[i], rr, frag, q < nq, m, q, nq, xbuf, xsum);
        }
    }
    cons_sync();
}

// RMSNorm input of in_proj / lm_head, with the previous layer's residual folded in:
// per sequence m, hidden[k] = half(hidden[k] + half(sum_c opart[c][m][k])) (the out_proj
// output rounded to fp16, then hidden += block_out, mamba2_block.cpp:274-276), or
// hidden = embed[tok[m]] at layer 0. `hid` (shared memory) keeps the updated vector for
// the next layer; the normalised fp16 values go to xbuf as in stage_norm. Every SM
// computes the same vector (same inputs, same order of additions). The residual pass
// works on 4-element quads (<= NOCT per thread: K <= 2560), all slot loads in flight at once.
template <uint32_t NB>
__device__ void stage_norm_h(const float* opart, uint32_t nch, const uint32_t* tok, const __half* embed, __half* hid,
                             const __half* w, uint32_t K, bool frag, uint8_t* xbuf, float* xsum, float* red) {
    const uint32_t tid = threadIdx.x, nq = K / 8, n4 = K / 4;
    uint4 wv[NOCT];
#pragma unroll
    for (int i = 0; i < (int)NOCT; ++i) {
        const uint32_t q = tid + i * CONS;
        if (q < nq) wv[i] = __ldg(reinterpret_cast<const uint4*>(w) + q);
    }
    // slots loaded two at a time (at most 2 x NOCT float4 loads in flight per thread)
    constexpr uint32_t CB = 2;
    for (uint32_t m = 0; m < NB; ++m) {
        __half* hrow = hid + (uint64_t)m * K;
        uint2 hv[NOCT];
        float4 o[NOCT];
        // slots summed in chunk order c = 0, 1, 2, 3 (fixed)
#pragma unroll
        for (uint32_t c0 = 0; c0 < NCH_MAX; c0 += CB) {
            if (tok || c0 >= nch) break;
            float4 pa[NOCT][CB];
#pragma unroll
            for (int i = 0; i < (int)NOCT; ++i) {
                const uint32_t q = tid + i * CONS;
                if (q >= n4) continue;
#pragma unroll
                for (uint32_t c = 0; c < CB; ++c)
                    if (c0 + c < nch)
                        pa[i][c] = __ldcg(reinterpret_cast<const float4*>(opart + ((uint64_t)(c0 + c) * NB + m) * K) + q);
            }
#pragma unroll
            for (int i = 0; i < (int)NOCT; ++i) {
                const uint32_t q = tid + i * CONS;
                if (q >= n4) continue;
#pragma unroll
                for (uint32_t c = 0; c < CB; ++c) {
                    if (c0 + c >= nch) continue;
                    if (c0 + c == 0) o[i] = pa[i][0];
                    else { o[i].x += pa[i][c].x; o[i].y += pa[i][c].y; o[i].z += pa[i][c].z; o[i].w += pa[i][c].w; }
                }
            }
        }
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < (int)NOCT; ++i) {
            const uint32_t q = tid + i * CONS;
            if (q >= n4) continue;
            hv[i] = tok ? __ldcg(reinterpret_cast<const uint2*>(embed + (uint64_t)tok[m] * K) + q)
                        : reinterpret_cast<const uint2*>(hrow)[q];
            __half* h4 = reinterpret_cast<__half*>(&hv[i]);
            if (!tok) {
                const float ov[4] = {o[i].x, o[i].y, o[i].z, o[i].w};
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    h4[j] = __float2half_rn(__half2float(h4[j]) + __half2float(__float2half_rn(ov[j])));
            }
            reinterpret_cast<uint2*>(hrow)[q] = hv[i];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float f = __half2float(h4[j]);
                ss += f * f;
            }
        }
        ss = warp_sum(ss);
        if ((tid & 31) == 0) red[tid >> 5] = ss;
        cons_sync();   // also publishes hrow
        float tot = 0.0f;
#pragma unroll
        for (int i = 0; i < CONS_WARPS; ++i) tot += red[i];
        const float rr = rsqrtf(tot / (float)K + 1e-5f);
#pragma unroll
        for (int i = 0; i < (int)NOCT; ++i) {
            const uint32_t q = tid + i * CONS;
            const uint4 xv = q < nq ? reinterpret_cast<const uint4*>(hrow)[q] : make_uint4(0, 0, 0, 0);
            stage_octet(xv, wv[i], rr, frag, q < nq, m, q, nq, xbuf, xsum);
        }
        cons_sync();
    }
}

// In_proj work of CTA s (owner computes): channel units of 8 d_inner channels are dealt in
// contiguous ranges; the z rows and x rows of a unit form one 16-row tile (two 8-row
// halves), so the CTA that runs the ssd rows of a channel also computes its x and z. The
// "special" tiles hold the B, C and dt rows (16 rows at 2 d_inner + 16 k); each CTA runs
// its special tiles first, as a group of their own, so the rows every CTA polls are written
// early. That extra group costs about one more tile, so a CTA with a special tile is
// charged two units: with T = ceil((units + 2 * special tiles) / G), special tile k goes to
// CTA k, which takes T - 2 units, the other CTAs take T, and the last E CTAs one fewer
// (E = G * T - 2 * special - units). Shapes where that does not fit (more special tiles
// than CTAs, T < 2, or the reduced CTAs reaching the special ones) deal the units evenly
// (the first NU % G CTAs one more) and the special tiles to CTAs with fewer units.
struct InTiles {
    uint32_t ub, nu;      // first unit, units
    uint32_t kfirst, nsp; // first special tile index, special tiles (k = kfirst + i * G)
};
struct InPlan {
    uint32_t T, E;
    bool fold;            // special tiles charged as two units (else the even deal)
};
__host__ __device__ __forceinline__ InPlan in_plan(uint32_t G, uint32_t di, uint32_t nspec) {
    const uint32_t NU = di / 8;
    InPlan q;
    q.T = (NU + 2 * nspec + G - 1) / G;
    q.E = G * q.T - 2 * nspec - NU;
    q.fold = nspec <= G && nspec + q.E <= G && q.T >= 2;
    return q;
}
__host__ __device__ __forceinline__ InTiles in_tiles(uint32_t s, uint32_t G, uint32_t di, uint32_t nspec) {
    const InPlan q = in_plan(G, di, nspec);
    InTiles t;
    if (q.fold) {
        const uint32_t cut = G - q.E;   // CTAs >= cut take one unit fewer
        t.nsp = s < nspec ? 1u : 0u;
        t.kfirst = s;
        t.nu = q.T - 2 * t.nsp - (s >= cut ? 1u : 0u);
        t.ub = s * q.T - 2 * (s < nspec ? s : nspec) - (s > cut ? s - cut : 0u);
        return t;
    }
    const uint32_t NU = di / 8, base = NU / G, extra = NU % G;
    t.nu = base + (s < extra ? 1u : 0u);
    t.ub = s * base + (s < extra ? s : extra);
    t.kfirst = (s + G - (extra % G)) % G;
    t.nsp = t.kfirst < nspec ? (nspec - 1 - t.kfirst) / G + 1 : 0;
    return t;
}
// Upper bounds over the CTAs of units and of in_proj tiles (special + units) per CTA.
__host__ __device__ __forceinline__ uint32_t in_max_units(uint32_t G, uint32_t di, uint32_t nspec) {
    const InPlan q = in_plan(G, di, nspec);
    return q.fold ? q.T : (di / 8 + G - 1) / G;
}
__host__ __device__ __forceinline__ uint32_t in_max_tiles(uint32_t G, uint32_t di, uint32_t nspec) {
    const InPlan q = in_plan(G, di, nspec);
    return q.fold ? q.T : (di / 8 + G - 1) / G + (nspec + G - 1) / G;
}
// Row starts of the two 8-row halves of tile ti of a CTA.
__device__ __forceinline__ void in_tile_rows(const InTiles& t, uint32_t ti, uint32_t G, uint32_t di, uint32_t& h0,
                                             uint32_t& h1) {
    if (ti < t.nsp) {
        h0 = 2 * di + 16 * (t.kfirst + ti * G);
        h1 = h0 + 8;
    } else {
        const uint32_t u = t.ub + ti - t.nsp;
        h0 = 8 * u;
        h1 = di + 8 * u;
    }
}

// First-max argmax step: (v, i) replaces (bv, bi) when larger, or equal with a lower index.
__device__ __forceinline__ void argmax_take(float& bv, uint32_t& bi, float v, uint32_t i) {
    if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
}
// Warp-wide first-max over lanes of the same sequence (lane % B), B in {1, 2}.
__device__ __forceinline__ void warp_argmax(float& v, uint32_t& i, uint32_t B) {
    for (uint32_t off = 16; off >= B; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, off);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, i, off);
        argmax_take(v, i, ov, oi);
    }
}

}  // namespace

// NB = sequences (1 or 2), a template parameter so that the one-sequence kernel keeps only
// the accumulators it uses (11 warps allow 168 registers per thread); TR = the phase trace
// is recorded (p.trace set), so the untraced kernel carries no timer state.
template <uint32_t NB, bool TR>
__global__ void __launch_bounds__(THREADS, 1) k_decode_persist(PParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    uint64_t* empty = full + RING;
    uint64_t* sfull = empty + RING;       // ssd state rows landed
    uint64_t* sempty = sfull + 1;         // ssd state buffer released by the consumers
    float* red = reinterpret_cast<float*>(smem + OFF_MISC);              // 2 x 16 floats
    uint32_t* tok = reinterpret_cast<uint32_t*>(red + 32);                 // 2 tokens
    volatile int* abort = reinterpret_cast<volatile int*>(tok + 2);
    uint32_t* nslot_s = reinterpret_cast<uint32_t*>(tok + 3);
    float* argv = reinterpret_cast<float*>(smem + OFF_MISC + 256);         // 32 floats
    uint32_t* argi = reinterpret_cast<uint32_t*>(argv + 32);              // 32 ids
    PLayer* LT = reinterpret_cast<PLayer*>(smem + OFF_LT);
    float* part = reinterpret_cast<float*>(smem + OFF_PART);
    float* xsum = reinterpret_cast<float*>(smem + OFF_XSUM);
    uint8_t* xbuf = smem + OFF_X;
    float* sstate = reinterpret_cast<float*>(smem + OFF_S);
    __half* hid = reinterpret_cast<__half*>(smem + OFF_H);
    __half* bcs = reinterpret_cast<__half*>(smem + OFF_BC);
    float* rowv = reinterpret_cast<float*>(smem + OFF_ROWV);
    uint8_t* rslot = smem + OFF_RSLOT;                                     // per state row: B / C slot
    uint32_t* skey = reinterpret_cast<uint32_t*>(smem + OFF_RSLOT + 96);  // per slot: m * G + g
    const CUtensorMap* maps = static_cast<const CUtensorMap*>(p.maps);

    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t G = gridDim.x, cta = blockIdx.x;
    const uint32_t nC = (p.dm + 15) / 16, nL = (p.V + 15) / 16;
    const uint32_t nchA = p.dm / (p.seg_in * 256), nchC = p.di / (p.seg_out * 256), nchL = p.dm / (p.seg_lm * 64);
    const uint32_t uC = nC * nchC;                                  // out_proj (tile, chunk) units
    const uint32_t nspec = (2 * p.G * p.N + p.H + 15) / 16;        // B / C / dt tiles
    const InTiles tt = in_tiles(cta, G, p.di, nspec);
    const uint32_t ntA = tt.nsp + tt.nu;                            // this CTA's in_proj tiles
    const uint32_t nuC = cta < uC ? (uC - 1 - cta) / G + 1 : 0;    // this CTA's out_proj units
    const uint32_t ntL = cta < nL ? (nL - 1 - cta) / G + 1 : 0;    // lm_head tiles
    // state rows: the channels of this CTA's units, for each sequence (local row j: sequence
    // j / (8 nu), channel 8 ub + j % (8 nu))
    const uint32_t urows = 8 * tt.nu, nrows = NB * urows;
    const uint32_t GN = p.G * p.N, hpg = p.H / p.G;

    // Shapes the host checks before choosing this kernel, re-checked (identically in
    // every CTA) so a bad launch reports an error instead of overrunning shared memory.
    if (p.dconv > 4 || p.dconv < 1 || NB > 2 || NB < 1 || p.N != 128 || p.P < 32 || p.P > 256 || p.H > 65535 ||
        NB * 8 * in_max_units(G, p.di, nspec) > SROWS || p.di % 8 || p.H * p.P != p.di ||
        p.n_layer > LT_MAX || (uint64_t)NB * max(p.dm, p.di) * 2 > XBUF || (uint64_t)NB * p.dm * 2 > HBUF ||
        p.dm / 8 > NOCT * CONS || p.di / 8 > NOCT * CONS || p.seg_in > SEG_MAX || p.seg_out > SEG_MAX ||
        p.seg_lm > SEG_MAX || !(p.seg_in & 1) || !(p.seg_out & 1) || !(p.seg_lm & 1) || nchA * p.seg_in * 256 != p.dm ||
        nchC * p.seg_out * 256 != p.di || nchL * p.seg_lm * 64 != p.dm || nchC > NCH_MAX ||
        p.H % p.G || in_max_tiles(G, p.di, nspec) * 16 * NB > EPI_T || p.dm / 4 > NOCT * CONS ||
        p.proj >= (1u << 20)) {
        if (tid == 0) atomicExch(p.err, 1);
        return;
    }

    if (tid == 0) {
        for (int s = 0; s < RING; ++s) {
            mbar_init1(smem_u32(&full[s]), 1);
            mbar_init1(smem_u32(&empty[s]), HALF_WARPS);
        }
        mbar_init1(smem_u32(sfull), 1);
        mbar_init1(smem_u32(sempty), 1);
        *reinterpret_cast<uint4*>(smem + OFF_ZERO) = make_uint4(0, 0, 0, 0);
        *abort = 0;
        // distinct (seq, group) pairs of this CTA's state rows -> B / C slots
        uint32_t ns = 0;
        for (uint32_t j = 0; j < nrows; ++j) {
            const uint32_t m = j / urows, c = 8 * tt.ub + j % urows, h = c / p.P, pp = c % p.P;
            const uint32_t key = m * p.G + h / hpg;
            uint32_t sl = 0;
            while (sl < ns && skey[sl] != key) ++sl;
            if (sl == ns) {
                if (ns == BSLOTS) { atomicExch(p.err, 1); *abort = 1; break; }
                skey[ns++] = key;
            }
            rslot[j] = (uint8_t)sl;
            // (seq m, head h, channel pp) of the row, packed once: no divisions in phase B
            reinterpret_cast<uint32_t*>(rowv)[j * 6 + 5] = (m << 24) | (pp << 16) | h;
        }
        *nslot_s = ns;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (tid < NB) tok[tid] = p.cur[tid];
    for (uint32_t i = tid; i < p.n_layer * (uint32_t)(sizeof(PLayer) / 8); i += THREADS)
        reinterpret_cast<uint64_t*>(LT)[i] = reinterpret_cast<const uint64_t*>(p.layers)[i];
    __syncthreads();
    if (*abort) return;
    const uint32_t nslot = *nslot_s;

    const uint64_t tbase = (uint64_t)cta * (p.n_layer * TRACE_PER_LAYER + TRACE_LM);
    const uint32_t lmb = p.n_layer * TRACE_PER_LAYER;

    if (tid >= CONS) {
        // ------------------------------------------------------------ producer
        if (tid == CONS) {
            const uint64_t pol = evict_first_policy();
            uint32_t slot = 0, phase = 0, sphase = 0;
            int last_phase[RING];
            for (int s = 0; s < RING; ++s) last_phase[s] = -1;
            bool state_issued = false;
            // next free stage (bounded wait); ~0u on abort
            auto take = [&]() -> uint32_t {
                if (!mbar_wait_ab(smem_u32(&empty[slot]), phase ^ 1, abort)) return ~0u;
                return slot;
            };
            auto advance = [&]() {
                last_phase[slot] = (int)phase;
                if (++slot == RING) { slot = 0; phase ^= 1; }
            };
            // one in_proj (tile, chunk): two 8-row halves starting at rows h0 and h1
            auto put_in = [&](const CUtensorMap* mw, uint32_t seg, uint32_t h0, uint32_t h1, uint32_t c) -> bool {
                const uint32_t s = take();
                if (s == ~0u) return false;
                const uint32_t dst = smem_u32(smem + OFF_RING + s * STAGE), bar = smem_u32(&full[s]);
                const int32_t cs = (int32_t)(c * seg);
                mbar_expect(bar, 16 * seg * (128 + 16));
                tma3(dst, mw, 0, cs, (int32_t)h0, bar, pol);
                tma3(dst + 8 * seg * 128, mw, 0, cs, (int32_t)h1, bar, pol);
                tma2(dst + 16 * seg * 128, mw + 1, cs * 8, (int32_t)h0, bar, pol);
                tma2(dst + 16 * seg * 128 + 8 * seg * 16, mw + 1, cs * 8, (int32_t)h1, bar, pol);
                advance();
                return true;
            };
            // one INT4 (tile, chunk) unit: weights (3-D, swizzled) + scales (2-D)
            auto put_int4 = [&](const CUtensorMap* mw, uint32_t seg, uint32_t u, uint32_t nch) -> bool {
                const uint32_t s = take();
                if (s == ~0u) return false;
                const uint32_t dst = smem_u32(smem + OFF_RING + s * STAGE), bar = smem_u32(&full[s]);
                const int32_t row0 = (int32_t)((u / nch) * 16), c = (int32_t)(u % nch);
                mbar_expect(bar, 16 * seg * (128 + 16));
                tma3(dst, mw, 0, c * (int32_t)seg, row0, bar, pol);
                tma2(dst + 16 * seg * 128, mw + 1, c * (int32_t)seg * 8, row0, bar, pol);
                advance();
                return true;
            };
            const uint32_t sbytes = nrows * p.N * 4;
            bool ok = true;
            for (uint32_t step = 0; step < p.n_steps && ok; ++step) {
                for (uint32_t l = 0; l < p.n_layer && ok; ++l) {
                    const CUtensorMap* mp = maps + 4 * l;
                    // this layer's ssd state rows, as soon as the previous layer's are released
                    // (ahead of this layer's weights, so the state lands long before phase B)
                    if (!mbar_wait_ab(smem_u32(sempty), sphase ^ 1, abort)) { ok = false; break; }
                    if (sbytes) {
                        mbar_expect(smem_u32(sfull), sbytes);
                        for (uint32_t m = 0; m < NB; ++m)
                            bulk_g2s(smem_u32(smem + OFF_S + m * urows * p.N * 4),
                                     LT[l].ssd_state + ((uint64_t)m * p.di + 8 * tt.ub) * p.N, urows * p.N * 4,
                                     smem_u32(sfull));
                    } else {
                        mbar_arrive1(smem_u32(sfull));
                    }
                    state_issued = true;
                    sphase ^= 1;
                    for (uint32_t ti = 0; ti < ntA && ok; ++ti)
                        for (uint32_t c = 0; c < nchA && ok; ++c) {
                            uint32_t h0, h1;
                            in_tile_rows(tt, ti, G, p.di, h0, h1);
                            ok = put_in(mp, p.seg_in, h0, h1, c);
                            if (TR && step == 0 && ti == 0 && c == 0)
                                p.trace[tbase + l * TRACE_PER_LAYER + 8] = gtimer();
                        }
                    if (!ok) break;
                    for (uint32_t i = 0; i < nuC && ok; ++i) ok = put_int4(mp + 2, p.seg_out, cta + i * G, nchC);
                }
                const CUtensorMap* ml = maps + 4 * p.n_layer;
                for (uint32_t ti = 0; ti < ntL && ok; ++ti)
                    for (uint32_t c = 0; c < nchL && ok; ++c) {
                        const uint32_t s = take();
                        if (s == ~0u) { ok = false; break; }
                        const uint32_t dst = smem_u32(smem + OFF_RING + s * STAGE), bar = smem_u32(&full[s]);
                        mbar_expect(bar, 16 * p.seg_lm * 128);
                        tma3(dst, ml, 0, (int32_t)(c * p.seg_lm), (int32_t)((cta + ti * G) * 16), bar, pol);
                        advance();
                        if (TR && step == 0 && ti == 0 && c == 0) p.trace[tbase + lmb + 5] = gtimer();
                    }
            }
            // every issued copy must land before the CTA exits (bounded)
            for (int s = 0; s < RING; ++s)
                if (last_phase[s] >= 0) bar_wait_bounded(smem_u32(&full[s]), (uint32_t)last_phase[s]);
            if (state_issued) bar_wait_bounded(smem_u32(sfull), sphase ^ 1);
        }
        return;
    }

    // ---------------------------------------------------------------- consumers
    uint32_t slot = 0, phase = 0, gen = 0, sphase = 0;
    uint32_t sn = 0;                       // ring stages passed (all consumers alike)
    const uint32_t half = warp / HALF_WARPS;   // this warp consumes the stages sn with sn % 2 == half
    uint64_t wait_ns = 0;   // trace: warp 0's time blocked on the ring in this layer

    // Consume `nt` (<= TG) units of this CTA starting at unit ordinal i0: units are
    // (tile, chunk) pairs when `split` (one chunk each), else whole tiles of `nch`
    // chunks. Each stage is consumed by one half of the warps (alternating); accumulated
    // per unit in registers; every warp's partial sums (zero for units it had no stage of)
    // then go to shared memory (readable after the closing barrier).
    auto consume_group = [&](bool int4, uint32_t seg, uint32_t nch, uint32_t K, bool split, uint32_t i0,
                             uint32_t nt) -> bool {
        float acc[TG][4];
        bool bad = false;   // a bounded ring wait gave up: skip the rest, leave together below
#pragma unroll
        for (uint32_t ti = 0; ti < TG; ++ti) {
            acc[ti][0] = acc[ti][1] = acc[ti][2] = acc[ti][3] = 0.0f;
            if (ti < nt && !bad) {
                const uint32_t u = cta + (i0 + ti) * G;
                const uint32_t c0 = split ? u % nch : 0, c1 = split ? c0 + 1 : nch;
                for (uint32_t c = c0; c < c1; ++c) {
                    if ((sn & 1) == half) {
                        const uint64_t w0 = (TR && tid == 0) ? gtimer() : 0;
                        if (!mbar_wait_ab(smem_u32(&full[slot]), phase, abort)) { bad = true; break; }
                        if (TR && tid == 0) wait_ns += gtimer() - w0;
                        const uint8_t* stage = smem + OFF_RING + slot * STAGE;
                        if (int4)
                            consume_int4(stage, seg, c, reinterpret_cast<const uint4*>(xbuf), xsum, K / 8, K / 32,
                                         NB, smem_u32(smem + OFF_ZERO), acc[ti]);
                        else consume_f16(stage, seg, c, reinterpret_cast<const __half*>(xbuf), K, NB, acc[ti]);
                        __syncwarp();
                        if (lane == 0) mbar_arrive1(smem_u32(&empty[slot]));
                    }
                    ++sn;
                    if (++slot == RING) { slot = 0; phase ^= 1; }
                }
            }
        }
        // per-warp results of rows g / g + 8 -> part[ti][warp][g] = {(g, m0), (g, m1), (g+8, m0), (g+8, m1)}:
        // INT4 columns are (block, sequence) pairs, summed over the quad's lanes; fp16 (lm_head)
        // columns are the sequences themselves, held by the quad's lane c = 0
#pragma unroll
        for (uint32_t ti = 0; ti < TG; ++ti) {
            if (ti >= nt) continue;
            float v[4] = {acc[ti][0], acc[ti][1], acc[ti][2], acc[ti][3]};
            if (int4) {
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    v[q] += __shfl_xor_sync(0xffffffffu, v[q], 1);
                    v[q] += __shfl_xor_sync(0xffffffffu, v[q], 2);
                }
            }
            if ((lane & 3) == 0)
                *reinterpret_cast<float4*>(part + ((ti * CONS_WARPS + warp) * 8 + (lane >> 2)) * 4) =
                    make_float4(v[0], v[1], v[2], v[3]);
        }
        return !cons_any(bad || *abort);
    };
    // Cross-warp sum of output (unit ordinal ti within the group, row, sequence m).
    auto reduce_item = [&](uint32_t ti, uint32_t row, uint32_t m) -> float {
        const uint32_t idx = ((row >> 3) << 1) + m;
        float s = 0.0f;
#pragma unroll
        for (int w = 0; w < CONS_WARPS; ++w) s += part[((ti * CONS_WARPS + w) * 8 + (row & 7)) * 4 + idx];
        return s;
    };
    // All units of a split-K GEMV phase: groups of TG units -> partial-sum slots
    // slots[(chunk * B + m) * N + row].
    auto gemv_phase = [&](uint32_t seg, uint32_t nch, uint32_t K, uint32_t N, uint32_t nu, float* slots) -> bool {
        for (uint32_t i0 = 0; i0 < nu; i0 += TG) {
            const uint32_t nt = min(TG, nu - i0);
            if (!consume_group(true, seg, nch, K, true, i0, nt)) return false;
            if (tid < nt * 16 * NB) {
                const uint32_t ti = tid / (16 * NB), row = (tid / NB) % 16, m = tid % NB;
                const uint32_t u = cta + (i0 + ti) * G, r = (u / nch) * 16 + row;
                if (r < N) slots[((uint64_t)(u % nch) * NB + m) * N + r] = reduce_item(ti, row, m);
            }
            cons_sync();   // partial sums reused by the next group
        }
        return true;
    };
    // Each thread t < EPI_T owns one (tile ordinal, row, seq) output of in_proj for the
    // epilogue; its mapping is packed into shared memory once, so no registers carry it
    // through the layer loop.
    const uint32_t tiA = tid / (16 * NB), rowA = (tid / NB) % 16, mA = tid % NB;
    if (tid < EPI_T) {
        uint32_t w = 0;
        if (tiA < ntA) {
            uint32_t hA0, hA1;
            in_tile_rows(tt, tiA, G, p.di, hA0, hA1);
            const uint32_t rA = rowA < 8 ? hA0 + rowA : hA1 + rowA - 8;   // in_proj output row
            w = rA | EPI_OWN;
            if (rA >= p.di && rA < p.di + p.xd) w |= EPI_CONV;
            if (tiA < tt.nsp) w |= EPI_SPEC;                               // B / C / dt rows: published
            else w |= (mA * urows + (tiA - tt.nsp) * 8 + (rowA & 7)) << 24;   // unit rows: local state row
        }
        reinterpret_cast<uint32_t*>(smem + OFF_EPI)[tid] = w;
    }

    bool ok = true;
    for (uint32_t step = 0; step < p.n_steps && ok; ++step) {
        const bool tr = TR && step == 0 && tid == 0;
        auto stamp = [&](uint32_t idx) {
            if (tr) p.trace[tbase + idx] = gtimer();
        };
        for (uint32_t l = 0; l < p.n_layer && ok; ++l) {
            const PLayer& L = LT[l];
            const uint32_t lb = l * TRACE_PER_LAYER;
            const uint32_t ep = p.epoch0 + step * p.n_layer + l;   // tag of this layer's in_proj exchange words
            stamp(lb + 0);
            wait_ns = 0;
            // ---- loads consumed only in this layer's in_proj epilogue (issued first, waited
            // late; kept as raw fp16 bits so no conversion waits on them)
            __half cwh[4], csh[4], cbh = __ushort_as_half(0);
#pragma unroll
            for (uint32_t k = 0; k < 4; ++k) cwh[k] = csh[k] = __ushort_as_half(0);
            const uint32_t ew0 = tid < EPI_T ? reinterpret_cast<const uint32_t*>(smem + OFF_EPI)[tid] : 0u;
            const bool convA = ew0 & EPI_CONV;
            if (convA) {
                const uint32_t dA = (ew0 & 0xFFFFFu) - p.di;
                const __half* wrow = L.conv_w + (uint64_t)dA * p.dconv;
                const __half* srow = L.conv_state + ((uint64_t)mA * p.xd + dA) * p.dconv;
#pragma unroll
                for (uint32_t k = 0; k < 4; ++k)
                    if (k < p.dconv) { cwh[k] = wrow[k]; csh[k] = srow[k]; }
                cbh = L.conv_b[dA];
            }
            // ---- A: residual + RMSNorm, in_proj tiles (all K chunks of a tile), epilogue:
            // z / dt and, for xBC rows, conv-state roll + conv + SiLU -> exchange words
            stage_norm_h<NB>(p.opart, nchC, l == 0 ? tok : nullptr, p.embed, hid, L.norm_w, p.dm, true, xbuf, xsum,
                         red);
            // park the conv inputs in this thread's shared-memory slot: no registers held across in_proj
            if (convA) {
                const __half2 c01 = __halves2half2(cwh[0], cwh[1]), c23 = __halves2half2(cwh[2], cwh[3]);
                const __half2 s12 = __halves2half2(csh[1], csh[2]), s3b = __halves2half2(csh[3], cbh);
                *reinterpret_cast<uint4*>(smem + OFF_CONV + tid * 16) =
                    make_uint4(*reinterpret_cast<const uint32_t*>(&c01), *reinterpret_cast<const uint32_t*>(&c23),
                               *reinterpret_cast<const uint32_t*>(&s12), *reinterpret_cast<const uint32_t*>(&s3b));
            }
            stamp(lb + 1);
            // special tiles form their own group(s), so their rows are published before the units run
            for (uint32_t g0 = 0, nt = 0; g0 < ntA && ok; g0 += nt) {
                nt = g0 < tt.nsp ? min(TG, tt.nsp - g0) : min(TG, ntA - g0);
                if (!consume_group(true, p.seg_in, nchA, p.dm, false, g0, nt)) { ok = false; break; }
                const uint32_t ew = tid < EPI_T ? reinterpret_cast<const uint32_t*>(smem + OFF_EPI)[tid] : 0u;
                const uint32_t rA = ew & 0xFFFFFu;
                if ((ew & EPI_OWN) && tiA >= g0 && tiA < g0 + nt && rA < p.proj) {
                    __half vh = __float2half_rn(reduce_item(tiA - g0, rowA, mA));
                    if (ew & EPI_CONV) {
                        const uint32_t dA = rA - p.di;
                        // conv-state roll + depthwise conv + SiLU (k_conv_update_silu_split arithmetic)
                        const uint4 cv = *reinterpret_cast<const uint4*>(smem + OFF_CONV + tid * 16);
                        const __half* cvh = reinterpret_cast<const __half*>(&cv);
                        const __half cwh[4] = {cvh[0], cvh[1], cvh[2], cvh[3]};
                        const __half csh[4] = {__ushort_as_half(0), cvh[4], cvh[5], cvh[6]};
                        const __half cbh = cvh[7];
                        __half* st = L.conv_state + ((uint64_t)mA * p.xd + dA) * p.dconv;
                        float acc = __half2float(cbh);
#pragma unroll
                        for (uint32_t k = 0; k < 3; ++k)
                            if (k + 1 < p.dconv) {
                                st[k] = csh[k + 1];
                                acc += __half2float(csh[k + 1]) * __half2float(cwh[k]);
                            }
                        st[p.dconv - 1] = vh;
                        __half wl = cwh[0];
#pragma unroll
                        for (uint32_t k = 1; k < 4; ++k)
                            if (k == p.dconv - 1) wl = cwh[k];
                        acc += __half2float(vh) * __half2float(wl);
                        vh = __float2half_rn(silu(__half2float(__float2half_rn(acc))));
                    }
                    if (ew & EPI_SPEC) mb_put(p.mb_in + (uint64_t)mA * p.proj + rA, mb_word(__half_as_ushort(vh), ep));
                    else rowv[(ew >> 24) * 6 + (rowA < 8 ? 4 : 3)] = __half2float(vh);   // z / x of an own row
                }
                cons_sync();   // partial sums reused by the next group
            }
            stamp(lb + 2);
            if (tr) p.trace[tbase + lb + 9] = wait_ns;   // warp 0's ring wait during in_proj
            if (!ok) break;
            // ---- B: ssd_step + gate over this CTA's state rows. No grid barrier: the B / C
            // vectors of its (seq, group) slots and each row's x, z and dt are polled from the
            // exchange words of this layer (one parallel round of loads, then re-reads of any
            // word not yet written)
            {
                if (tid < nslot * 64) {
                    const uint32_t sl = tid >> 6, w = tid & 63, key = skey[sl], m = key / p.G, g = key % p.G;
                    const uint64_t* a = p.mb_in + (uint64_t)m * p.proj + 2 * p.di + (w < 32 ? 0 : GN) + g * p.N +
                                        (w & 31) * 4;
                    uint64_t v[4];
                    mb_ld2(a, v[0], v[1]);
                    mb_ld2(a + 2, v[2], v[3]);
#pragma unroll
                    for (int j = 0; j < 4; ++j) mb_need(a + j, ep, v[j], abort, p.err);
                    *reinterpret_cast<uint2*>(bcs + sl * 256 + (w < 32 ? 0 : 128) + (w & 31) * 4) =
                        make_uint2((uint32_t)(v[0] & 0xFFFF) | ((uint32_t)v[1] << 16),
                                   (uint32_t)(v[2] & 0xFFFF) | ((uint32_t)v[3] << 16));
                }
                if (tid < nrows) {
                    // x and z of the row came from this CTA's own in_proj epilogue (rv[3], rv[4])
                    const uint32_t info = reinterpret_cast<const uint32_t*>(rowv)[tid * 6 + 5];
                    const uint32_t m = info >> 24, h = info & 0xFFFF;
                    const uint64_t* adt = p.mb_in + (uint64_t)m * p.proj + p.di + p.xd + h;   // dt (raw)
                    uint64_t wdt = mb_ld(adt);
                    const float A = -expf(__half2float(L.A_log[h]));
                    const float dtb = __half2float(L.dt_bias[h]), Dh = __half2float(L.D[h]);
                    mb_need(adt, ep, wdt, abort, p.err);
                    const float dt =
                        fminf(fmaxf(softplus(__half2float(__ushort_as_half((uint16_t)wdt)) + dtb), 1e-6f), 1e6f);
                    float* rv = rowv + tid * 6;
                    const float xv = rv[3];
                    rv[0] = expf(A * dt);
                    rv[1] = dt * xv;
                    rv[2] = Dh;
                }
                const bool sbad = !mbar_wait_ab(smem_u32(sfull), sphase, abort);
                sphase ^= 1;
                if (cons_any(sbad || *abort)) { ok = false; break; }
                stamp(lb + 3);
                for (uint32_t j0 = warp; j0 < nrows; j0 += 2 * CONS_WARPS) {
                    float a2[2];
                    float4 v2[2];
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        const uint32_t j = min(j0 + q * CONS_WARPS, nrows - 1);
                        const __half* bv = bcs + rslot[j] * 256;
                        const float* rv = rowv + j * 6;
                        const uint2 bu = *reinterpret_cast<const uint2*>(bv + lane * 4);
                        const uint2 cu = *reinterpret_cast<const uint2*>(bv + 128 + lane * 4);
                        const float2 b01 = __half22float2(*reinterpret_cast<const __half2*>(&bu.x));
                        const float2 b23 = __half22float2(*reinterpret_cast<const __half2*>(&bu.y));
                        const float2 c01 = __half22float2(*reinterpret_cast<const __half2*>(&cu.x));
                        const float2 c23 = __half22float2(*reinterpret_cast<const __half2*>(&cu.y));
                        const float dec = rv[0], dtx = rv[1];
                        float4 v = *reinterpret_cast<const float4*>(sstate + (uint64_t)j * p.N + lane * 4);
                        v.x = dec * v.x + b01.x * dtx;
                        v.y = dec * v.y + b01.y * dtx;
                        v.z = dec * v.z + b23.x * dtx;
                        v.w = dec * v.w + b23.y * dtx;
                        v2[q] = v;
                        a2[q] = c01.x * v.x + c01.y * v.y + c23.x * v.z + c23.y * v.w;
                    }
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) {
                        a2[0] += __shfl_xor_sync(0xffffffffu, a2[0], o);
                        a2[1] += __shfl_xor_sync(0xffffffffu, a2[1], o);
                    }
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        const uint32_t j = j0 + q * CONS_WARPS;
                        if (j >= nrows) continue;
                        const float* rv = rowv + j * 6;
                        const uint32_t info = reinterpret_cast<const uint32_t*>(rv)[5];
                        const uint32_t m = info >> 24, pp = (info >> 16) & 0xFF, h = info & 0xFFFF;
                        // the new state goes back into the shared buffer; one bulk copy per
                        // sequence stores the rows after the loop
                        *reinterpret_cast<float4*>(sstate + (uint64_t)j * p.N + lane * 4) = v2[q];
                        if (lane == 0) {
                            const float yh = __half2float(__float2half_rn(a2[q] + rv[2] * rv[3]));
                            p.gated[(uint64_t)m * p.di + h * p.P + pp] = __float2half_rn(silu(rv[4]) * yh);
                        }
                    }
                }
            }
            if (!ok) break;
            // the updated state rows (shared memory, generic proxy) are stored by the async proxy:
            // bulk copies issued here, not waited for by the grid barrier's fence, and completed
            // before the buffer is handed back to the producer
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            cons_sync();
            if (tid == 0 && urows) {
                for (uint32_t m = 0; m < NB; ++m)
                    bulk_s2g(L.ssd_state + ((uint64_t)m * p.di + 8 * tt.ub) * p.N,
                             smem_u32(smem + OFF_S + m * urows * p.N * 4), urows * p.N * 4);
                bulk_commit();
            }
            stamp(lb + 4);
            if (!grid_sync(p, gen, abort)) { ok = false; break; }
            if (tid == 0) {
                bulk_wait_all();
                mbar_arrive1(smem_u32(sempty));   // state stored; the buffer may be refilled
            }
            stamp(lb + 5);
            // ---- C: RMSNorm(gated), out_proj (tile, chunk) units -> out_proj slots
            stage_norm(p.gated, p.di, nullptr, nullptr, L.mixer_norm_w, NB, p.di, true, xbuf, xsum, red);
            stamp(lb + 6);
            if (!gemv_phase(p.seg_out, nchC, p.di, p.dm, nuC, p.opart)) { ok = false; break; }
            stamp(lb + 7);

            if (!grid_sync(p, gen, abort)) { ok = false; break; }
        }
        if (!ok) break;
        // ---- residual + norm_f + lm_head + first-max argmax partials
        wait_ns = 0;
        stage_norm_h<NB>(p.opart, nchC, nullptr, p.embed, hid, p.norm_f, p.dm, false, xbuf, xsum, red);
        stamp(lmb + 0);
        float bv = -INFINITY;
        uint32_t bi = 0xFFFFFFFFu;
        for (uint32_t g0 = 0; g0 < ntL && ok; g0 += TG) {
            const uint32_t nt = min(TG, ntL - g0);
            if (!consume_group(false, p.seg_lm, nchL, p.dm, false, g0, nt)) { ok = false; break; }
            if (tid < nt * 16 * NB) {
                const uint32_t ti = tid / (16 * NB), row = (tid / NB) % 16, m = tid % NB;
                const uint32_t r = (cta + (g0 + ti) * G) * 16 + row;
                if (r < p.V) {
                    const __half vh = __float2half_rn(reduce_item(ti, row, m));
                    p.logits[(uint64_t)m * p.V + r] = vh;
                    const float f = __half2float(vh);
                    if (f > bv) { bv = f; bi = r; }        // rows arrive in increasing order per thread
                }
            }
            cons_sync();
        }
        if (!ok) break;
        if (tr) p.trace[tbase + lmb + 4] = wait_ns;
        // CTA first-max per sequence (thread tid serves sequence tid % B)
        warp_argmax(bv, bi, NB);
        if (lane < NB) { argv[warp * 2 + lane] = bv; argi[warp * 2 + lane] = bi; }
        cons_sync();
        if (tid < NB) {
            float v = -INFINITY;
            uint32_t ix = 0xFFFFFFFFu;
            for (uint32_t w = 0; w < CONS_WARPS; ++w) argmax_take(v, ix, argv[w * 2 + tid], argi[w * 2 + tid]);
            p.part_val[(uint64_t)cta * NB + tid] = v;
            p.part_idx[(uint64_t)cta * NB + tid] = ix;
        }
        stamp(lmb + 1);
        if (!grid_sync(p, gen, abort)) { ok = false; break; }
        stamp(lmb + 2);
        {
            // all CTAs' partials in one parallel round of loads (entry e serves sequence e % B)
            float v = -INFINITY;
            uint32_t ix = 0xFFFFFFFFu;
            for (uint32_t e = tid; e < G * NB; e += CONS)
                argmax_take(v, ix, __ldcg(p.part_val + e), __ldcg(p.part_idx + e));
            warp_argmax(v, ix, NB);
            if (lane < NB) { argv[warp * 2 + lane] = v; argi[warp * 2 + lane] = ix; }
            cons_sync();
            if (tid < NB) {
                const uint32_t m = tid;
                float bv2 = -INFINITY;
                uint32_t bi2 = 0xFFFFFFFFu;
                for (uint32_t w = 0; w < CONS_WARPS; ++w) argmax_take(bv2, bi2, argv[w * 2 + m], argi[w * 2 + m]);
                const float l0 = __half2float(__ldcg(p.logits + (uint64_t)m * p.V));
                uint32_t pick = bi2 == 0xFFFFFFFFu ? 0u : bi2;
                if (l0 != l0) pick = 0;
                tok[m] = pick;
                if (cta == 0) {
                    p.history[(uint64_t)m * p.hist_stride + step] = pick;
                    p.cur[m] = pick;
                }
            }
            cons_sync();
        }
        stamp(lmb + 3);
    }
    if (tid == 0) bulk_wait_all();   // no state store still reading shared memory at exit
    if (!ok) {
        *abort = 1;
        if (tid == 0) atomicExch(p.err, 1);
    }
}

// Host launcher: cooperative launch with one CTA per SM (co-residency guaranteed or
// the launch fails, so the grid barriers cannot wait on a CTA that never runs).
cudaError_t launch_decode_persist(const PParams& prm, int sm_count, cudaStream_t s) {
    if (prm.B < 1 || prm.B > 2) return cudaErrorInvalidValue;
    const bool tr = prm.trace != nullptr;
    const void* fn = prm.B == 1 ? (tr ? (const void*)k_decode_persist<1, true> : (const void*)k_decode_persist<1, false>)
                                : (tr ? (const void*)k_decode_persist<2, true> : (const void*)k_decode_persist<2, false>);
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, THREADS, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorNotSupported;
    PParams p = prm;
    void* args[] = {&p};
    return cudaLaunchCooperativeKernel(fn, dim3(sm_count), dim3(THREADS), args, SMEM_BYTES, s);
}

// ---------------------------------------------------------------------------
//  Host helpers: shape plan and tensor maps
// ---------------------------------------------------------------------------
namespace {

// Largest odd segment count <= SEG_MAX that divides `total` segments.
uint32_t odd_seg(uint32_t total) {
    for (uint32_t s = SEG_MAX; s >= 1; s -= 2)
        if (total % s == 0) return s;
    return 1;
}

// [rows][segs][128 B] view of a row-major matrix with `row_bytes` per row; box = 16 rows
// x seg segments, 128-byte swizzle; f16 selects the element type (fp16 rows, or bytes
// holding INT4 nibble pairs).
bool map_rows(CUtensorMap* m, const void* base, uint64_t rows, uint64_t row_bytes, uint32_t seg, bool f16,
              uint32_t box_rows = 16) {
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    const uint64_t esz = f16 ? 2 : 1;
    cuuint64_t dims[3] = {128 / esz, row_bytes / 128, rows};
    cuuint64_t strides[2] = {128, row_bytes};
    cuuint32_t box[3] = {(cuuint32_t)(128 / esz), seg, box_rows};
    cuuint32_t estr[3] = {1, 1, 1};
    return enc(m, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base),
               dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// INT4_B32 scales [rows][K/32] fp16; box = 16 rows x seg*8 scales, no swizzle.
bool map_scales(CUtensorMap* m, const void* base, uint64_t rows, uint64_t K, uint32_t seg, uint32_t box_rows = 16) {
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    cuuint64_t dims[2] = {K / 32, rows};
    cuuint64_t strides[1] = {K / 16};
    cuuint32_t box[2] = {seg * 8, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

const char* decode_persist_plan(const PersistShape& sh, uint32_t* seg_in, uint32_t* seg_out, uint32_t* seg_lm) {
    const uint32_t G = sh.sm_count;
    if (sh.B < 1 || sh.B > 2) return "batch must be 1 or 2";
    if (sh.N != 128) return "d_state must be 128";
    if (sh.P < 32 || sh.P > 256) return "d_head must be 32..256";
    if (sh.H > 65535) return "more than 65535 heads";
    if (sh.dconv < 1 || sh.dconv > 4) return "d_conv must be 1..4";
    if (sh.dm % 256 || sh.di % 256) return "d_model and d_inner must be multiples of 256";
    if (sh.dm / 8 > NOCT * CONS || sh.di / 8 > NOCT * CONS) return "d_model / d_inner too wide for the staged RMSNorm";
    if ((uint64_t)sh.B * (sh.dm > sh.di ? sh.dm : sh.di) * 2 > XBUF) return "staged activations exceed 20 KB";
    if (sh.n_layer > LT_MAX) return "more than 64 layers";
    if ((uint64_t)sh.B * sh.dm * 2 > HBUF) return "hidden vectors exceed 10 KB";
    if (sh.di % 8 || sh.H * sh.P != sh.di) return "d_inner must be n_heads x d_head, a multiple of 8";
    const uint32_t nspec = (2 * sh.G * sh.N + sh.H + 15) / 16;
    if (in_max_tiles(G, sh.di, nspec) * 16 * sh.B > EPI_T) return "too many in_proj rows per SM";
    if (sh.proj >= (1u << 20)) return "in_proj wider than 2^20 rows";
    if (sh.dm / 4 > NOCT * CONS) return "d_model too wide for the residual pass (<= 2560)";
    if (sh.H % sh.G) return "n_heads not divisible by n_groups";
    if ((uint64_t)sh.B * 8 * in_max_units(G, sh.di, nspec) > SROWS) return "ssd state rows per SM exceed 40 KB";
    *seg_in = odd_seg(sh.dm / 256);
    *seg_out = odd_seg(sh.di / 256);
    *seg_lm = odd_seg(sh.dm / 64);
    if (sh.di / 256 / *seg_out > NCH_MAX) return "too many out_proj K chunks per row";
    return "";
}

size_t decode_persist_maps_bytes(uint32_t n_layer) { return (size_t)(4 * n_layer + 1) * sizeof(CUtensorMap); }

bool decode_persist_encode_maps(void* out, const PLayer* layers, const void* lm_head, const PersistShape& sh,
                                uint32_t seg_in, uint32_t seg_out, uint32_t seg_lm) {
    CUtensorMap* m = static_cast<CUtensorMap*>(out);
    for (uint32_t l = 0; l < sh.n_layer; ++l) {
        const uint8_t* in_w = layers[l].in_w;
        const uint8_t* out_w = layers[l].out_w;
        // in_proj: 8-row boxes (a stage holds two 8-row halves: z / x rows of one channel unit)
        if (!map_rows(&m[4 * l + 0], in_w, sh.proj, sh.dm / 2, seg_in, false, 8) ||
            !map_scales(&m[4 * l + 1], in_w + (size_t)sh.proj * sh.dm / 2, sh.proj, sh.dm, seg_in, 8) ||
            !map_rows(&m[4 * l + 2], out_w, sh.dm, sh.di / 2, seg_out, false) ||
            !map_scales(&m[4 * l + 3], out_w + (size_t)sh.dm * sh.di / 2, sh.dm, sh.di, seg_out))
            return false;
    }
    return map_rows(&m[4 * sh.n_layer], lm_head, sh.V, (uint64_t)sh.dm * 2, seg_lm, true);
}

}  // namespace lssm

// The in_proj work the persistent decode kernel deals to CTA s of G (the same function the
// kernel calls): out = {first unit, units, first B / C / dt tile, B / C / dt tiles}.
extern "C" void lssm_persist_in_deal(uint32_t s, uint32_t G, uint32_t d_inner, uint32_t n_spec, uint32_t* out) {
    const lssm::InTiles t = lssm::in_tiles(s, G, d_inner, n_spec);
    out[0] = t.ub;
    out[1] = t.nu;
    out[2] = t.kfirst;
    out[3] = t.nsp;
}
