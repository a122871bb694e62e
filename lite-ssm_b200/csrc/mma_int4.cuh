// mma_int4.cuh — register-operand INT4_B32 dequantisation + mma.sync helpers, bulk and
// tensor-map TMA copies, shared by the GEMV kernels and the persistent decode kernel.
//
// INT4_B32 nibble q for (row, k): byte row*(K/2) + k/2, low nibble = even k,
// q = nib < 8 ? nib : nib - 16 (shaders/linear.metal:38-61). A 32-bit word holds 8
// consecutive k. dequant_word turns it into four exact fp16 pairs (n0,n4) (n1,n5)
// (n2,n6) (n3,n7): lop3 places (nib ^ 8) in the mantissa of 1024.0 (or 16*(nib ^ 8)
// for the high nibble of each byte), one HSUB2 / HFMA2 removes the bias.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>

namespace lssm {

__device__ __forceinline__ uint32_t lop3_6a(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ void dequant_word(uint32_t w, uint32_t q[4]) {
    const uint32_t LO = 0x000F000Fu, HI = 0x00F000F0u;
    const uint32_t MLO = 0x64086408u, MHI = 0x64806480u;
    const __half2 sub_lo = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));  // 1032
    const __half2 mul_hi = __halves2half2(__ushort_as_half(0x2C00), __ushort_as_half(0x2C00));  // 1/16
    const __half2 add_hi = __halves2half2(__ushort_as_half(0xD480), __ushort_as_half(0xD480));  // -72
    uint32_t p0 = lop3_6a(w, LO, MLO);
    uint32_t p1 = lop3_6a(w, HI, MHI);
    const uint32_t w8 = w >> 8;
    uint32_t p2 = lop3_6a(w8, LO, MLO);
    uint32_t p3 = lop3_6a(w8, HI, MHI);
    __half2 h0 = __hsub2(*reinterpret_cast<__half2*>(&p0), sub_lo);
    __half2 h1 = __hfma2(*reinterpret_cast<__half2*>(&p1), mul_hi, add_hi);
    __half2 h2 = __hsub2(*reinterpret_cast<__half2*>(&p2), sub_lo);
    __half2 h3 = __hfma2(*reinterpret_cast<__half2*>(&p3), mul_hi, add_hi);
    q[0] = *reinterpret_cast<uint32_t*>(&h0);
    q[1] = *reinterpret_cast<uint32_t*>(&h1);
    q[2] = *reinterpret_cast<uint32_t*>(&h2);
    q[3] = *reinterpret_cast<uint32_t*>(&h3);
}

// Bias-folding dequantisation of one packed word (nibbles u = q + 8 of k0..k7, q signed) into the
// MMA pairs (k0,k4) (k1,k5) (k2,k6) (k3,k7) with one shift: the even nibbles k0 / k4 and (after
// w >> 8) k2 / k6 sit in bits 0..3 of their fp16 lanes and are written under the exponent of 1024
// (unit 1 there), the odd ones sit in bits 4..7 and are written under the exponent of 64 (unit 1
// there). The values are exact: 1032 + q for even k, 72 + q for odd k, so a block's dot product
// with x equals sum(q * x) + 1032 * sum(x_even) + 72 * sum(x_odd): the caller starts the MMA
// accumulator at fold_bias of the block's even / odd activation sums. 5 instructions per word
// (dequant_word: 9). The folded bias stays small next to fp32's 24 bits, so the products keep
// their precision.
__device__ __forceinline__ void dequant_word_fold(uint32_t w, uint32_t q[4]) {
    const uint32_t LO = 0x000F000Fu, HI = 0x00F000F0u, M1024 = 0x64086408u, M64 = 0x54805480u;
    const uint32_t w8 = w >> 8;
    q[0] = lop3_6a(w, LO, M1024);
    q[1] = lop3_6a(w, HI, M64);
    q[2] = lop3_6a(w8, LO, M1024);
    q[3] = lop3_6a(w8, HI, M64);
}
// Accumulator start of a block from its {even k, odd k} activation sums.
__device__ __forceinline__ float fold_bias(float even_sum, float odd_sum) {
    return fmaf(-1032.0f, even_sum, -72.0f * odd_sum);
}

// D += A(16x16, f16) * B(16x8, f16), fp32 accumulate.
__device__ __forceinline__ void mma_16816(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Non-tensor bulk copy global -> shared, completing on an mbarrier (16-B aligned, size % 16 == 0).
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
                 : "memory");
}

// Non-tensor bulk copy shared -> global in the thread's bulk async-group (16-B aligned,
// size % 16 == 0); bulk_commit closes the group, bulk_wait_all waits for every group to complete.
__device__ __forceinline__ void bulk_s2g(void* dst, uint32_t src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(reinterpret_cast<uint64_t>(dst)),
                 "r"(src), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// mbarrier phase wait that gives up after 2 s of %globaltimer.
__device__ __forceinline__ bool bar_wait_bounded(uint32_t bar, uint32_t parity) {
    uint32_t ok = 0;
    uint64_t t0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    while (true) {
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
            : "=r"(ok)
            : "r"(bar), "r"(parity)
            : "memory");
        if (ok) return true;
        uint64_t t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        if (t - t0 > 2000000000ull) return false;
    }
}

// L2 evict-first policy for weight streams read once per step.
__device__ __forceinline__ uint64_t evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ void tma3(uint32_t dst, const CUtensorMap* map, int32_t c0, int32_t c1, int32_t c2,
                                     uint32_t bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar), "l"(pol)
        : "memory");
}
__device__ __forceinline__ void tma2(uint32_t dst, const CUtensorMap* map, int32_t c0, int32_t c1, uint32_t bar,
                                     uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar), "l"(pol)
        : "memory");
}

}  // namespace lssm
