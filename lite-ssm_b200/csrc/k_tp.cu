// k_tp.cu — the greedy pick and the small kernels of the head-tensor-parallel model path
// (one rank per GPU, the heads, groups and d_inner channels of every layer split over the
// ranks). The pick compares fp16 logits, which is comparing the reference's fp32 logits
// (fp16 -> fp32 is exact, read_logits_fp32 mamba2_model.cpp:177-211):
//   * k_rowsumsq: fp32 sum of squares of each row of this rank's gated slice; the ranks'
//     sums are all-reduced, because the gated RMSNorm spans the full d_inner
//     (src/model/mamba2_block.cpp:235-238)
//   * k_rmsnorm_total: y = half(x * w * rsqrt(sumsq_total / dim_total + eps)), the
//     rmsnorm_f16 arithmetic (shaders/norm.metal:51-79) with the all-reduced sum
//   * k_residual_f32: hidden = half(hidden + half(sum of the ranks' fp32 out_proj
//     partials)), block_out rounded to fp16 then added (mamba2_block.cpp:274-276)
//   * k_argmax_chunks / k_argmax_merge: first-max argmax over vocab chunks of this rank's
//     logits (many CTAs per row), then over the ranks' (value, index) pairs (one rank
//     without tensor parallelism), with the strict `>` / lowest-index rule
//     and the NaN-at-index-0 case of src/runtime/sampler.cpp:13-21; the merge writes the
//     token, the history slot and the next token's embedding row.
#include <cuda_fp16.h>

#include "device_util.cuh"
#include "lssm_internal.h"

namespace lssm {

int* tc_error_word();

namespace {

__global__ void k_rowsumsq(const __half* __restrict__ x, uint64_t stride, uint32_t rows, uint32_t dim,
                           float* __restrict__ out) {
    const uint32_t row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= rows) return;
    const __half* xr = x + (uint64_t)row * stride;
    float s = 0.0f;
    for (uint32_t k = lane; k < dim; k += 32) {
        const float v = __half2float(xr[k]);
        s += v * v;
    }
    s = warp_sum(s);
    if (lane == 0) out[row] = s;
}

__global__ void k_rmsnorm_total(const __half* __restrict__ x, uint64_t stride, const __half* __restrict__ w,
                                const float* __restrict__ sumsq, uint32_t rows, uint32_t dim, float dim_total, float eps,
                                __half* __restrict__ y) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (uint64_t)rows * dim) return;
    const uint32_t row = (uint32_t)(i / dim), k = (uint32_t)(i % dim);
    const float rr = rsqrtf(sumsq[row] / dim_total + eps);
    y[i] = __float2half_rn(__half2float(x[(uint64_t)row * stride + k]) * __half2float(w[k]) * rr);
}

__global__ void k_residual_f32(__half* __restrict__ hidden, const float* __restrict__ part, uint64_t n) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float o = __half2float(__float2half_rn(part[i]));
    hidden[i] = __float2half_rn(__half2float(hidden[i]) + o);
}

constexpr uint32_t AMX_CHUNK = 4096;

__device__ __forceinline__ void take(float& bv, uint32_t& bi, float v, uint32_t i) {
    if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
}

// First-max argmax of logits[row][0..Vr) in AMX_CHUNK-wide chunks: grid (chunks, rows).
// Each CTA reduces its chunk to a (value, global index) pair with 16-byte loads when the
// rows allow it; the last CTA of a row to finish (atomic ticket) merges the row's chunk
// pairs into out[row] and re-arms the ticket. Pairs are (float bits, index). The rank
// whose slice holds global index 0 reports (+inf, 0) when that logit is NaN: the
// reference's loop never replaces a NaN first element (src/runtime/sampler.cpp:13-21).
__global__ void __launch_bounds__(256) k_argmax_chunks(const __half* __restrict__ logits, uint32_t ld, uint32_t Vr,
                                                       uint32_t v_off, uint2* __restrict__ cpair,
                                                       uint32_t* __restrict__ ticket, uint2* __restrict__ out) {
    __shared__ float sv[8];
    __shared__ uint32_t si[8];
    __shared__ bool last;
    const uint32_t ch = blockIdx.x, b = blockIdx.y, nch = gridDim.x;
    const __half* lg = logits + (uint64_t)b * ld;
    const uint32_t lo = ch * AMX_CHUNK, hi = min(Vr, lo + AMX_CHUNK);
    float bv = -INFINITY;
    uint32_t bi = 0xFFFFFFFFu;
    const bool vec = (ld % 8 == 0) && ((reinterpret_cast<uintptr_t>(logits) & 15) == 0);
    if (vec) {
        for (uint32_t i = lo + 8 * threadIdx.x; i < hi; i += 8 * blockDim.x) {
            if (i + 8 <= hi) {
                const uint4 u = __ldcs(reinterpret_cast<const uint4*>(lg + i));
                const __half* h = reinterpret_cast<const __half*>(&u);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float v = __half2float(h[j]);
                    if (v > bv) { bv = v; bi = v_off + i + j; }
                }
            } else {
                for (uint32_t j = i; j < hi; ++j) {
                    const float v = __half2float(lg[j]);
                    if (v > bv) { bv = v; bi = v_off + j; }
                }
            }
        }
    } else {
        for (uint32_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
            const float v = __half2float(lg[i]);
            if (v > bv) { bv = v; bi = v_off + i; }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) take(bv, bi, __shfl_xor_sync(0xffffffffu, bv, o), __shfl_xor_sync(0xffffffffu, bi, o));
    const uint32_t lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    if (lane == 0) { sv[wid] = bv; si[wid] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (uint32_t w = 1; w < (blockDim.x >> 5); ++w) take(bv, bi, sv[w], si[w]);
        if (ch == 0 && v_off == 0 && __half2float(lg[0]) != __half2float(lg[0])) { bv = INFINITY; bi = 0; }
        cpair[(uint64_t)b * nch + ch] = make_uint2(__float_as_uint(bv), bi);
        __threadfence();
        last = atomicAdd(&ticket[b], 1u) == nch - 1;
    }
    __syncthreads();
    if (!last) return;
    if (wid == 0) {
        __threadfence();
        bv = -INFINITY;
        bi = 0xFFFFFFFFu;
        for (uint32_t c = lane; c < nch; c += 32) {
            const uint2 p = __ldcg(cpair + (uint64_t)b * nch + c);
            take(bv, bi, __uint_as_float(p.x), p.y);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
            take(bv, bi, __shfl_xor_sync(0xffffffffu, bv, o), __shfl_xor_sync(0xffffffffu, bi, o));
        if (lane == 0) {
            out[b] = make_uint2(__float_as_uint(bv), bi);
            ticket[b] = 0;
        }
    }
}

// pairs laid out [rank][row] (the all-gather order). One thread block per row.
__global__ void k_argmax_merge(const uint2* __restrict__ pairs, uint32_t world,
                               uint32_t B, uint32_t* __restrict__ cur, uint32_t* __restrict__ history,
                               uint32_t hist_stride, const uint32_t* __restrict__ step, const __half* __restrict__ embed,
                               __half* __restrict__ hidden, uint32_t d_model) {
    __shared__ uint32_t pick;
    const uint32_t b = blockIdx.x;
    if (threadIdx.x == 0) {
        float bv = -INFINITY;
        uint32_t bi = 0xFFFFFFFFu;
        for (uint32_t r = 0; r < world; ++r) {
            const uint2 p = pairs[(uint64_t)r * B + b];
            take(bv, bi, __uint_as_float(p.x), p.y);
        }
        const uint32_t p = bi == 0xFFFFFFFFu ? 0u : bi;
        pick = p;
        cur[b] = p;
        if (history && step) history[(uint64_t)b * hist_stride + *step] = p;
    }
    __syncthreads();
    if (embed && hidden)
        for (uint32_t k = threadIdx.x; k < d_model; k += blockDim.x)
            hidden[(uint64_t)b * d_model + k] = embed[(uint64_t)pick * d_model + k];
}

// Peer-memory sum-all-reduce of n fp32 (n <= 1024 * P2P_BLOCKS) for the tensor-parallel
// decode step; CTA b owns floats [1024 b, 1024 b + 1024). Every value travels as one 8-byte
// word (epoch << 32 | float bits): the receiver polls its words until they carry the
// current epoch, so data and readiness arrive in the same store and no fence or separate
// flag is needed. Per call CTA b takes the next epoch e of its own counter (every rank runs
// the same calls, so the epochs agree), writes its words into parity e & 1 of every peer's
// receive area (peer stores over NVLink), then reads its peers' words here and sums the
// values in rank order (the same order on every rank: identical results). Two parities
// suffice: a rank reaches epoch e + 2 only after reading every peer's epoch e + 1 words,
// which that peer writes after its epoch-e kernel, reads included, has finished.
// Residual form (hidden): hidden = half(hidden + half(sum)), the out_proj residual of
// mamba2_block.cpp:274-276; else out = sum (may alias part). Each poll is bounded by
// spin_ns; a timeout sets *err (the host reports LSSM_ERR_TIMEOUT) and the value counts 0.
__global__ void __launch_bounds__(256) k_p2p_allreduce(P2PPeers peers, const uint64_t* recv_local,
                                                       uint32_t* __restrict__ epochs, int rank, int world, uint64_t cap,
                                                       const float* part, uint32_t n, float* out,
                                                       __half* __restrict__ hidden, uint64_t spin_ns,
                                                       int* __restrict__ err) {
    __shared__ uint32_t e_sh;
    const uint32_t tid = threadIdx.x, blk = blockIdx.x;
    if (tid == 0) e_sh = ++epochs[blk];
    __syncthreads();
    const uint32_t e = e_sh, par = e & 1;
    const uint32_t lo = blk * 1024, hi = min(n, lo + 1024);
    for (uint32_t i = lo + tid; i < hi; i += 256) {
        const uint64_t w = ((uint64_t)e << 32) | __float_as_uint(part[i]);
        for (int r = 0; r < world; ++r) {
            if (r == rank) continue;
            uint64_t* dst = peers.recv[r] + ((uint64_t)par * world + rank) * cap + i;
            asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(dst), "l"(w) : "memory");
        }
    }
    for (uint32_t i = lo + tid; i < hi; i += 256) {
        float acc = 0.0f;
        for (int r = 0; r < world; ++r) {
            float v;
            if (r == rank) {
                v = part[i];
            } else {
                const uint64_t* src = recv_local + ((uint64_t)par * world + r) * cap + i;
                uint64_t w;
                uint64_t t0 = 0;
                for (uint32_t k = 0;; ++k) {
                    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(src) : "memory");
                    if ((uint32_t)(w >> 32) == e) break;
                    if ((k & 255) == 0) {
                        uint64_t t;
                        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
                        if (k == 0) {
                            t0 = t;
                        } else if (t - t0 > spin_ns) {
                            atomicExch(err, 1);
                            w = 0;
                            break;
                        }
                    }
                }
                v = __uint_as_float((uint32_t)w);
            }
            acc += v;
        }
        if (hidden) {
            const float o = __half2float(__float2half_rn(acc));
            hidden[i] = __float2half_rn(__half2float(hidden[i]) + o);
        } else {
            out[i] = acc;
        }
    }
}

__global__ void k_step_inc(uint32_t* step) { *step += 1; }

}  // namespace

cudaError_t launch_rowsumsq(const void* x, uint64_t stride, uint32_t rows, uint32_t dim, float* out, cudaStream_t s) {
    if (!rows) return cudaSuccess;
    k_rowsumsq<<<(rows + 7) / 8, 256, 0, s>>>(static_cast<const __half*>(x), stride, rows, dim, out);
    return cudaGetLastError();
}

cudaError_t launch_rmsnorm_total(const void* x, uint64_t stride, const void* w, const float* sumsq, uint32_t rows,
                                 uint32_t dim, uint32_t dim_total, float eps, void* y, cudaStream_t s) {
    const uint64_t n = (uint64_t)rows * dim;
    if (!n) return cudaSuccess;
    k_rmsnorm_total<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(static_cast<const __half*>(x), stride,
                                                               static_cast<const __half*>(w), sumsq, rows, dim,
                                                               (float)dim_total, eps, static_cast<__half*>(y));
    return cudaGetLastError();
}

cudaError_t launch_residual_f32(void* hidden, const float* part, uint64_t n, cudaStream_t s) {
    if (!n) return cudaSuccess;
    k_residual_f32<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(static_cast<__half*>(hidden), part, n);
    return cudaGetLastError();
}

uint32_t argmax_chunks(uint32_t Vr) { return Vr ? (Vr + AMX_CHUNK - 1) / AMX_CHUNK : 1; }

cudaError_t launch_argmax_chunks(const void* logits, uint32_t ld, uint32_t B, uint32_t Vr, uint32_t v_off, uint2* cpair,
                                 uint32_t* ticket, uint2* out, cudaStream_t s) {
    if (!B) return cudaSuccess;
    k_argmax_chunks<<<dim3(argmax_chunks(Vr), B), 256, 0, s>>>(static_cast<const __half*>(logits), ld, Vr, v_off, cpair,
                                                               ticket, out);
    return cudaGetLastError();
}

cudaError_t launch_argmax_merge(const uint2* pairs, uint32_t world, uint32_t B, uint32_t* cur, uint32_t* history,
                                uint32_t hist_stride, uint32_t* step, const void* embed, void* hidden, uint32_t d_model,
                                cudaStream_t s) {
    if (!B) return cudaSuccess;
    k_argmax_merge<<<B, 256, 0, s>>>(pairs, world, B, cur, history, hist_stride, step,
                                     static_cast<const __half*>(embed), static_cast<__half*>(hidden), d_model);
    if (step) k_step_inc<<<1, 1, 0, s>>>(step);
    return cudaGetLastError();
}

cudaError_t launch_p2p_allreduce(const P2PPeers& peers, const uint64_t* recv_local, uint32_t* epochs, int rank,
                                 int world, size_t cap, const float* part, uint32_t n, float* out, __half* hidden,
                                 uint64_t spin_ns, cudaStream_t s) {
    if (!n) return cudaSuccess;
    const uint32_t blocks = (n + 1023) / 1024;
    if (blocks > P2P_BLOCKS || n > cap || world > P2P_MAX_RANKS) return cudaErrorInvalidValue;
    k_p2p_allreduce<<<blocks, 256, 0, s>>>(peers, recv_local, epochs, rank, world, cap, part, n, out, hidden, spin_ns,
                                           tc_error_word());
    return cudaGetLastError();
}

}  // namespace lssm
