// synth_rng.h — deterministic, platform-independent weight generator for the
// seeded random-init models (host and device produce bit-identical values).
//
// value(seed, stream, i, amp) = (2u - 1) * amp, u = top 24 bits of a splitmix64
// hash of (seed, stream, i) scaled by 2^-24. Every step is an exactly rounded IEEE
// operation with no contraction opportunity (2u-1 is exact, one multiply), so the
// CUDA kernel and a CPU loop agree bit for bit; fp16 rounding (round-to-nearest-even)
// and the INT4 quantiser are likewise exact IEEE operations.
#pragma once

#include <stdint.h>

#if defined(__CUDACC__)
#define LSSM_HD __host__ __device__ __forceinline__
#else
#define LSSM_HD static inline
#endif

LSSM_HD uint64_t synth_mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

LSSM_HD float synth_value(uint64_t seed, uint64_t stream, uint64_t i, float amp) {
    const uint64_t h = synth_mix64(synth_mix64(seed ^ (stream * 0x9E3779B97F4A7C15ull)) + i);
    const float u = (float)(uint32_t)(h >> 40) * (1.0f / 16777216.0f);
    return (2.0f * u - 1.0f) * amp;
}
