// oracle/lssm_oracle.cpp — CPU restatement of lite-ssm's Mamba-2 hot path.
//
// TEST INFRASTRUCTURE ONLY. This file is the parity checker and the timed CPU
// baseline. Only tests/, __graft_entry__.smoke() and bench.py's cpu-baseline /
// reference arm load it. The product library (lite-ssm_b200/liblssm_cuda.so)
// never links, calls or falls back to it.
//
// The reference has no CPU compute path: all of its math lives in Metal
// shaders. Every function below restates one shader's arithmetic in plain C++
// and cites the shader file:line it follows (paths inside the lite-ssm
// project). Two numeric modes exist where it matters:
//   * "faithful": fp16 rounding exactly where the Metal kernels store `half`
//     (activations, the fp16-staged SSD state of ssd_chunked, the fp16
//     dequantised GEMM weight tile), fp32 accumulation;
//   * "exact": double accumulation and no intermediate rounding, used to
//     measure how far any implementation sits from the true value.
//
// Parity pins: the format side is pinned against the reference's own Python
// writer (tools/ssm_format.py, tools/export_mamba2.py) through fixtures in
// tests/golden; the model math is pinned against HF transformers'
// Mamba2ForCausalLM (the ground truth the reference's own parity test uses,
// tools/dump_parity.py:26-70) through logits fixtures in tests/golden.
//
// Build: g++ -O3 -fopenmp -fPIC -shared (see oracle/build_oracle.py).

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

extern "C" {

// ---------------------------------------------------------------------------
//  IEEE binary16 / bfloat16 conversions (round to nearest even), own code.
// ---------------------------------------------------------------------------
static inline float h2f(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t mant = h & 0x3FFu;
    uint32_t f;
    if (exp == 0) {
        if (mant == 0) {
            f = sign;
        } else {
            int e = -1;
            do { mant <<= 1; ++e; } while ((mant & 0x400u) == 0);
            mant &= 0x3FFu;
            f = sign | ((uint32_t)(127 - 15 - e) << 23) | (mant << 13);
        }
    } else if (exp == 0x1F) {
        f = sign | 0x7F800000u | (mant << 13);
    } else {
        f = sign | ((exp + 127 - 15) << 23) | (mant << 13);
    }
    float out;
    std::memcpy(&out, &f, 4);
    return out;
}

static inline uint16_t f2h(float v) {
    uint32_t x;
    std::memcpy(&x, &v, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t absx = x & 0x7FFFFFFFu;
    if (absx >= 0x7F800000u) {                       // inf / nan
        return (uint16_t)(sign | 0x7C00u | (absx > 0x7F800000u ? 0x200u : 0u));
    }
    if (absx >= 0x477FF000u) {                       // rounds to >= 65520 -> inf
        return (uint16_t)(sign | 0x7C00u);
    }
    if (absx < 0x38800000u) {                        // subnormal half (< 2^-14)
        if (absx < 0x33000000u) return (uint16_t)sign;   // < 2^-25 -> 0
        uint32_t e = absx >> 23;
        uint32_t m = (absx & 0x7FFFFFu) | 0x800000u;
        uint32_t shift = 126 - e;                    // 14 - (e - 127) + 13 - 1 + ... (see below)
        // value = m * 2^(e-150); half subnormal unit = 2^-24 -> q = m * 2^(e-126)
        uint32_t q = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (q & 1u))) ++q;
        return (uint16_t)(sign | q);
    }
    uint32_t e = (absx >> 23) - 127 + 15;
    uint32_t m = absx & 0x7FFFFFu;
    uint32_t q = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) ++q;
    return (uint16_t)(sign | q);
}

static inline float hr(float v) { return h2f(f2h(v)); }   // round through fp16

static inline float bf2f(uint16_t b) {
    uint32_t f = (uint32_t)b << 16;
    float out;
    std::memcpy(&out, &f, 4);
    return out;
}

static inline uint16_t f2bf(float v) {
    uint32_t x;
    std::memcpy(&x, &v, 4);
    if ((x & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((x >> 16) | 0x40u);
    uint32_t lsb = (x >> 16) & 1u;
    x += 0x7FFFu + lsb;
    return (uint16_t)(x >> 16);
}

// Exposed for the host-side tests of the conversions themselves.
float lssm_oracle_h2f(uint16_t h) { return h2f(h); }
uint16_t lssm_oracle_f2h(float v) { return f2h(v); }
float lssm_oracle_bf2f(uint16_t b) { return bf2f(b); }
uint16_t lssm_oracle_f2bf(float v) { return f2bf(v); }

void lssm_oracle_f16_to_f32(const uint16_t* in, float* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = h2f(in[i]);
}
void lssm_oracle_f32_to_f16(const float* in, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = f2h(in[i]);
}

int lssm_oracle_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void lssm_oracle_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

// ---------------------------------------------------------------------------
//  Scalar helpers — shaders/common.metal:48-61, shaders/ssd_step.metal:29-31.
// ---------------------------------------------------------------------------
static inline float silu_f(float x) { return x / (1.0f + std::exp(-x)); }
static inline float softplus_f(float x) { return (x > 20.0f) ? x : std::log(1.0f + std::exp(x)); }
static inline float clampf(float v, float lo, float hi) { return std::min(std::max(v, lo), hi); }

// ---------------------------------------------------------------------------
//  RMSNorm — shaders/norm.metal:51-79.  y = half(x * w * rsqrt(mean(x^2)+eps)).
// ---------------------------------------------------------------------------
void lssm_oracle_rmsnorm_f16(const uint16_t* x, const uint16_t* w, uint16_t* y,
                             uint32_t rows, uint32_t dim, float eps) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < (int64_t)rows; ++r) {
        const uint16_t* xr = x + (size_t)r * dim;
        uint16_t* yr = y + (size_t)r * dim;
        float ss = 0.0f;
        for (uint32_t i = 0; i < dim; ++i) { float v = h2f(xr[i]); ss += v * v; }
        float rrms = 1.0f / std::sqrt(ss / (float)dim + eps);
        for (uint32_t i = 0; i < dim; ++i) yr[i] = f2h(h2f(xr[i]) * h2f(w[i]) * rrms);
    }
}

// ---------------------------------------------------------------------------
//  INT4_B32 dequant — shaders/linear.metal:38-61 (layout), tools/export_mamba2.py:68-103
//  (packing). Nibble for (row, col): byte row*(K/2) + col/2, low nibble = even col;
//  q = nib < 8 ? nib : nib - 16; scale = scales[row*(K/32) + col/32].
// ---------------------------------------------------------------------------
static inline int q4_at(const uint8_t* packed, uint32_t K, uint32_t row, uint32_t col) {
    uint8_t b = packed[(size_t)row * (K / 2) + (col >> 1)];
    uint32_t nib = (col & 1u) ? (uint32_t)(b >> 4) : (uint32_t)(b & 0x0Fu);
    return nib < 8u ? (int)nib : (int)nib - 16;
}

void lssm_oracle_int4_dequant(const uint8_t* packed, const uint16_t* scales, float* out,
                              uint32_t N, uint32_t K) {
    const uint32_t bpr = K / 32;
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < (int64_t)N; ++n)
        for (uint32_t k = 0; k < K; ++k)
            out[(size_t)n * K + k] = (float)q4_at(packed, K, (uint32_t)n, k) * h2f(scales[(size_t)n * bpr + k / 32]);
}

// Block-32 symmetric quantiser, restating tools/export_mamba2.py:68-103:
//   absmax = max(|w|) over the block (clamped to >= 1e-12), scale = absmax / 7 (fp32),
//   q = round_half_even(w / scale) clipped to [-8, 7], scale stored as fp16,
//   two nibbles per byte with the even column in the low nibble,
//   packed bytes first (N*K/2), then the fp16 scales (N*K/32).
void lssm_oracle_int4_quantize(const float* w, uint32_t N, uint32_t K,
                               uint8_t* packed_out, uint16_t* scales_out) {
    const uint32_t bpr = K / 32;
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < (int64_t)N; ++n) {
        for (uint32_t b = 0; b < bpr; ++b) {
            const float* blk = w + (size_t)n * K + (size_t)b * 32;
            float absmax = 0.0f;
            for (int i = 0; i < 32; ++i) absmax = std::max(absmax, std::fabs(blk[i]));
            absmax = std::max(absmax, 1e-12f);
            float scale = absmax / 7.0f;
            scales_out[(size_t)n * bpr + b] = f2h(scale);
            uint8_t* dst = packed_out + (size_t)n * (K / 2) + (size_t)b * 16;
            for (int i = 0; i < 16; ++i) {
                float q0 = std::nearbyint(blk[2 * i] / scale);
                float q1 = std::nearbyint(blk[2 * i + 1] / scale);
                int i0 = (int)std::min(std::max(q0, -8.0f), 7.0f);
                int i1 = (int)std::min(std::max(q1, -8.0f), 7.0f);
                dst[i] = (uint8_t)(((i1 & 0xF) << 4) | (i0 & 0xF));
            }
        }
    }
}

// ---------------------------------------------------------------------------
//  GEMV / GEMM.
//   linear_f16_gemv   shaders/linear.metal:82-109   y = half(sum_k w*x), fp32 acc
//   linear_int4_gemv  shaders/linear.metal:440-474  y = half(sum_k (q*s)*x), fp32 dequant
//   linear_f16_gemm   shaders/linear.metal:253-343  fp16 operands, fp32 acc
//   linear_int4_gemm  shaders/linear.metal:492-574  dequant tile rounded to fp16 (:538)
// All: Y[M,N] = X[M,K] . W[N,K]^T, row-major.
// ---------------------------------------------------------------------------
void lssm_oracle_linear_f16(const uint16_t* x, const uint16_t* w, uint16_t* y,
                            uint32_t M, uint32_t N, uint32_t K) {
    std::vector<float> xf((size_t)M * K);
    for (size_t i = 0; i < xf.size(); ++i) xf[i] = h2f(x[i]);
#pragma omp parallel
    {
        std::vector<float> wr(K);
#pragma omp for schedule(static)
        for (int64_t n = 0; n < (int64_t)N; ++n) {
            for (uint32_t k = 0; k < K; ++k) wr[k] = h2f(w[(size_t)n * K + k]);
            for (uint32_t m = 0; m < M; ++m) {
                const float* xr = xf.data() + (size_t)m * K;
                float acc = 0.0f;
                for (uint32_t k = 0; k < K; ++k) acc += wr[k] * xr[k];
                y[(size_t)m * N + n] = f2h(acc);
            }
        }
    }
}

// round_weight_f16: 1 = GEMM semantics (dequantised weight rounded to fp16), 0 = GEMV (fp32).
void lssm_oracle_linear_int4(const uint16_t* x, const uint8_t* packed, const uint16_t* scales,
                             uint16_t* y, uint32_t M, uint32_t N, uint32_t K, int round_weight_f16) {
    std::vector<float> xf((size_t)M * K);
    for (size_t i = 0; i < xf.size(); ++i) xf[i] = h2f(x[i]);
    const uint32_t bpr = K / 32;
#pragma omp parallel
    {
        std::vector<float> wr(K);
#pragma omp for schedule(static)
        for (int64_t n = 0; n < (int64_t)N; ++n) {
            for (uint32_t k = 0; k < K; ++k) {
                float v = (float)q4_at(packed, K, (uint32_t)n, k) * h2f(scales[(size_t)n * bpr + k / 32]);
                wr[k] = round_weight_f16 ? hr(v) : v;
            }
            for (uint32_t m = 0; m < M; ++m) {
                const float* xr = xf.data() + (size_t)m * K;
                float acc = 0.0f;
                for (uint32_t k = 0; k < K; ++k) acc += wr[k] * xr[k];
                y[(size_t)m * N + n] = f2h(acc);
            }
        }
    }
}

// ---------------------------------------------------------------------------
//  Elementwise — shaders/activations.metal:12-87.
// ---------------------------------------------------------------------------
void lssm_oracle_silu_f16(const uint16_t* x, uint16_t* y, uint32_t n) {
    for (uint32_t i = 0; i < n; ++i) y[i] = f2h(silu_f(h2f(x[i])));
}
void lssm_oracle_add_inplace_f16(uint16_t* y, const uint16_t* x, uint32_t n) {
    for (uint32_t i = 0; i < n; ++i) y[i] = f2h(h2f(y[i]) + h2f(x[i]));
}
void lssm_oracle_silu_gated_f16(const uint16_t* z, const uint16_t* gate, uint16_t* y, uint32_t n) {
    for (uint32_t i = 0; i < n; ++i) y[i] = f2h(silu_f(h2f(z[i])) * h2f(gate[i]));
}
void lssm_oracle_split_silu_xBC_f16(const uint16_t* xBC, uint16_t* x_out, uint16_t* B_out, uint16_t* C_out,
                                    uint32_t L, uint32_t d_inner, uint32_t d_state, uint32_t n_groups) {
    const uint32_t GN = n_groups * d_state, D = d_inner + 2 * GN;
    for (uint32_t t = 0; t < L; ++t)
        for (uint32_t f = 0; f < D; ++f) {
            uint16_t v = f2h(silu_f(h2f(xBC[(size_t)t * D + f])));
            if (f < d_inner) x_out[(size_t)t * d_inner + f] = v;
            else if (f < d_inner + GN) B_out[(size_t)t * GN + (f - d_inner)] = v;
            else C_out[(size_t)t * GN + (f - d_inner - GN)] = v;
        }
}

// ---------------------------------------------------------------------------
//  Causal conv1d — shaders/conv1d.metal:35-137.
//  x,y (B, L, D); w (D, K); state (B, D, K) oldest first.
// ---------------------------------------------------------------------------
void lssm_oracle_causal_conv1d_f16(const uint16_t* x, const uint16_t* w, const uint16_t* bias, uint16_t* y,
                                   uint32_t B, uint32_t L, uint32_t D, uint32_t K) {
    for (uint32_t b = 0; b < B; ++b)
        for (uint32_t t = 0; t < L; ++t)
            for (uint32_t d = 0; d < D; ++d) {
                float acc = bias ? h2f(bias[d]) : 0.0f;
                for (uint32_t tap = 0; tap < K; ++tap) {
                    int src = (int)t - (int)(K - 1 - tap);
                    float v = src >= 0 ? h2f(x[((size_t)b * L + (uint32_t)src) * D + d]) : 0.0f;
                    acc += h2f(w[(size_t)d * K + tap]) * v;
                }
                y[((size_t)b * L + t) * D + d] = f2h(acc);
            }
}

void lssm_oracle_causal_conv1d_update_f16(const uint16_t* x_new, uint16_t* state, const uint16_t* w,
                                          const uint16_t* bias, uint16_t* y,
                                          uint32_t B, uint32_t D, uint32_t K) {
    for (uint32_t b = 0; b < B; ++b)
        for (uint32_t d = 0; d < D; ++d) {
            uint16_t* sd = state + ((size_t)b * D + d) * K;
            for (uint32_t k = 0; k + 1 < K; ++k) sd[k] = sd[k + 1];
            sd[K - 1] = x_new[(size_t)b * D + d];
            float acc = bias ? h2f(bias[d]) : 0.0f;
            for (uint32_t k = 0; k < K; ++k) acc += h2f(sd[k]) * h2f(w[(size_t)d * K + k]);
            y[(size_t)b * D + d] = f2h(acc);
        }
}

void lssm_oracle_seed_conv_state_f16(const uint16_t* xBC, uint16_t* state, uint32_t L, uint32_t D, uint32_t K) {
    for (uint32_t d = 0; d < D; ++d)
        for (uint32_t k = 0; k < K; ++k) {
            int src = (int)L - (int)K + (int)k;
            state[(size_t)d * K + k] = src >= 0 ? xBC[(size_t)src * D + d] : (uint16_t)0;
        }
}

// ---------------------------------------------------------------------------
//  Fused in_proj — shaders/fused.metal:43-165. The matmul stays fp32 in the
//  threadgroup tile (Cmm) and the conv reads those fp32 values; z, dt and the
//  pre-conv copy are rounded to fp16 on store.
// ---------------------------------------------------------------------------
void lssm_oracle_inproj_fused_f16(const uint16_t* normed, const uint16_t* W, const uint16_t* Wc,
                                  const uint16_t* cb, uint16_t* z, uint16_t* xs, uint16_t* Bs, uint16_t* Cs,
                                  uint16_t* dt, uint16_t* xBC_pre,
                                  uint32_t L, uint32_t d_model, uint32_t d_inner, uint32_t d_state,
                                  uint32_t n_groups, uint32_t n_heads, uint32_t d_conv) {
    const uint32_t GN = n_groups * d_state, xd = d_inner + 2 * GN, proj = d_inner + xd + n_heads;
    std::vector<float> mm((size_t)L * proj);
#pragma omp parallel for schedule(static)
    for (int64_t c = 0; c < (int64_t)proj; ++c)
        for (uint32_t m = 0; m < L; ++m) {
            float acc = 0.0f;
            for (uint32_t k = 0; k < d_model; ++k)
                acc += h2f(normed[(size_t)m * d_model + k]) * h2f(W[(size_t)c * d_model + k]);
            mm[(size_t)m * proj + c] = acc;
        }
    for (uint32_t m = 0; m < L; ++m)
        for (uint32_t c = 0; c < proj; ++c) {
            float v = mm[(size_t)m * proj + c];
            if (c < d_inner) {
                z[(size_t)m * d_inner + c] = f2h(v);
            } else if (c < d_inner + xd) {
                uint32_t f = c - d_inner;
                xBC_pre[(size_t)m * xd + f] = f2h(v);
                float s = h2f(cb[f]);
                for (uint32_t kk = 0; kk < d_conv; ++kk) {
                    int sm = (int)m - (int)(d_conv - 1 - kk);
                    if (sm >= 0) s += h2f(Wc[(size_t)f * d_conv + kk]) * mm[(size_t)sm * proj + c];
                }
                uint16_t o = f2h(silu_f(s));
                if (f < d_inner) xs[(size_t)m * d_inner + f] = o;
                else if (f < d_inner + GN) Bs[(size_t)m * GN + (f - d_inner)] = o;
                else Cs[(size_t)m * GN + (f - d_inner - GN)] = o;
            } else {
                dt[(size_t)m * n_heads + (c - d_inner - xd)] = f2h(v);
            }
        }
}

// ---------------------------------------------------------------------------
//  SSD decode step — shaders/ssd_step.metal:33-77.
//  x (H,P), B/C (G,N), dt_raw/dt_bias/A_log/D (H) fp16; state (H,P,N) fp32 RW; y (H,P) fp16.
// ---------------------------------------------------------------------------
void lssm_oracle_ssd_step_f16(const uint16_t* x, const uint16_t* Bp, const uint16_t* Cp,
                              const uint16_t* dt_raw, const uint16_t* dt_bias, const uint16_t* A_log,
                              const uint16_t* D_skip, float* state, uint16_t* y,
                              uint32_t H, uint32_t P, uint32_t N, uint32_t G,
                              float dt_min, float dt_max, uint32_t has_D) {
    const uint32_t hpg = std::max(1u, H / G);
#pragma omp parallel for schedule(static)
    for (int64_t h = 0; h < (int64_t)H; ++h) {
        const uint32_t g = (uint32_t)h / hpg;
        const float A = -std::exp(h2f(A_log[h]));
        const float dt = clampf(softplus_f(h2f(dt_raw[h]) + h2f(dt_bias[h])), dt_min, dt_max);
        const float decay = std::exp(A * dt);
        const float Dh = has_D ? h2f(D_skip[h]) : 0.0f;
        for (uint32_t p = 0; p < P; ++p) {
            const float xv = h2f(x[(size_t)h * P + p]);
            float* S = state + ((size_t)h * P + p) * N;
            float ys = 0.0f;
            for (uint32_t n = 0; n < N; ++n) {
                float s = decay * S[n] + dt * h2f(Bp[(size_t)g * N + n]) * xv;
                S[n] = s;
                ys += h2f(Cp[(size_t)g * N + n]) * s;
            }
            y[(size_t)h * P + p] = f2h(ys + Dh * xv);
        }
    }
}

// ---------------------------------------------------------------------------
//  SSD chunked prefill, faithful — shaders/ssd_chunked.metal:82-297.
//  The state is staged in fp16 between chunks (:116, :127, :287), M is fp16
//  (:121, :218), Y is fp16, the persisted state is fp32 of the fp16 stage (:295).
//  X (L,H,P), B/C (L,G,N), dt_raw (L,H), dt_bias/A_log/D (H), state_io (H,P,N) fp32.
// ---------------------------------------------------------------------------
void lssm_oracle_ssd_chunked_f16(const uint16_t* X, const uint16_t* Bp, const uint16_t* Cp,
                                 const uint16_t* dt_raw, const uint16_t* dt_bias, const uint16_t* A_log,
                                 const uint16_t* D_skip, uint16_t* Y, float* state_io,
                                 uint32_t L, uint32_t H, uint32_t P, uint32_t N, uint32_t G,
                                 uint32_t C, float dt_min, float dt_max, uint32_t has_D) {
    const uint32_t hpg = std::max(1u, H / G), GN = G * N;
    const uint32_t n_chunks = (L + C - 1) / C;
#pragma omp parallel for schedule(dynamic)
    for (int64_t hh = 0; hh < (int64_t)H; ++hh) {
        const uint32_t h = (uint32_t)hh, g = h / hpg;
        const float A = -std::exp(h2f(A_log[h]));
        const float db = h2f(dt_bias[h]);
        const float Dh = has_D ? h2f(D_skip[h]) : 0.0f;
        std::vector<float> S((size_t)P * N), DT(C), Lc(C), M((size_t)C * C);
        for (size_t i = 0; i < S.size(); ++i) S[i] = hr(state_io[(size_t)h * P * N + i]);
        for (uint32_t c = 0; c < n_chunks; ++c) {
            const uint32_t t0 = c * C, tl = std::min(C, L - t0);
            for (uint32_t t = 0; t < tl; ++t)
                DT[t] = clampf(softplus_f(h2f(dt_raw[(size_t)(t0 + t) * H + h]) + db), dt_min, dt_max);
            float run = 0.0f;
            for (uint32_t t = 0; t < tl; ++t) { run += A * DT[t]; Lc[t] = run; }
            const float Lend = Lc[tl - 1], dchunk = std::exp(Lend);
            for (uint32_t t = 0; t < tl; ++t)
                for (uint32_t j = 0; j < tl; ++j) {
                    if (j > t) { M[(size_t)t * tl + j] = 0.0f; continue; }
                    float cb = 0.0f;
                    for (uint32_t n = 0; n < N; ++n)
                        cb += h2f(Cp[(size_t)(t0 + t) * GN + g * N + n]) * h2f(Bp[(size_t)(t0 + j) * GN + g * N + n]);
                    M[(size_t)t * tl + j] = hr(cb * std::exp(Lc[t] - Lc[j]) * DT[j]);
                }
            for (uint32_t t = 0; t < tl; ++t)
                for (uint32_t p = 0; p < P; ++p) {
                    float yi = 0.0f;
                    for (uint32_t j = 0; j <= t; ++j)
                        yi += M[(size_t)t * tl + j] * h2f(X[((size_t)(t0 + j) * H + h) * P + p]);
                    float ye = 0.0f;
                    for (uint32_t n = 0; n < N; ++n)
                        ye += h2f(Cp[(size_t)(t0 + t) * GN + g * N + n]) * S[(size_t)p * N + n];
                    ye *= std::exp(Lc[t]);
                    float xc = h2f(X[((size_t)(t0 + t) * H + h) * P + p]);
                    Y[((size_t)(t0 + t) * H + h) * P + p] = f2h(yi + ye + Dh * xc);
                }
            for (uint32_t p = 0; p < P; ++p)
                for (uint32_t n = 0; n < N; ++n) {
                    float acc = dchunk * S[(size_t)p * N + n];
                    for (uint32_t j = 0; j < tl; ++j) {
                        float wj = std::exp(Lend - Lc[j]) * DT[j];
                        acc += wj * h2f(Bp[(size_t)(t0 + j) * GN + g * N + n]) *
                               h2f(X[((size_t)(t0 + j) * H + h) * P + p]);
                    }
                    S[(size_t)p * N + n] = hr(acc);
                }
        }
        for (size_t i = 0; i < S.size(); ++i) state_io[(size_t)h * P * N + i] = S[i];
    }
}

// ---------------------------------------------------------------------------
//  SSD, generic precision (the standalone SSD-op benchmark configuration and the exact check).
//  Same recurrence as ssd_step/ssd_chunked, written as the chunked algorithm
//  (chunk C) with fp32 or double accumulation and no intermediate rounding.
//  Inputs are pre-converted to fp32 by the caller (bf16 / fp16 sources).
//  Layout with a batch dim: X (Bt,L,H,P), B/C (Bt,L,G,N), dt (Bt,L,H) *raw* (softplus
//  applied here with dt_bias), state (Bt,H,P,N) fp32 in/out, Y (Bt,L,H,P) fp32.
//  use_double: 1 = double accumulators (the "exact" mode).
// ---------------------------------------------------------------------------
}  // extern "C" (templates need C++ linkage)

template <typename Acc>
static void ssd_chunked_generic(const float* X, const float* Bp, const float* Cp, const float* dt_raw,
                                const float* dt_bias, const float* A_log, const float* D_skip,
                                float* Y, float* state, uint32_t Bt, uint32_t L, uint32_t H,
                                uint32_t P, uint32_t N, uint32_t G, uint32_t C,
                                float dt_min, float dt_max, uint32_t has_D) {
    const uint32_t hpg = std::max(1u, H / G), GN = G * N;
    const uint32_t n_chunks = (L + C - 1) / C;
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int64_t b = 0; b < (int64_t)Bt; ++b)
        for (int64_t hh = 0; hh < (int64_t)H; ++hh) {
            const uint32_t h = (uint32_t)hh, g = h / hpg;
            const Acc A = -std::exp((Acc)A_log[h]);
            const Acc Dh = has_D ? (Acc)D_skip[h] : (Acc)0;
            const float* Xb = X + (size_t)b * L * H * P;
            const float* Bb = Bp + (size_t)b * L * GN;
            const float* Cb = Cp + (size_t)b * L * GN;
            const float* dtb = dt_raw + (size_t)b * L * H;
            float* Yb = Y + (size_t)b * L * H * P;
            float* Sio = state + ((size_t)b * H + h) * P * N;
            std::vector<Acc> S((size_t)P * N), DT(C), Lc(C), M((size_t)C * C), SN((size_t)P * N);
            for (size_t i = 0; i < S.size(); ++i) S[i] = (Acc)Sio[i];
            for (uint32_t c = 0; c < n_chunks; ++c) {
                const uint32_t t0 = c * C, tl = std::min(C, L - t0);
                for (uint32_t t = 0; t < tl; ++t) {
                    Acc d = (Acc)dtb[(size_t)(t0 + t) * H + h] + (Acc)dt_bias[h];
                    Acc sp = d > (Acc)20 ? d : std::log1p(std::exp(d));
                    DT[t] = std::min(std::max(sp, (Acc)dt_min), (Acc)dt_max);
                }
                Acc run = 0;
                for (uint32_t t = 0; t < tl; ++t) { run += A * DT[t]; Lc[t] = run; }
                const Acc Lend = Lc[tl - 1];
                for (uint32_t t = 0; t < tl; ++t)
                    for (uint32_t j = 0; j <= t; ++j) {
                        Acc cb = 0;
                        const float* cr = Cb + (size_t)(t0 + t) * GN + g * N;
                        const float* br = Bb + (size_t)(t0 + j) * GN + g * N;
                        for (uint32_t n = 0; n < N; ++n) cb += (Acc)cr[n] * (Acc)br[n];
                        M[(size_t)t * C + j] = cb * std::exp(Lc[t] - Lc[j]) * DT[j];
                    }
                for (uint32_t t = 0; t < tl; ++t) {
                    const Acc eL = std::exp(Lc[t]);
                    const float* cr = Cb + (size_t)(t0 + t) * GN + g * N;
                    for (uint32_t p = 0; p < P; ++p) {
                        Acc yi = 0;
                        for (uint32_t j = 0; j <= t; ++j)
                            yi += M[(size_t)t * C + j] * (Acc)Xb[((size_t)(t0 + j) * H + h) * P + p];
                        Acc ye = 0;
                        const Acc* Sr = S.data() + (size_t)p * N;
                        for (uint32_t n = 0; n < N; ++n) ye += (Acc)cr[n] * Sr[n];
                        Acc xc = (Acc)Xb[((size_t)(t0 + t) * H + h) * P + p];
                        Yb[((size_t)(t0 + t) * H + h) * P + p] = (float)(yi + ye * eL + Dh * xc);
                    }
                }
                const Acc dch = std::exp(Lend);
                for (size_t i = 0; i < SN.size(); ++i) SN[i] = dch * S[i];
                for (uint32_t j = 0; j < tl; ++j) {
                    const Acc wj = std::exp(Lend - Lc[j]) * DT[j];
                    const float* br = Bb + (size_t)(t0 + j) * GN + g * N;
                    for (uint32_t p = 0; p < P; ++p) {
                        const Acc xw = wj * (Acc)Xb[((size_t)(t0 + j) * H + h) * P + p];
                        Acc* Sr = SN.data() + (size_t)p * N;
                        for (uint32_t n = 0; n < N; ++n) Sr[n] += xw * (Acc)br[n];
                    }
                }
                S.swap(SN);
            }
            for (size_t i = 0; i < S.size(); ++i) Sio[i] = (float)S[i];
        }
}

extern "C" {

void lssm_oracle_ssd_chunked_f32(const float* X, const float* Bp, const float* Cp, const float* dt_raw,
                                 const float* dt_bias, const float* A_log, const float* D_skip,
                                 float* Y, float* state, uint32_t Bt, uint32_t L, uint32_t H,
                                 uint32_t P, uint32_t N, uint32_t G, uint32_t C,
                                 float dt_min, float dt_max, uint32_t has_D, int use_double) {
    if (use_double)
        ssd_chunked_generic<double>(X, Bp, Cp, dt_raw, dt_bias, A_log, D_skip, Y, state, Bt, L, H, P, N, G, C,
                                    dt_min, dt_max, has_D);
    else
        ssd_chunked_generic<float>(X, Bp, Cp, dt_raw, dt_bias, A_log, D_skip, Y, state, Bt, L, H, P, N, G, C,
                                   dt_min, dt_max, has_D);
}

// Token-by-token recurrence in double (the definition; ssd_step applied L times).
void lssm_oracle_ssd_sequential_f64(const float* X, const float* Bp, const float* Cp, const float* dt_raw,
                                    const float* dt_bias, const float* A_log, const float* D_skip,
                                    float* Y, float* state, uint32_t Bt, uint32_t L, uint32_t H,
                                    uint32_t P, uint32_t N, uint32_t G,
                                    float dt_min, float dt_max, uint32_t has_D) {
    const uint32_t hpg = std::max(1u, H / G), GN = G * N;
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int64_t b = 0; b < (int64_t)Bt; ++b)
        for (int64_t hh = 0; hh < (int64_t)H; ++hh) {
            const uint32_t h = (uint32_t)hh, g = h / hpg;
            const double A = -std::exp((double)A_log[h]);
            const double Dh = has_D ? (double)D_skip[h] : 0.0;
            std::vector<double> S((size_t)P * N);
            float* Sio = state + ((size_t)b * H + h) * P * N;
            for (size_t i = 0; i < S.size(); ++i) S[i] = Sio[i];
            for (uint32_t t = 0; t < L; ++t) {
                double d = (double)dt_raw[((size_t)b * L + t) * H + h] + (double)dt_bias[h];
                double sp = d > 20.0 ? d : std::log1p(std::exp(d));
                double dt = std::min(std::max(sp, (double)dt_min), (double)dt_max);
                double decay = std::exp(A * dt);
                const float* br = Bp + ((size_t)b * L + t) * GN + g * N;
                const float* cr = Cp + ((size_t)b * L + t) * GN + g * N;
                for (uint32_t p = 0; p < P; ++p) {
                    double xv = X[(((size_t)b * L + t) * H + h) * P + p];
                    double ys = 0.0;
                    for (uint32_t n = 0; n < N; ++n) {
                        double s = decay * S[(size_t)p * N + n] + dt * br[n] * xv;
                        S[(size_t)p * N + n] = s;
                        ys += cr[n] * s;
                    }
                    Y[(((size_t)b * L + t) * H + h) * P + p] = (float)(ys + Dh * xv);
                }
            }
            for (size_t i = 0; i < S.size(); ++i) Sio[i] = (float)S[i];
        }
}

// ---------------------------------------------------------------------------
//  Greedy argmax — src/runtime/sampler.cpp:13-21 (strict '>' => first max wins).
// ---------------------------------------------------------------------------
uint32_t lssm_oracle_argmax_f32(const float* v, uint32_t n) {
    uint32_t best = 0;
    float bv = v[0];
    for (uint32_t i = 1; i < n; ++i)
        if (v[i] > bv) { bv = v[i]; best = i; }
    return best;
}

// ---------------------------------------------------------------------------
//  Whole-model forward (faithful mode): restates src/model/mamba2_block.cpp:51-327,
//  src/model/mamba2_model.cpp:128-211, src/runtime/inference.cpp:14-70.
//
//  The caller passes the raw bytes of a .ssm file's payload arena (`base`, the
//  whole file) and a table of per-layer tensor offsets (filled by the Python
//  side from the .ssm index). Activations are fp16 at the workspace rounding
//  points; conv state fp16; SSD state fp32 (fp16-staged inside a prefill, as
//  the shader does).
// ---------------------------------------------------------------------------
struct OracleLayerOffsets {
    uint64_t norm_w, in_proj_w, conv1d_w, conv1d_b, dt_bias, A_log, D, mixer_norm_w, out_proj_w;
    uint32_t in_proj_int4, out_proj_int4;
};

struct OracleModelDesc {
    uint32_t d_model, n_layer, d_state, d_conv, expand, vocab, n_heads, d_head, chunk, n_groups;
    uint64_t embed_off, norm_f_off, lm_head_off;
    uint32_t lm_head_int4;
    // mode: 0 = faithful (fp16 activations, reference chunk cap 64 and fp16-staged
    //       prefill state), 1 = fp32 (no intermediate fp16 rounding of activations;
    //       the 130M-shape fp32 parity configuration; weights are read as stored).
    uint32_t mode;
};

struct OracleState {
    std::vector<uint16_t> conv;   // n_layer * xBC * d_conv   (faithful)
    std::vector<float> convf;     // same, fp32 mode
    std::vector<float> ssd;       // n_layer * H * P * N
};

static inline float act_round(const OracleModelDesc& md, float v) { return md.mode == 0 ? hr(v) : v; }

// Linear on fp32 activations with the weight in the file's format.
static void linear_any(const OracleModelDesc& md, const uint8_t* base, uint64_t w_off, int is_int4,
                       uint32_t N_total, uint32_t row0, uint32_t N, uint32_t K,
                       const float* x, uint32_t M, float* y, bool gemm_semantics) {
    const uint8_t* wbytes = base + w_off;
#pragma omp parallel
    {
        std::vector<float> wr(K);
#pragma omp for schedule(static)
        for (int64_t nn = 0; nn < (int64_t)N; ++nn) {
            const uint32_t n = row0 + (uint32_t)nn;
            if (is_int4) {
                const uint8_t* packed = wbytes;
                const uint16_t* scales = reinterpret_cast<const uint16_t*>(wbytes + (size_t)N_total * (K / 2));
                for (uint32_t k = 0; k < K; ++k) {
                    float v = (float)q4_at(packed, K, n, k) * h2f(scales[(size_t)n * (K / 32) + k / 32]);
                    wr[k] = (gemm_semantics && md.mode == 0) ? hr(v) : v;
                }
            } else {
                const uint16_t* w = reinterpret_cast<const uint16_t*>(wbytes);
                for (uint32_t k = 0; k < K; ++k) wr[k] = h2f(w[(size_t)n * K + k]);
            }
            for (uint32_t m = 0; m < M; ++m) {
                float acc = 0.0f;
                const float* xr = x + (size_t)m * K;
                for (uint32_t k = 0; k < K; ++k) acc += wr[k] * xr[k];
                y[(size_t)m * N + nn] = act_round(md, acc);
            }
        }
    }
}

static void rmsnorm_rows(const OracleModelDesc& md, const float* x, const uint16_t* w, float* y,
                         uint32_t rows, uint32_t dim) {
    for (uint32_t r = 0; r < rows; ++r) {
        float ss = 0.0f;
        for (uint32_t i = 0; i < dim; ++i) ss += x[(size_t)r * dim + i] * x[(size_t)r * dim + i];
        float rrms = 1.0f / std::sqrt(ss / (float)dim + 1e-5f);
        for (uint32_t i = 0; i < dim; ++i)
            y[(size_t)r * dim + i] = act_round(md, x[(size_t)r * dim + i] * h2f(w[i]) * rrms);
    }
}

// One Mamba-2 block over L tokens (decode when `decode` != 0 and L == 1).
static void run_block(const OracleModelDesc& md, const uint8_t* base, const OracleLayerOffsets& lo,
                      OracleState& st, uint32_t layer, float* hidden, uint32_t L, bool decode) {
    const uint32_t dm = md.d_model, di = md.expand * md.d_model, N = md.d_state, H = md.n_heads,
                   G = md.n_groups, P = md.d_head, Kc = md.d_conv;
    const uint32_t GN = G * N, xd = di + 2 * GN, proj = di + xd + H;
    std::vector<float> normed((size_t)L * dm), z((size_t)L * di), xbc((size_t)L * xd), dtv((size_t)L * H);
    rmsnorm_rows(md, hidden, reinterpret_cast<const uint16_t*>(base + lo.norm_w), normed.data(), L, dm);
    const bool gemm = !(decode || L == 1);
    linear_any(md, base, lo.in_proj_w, lo.in_proj_int4, proj, 0, di, dm, normed.data(), L, z.data(), gemm);
    linear_any(md, base, lo.in_proj_w, lo.in_proj_int4, proj, di, xd, dm, normed.data(), L, xbc.data(), gemm);
    linear_any(md, base, lo.in_proj_w, lo.in_proj_int4, proj, di + xd, H, dm, normed.data(), L, dtv.data(), gemm);

    const uint16_t* cw = reinterpret_cast<const uint16_t*>(base + lo.conv1d_w);
    const uint16_t* cbias = reinterpret_cast<const uint16_t*>(base + lo.conv1d_b);
    std::vector<float> conv((size_t)L * xd);
    if (!gemm) {
        for (uint32_t d = 0; d < xd; ++d) {
            size_t so = ((size_t)layer * xd + d) * Kc;
            float acc = h2f(cbias[d]);
            if (md.mode == 0) {
                uint16_t* s = st.conv.data() + so;
                for (uint32_t k = 0; k + 1 < Kc; ++k) s[k] = s[k + 1];
                s[Kc - 1] = f2h(xbc[d]);
                for (uint32_t k = 0; k < Kc; ++k) acc += h2f(s[k]) * h2f(cw[(size_t)d * Kc + k]);
            } else {
                float* s = st.convf.data() + so;
                for (uint32_t k = 0; k + 1 < Kc; ++k) s[k] = s[k + 1];
                s[Kc - 1] = xbc[d];
                for (uint32_t k = 0; k < Kc; ++k) acc += s[k] * h2f(cw[(size_t)d * Kc + k]);
            }
            conv[d] = act_round(md, acc);
        }
    } else {
        for (uint32_t t = 0; t < L; ++t)
            for (uint32_t d = 0; d < xd; ++d) {
                float acc = h2f(cbias[d]);
                for (uint32_t tap = 0; tap < Kc; ++tap) {
                    int src = (int)t - (int)(Kc - 1 - tap);
                    if (src >= 0) acc += h2f(cw[(size_t)d * Kc + tap]) * xbc[(size_t)src * xd + d];
                }
                conv[(size_t)t * xd + d] = act_round(md, acc);
            }
    }
    std::vector<float> xs((size_t)L * di), Bs((size_t)L * GN), Cs((size_t)L * GN);
    for (uint32_t t = 0; t < L; ++t)
        for (uint32_t f = 0; f < xd; ++f) {
            float v = act_round(md, silu_f(conv[(size_t)t * xd + f]));
            if (f < di) xs[(size_t)t * di + f] = v;
            else if (f < di + GN) Bs[(size_t)t * GN + f - di] = v;
            else Cs[(size_t)t * GN + f - di - GN] = v;
        }

    const uint16_t* dtb = reinterpret_cast<const uint16_t*>(base + lo.dt_bias);
    const uint16_t* alog = reinterpret_cast<const uint16_t*>(base + lo.A_log);
    const uint16_t* Dsk = reinterpret_cast<const uint16_t*>(base + lo.D);
    float* S0 = st.ssd.data() + (size_t)layer * H * P * N;
    std::vector<float> ys((size_t)L * di);
    const uint32_t hpg = std::max(1u, H / G);
    if (!gemm) {
        for (uint32_t h = 0; h < H; ++h) {
            const uint32_t g = h / hpg;
            const float A = -std::exp(h2f(alog[h]));
            const float dt = clampf(softplus_f(dtv[h] + h2f(dtb[h])), 1e-6f, 1e6f);
            const float decay = std::exp(A * dt), Dh = h2f(Dsk[h]);
            for (uint32_t p = 0; p < P; ++p) {
                float xv = xs[(size_t)h * P + p];
                float* S = S0 + ((size_t)h * P + p) * N;
                float acc = 0.0f;
                for (uint32_t n = 0; n < N; ++n) {
                    float s = decay * S[n] + dt * Bs[(size_t)g * N + n] * xv;
                    S[n] = s;
                    acc += Cs[(size_t)g * N + n] * s;
                }
                ys[(size_t)h * P + p] = act_round(md, acc + Dh * xv);
            }
        }
    } else {
        // Reference prefill caps the chunk at 64 (mamba2_block.cpp:203-206) and stages
        // the state in fp16 (ssd_chunked.metal:116). fp32 mode uses the config chunk.
        const uint32_t C = md.mode == 0 ? std::min(std::min(md.chunk, L), 64u) : std::min(md.chunk, L);
        const uint32_t nch = (L + C - 1) / C;
#pragma omp parallel for schedule(dynamic)
        for (int64_t hh = 0; hh < (int64_t)H; ++hh) {
            const uint32_t h = (uint32_t)hh, g = h / hpg;
            const float A = -std::exp(h2f(alog[h])), Dh = h2f(Dsk[h]), db = h2f(dtb[h]);
            std::vector<float> S((size_t)P * N), DT(C), Lc(C), M((size_t)C * C);
            float* Sg = S0 + (size_t)h * P * N;
            for (size_t i = 0; i < S.size(); ++i) S[i] = act_round(md, Sg[i]);
            for (uint32_t c = 0; c < nch; ++c) {
                const uint32_t t0 = c * C, tl = std::min(C, L - t0);
                for (uint32_t t = 0; t < tl; ++t) DT[t] = clampf(softplus_f(dtv[(size_t)(t0 + t) * H + h] + db), 1e-6f, 1e6f);
                float run = 0.0f;
                for (uint32_t t = 0; t < tl; ++t) { run += A * DT[t]; Lc[t] = run; }
                const float Lend = Lc[tl - 1];
                for (uint32_t t = 0; t < tl; ++t)
                    for (uint32_t j = 0; j <= t; ++j) {
                        float cb = 0.0f;
                        for (uint32_t n = 0; n < N; ++n)
                            cb += Cs[(size_t)(t0 + t) * GN + g * N + n] * Bs[(size_t)(t0 + j) * GN + g * N + n];
                        M[(size_t)t * C + j] = act_round(md, cb * std::exp(Lc[t] - Lc[j]) * DT[j]);
                    }
                for (uint32_t t = 0; t < tl; ++t)
                    for (uint32_t p = 0; p < P; ++p) {
                        float yi = 0.0f;
                        for (uint32_t j = 0; j <= t; ++j) yi += M[(size_t)t * C + j] * xs[(size_t)(t0 + j) * di + h * P + p];
                        float ye = 0.0f;
                        for (uint32_t n = 0; n < N; ++n) ye += Cs[(size_t)(t0 + t) * GN + g * N + n] * S[(size_t)p * N + n];
                        ye *= std::exp(Lc[t]);
                        ys[(size_t)(t0 + t) * di + h * P + p] =
                            act_round(md, yi + ye + Dh * xs[(size_t)(t0 + t) * di + h * P + p]);
                    }
                std::vector<float> SN((size_t)P * N);
                for (uint32_t p = 0; p < P; ++p)
                    for (uint32_t n = 0; n < N; ++n) {
                        float acc = std::exp(Lend) * S[(size_t)p * N + n];
                        for (uint32_t j = 0; j < tl; ++j)
                            acc += std::exp(Lend - Lc[j]) * DT[j] * Bs[(size_t)(t0 + j) * GN + g * N + n] *
                                   xs[(size_t)(t0 + j) * di + h * P + p];
                        SN[(size_t)p * N + n] = act_round(md, acc);
                    }
                S.swap(SN);
            }
            for (size_t i = 0; i < S.size(); ++i) Sg[i] = S[i];
        }
    }

    // gate then norm over full d_inner (mamba2_block.cpp:231-238)
    std::vector<float> gated((size_t)L * di), mo((size_t)L * di);
    for (size_t i = 0; i < gated.size(); ++i) gated[i] = act_round(md, silu_f(z[i]) * ys[i]);
    rmsnorm_rows(md, gated.data(), reinterpret_cast<const uint16_t*>(base + lo.mixer_norm_w), mo.data(), L, di);
    std::vector<float> bo((size_t)L * dm);
    linear_any(md, base, lo.out_proj_w, lo.out_proj_int4, dm, 0, dm, di, mo.data(), L, bo.data(), gemm);
    for (size_t i = 0; i < bo.size(); ++i) hidden[i] = act_round(md, hidden[i] + bo[i]);

    if (!decode) {  // seed conv state from pre-conv xBC (mamba2_block.cpp:285-289)
        for (uint32_t d = 0; d < xd; ++d)
            for (uint32_t k = 0; k < Kc; ++k) {
                int src = (int)L - (int)Kc + (int)k;
                float v = src >= 0 ? xbc[(size_t)src * xd + d] : 0.0f;
                size_t so = ((size_t)layer * xd + d) * Kc + k;
                if (md.mode == 0) st.conv[so] = f2h(v); else st.convf[so] = v;
            }
    }
}

static void compute_logits(const OracleModelDesc& md, const uint8_t* base, const float* hrow, float* logits) {
    std::vector<float> nr(md.d_model);
    rmsnorm_rows(md, hrow, reinterpret_cast<const uint16_t*>(base + md.norm_f_off), nr.data(), 1, md.d_model);
    std::vector<float> out(md.vocab);
    linear_any(md, base, md.lm_head_off, md.lm_head_int4, md.vocab, 0, md.vocab, md.d_model, nr.data(), 1,
               out.data(), false);
    for (uint32_t i = 0; i < md.vocab; ++i) logits[i] = out[i];
}

static void embed_row(const OracleModelDesc& md, const uint8_t* base, uint32_t tok, float* dst) {
    const uint16_t* e = reinterpret_cast<const uint16_t*>(base + md.embed_off) + (size_t)tok * md.d_model;
    for (uint32_t i = 0; i < md.d_model; ++i) dst[i] = h2f(e[i]);
}

// Prefill `L` prompt tokens then greedily decode `n_new` tokens (inference.cpp:14-70,
// eos disabled). Writes the generated ids to `out_tokens` (n_new entries) and, when
// non-null, the logits of the last prompt position to `prefill_logits` (vocab) and
// the logits of every decode position to `step_logits` (n_new-1 rows of vocab).
// When `teacher` is non-null, the decode input at step i is teacher[i] instead of the
// greedy pick (teacher-forced comparison); out_tokens still records the greedy picks.
int lssm_oracle_generate(const uint8_t* base, const OracleModelDesc* mdp, const OracleLayerOffsets* layers,
                         const uint32_t* prompt, uint32_t L, uint32_t n_new, const uint32_t* teacher,
                         uint32_t* out_tokens, float* prefill_logits, float* step_logits) {
    const OracleModelDesc& md = *mdp;
    if (L == 0 || n_new == 0) return 1;
    const uint32_t di = md.expand * md.d_model, xd = di + 2 * md.n_groups * md.d_state;
    OracleState st;
    if (md.mode == 0) st.conv.assign((size_t)md.n_layer * xd * md.d_conv, 0);
    else st.convf.assign((size_t)md.n_layer * xd * md.d_conv, 0.0f);
    st.ssd.assign((size_t)md.n_layer * md.n_heads * md.d_head * md.d_state, 0.0f);
    std::vector<float> hidden((size_t)L * md.d_model), logits(md.vocab);
    for (uint32_t i = 0; i < L; ++i) {
        if (prompt[i] >= md.vocab) return 2;
        embed_row(md, base, prompt[i], hidden.data() + (size_t)i * md.d_model);
    }
    for (uint32_t l = 0; l < md.n_layer; ++l) run_block(md, base, layers[l], st, l, hidden.data(), L, false);
    compute_logits(md, base, hidden.data() + (size_t)(L - 1) * md.d_model, logits.data());
    if (prefill_logits) std::memcpy(prefill_logits, logits.data(), sizeof(float) * md.vocab);
    uint32_t next = lssm_oracle_argmax_f32(logits.data(), md.vocab);
    out_tokens[0] = next;
    std::vector<float> h1(md.d_model);
    for (uint32_t s = 1; s < n_new; ++s) {
        uint32_t inp = teacher ? teacher[s - 1] : next;
        embed_row(md, base, inp, h1.data());
        for (uint32_t l = 0; l < md.n_layer; ++l) run_block(md, base, layers[l], st, l, h1.data(), 1, true);
        compute_logits(md, base, h1.data(), logits.data());
        if (step_logits) std::memcpy(step_logits + (size_t)(s - 1) * md.vocab, logits.data(), sizeof(float) * md.vocab);
        next = lssm_oracle_argmax_f32(logits.data(), md.vocab);
        out_tokens[s] = next;
    }
    return 0;
}

// ---------------------------------------------------------------------------
//  Seeded synthetic weights on the CPU: the same recipe as the GPU generator
//  (lite-ssm_b200/csrc/synth_rng.h), so the CPU baseline and the parity tests can
//  build a bit-identical copy of a synthesized model without a GPU.
//  f16: out[i] = half(value(seed, stream, i, amp)).
//  int4: values rounded to fp16, then the block-32 quantiser above.
// ---------------------------------------------------------------------------
}  // extern "C"
#include "../lite-ssm_b200/csrc/synth_rng.h"
extern "C" {

void lssm_oracle_synth_f32(float* out, uint64_t n, uint64_t seed, uint64_t stream, float amp) {
    for (uint64_t i = 0; i < n; ++i) out[i] = synth_value(seed, stream, i, amp);
}

void lssm_oracle_synth_f16(uint16_t* out, uint64_t n, uint64_t seed, uint64_t stream, float amp) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) out[i] = f2h(synth_value(seed, stream, (uint64_t)i, amp));
}

void lssm_oracle_synth_int4(uint8_t* out, uint32_t N, uint32_t K, uint64_t seed, uint64_t stream, float amp) {
    uint16_t* scales = reinterpret_cast<uint16_t*>(out + (size_t)N * K / 2);
    const uint32_t nb = K / 32;
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < (int64_t)N; ++n) {
        float v[32];
        for (uint32_t b = 0; b < nb; ++b) {
            float absmax = 0.0f;
            for (int j = 0; j < 32; ++j) {
                v[j] = hr(synth_value(seed, stream, (uint64_t)n * K + b * 32 + j, amp));
                absmax = std::max(absmax, std::fabs(v[j]));
            }
            absmax = std::max(absmax, 1e-12f);
            const float scale = absmax / 7.0f;
            scales[(size_t)n * nb + b] = f2h(scale);
            uint8_t* dst = out + (size_t)n * (K / 2) + (size_t)b * 16;
            for (int j = 0; j < 16; ++j) {
                const float q0 = std::min(std::max(std::nearbyint(v[2 * j] / scale), -8.0f), 7.0f);
                const float q1 = std::min(std::max(std::nearbyint(v[2 * j + 1] / scale), -8.0f), 7.0f);
                dst[j] = (uint8_t)((((int)q1 & 0xF) << 4) | ((int)q0 & 0xF));
            }
        }
    }
}

uint32_t lssm_oracle_sizeof_layer_offsets(void) { return (uint32_t)sizeof(OracleLayerOffsets); }
uint32_t lssm_oracle_sizeof_model_desc(void) { return (uint32_t)sizeof(OracleModelDesc); }

}  // extern "C"
