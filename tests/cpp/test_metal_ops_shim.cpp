// Self-checking test of the C++ drop-in class lite_ssm::MetalOps
// (include/lite_ssm_b200/ops.hpp over liblssm_cuda.so), written the way the reference's
// own C++ tests drive its backend (tests/test_metal_ops.cpp:31-49 kernel list).
//
//   test_metal_ops_shim cpu   -- no GPU: construction must throw std::runtime_error
//   test_metal_ops_shim gpu   -- kernel list, ops against host reference loops, batching,
//                                and the dims-check exceptions
//
// Exit status 0 = pass. Host reference math is fp32 with fp16 rounding at the kernels'
// storage points; tolerances are stated at each check.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include "lite_ssm_b200/ops.hpp"

using namespace lite_ssm;

namespace {

int g_fail = 0;
#define CHECK(cond, ...)                                   \
    do {                                                   \
        if (!(cond)) {                                     \
            std::printf("FAIL %s:%d: ", __FILE__, __LINE__); \
            std::printf(__VA_ARGS__);                      \
            std::printf("\n");                             \
            ++g_fail;                                      \
        }                                                  \
    } while (0)

// IEEE binary16 <-> binary32, round to nearest even.
uint16_t f2h(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    int32_t e = (int32_t)((x >> 23) & 0xFF) - 127 + 15;
    uint32_t m = x & 0x7FFFFFu;
    if (((x >> 23) & 0xFF) == 0xFF) return (uint16_t)(sign | 0x7C00u | (m ? 0x200u : 0));
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        m |= 0x800000u;
        const int shift = 14 - e;
        uint32_t r = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (r & 1))) ++r;
        return (uint16_t)(sign | r);
    }
    uint32_t r = ((uint32_t)e << 10) | (m >> 13);
    const uint32_t rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1))) ++r;
    return (uint16_t)(sign | r);
}

float h2f(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1F, m = h & 0x3FFu;
    uint32_t x;
    if (e == 0) {
        if (m == 0) x = sign;
        else {
            int ee = -1;
            do { m <<= 1; ++ee; } while (!(m & 0x400u));
            x = sign | ((uint32_t)(127 - 15 - ee) << 23) | ((m & 0x3FFu) << 13);
        }
    } else if (e == 31) {
        x = sign | 0x7F800000u | (m << 13);
    } else {
        x = sign | ((e - 15 + 127) << 23) | (m << 13);
    }
    float f;
    std::memcpy(&f, &x, 4);
    return f;
}

float rh(float f) { return h2f(f2h(f)); }   // round through fp16

std::vector<uint16_t> rand_h(size_t n, std::mt19937& g, float lo = -1.0f, float hi = 1.0f) {
    std::uniform_real_distribution<float> u(lo, hi);
    std::vector<uint16_t> v(n);
    for (auto& x : v) x = f2h(u(g));
    return v;
}

template <class T>
std::vector<T> down(const DeviceBuffer& b, size_t n) {
    std::vector<T> v(n);
    b.download(v.data(), n * sizeof(T));
    return v;
}

int run_gpu() {
    MetalOps ops;
    CHECK(ops.metallib_loaded(), "kernels not loaded for this GPU");
    std::printf("[shim] kernel library: %s\n", ops.metallib_path().c_str());
    const char* kernels[] = {"lite_ssm_common_noop", "rmsnorm_f16", "silu_f16", "silu_gated_f16", "linear_f16_gemv",
                             "linear_silu_f16_gemv", "rmsnorm_linear_f16_gemv", "linear_f16_gemm",
                             "linear_silu_f16_gemm", "causal_conv1d_f16", "causal_conv1d_update_f16",
                             "ssd_chunked_f16", "ssd_step_f16", "linear_int4_gemv", "linear_int4_gemm",
                             "seed_conv_state_f16", "inproj_fused_f16"};
    for (const char* k : kernels) CHECK(ops.has_pipeline(k), "missing kernel %s", k);
    CHECK(!ops.has_pipeline("no_such_kernel"), "has_pipeline accepted an unknown name");

    std::mt19937 g(7);
    // ---- rmsnorm_f16: y = x * w * rsqrt(mean(x^2) + eps), rows 3 x dim 256 (|err| <= 2 fp16 ulp)
    {
        const uint32_t rows = 3, dim = 256;
        auto x = rand_h(rows * dim, g), w = rand_h(dim, g, 0.5f, 1.5f);
        DeviceBuffer bx(ops, x.size() * 2), bw(ops, w.size() * 2), by(ops, x.size() * 2);
        bx.upload(x.data(), x.size() * 2);
        bw.upload(w.data(), w.size() * 2);
        ops.rmsnorm_f16(bx.metal_buffer(), 0, bw.metal_buffer(), 0, by.metal_buffer(), 0, {rows, dim, 1e-5f});
        auto y = down<uint16_t>(by, x.size());
        double worst = 0;
        for (uint32_t r = 0; r < rows; ++r) {
            double ss = 0;
            for (uint32_t k = 0; k < dim; ++k) ss += (double)h2f(x[r * dim + k]) * h2f(x[r * dim + k]);
            const float rr = 1.0f / std::sqrt((float)(ss / dim) + 1e-5f);
            for (uint32_t k = 0; k < dim; ++k) {
                const float ref = rh(h2f(x[r * dim + k]) * h2f(w[k]) * rr);
                worst = std::max(worst, (double)std::fabs(h2f(y[r * dim + k]) - ref) / (std::fabs(ref) * 9.8e-4 + 1e-6));
            }
        }
        CHECK(worst <= 2.0, "rmsnorm_f16 off by %.2f fp16 ulps", worst);
    }
    // ---- silu_f16 and add_inplace_f16 inside one batch (|err| <= 2 ulp)
    {
        const uint32_t n = 1000;
        auto a = rand_h(n, g, -4, 4), b = rand_h(n, g);
        DeviceBuffer ba(ops, n * 2), bb(ops, n * 2), bs(ops, n * 2);
        ba.upload(a.data(), n * 2);
        bb.upload(b.data(), n * 2);
        ops.begin_batch();
        CHECK(ops.batch_active(), "batch_active() false inside a batch");
        ops.silu_f16(ba.metal_buffer(), 0, bs.metal_buffer(), 0, n);
        ops.add_inplace_f16(bs.metal_buffer(), 0, bb.metal_buffer(), 0, n);
        ops.commit_and_wait();
        CHECK(!ops.batch_active(), "batch_active() true after commit_and_wait");
        auto s = down<uint16_t>(bs, n);
        double worst = 0;
        for (uint32_t i = 0; i < n; ++i) {
            const float av = h2f(a[i]);
            const float silu = rh(av / (1.0f + std::exp(-av)));
            const float ref = rh(silu + h2f(b[i]));
            worst = std::max(worst, (double)std::fabs(h2f(s[i]) - ref) / (std::fabs(ref) * 9.8e-4 + 1e-4));
        }
        CHECK(worst <= 2.0, "silu + add_inplace off by %.2f ulps", worst);
    }
    // ---- linear_int4_gemv: y[n] = sum_k q(n,k) * scale(n,k/32) * x[k] (shaders/linear.metal:440-474), rtol 2e-3
    {
        const uint32_t N = 96, K = 512;
        std::vector<uint8_t> packed(N * K / 2);
        std::vector<uint16_t> scales(N * K / 32);
        std::uniform_int_distribution<int> nib(0, 255);
        for (auto& v : packed) v = (uint8_t)nib(g);
        for (auto& v : scales) v = f2h(std::uniform_real_distribution<float>(0.01f, 0.05f)(g));
        auto x = rand_h(K, g);
        std::vector<uint8_t> wbuf(packed.size() + scales.size() * 2);
        std::memcpy(wbuf.data(), packed.data(), packed.size());
        std::memcpy(wbuf.data() + packed.size(), scales.data(), scales.size() * 2);
        DeviceBuffer bw(ops, wbuf.size()), bx(ops, K * 2), by(ops, N * 2);
        bw.upload(wbuf.data(), wbuf.size());
        bx.upload(x.data(), K * 2);
        ops.linear_int4_gemv(bx.metal_buffer(), 0, bw.metal_buffer(), 0, bw.metal_buffer(), packed.size(),
                             by.metal_buffer(), 0, {1, N, K});
        auto y = down<uint16_t>(by, N);
        double worst = 0;
        for (uint32_t n = 0; n < N; ++n) {
            double acc = 0, mag = 0;
            for (uint32_t k = 0; k < K; ++k) {
                const uint8_t byte = packed[n * (K / 2) + k / 2];
                const int v = (k & 1) ? (byte >> 4) : (byte & 0xF);
                const int q = v < 8 ? v : v - 16;
                const double w = q * (double)h2f(scales[n * (K / 32) + k / 32]);
                acc += w * h2f(x[k]);
                mag += std::fabs(w * h2f(x[k]));
            }
            worst = std::max(worst, std::fabs(h2f(y[n]) - acc) / (mag * 2e-3 + 1e-3));
        }
        CHECK(worst <= 1.0, "linear_int4_gemv error %.2f x tolerance", worst);
    }
    // ---- ssd_step_f16 (shaders/ssd_step.metal:55-76), H 4, P 8, N 16, G 2, fp32 state; rtol 4e-3
    {
        const uint32_t H = 4, P = 8, N = 16, G = 2;
        auto x = rand_h(H * P, g), Bm = rand_h(G * N, g), Cm = rand_h(G * N, g), dt = rand_h(H, g, -2, 0);
        auto db = rand_h(H, g, -0.5f, 0.5f), al = rand_h(H, g, 0, 2), D = rand_h(H, g);
        std::vector<float> S(H * P * N);
        for (auto& v : S) v = std::uniform_real_distribution<float>(-1, 1)(g);
        DeviceBuffer bx(ops, x.size() * 2), bB(ops, Bm.size() * 2), bC(ops, Cm.size() * 2), bdt(ops, H * 2),
            bdb(ops, H * 2), bal(ops, H * 2), bD(ops, H * 2), bS(ops, S.size() * 4), by(ops, H * P * 2);
        bx.upload(x.data(), x.size() * 2);
        bB.upload(Bm.data(), Bm.size() * 2);
        bC.upload(Cm.data(), Cm.size() * 2);
        bdt.upload(dt.data(), H * 2);
        bdb.upload(db.data(), H * 2);
        bal.upload(al.data(), H * 2);
        bD.upload(D.data(), H * 2);
        bS.upload(S.data(), S.size() * 4);
        ops.ssd_step_f16(bx.metal_buffer(), 0, bB.metal_buffer(), 0, bC.metal_buffer(), 0, bdt.metal_buffer(), 0,
                         bdb.metal_buffer(), 0, bal.metal_buffer(), 0, bD.metal_buffer(), 0, bS.metal_buffer(), 0,
                         by.metal_buffer(), 0, {H, P, N, G, 1e-6f, 1e6f, 1});
        auto y = down<uint16_t>(by, H * P);
        auto S2 = down<float>(bS, S.size());
        double worst_y = 0, worst_s = 0;
        for (uint32_t h = 0; h < H; ++h) {
            const uint32_t gg = h / (H / G);
            const float t = h2f(dt[h]) + h2f(db[h]);
            const float sp = t > 20.0f ? t : std::log(1.0f + std::exp(t));
            const float d = std::fmin(std::fmax(sp, 1e-6f), 1e6f);
            const float decay = std::exp(-std::exp(h2f(al[h])) * d);
            for (uint32_t p = 0; p < P; ++p) {
                double acc = 0, mag = 0;
                const float xv = h2f(x[h * P + p]);
                for (uint32_t n = 0; n < N; ++n) {
                    const size_t i = ((size_t)h * P + p) * N + n;
                    const float s = decay * S[i] + d * h2f(Bm[gg * N + n]) * xv;
                    worst_s = std::max(worst_s, (double)std::fabs(S2[i] - s) / (std::fabs(s) * 4e-3 + 1e-4));
                    acc += (double)h2f(Cm[gg * N + n]) * s;
                    mag += std::fabs((double)h2f(Cm[gg * N + n]) * s);
                }
                acc += h2f(D[h]) * xv;
                worst_y = std::max(worst_y, std::fabs(h2f(y[h * P + p]) - acc) / (mag * 4e-3 + 2e-3));
            }
        }
        CHECK(worst_s <= 1.0 && worst_y <= 1.0, "ssd_step_f16 state %.2f / y %.2f x tolerance", worst_s, worst_y);
    }
    // ---- dims checks throw std::runtime_error with the backend's message (ops.mm:179-181)
    {
        DeviceBuffer b(ops, 64);
        bool threw = false;
        try {
            ops.rmsnorm_f16(b.metal_buffer(), 0, b.metal_buffer(), 0, b.metal_buffer(), 0, {1, 6, 1e-5f});
        } catch (const std::runtime_error& e) {
            threw = std::strlen(e.what()) > 0;
            std::printf("[shim] expected error: %s\n", e.what());
        }
        CHECK(threw, "rmsnorm_f16 with dim 6 (not a multiple of 4) did not throw");
        threw = false;
        try {
            ops.linear_int4_gemv(b.metal_buffer(), 0, b.metal_buffer(), 0, b.metal_buffer(), 0, b.metal_buffer(), 0,
                                 {1, 8, 33});
        } catch (const std::runtime_error&) {
            threw = true;
        }
        CHECK(threw, "linear_int4_gemv with K not a multiple of 32 did not throw");
    }
    return g_fail;
}

int run_cpu() {
    // Without a CUDA device the constructor reports the failure the way the Metal backend
    // reports a missing device: a std::runtime_error, not a crash.
    try {
        MetalOps ops;
        std::printf("[shim] a CUDA device is present; construction succeeded\n");
        return ops.metallib_loaded() ? 0 : 1;
    } catch (const std::runtime_error& e) {
        std::printf("[shim] no device: %s\n", e.what());
        return std::strlen(e.what()) > 0 ? 0 : 1;
    }
}

}  // namespace

int main(int argc, char** argv) {
    const std::string mode = argc > 1 ? argv[1] : "gpu";
    const int rc = mode == "cpu" ? run_cpu() : run_gpu();
    std::printf("[shim] %s: %s\n", mode.c_str(), rc == 0 ? "PASS" : "FAIL");
    return rc == 0 ? 0 : 1;
}
