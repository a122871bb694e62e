// capi_noalloc.cu — lssm_inproj_fused_f16_noalloc: the fused in_proj op with its
// scratch in a fixed device array instead of memory allocated at call time.
//
// Who needs this: callers that cannot allocate device memory when they call an op.
// Examples are a host framework whose own allocator owns the whole device-memory
// budget, a serving loop where cudaMalloc / cudaFree would block or synchronise the
// device in the middle of a request, and a process that must not fail with
// out-of-memory once it is running. lssm_inproj_fused_f16 grows a scratch buffer
// with cudaMalloc on demand; this variant never allocates.
//
// The scratch is `g_inproj_tile`, a file-scope __device__ array of
// LSSM_NOALLOC_SCRATCH_BYTES (4 MiB). Every GPU that loads this library holds it
// until the process exits. It holds the fp32 matmul tile of one call (L x proj_dim
// floats), so a call needs L * proj_dim * 4 <= 4 MiB (with L <= 16 that allows
// proj_dim up to 65536); larger requests are rejected with LSSM_ERR_INVALID_ARGUMENT.
//
// The device address of the array is looked up once per device with
// cudaGetSymbolAddress, on that device's first call (the lookup is host-side only
// and allocates nothing). All calls on a device share the one array and it keeps
// the last call's contents; every element a call reads is written earlier in the
// same call, so nothing needs clearing. Calls that overlap on the GPU (two streams,
// or two host threads with their own contexts) race on the array and must be
// serialised by the caller.
#include <cuda_fp16.h>

#include <mutex>

#include "lssm_internal.h"

#define LSSM_NOALLOC_SCRATCH_BYTES (4u << 20)

static __device__ __align__(256) uint8_t g_inproj_tile[LSSM_NOALLOC_SCRATCH_BYTES];

namespace lssm {
cudaError_t launch_gemv_f16_f32out(const void* x, const void* w, float* y, uint32_t M, uint32_t N, uint32_t K,
                                   cudaStream_t s);
cudaError_t launch_inproj_route(const float* mm, const void* wconv, const void* cbias, void* z, void* xs, void* Bs,
                                void* Cs, void* dt, void* xbc_pre, uint32_t L, uint32_t d_inner, uint32_t GN,
                                uint32_t H, uint32_t K, cudaStream_t s);
}  // namespace lssm

using namespace lssm;

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_lookup_mutex;
float* g_tile_ptr[kMaxDevices] = {};

// Device address of g_inproj_tile for the current device (looked up once per device).
lssm_status tile_for_device(int device, float** out) {
    if (device < 0 || device >= kMaxDevices) return fail(LSSM_ERR_INVALID_ARGUMENT, "inproj_fused_f16_noalloc: device %d out of range", device);
    std::lock_guard<std::mutex> lock(g_lookup_mutex);
    if (!g_tile_ptr[device]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_inproj_tile);
        if (e != cudaSuccess) return cuda_fail(e, "inproj_fused_f16_noalloc: cudaGetSymbolAddress");
        g_tile_ptr[device] = static_cast<float*>(p);
    }
    *out = g_tile_ptr[device];
    return LSSM_OK;
}

}  // namespace

extern "C" lssm_status lssm_inproj_fused_f16_noalloc(lssm_ctx* ctx, const void* normed, size_t normed_off,
                                                     const void* W_in, size_t w_in_off, const void* W_conv,
                                                     size_t w_conv_off, const void* conv_b, size_t conv_b_off,
                                                     void* proj_z, size_t z_off, void* ssd_x, size_t x_off,
                                                     void* ssd_B, size_t b_off, void* ssd_C, size_t c_off,
                                                     void* proj_dt, size_t dt_off, void* proj_xBC, size_t xBC_off,
                                                     lssm_fused_inproj_dims d) {
    if (!ctx) return fail(LSSM_ERR_INVALID_ARGUMENT, "inproj_fused_f16_noalloc: null context");
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e != cudaSuccess) return cuda_fail(e, "inproj_fused_f16_noalloc");
    const uint32_t GN = d.n_groups * d.d_state, xd = d.d_inner + 2 * GN;
    if (d.proj_dim != d.d_inner + xd + d.n_heads)
        return fail(LSSM_ERR_INVALID_ARGUMENT, "inproj_fused_f16_noalloc: proj_dim != d_inner + xBC_dim + n_heads");
    if (d.L > 16) return fail(LSSM_ERR_INVALID_ARGUMENT, "inproj_fused_f16_noalloc: L must be <= 16");
    const uint64_t need = (uint64_t)d.L * d.proj_dim * sizeof(float);
    if (need > LSSM_NOALLOC_SCRATCH_BYTES)
        return fail(LSSM_ERR_INVALID_ARGUMENT,
                    "inproj_fused_f16_noalloc: L * proj_dim * 4 = %llu bytes exceeds the %u-byte static scratch",
                    (unsigned long long)need, LSSM_NOALLOC_SCRATCH_BYTES);
    if (d.L == 0) return finish_op(ctx, "inproj_fused_f16_noalloc");
    float* mm = nullptr;
    if (lssm_status st = tile_for_device(ctx->device, &mm)) return st;
    for (uint32_t m0 = 0; m0 < d.L; m0 += 8) {
        const uint32_t mr = d.L - m0 < 8 ? d.L - m0 : 8;
        e = launch_gemv_f16_f32out(bp(normed, normed_off + (size_t)m0 * d.d_model * 2), bp(W_in, w_in_off),
                                   mm + (size_t)m0 * d.proj_dim, mr, d.proj_dim, d.d_model, ctx->stream);
        if (e != cudaSuccess) return cuda_fail(e, "inproj_fused_f16_noalloc");
    }
    e = launch_inproj_route(mm, bp(W_conv, w_conv_off), bp(conv_b, conv_b_off), bp(proj_z, z_off), bp(ssd_x, x_off),
                            bp(ssd_B, b_off), bp(ssd_C, c_off), bp(proj_dt, dt_off), bp(proj_xBC, xBC_off), d.L,
                            d.d_inner, GN, d.n_heads, d.d_conv, ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "inproj_fused_f16_noalloc");
    // the same completion path as every other op: launch error check, then (outside a
    // batch) wait for the stream and read the device error word
    return finish_op(ctx, "inproj_fused_f16_noalloc");
}
