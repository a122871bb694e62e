// capi_ops.cu — extern "C" op entry points (include/lssm_cuda.h), one per
// lite_ssm::MetalOps method (include/lite_ssm/ops.hpp:57-244), plus context,
// memory and batching. Dims validation and its wording follow
// src/backend/metal/ops.mm; execution semantics follow ops.mm:82-149 (one-shot
// outside a batch, enqueue-only inside).
#include <cuda_fp16.h>

#include <cstring>
#include <mutex>

#include "device_util.cuh"
#include "lssm_internal.h"

namespace lssm {

static thread_local std::string g_last_error;

void set_error(const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
}

lssm_status fail(lssm_status st, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return st;
}

lssm_status cuda_fail(cudaError_t e, const char* what) {
    if (e == cudaErrorMemoryAllocation)
        return fail(LSSM_ERR_OUT_OF_MEMORY, "%s: %s", what, cudaGetErrorString(e));
    if (e == cudaErrorInvalidValue)
        return fail(LSSM_ERR_INVALID_ARGUMENT, "%s: unsupported shape or layout (%s)", what, cudaGetErrorString(e));
    return fail(LSSM_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int* tc_error_word();

lssm_status finish_op(lssm_ctx* ctx, const char* name) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, name);
    if (ctx->batch_active) return LSSM_OK;
    e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, name);
    int* ew = tc_error_word();
    if (ew) {
        int h = 0;
        cudaMemcpy(&h, ew, sizeof(int), cudaMemcpyDeviceToHost);
        if (h) {
            cudaMemset(ew, 0, sizeof(int));
            return fail(LSSM_ERR_TIMEOUT, "%s: a bounded device wait timed out", name);
        }
    }
    return LSSM_OK;
}

// The context's device scratch (see lssm_ctx::scratch). Growing it never frees a block
// that a kept graph may replay; growing it inside a graph capture is refused, because the
// allocation would not be part of the graph and the old block's users would be recorded.
static lssm_status scratch_reserve(lssm_ctx* ctx, size_t n, void** out) {
    if (ctx->scratch_size < n) {
        if (ctx->capturing)
            return fail(LSSM_ERR_STATE,
                        "scratch of %zu bytes needed inside a captured batch (have %zu): make one call of this "
                        "shape outside the batch first",
                        n, ctx->scratch_size);
        if (ctx->scratch) {
            if (ctx->last_graph) {
                ctx->scratch_retired.push_back(ctx->scratch);
            } else {
                cudaStreamSynchronize(ctx->stream);
                cudaFree(ctx->scratch);
            }
            ctx->scratch = nullptr;
            ctx->scratch_size = 0;
        }
        cudaError_t e = cudaMalloc(&ctx->scratch, n);
        if (e != cudaSuccess) { ctx->scratch = nullptr; return cuda_fail(e, "scratch allocation"); }
        ctx->scratch_size = n;
    }
    *out = ctx->scratch;
    return LSSM_OK;
}

// Scratch for an optional fast path: the context's scratch when it already holds n bytes, or
// after growing it outside a capture; nullptr (no error recorded) when it cannot be had, and
// the op then takes its path without scratch.
static void* scratch_try(lssm_ctx* ctx, size_t n) {
    if (ctx->scratch_size < n && ctx->capturing) return nullptr;
    void* p = nullptr;
    if (scratch_reserve(ctx, n, &p) != LSSM_OK) {
        set_error("");
        return nullptr;
    }
    return p;
}

// Frees the scratch blocks only the (now replaced or destroyed) kept graph referred to.
static void scratch_release_retired(lssm_ctx* ctx) {
    if (ctx->scratch_retired.empty()) return;
    cudaStreamSynchronize(ctx->stream);
    for (void* p : ctx->scratch_retired) cudaFree(p);
    ctx->scratch_retired.clear();
}

cudaError_t launch_gemv_int4_ex(const void* x, const void* packed, const void* scales, void* y, uint32_t M,
                                uint32_t N, uint32_t K, const void* norm_w, float eps, int epilogue,
                                cudaStream_t s);
cudaError_t launch_gemv_f16_f32out(const void* x, const void* w, float* y, uint32_t M, uint32_t N, uint32_t K,
                                   cudaStream_t s);
cudaError_t launch_inproj_route(const float* mm, const void* wconv, const void* cbias, void* z, void* xs, void* Bs,
                                void* Cs, void* dt, void* xbc_pre, uint32_t L, uint32_t d_inner, uint32_t GN,
                                uint32_t H, uint32_t K, cudaStream_t s);

}  // namespace lssm

using namespace lssm;

#define CHECK_CTX(ctx)                                                                         \
    do {                                                                                       \
        if (!(ctx)) return fail(LSSM_ERR_INVALID_ARGUMENT, "%s: null context", __func__);    \
        cudaSetDevice((ctx)->device);                                                          \
    } while (0)

#define LAUNCH(name, expr)                                  \
    do {                                                    \
        cudaError_t _e = (expr);                            \
        if (_e != cudaSuccess) return cuda_fail(_e, name);  \
        return finish_op(ctx, name);                        \
    } while (0)

extern "C" {

const char* lssm_last_error(void) { return g_last_error.c_str(); }
const char* lssm_version(void) { return "lite-ssm-b200 0.1 (sm_100a)"; }

lssm_status lssm_ctx_create(int device, lssm_ctx** out) {
    if (!out) return fail(LSSM_ERR_INVALID_ARGUMENT, "lssm_ctx_create: null out");
    *out = nullptr;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0) return fail(LSSM_ERR_CUDA, "lssm_ctx_create: no CUDA device");
    if (device < 0 || device >= n) return fail(LSSM_ERR_INVALID_ARGUMENT, "lssm_ctx_create: bad device %d", device);
    e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_fail(e, "lssm_ctx_create");
    auto* c = new lssm_ctx();
    c->device = device;
    e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) { delete c; return cuda_fail(e, "lssm_ctx_create: stream"); }
    c->owns_stream = true;
    cudaDeviceGetAttribute(&c->sm_count, cudaDevAttrMultiProcessorCount, device);
    // The device error word of the bounded waits is allocated here, never lazily
    // inside a later op (which might be running under stream capture).
    if (!tc_error_word()) { lssm_ctx_destroy(c); return fail(LSSM_ERR_OUT_OF_MEMORY, "lssm_ctx_create: error word"); }
    // Likewise the driver entry point of the tensor-map encoder: looked up here, outside
    // any capture, so the first tensor-map kernel may be captured into a graph.
    (void)tensor_map_encoder();
    gemv_init();
    cudaGetLastError();
    *out = c;
    return LSSM_OK;
}

lssm_status lssm_ctx_destroy(lssm_ctx* ctx) {
    if (!ctx) return LSSM_OK;
    cudaSetDevice(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    if (ctx->last_graph) cudaGraphExecDestroy(ctx->last_graph);
    ctx->last_graph = nullptr;
    scratch_release_retired(ctx);
    if (ctx->scratch) cudaFree(ctx->scratch);
    if (ctx->owns_stream && ctx->stream) cudaStreamDestroy(ctx->stream);
    delete ctx;
    return LSSM_OK;
}

lssm_status lssm_ctx_set_stream(lssm_ctx* ctx, void* stream) {
    CHECK_CTX(ctx);
    if (ctx->owns_stream && ctx->stream) {
        cudaStreamSynchronize(ctx->stream);
        cudaStreamDestroy(ctx->stream);
    }
    ctx->stream = static_cast<cudaStream_t>(stream);
    ctx->owns_stream = false;
    return LSSM_OK;
}

void* lssm_ctx_stream(lssm_ctx* ctx) { return ctx ? ctx->stream : nullptr; }

int lssm_backend_loaded(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return 0;
    int dev = 0, major = 0, minor = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    return (major == 10 && minor == 0) ? 1 : 0;
}

int lssm_has_kernel(const char* name) {
    static const char* kNames[] = {
        "lite_ssm_common_noop", "rmsnorm_f16",         "silu_f16",          "silu_gated_f16",
        "linear_f16_gemv",      "linear_silu_f16_gemv", "rmsnorm_linear_f16_gemv", "linear_f16_gemm",
        "linear_silu_f16_gemm", "causal_conv1d_f16",   "causal_conv1d_update_f16", "ssd_chunked_f16",
        "ssd_step_f16",         "linear_int4_gemv",    "linear_int4_gemm",  "seed_conv_state_f16",
        "inproj_fused_f16",     "add_inplace_f16",     "split_silu_xBC_f16"};
    if (!name) return 0;
    for (const char* k : kNames)
        if (std::strcmp(k, name) == 0) return 1;
    return 0;
}

lssm_status lssm_begin_batch(lssm_ctx* ctx) {
    CHECK_CTX(ctx);
    if (ctx->batch_active) return fail(LSSM_ERR_STATE, "MetalOps: begin_batch called while batch already active");
    if (ctx->capture_batches) {
        cudaError_t e = cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal);
        if (e != cudaSuccess) return cuda_fail(e, "begin_batch: stream capture");
        ctx->capturing = true;
    }
    ctx->batch_active = true;
    return LSSM_OK;
}

lssm_status lssm_commit_and_wait(lssm_ctx* ctx) {
    CHECK_CTX(ctx);
    if (!ctx->batch_active) return fail(LSSM_ERR_STATE, "MetalOps: commit_and_wait without an active batch");
    ctx->batch_active = false;
    if (ctx->capturing) {
        ctx->capturing = false;
        cudaGraph_t g = nullptr;
        cudaError_t e = cudaStreamEndCapture(ctx->stream, &g);
        if (e != cudaSuccess) return cuda_fail(e, "commit_and_wait: end capture");
        if (ctx->last_graph) { cudaGraphExecDestroy(ctx->last_graph); ctx->last_graph = nullptr; }
        scratch_release_retired(ctx);   // only the replaced graph could still use them
        e = cudaGraphInstantiate(&ctx->last_graph, g, 0);
        cudaGraphDestroy(g);
        if (e != cudaSuccess) { ctx->last_graph = nullptr; return cuda_fail(e, "commit_and_wait: instantiate"); }
        e = cudaGraphLaunch(ctx->last_graph, ctx->stream);
        if (e != cudaSuccess) return cuda_fail(e, "commit_and_wait: graph launch");
    }
    return finish_op(ctx, "forward batch");
}

lssm_status lssm_ctx_set_graph_batching(lssm_ctx* ctx, int enable) {
    CHECK_CTX(ctx);
    if (ctx->batch_active) return fail(LSSM_ERR_STATE, "set_graph_batching: a batch is active");
    ctx->capture_batches = enable != 0;
    return LSSM_OK;
}

lssm_status lssm_replay_batch(lssm_ctx* ctx, uint32_t times) {
    CHECK_CTX(ctx);
    if (!ctx->last_graph) return fail(LSSM_ERR_STATE, "replay_batch: no captured batch");
    if (ctx->batch_active) return fail(LSSM_ERR_STATE, "replay_batch: a batch is active");
    for (uint32_t i = 0; i < times; ++i) {
        cudaError_t e = cudaGraphLaunch(ctx->last_graph, ctx->stream);
        if (e != cudaSuccess) return cuda_fail(e, "replay_batch");
    }
    return LSSM_OK;
}

int lssm_batch_active(lssm_ctx* ctx) { return ctx && ctx->batch_active ? 1 : 0; }

lssm_status lssm_alloc(lssm_ctx* ctx, size_t nbytes, void** dptr) {
    CHECK_CTX(ctx);
    if (!dptr) return fail(LSSM_ERR_INVALID_ARGUMENT, "lssm_alloc: null out");
    cudaError_t e = cudaMalloc(dptr, nbytes ? nbytes : 1);
    if (e != cudaSuccess) return cuda_fail(e, "lssm_alloc");
    return LSSM_OK;
}

lssm_status lssm_free(lssm_ctx* ctx, void* dptr) {
    CHECK_CTX(ctx);
    if (!dptr) return LSSM_OK;
    cudaStreamSynchronize(ctx->stream);
    cudaError_t e = cudaFree(dptr);
    if (e != cudaSuccess) return cuda_fail(e, "lssm_free");
    return LSSM_OK;
}

lssm_status lssm_upload(lssm_ctx* ctx, void* dst, size_t off, const void* src, size_t n) {
    CHECK_CTX(ctx);
    cudaError_t e = cudaMemcpyAsync(bp(dst, off), src, n, cudaMemcpyHostToDevice, ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "lssm_upload");
    e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "lssm_upload");
    return LSSM_OK;
}

lssm_status lssm_download(lssm_ctx* ctx, void* dst, const void* src, size_t off, size_t n) {
    CHECK_CTX(ctx);
    cudaError_t e = cudaMemcpyAsync(dst, bp(src, off), n, cudaMemcpyDeviceToHost, ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "lssm_download");
    e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "lssm_download");
    return LSSM_OK;
}

lssm_status lssm_memset(lssm_ctx* ctx, void* dst, size_t off, int value, size_t n) {
    CHECK_CTX(ctx);
    LAUNCH("lssm_memset", cudaMemsetAsync(bp(dst, off), value, n, ctx->stream));
}

// ---- ops ----------------------------------------------------------------
lssm_status lssm_rmsnorm_f16(lssm_ctx* ctx, const void* x, size_t x_off, const void* w, size_t w_off, void* y,
                             size_t y_off, lssm_rmsnorm_dims d) {
    CHECK_CTX(ctx);
    if (d.dim % 4 != 0) return fail(LSSM_ERR_INVALID_ARGUMENT, "rmsnorm_f16: dim must be a multiple of 4");
    LAUNCH("rmsnorm_f16", launch_rmsnorm_f16(bp(x, x_off), bp(w, w_off), bp(y, y_off), d.rows, d.dim, d.eps,
                                             ctx->stream));
}

static lssm_status gemv_checks(lssm_linear_dims d) {
    if (d.M != 1) return fail(LSSM_ERR_INVALID_ARGUMENT, "dispatch_gemv: M must be 1");
    if (d.K % 4 != 0) return fail(LSSM_ERR_INVALID_ARGUMENT, "dispatch_gemv: K must be a multiple of 4");
    return LSSM_OK;
}

lssm_status lssm_linear_f16_gemv(lssm_ctx* ctx, const void* x, size_t x_off, const void* w, size_t w_off, void* y,
                                 size_t y_off, lssm_linear_dims d) {
    CHECK_CTX(ctx);
    if (lssm_status st = gemv_checks(d)) return st;
    LAUNCH("linear_f16_gemv", launch_gemv_f16(bp(x, x_off), bp(w, w_off), bp(y, y_off), 1, d.N, d.K, nullptr, 0.0f,
                                              0, ctx->stream));
}

lssm_status lssm_linear_silu_f16_gemv(lssm_ctx* ctx, const void* x, size_t x_off, const void* w, size_t w_off,
                                      void* y, size_t y_off, lssm_linear_dims d) {
    CHECK_CTX(ctx);
    if (lssm_status st = gemv_checks(d)) return st;
    LAUNCH("linear_silu_f16_gemv", launch_gemv_f16(bp(x, x_off), bp(w, w_off), bp(y, y_off), 1, d.N, d.K, nullptr,
                                                   0.0f, 1, ctx->stream));
}

lssm_status lssm_rmsnorm_linear_f16_gemv(lssm_ctx* ctx, const void* x, size_t x_off, const void* w_norm,
                                         size_t w_norm_off, const void* w, size_t w_off, void* y, size_t y_off,
                                         lssm_rmslinear_dims d) {
    CHECK_CTX(ctx);
    if (d.K % 4 != 0) return fail(LSSM_ERR_INVALID_ARGUMENT, "rmsnorm_linear_f16_gemv: K must be a multiple of 4");
    LAUNCH("rmsnorm_linear_f16_gemv", launch_gemv_f16(bp(x, x_off), bp(w, w_off), bp(y, y_off), 1, d.N, d.K,
                                                      bp(w_norm, w_norm_off), d.eps, 0, ctx->stream));
}

lssm_status lssm_linear_f16_gemm(lssm_ctx* ctx, const void* x, size_t x_off, const void* w, size_t w_off, void* y,
                                 size_t y_off, lssm_linear_dims d) {
    CHECK_CTX(ctx);
    LAUNCH("linear_f16_gemm", launch_gemm_f16(bp(x, x_off), bp(w, w_off), bp(y, y_off), d.M, d.N, d.K, 0,
                                              ctx->stream));
}

lssm_status lssm_linear_silu_f16_gemm(lssm_ctx* ctx, const void* x, size_t x_off, const void* w, size_t w_off,
                                      void* y, size_t y_off, lssm_linear_dims d) {
    CHECK_CTX(ctx);
    LAUNCH("linear_silu_f16_gemm", launch_gemm_f16(bp(x, x_off), bp(w, w_off), bp(y, y_off), d.M, d.N, d.K, 1,
                                                   ctx->stream));
}

lssm_status lssm_linear_int4_gemv(lssm_ctx* ctx, const void* x, size_t x_off, const void* w, size_t w_packed_off,
                                  const void* w_scl, size_t w_scales_off, void* y, size_t y_off,
                                  lssm_linear_dims d) {
    CHECK_CTX(ctx);
    if (d.M != 1) return fail(LSSM_ERR_INVALID_ARGUMENT, "linear_int4_gemv: M must be 1");
    if (d.K % 32 != 0) return fail(LSSM_ERR_INVALID_ARGUMENT, "linear_int4_gemv: K must be a multiple of 32");
    LAUNCH("linear_int4_gemv", launch_gemv_int4(bp(x, x_off), bp(w, w_packed_off), bp(w_scl, w_scales_off),
                                                bp(y, y_off), 1, d.N, d.K, ctx->stream));
}

lssm_status lssm_linear_f16_gemv_rows(lssm_ctx* ctx, const void* x, size_t x_off, const void* w, size_t w_off,
                                      void* y, size_t y_off, lssm_linear_dims d) {
    CHECK_CTX(ctx);
    if (d.M < 1 || d.M > 8) return fail(LSSM_ERR_INVALID_ARGUMENT, "linear_f16_gemv_rows: M must be 1..8");
    LAUNCH("linear_f16_gemv_rows", launch_gemv_f16(bp(x, x_off), bp(w, w_off), bp(y, y_off), d.M, d.N, d.K, nullptr,
                                                   0.0f, 0, ctx->stream));
}

lssm_status lssm_linear_int4_gemv_rows(lssm_ctx* ctx, const void* x, size_t x_off, const void* w,
                                       size_t w_packed_off, const void* w_scl, size_t w_scales_off, void* y,
                                       size_t y_off, lssm_linear_dims d) {
    CHECK_CTX(ctx);
    if (d.M < 1 || d.M > 8) return fail(LSSM_ERR_INVALID_ARGUMENT, "linear_int4_gemv_rows: M must be 1..8");
    if (d.K % 32 != 0) return fail(LSSM_ERR_INVALID_ARGUMENT, "linear_int4_gemv_rows: K must be a multiple of 32");
    LAUNCH("linear_int4_gemv_rows", launch_gemv_int4(bp(x, x_off), bp(w, w_packed_off), bp(w_scl, w_scales_off),
                                                     bp(y, y_off), d.M, d.N, d.K, ctx->stream));
}

lssm_status lssm_linear_int4_gemm(lssm_ctx* ctx, const void* x, size_t x_off, const void* w, size_t w_packed_off,
                                  const void* w_scl, size_t w_scales_off, void* y, size_t y_off,
                                  lssm_linear_dims d) {
    CHECK_CTX(ctx);
    if (d.K % 32 != 0) return fail(LSSM_ERR_INVALID_ARGUMENT, "linear_int4_gemm: K must be a multiple of 32");
    if (d.M == 0 || d.N == 0) return finish_op(ctx, "linear_int4_gemm");
    {
        // decode-size M may split K over CTAs: fp32 partials (up to 8 splits) in the scratch
        void* ws = nullptr;
        const size_t ws_bytes = d.M <= 128 ? (size_t)8 * d.M * d.N * 4 : 0;
        if (ws_bytes)
            if (lssm_status st = scratch_reserve(ctx, ws_bytes, &ws)) return st;
        const cudaError_t e = launch_gemm_i4(bp(x, x_off), bp(w, w_packed_off), bp(w_scl, w_scales_off), bp(y, y_off),
                                             d.M, d.N, d.K, 0, ctx->stream, static_cast<float*>(ws), ws_bytes);
        if (e != cudaErrorNotSupported) {
            if (e != cudaSuccess) return cuda_fail(e, "linear_int4_gemm");
            return finish_op(ctx, "linear_int4_gemm");
        }
        cudaGetLastError();   // clear the not-supported status: dequantise, then the fp16 GEMM
    }
    void* scratch = nullptr;
    if (lssm_status st = scratch_reserve(ctx, (size_t)d.N * d.K * 2, &scratch)) return st;
    cudaError_t e = launch_int4_dequant_f16(bp(w, w_packed_off), bp(w_scl, w_scales_off), scratch, d.N, d.K,
                                            ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "linear_int4_gemm");
    LAUNCH("linear_int4_gemm", launch_gemm_f16(bp(x, x_off), scratch, bp(y, y_off), d.M, d.N, d.K, 0, ctx->stream));
}

lssm_status lssm_silu_f16(lssm_ctx* ctx, const void* x, size_t x_off, void* y, size_t y_off, uint32_t n) {
    CHECK_CTX(ctx);
    LAUNCH("silu_f16", launch_silu_f16(bp(x, x_off), bp(y, y_off), n, ctx->stream));
}

lssm_status lssm_add_inplace_f16(lssm_ctx* ctx, void* y, size_t y_off, const void* x, size_t x_off, uint32_t n) {
    CHECK_CTX(ctx);
    LAUNCH("add_inplace_f16", launch_add_inplace_f16(bp(y, y_off), bp(x, x_off), n, ctx->stream));
}

lssm_status lssm_split_silu_xBC_f16(lssm_ctx* ctx, const void* xBC, size_t xBC_off, void* x_out, size_t x_off,
                                    void* B_out, size_t B_off, void* C_out, size_t C_off, uint32_t L,
                                    uint32_t d_inner, uint32_t d_state, uint32_t n_groups) {
    CHECK_CTX(ctx);
    LAUNCH("split_silu_xBC_f16", launch_split_silu_xBC_f16(bp(xBC, xBC_off), bp(x_out, x_off), bp(B_out, B_off),
                                                           bp(C_out, C_off), L, d_inner, d_state, n_groups,
                                                           ctx->stream));
}

lssm_status lssm_silu_gated_f16(lssm_ctx* ctx, const void* x, size_t x_off, const void* gate, size_t gate_off,
                                void* y, size_t y_off, uint32_t n) {
    CHECK_CTX(ctx);
    LAUNCH("silu_gated_f16", launch_silu_gated_f16(bp(x, x_off), bp(gate, gate_off), bp(y, y_off), n, ctx->stream));
}

lssm_status lssm_causal_conv1d_f16(lssm_ctx* ctx, const void* x, size_t x_off, const void* w, size_t w_off,
                                   const void* bias, size_t bias_off, void* y, size_t y_off, lssm_conv1d_dims d) {
    CHECK_CTX(ctx);
    LAUNCH("causal_conv1d_f16", launch_causal_conv1d_f16(bp(x, x_off), bp(w, w_off), bias ? bp(bias, bias_off) : nullptr,
                                                         bp(y, y_off), d.B, d.L, d.D, d.K, ctx->stream));
}

lssm_status lssm_causal_conv1d_update_f16(lssm_ctx* ctx, const void* x_new, size_t x_off, void* state,
                                          size_t state_off, const void* w, size_t w_off, const void* bias,
                                          size_t bias_off, void* y, size_t y_off, lssm_conv1d_dims d) {
    CHECK_CTX(ctx);
    LAUNCH("causal_conv1d_update_f16",
           launch_causal_conv1d_update_f16(bp(x_new, x_off), bp(state, state_off), bp(w, w_off),
                                           bias ? bp(bias, bias_off) : nullptr, bp(y, y_off), d.B, d.D, d.K,
                                           ctx->stream));
}

lssm_status lssm_seed_conv_state_f16(lssm_ctx* ctx, const void* xBC, size_t xBC_off, void* state, size_t state_off,
                                     uint32_t L, uint32_t D, uint32_t K) {
    CHECK_CTX(ctx);
    LAUNCH("seed_conv_state_f16", launch_seed_conv_state_f16(bp(xBC, xBC_off), bp(state, state_off), L, D, K,
                                                             ctx->stream));
}

lssm_status lssm_inproj_fused_f16(lssm_ctx* ctx, const void* normed, size_t normed_off, const void* W_in,
                                  size_t w_in_off, const void* W_conv, size_t w_conv_off, const void* conv_b,
                                  size_t conv_b_off, void* proj_z, size_t z_off, void* ssd_x, size_t x_off,
                                  void* ssd_B, size_t b_off, void* ssd_C, size_t c_off, void* proj_dt,
                                  size_t dt_off, void* proj_xBC, size_t xBC_off, lssm_fused_inproj_dims d) {
    CHECK_CTX(ctx);
    const uint32_t GN = d.n_groups * d.d_state, xd = d.d_inner + 2 * GN;
    if (d.proj_dim != d.d_inner + xd + d.n_heads)
        return fail(LSSM_ERR_INVALID_ARGUMENT, "inproj_fused_f16: proj_dim != d_inner + xBC_dim + n_heads");
    if (d.L == 0) return finish_op(ctx, "inproj_fused_f16");
    if (d.L > 16) return fail(LSSM_ERR_INVALID_ARGUMENT, "inproj_fused_f16: L must be <= 16");
    void* scratch = nullptr;
    if (lssm_status st = scratch_reserve(ctx, (size_t)d.L * d.proj_dim * 4, &scratch)) return st;
    float* mm = static_cast<float*>(scratch);
    // fp32 matmul tile (the reference keeps it fp32 in threadgroup memory, fused.metal:76)
    for (uint32_t m0 = 0; m0 < d.L; m0 += 8) {
        const uint32_t mr = d.L - m0 < 8 ? d.L - m0 : 8;
        cudaError_t e = launch_gemv_f16_f32out(bp(normed, normed_off + (size_t)m0 * d.d_model * 2), bp(W_in, w_in_off),
                                               mm + (size_t)m0 * d.proj_dim, mr, d.proj_dim, d.d_model, ctx->stream);
        if (e != cudaSuccess) return cuda_fail(e, "inproj_fused_f16");
    }
    LAUNCH("inproj_fused_f16",
           launch_inproj_route(mm, bp(W_conv, w_conv_off), bp(conv_b, conv_b_off), bp(proj_z, z_off), bp(ssd_x, x_off),
                               bp(ssd_B, b_off), bp(ssd_C, c_off), bp(proj_dt, dt_off), bp(proj_xBC, xBC_off), d.L,
                               d.d_inner, GN, d.n_heads, d.d_conv, ctx->stream));
}

lssm_status lssm_ssd_chunked_f16(lssm_ctx* ctx, const void* X, size_t X_off, const void* B, size_t B_off,
                                 const void* C, size_t C_off, const void* dt_raw, size_t dt_off, const void* dt_bias,
                                 size_t db_off, const void* A_log, size_t A_off, const void* D_skip, size_t D_off,
                                 void* Y, size_t Y_off, void* state_io, size_t S_off, lssm_ssd_dims d) {
    CHECK_CTX(ctx);
    if (d.chunk_size == 0) return fail(LSSM_ERR_INVALID_ARGUMENT, "ssd_chunked_f16: chunk_size must be >= 1");
    SsdArgs a{};
    a.X = bp(X, X_off); a.B = bp(B, B_off); a.C = bp(C, C_off); a.dt_raw = bp(dt_raw, dt_off);
    a.dt_bias = bp(dt_bias, db_off); a.A_log = bp(A_log, A_off); a.D = bp(D_skip, D_off);
    a.Y = bp(Y, Y_off); a.state = reinterpret_cast<float*>(bp(state_io, S_off));
    a.batch = 1; a.L = d.L; a.H = d.H; a.P = d.P; a.N = d.N; a.G = d.n_groups ? d.n_groups : 1; a.chunk = d.chunk_size;
    a.dt_min = d.dt_min; a.dt_max = d.dt_max; a.has_D = d.has_D;
    a.x_dtype = 0; a.dt_dtype = 0; a.param_dtype = 0; a.y_dtype = 0;
    a.ws_bytes = ssd_chunked_cp_scratch(a.batch, a.H);
    a.ws = scratch_try(ctx, a.ws_bytes);
    a.sm_count = ctx->sm_count;
    LAUNCH("ssd_chunked_f16", launch_ssd_chunked(a, ctx->stream));
}

lssm_status lssm_ssd_step_f16(lssm_ctx* ctx, const void* x, size_t x_off, const void* B, size_t B_off, const void* C,
                              size_t C_off, const void* dt_raw, size_t dt_off, const void* dt_bias, size_t db_off,
                              const void* A_log, size_t A_off, const void* D_skip, size_t D_off, void* state,
                              size_t S_off, void* y, size_t y_off, lssm_ssd_step_dims d) {
    CHECK_CTX(ctx);
    LAUNCH("ssd_step_f16", launch_ssd_step(bp(x, x_off), bp(B, B_off), bp(C, C_off), bp(dt_raw, dt_off),
                                           bp(dt_bias, db_off), bp(A_log, A_off), bp(D_skip, D_off),
                                           reinterpret_cast<float*>(bp(state, S_off)), bp(y, y_off), 1, d.H, d.P, d.N,
                                           d.n_groups ? d.n_groups : 1, d.dt_min, d.dt_max, d.has_D, ctx->stream));
}

lssm_status lssm_ssd_chunked_batched(lssm_ctx* ctx, const void* X, const void* B, const void* C, const void* dt_raw,
                                     const void* dt_bias, const void* A_log, const void* D_skip, void* Y,
                                     void* state_io, lssm_ssd_batched_dims d) {
    CHECK_CTX(ctx);
    if (d.x_dtype > 1 || d.dt_dtype > 2 || d.param_dtype > 2 || d.y_dtype > 2)
        return fail(LSSM_ERR_INVALID_ARGUMENT, "ssd_chunked_batched: unsupported dtype code");
    SsdArgs a{};
    a.X = X; a.B = B; a.C = C; a.dt_raw = dt_raw; a.dt_bias = dt_bias; a.A_log = A_log; a.D = D_skip;
    a.Y = Y; a.state = static_cast<float*>(state_io);
    a.batch = d.batch; a.L = d.L; a.H = d.H; a.P = d.P; a.N = d.N; a.G = d.n_groups ? d.n_groups : 1;
    a.chunk = d.chunk_size; a.dt_min = d.dt_min; a.dt_max = d.dt_max; a.has_D = d.has_D;
    a.x_dtype = d.x_dtype; a.dt_dtype = d.dt_dtype; a.param_dtype = d.param_dtype; a.y_dtype = d.y_dtype;
    a.ws_bytes = ssd_chunked_cp_scratch(a.batch, a.H);
    a.ws = scratch_try(ctx, a.ws_bytes);
    a.sm_count = ctx->sm_count;
    LAUNCH("ssd_chunked_batched", launch_ssd_chunked(a, ctx->stream));
}

lssm_status lssm_ssd_step_batched(lssm_ctx* ctx, const void* x, const void* B, const void* C, const void* dt_raw,
                                  const void* dt_bias, const void* A_log, const void* D_skip, void* state_io, void* y,
                                  lssm_ssd_batched_dims d) {
    CHECK_CTX(ctx);
    if (!d.batch || !d.H || !d.P || !d.N) return LSSM_OK;
    const uint32_t G = d.n_groups ? d.n_groups : 1;
    if (d.H % G) return fail(LSSM_ERR_INVALID_ARGUMENT, "ssd_step_batched: n_heads must be a multiple of n_groups");
    StepArgs a{};
    a.x = static_cast<const __half*>(x); a.B = static_cast<const __half*>(B); a.C = static_cast<const __half*>(C);
    a.dt_raw = static_cast<const __half*>(dt_raw); a.dt_bias = static_cast<const __half*>(dt_bias);
    a.A_log = static_cast<const __half*>(A_log); a.D = static_cast<const __half*>(D_skip);
    a.state = static_cast<float*>(state_io); a.y = static_cast<__half*>(y); a.z = nullptr;
    a.batch = d.batch; a.H = d.H; a.P = d.P; a.N = d.N; a.G = G;
    a.dt_min = d.dt_min; a.dt_max = d.dt_max; a.has_D = d.has_D;
    a.x_bs = (uint64_t)d.H * d.P; a.bc_bs = (uint64_t)G * d.N; a.dt_bs = d.H; a.y_bs = (uint64_t)d.H * d.P; a.z_bs = 0;
    LAUNCH("ssd_step_batched", launch_ssd_step_ex(a, ctx->stream));
}

}  // extern "C"
