// metal_ops.cpp — lite_ssm::MetalOps on B200: each method forwards to the C ABI of
// liblssm_cuda.so (include/lssm_cuda.h) and turns a non-OK status into
// std::runtime_error carrying the C ABI's error text, the error behaviour of
// src/backend/metal/ops.mm (dims checks :179-181, :207-212, :323-324, :347;
// command-buffer errors :107-110, :144-147).
#include "lite_ssm_b200/ops.hpp"

#include <dlfcn.h>

#include <stdexcept>
#include <string>

#include "lssm_cuda.h"

namespace lite_ssm {

namespace {

void ok(lssm_status st) {
    if (st != LSSM_OK) throw std::runtime_error(lssm_last_error());
}

lssm_linear_dims cv(LinearDims d) { return {d.M, d.N, d.K}; }
lssm_rmsnorm_dims cv(RMSNormDims d) { return {d.rows, d.dim, d.eps}; }
lssm_rmslinear_dims cv(RMSLinearDims d) { return {d.N, d.K, d.eps}; }
lssm_conv1d_dims cv(Conv1dDims d) { return {d.B, d.L, d.D, d.K}; }
lssm_ssd_dims cv(SSDDims d) { return {d.L, d.H, d.P, d.N, d.n_groups, d.chunk_size, d.dt_min, d.dt_max, d.has_D}; }
lssm_ssd_step_dims cv(SSDStepDims d) { return {d.H, d.P, d.N, d.n_groups, d.dt_min, d.dt_max, d.has_D}; }
lssm_fused_inproj_dims cv(MetalOps::FusedInProjDims d) {
    return {d.L, d.d_model, d.d_inner, d.d_state, d.n_groups, d.n_heads, d.d_conv, d.proj_dim};
}

std::string library_path() {
    Dl_info info{};
    if (dladdr(reinterpret_cast<void*>(&lssm_version), &info) && info.dli_fname) return info.dli_fname;
    return "liblssm_cuda.so";
}

}  // namespace

struct MetalOps::Impl {
    lssm_ctx* ctx = nullptr;
    std::string path;
};

MetalOps::MetalOps() : MetalOps(0) {}

MetalOps::MetalOps(int device) : impl_(std::make_unique<Impl>()) {
    impl_->path = library_path();
    ok(lssm_ctx_create(device, &impl_->ctx));
}

MetalOps::~MetalOps() {
    if (impl_ && impl_->ctx) lssm_ctx_destroy(impl_->ctx);
}

bool MetalOps::metallib_loaded() const { return lssm_backend_loaded() == 1; }
bool MetalOps::has_pipeline(std::string_view name) { return lssm_has_kernel(std::string(name).c_str()) == 1; }
const std::string& MetalOps::metallib_path() const { return impl_->path; }

void MetalOps::begin_batch() { ok(lssm_begin_batch(impl_->ctx)); }
void MetalOps::commit_and_wait() { ok(lssm_commit_and_wait(impl_->ctx)); }
bool MetalOps::batch_active() const { return lssm_batch_active(impl_->ctx) == 1; }

void MetalOps::rmsnorm_f16(MetalBufferHandle x, std::size_t x_off, MetalBufferHandle w, std::size_t w_off,
                           MetalBufferHandle y, std::size_t y_off, RMSNormDims dims) {
    ok(lssm_rmsnorm_f16(impl_->ctx, x, x_off, w, w_off, y, y_off, cv(dims)));
}

void MetalOps::linear_f16_gemv(MetalBufferHandle x, std::size_t x_off, MetalBufferHandle w, std::size_t w_off,
                               MetalBufferHandle y, std::size_t y_off, LinearDims dims) {
    ok(lssm_linear_f16_gemv(impl_->ctx, x, x_off, w, w_off, y, y_off, cv(dims)));
}

void MetalOps::linear_silu_f16_gemv(MetalBufferHandle x, std::size_t x_off, MetalBufferHandle w, std::size_t w_off,
                                    MetalBufferHandle y, std::size_t y_off, LinearDims dims) {
    ok(lssm_linear_silu_f16_gemv(impl_->ctx, x, x_off, w, w_off, y, y_off, cv(dims)));
}

void MetalOps::rmsnorm_linear_f16_gemv(MetalBufferHandle x, std::size_t x_off, MetalBufferHandle w_norm,
                                       std::size_t w_norm_off, MetalBufferHandle w, std::size_t w_off,
                                       MetalBufferHandle y, std::size_t y_off, RMSLinearDims dims) {
    ok(lssm_rmsnorm_linear_f16_gemv(impl_->ctx, x, x_off, w_norm, w_norm_off, w, w_off, y, y_off, cv(dims)));
}

void MetalOps::linear_f16_gemm(MetalBufferHandle x, std::size_t x_off, MetalBufferHandle w, std::size_t w_off,
                               MetalBufferHandle y, std::size_t y_off, LinearDims dims) {
    ok(lssm_linear_f16_gemm(impl_->ctx, x, x_off, w, w_off, y, y_off, cv(dims)));
}

void MetalOps::linear_silu_f16_gemm(MetalBufferHandle x, std::size_t x_off, MetalBufferHandle w, std::size_t w_off,
                                    MetalBufferHandle y, std::size_t y_off, LinearDims dims) {
    ok(lssm_linear_silu_f16_gemm(impl_->ctx, x, x_off, w, w_off, y, y_off, cv(dims)));
}

void MetalOps::linear_int4_gemv(MetalBufferHandle x, std::size_t x_off, MetalBufferHandle w,
                                std::size_t w_packed_off, MetalBufferHandle w_scl, std::size_t w_scales_off,
                                MetalBufferHandle y, std::size_t y_off, LinearDims dims) {
    ok(lssm_linear_int4_gemv(impl_->ctx, x, x_off, w, w_packed_off, w_scl, w_scales_off, y, y_off, cv(dims)));
}

void MetalOps::linear_int4_gemm(MetalBufferHandle x, std::size_t x_off, MetalBufferHandle w,
                                std::size_t w_packed_off, MetalBufferHandle w_scl, std::size_t w_scales_off,
                                MetalBufferHandle y, std::size_t y_off, LinearDims dims) {
    ok(lssm_linear_int4_gemm(impl_->ctx, x, x_off, w, w_packed_off, w_scl, w_scales_off, y, y_off, cv(dims)));
}

void MetalOps::silu_f16(MetalBufferHandle x, std::size_t x_off, MetalBufferHandle y, std::size_t y_off, uint32_t n) {
    ok(lssm_silu_f16(impl_->ctx, x, x_off, y, y_off, n));
}

void MetalOps::add_inplace_f16(MetalBufferHandle y, std::size_t y_off, MetalBufferHandle x, std::size_t x_off,
                               uint32_t n) {
    ok(lssm_add_inplace_f16(impl_->ctx, y, y_off, x, x_off, n));
}

void MetalOps::split_silu_xBC_f16(MetalBufferHandle xBC, std::size_t xBC_off, MetalBufferHandle x_out,
                                  std::size_t x_off, MetalBufferHandle B_out, std::size_t B_off,
                                  MetalBufferHandle C_out, std::size_t C_off, uint32_t L, uint32_t d_inner,
                                  uint32_t d_state, uint32_t n_groups) {
    ok(lssm_split_silu_xBC_f16(impl_->ctx, xBC, xBC_off, x_out, x_off, B_out, B_off, C_out, C_off, L, d_inner,
                               d_state, n_groups));
}

void MetalOps::silu_gated_f16(MetalBufferHandle x, std::size_t x_off, MetalBufferHandle gate, std::size_t gate_off,
                              MetalBufferHandle y, std::size_t y_off, uint32_t n) {
    ok(lssm_silu_gated_f16(impl_->ctx, x, x_off, gate, gate_off, y, y_off, n));
}

void MetalOps::causal_conv1d_f16(MetalBufferHandle x, std::size_t x_off, MetalBufferHandle w, std::size_t w_off,
                                 MetalBufferHandle bias, std::size_t bias_off, MetalBufferHandle y, std::size_t y_off,
                                 Conv1dDims dims) {
    ok(lssm_causal_conv1d_f16(impl_->ctx, x, x_off, w, w_off, bias, bias_off, y, y_off, cv(dims)));
}

void MetalOps::causal_conv1d_update_f16(MetalBufferHandle x_new, std::size_t x_off, MetalBufferHandle state,
                                        std::size_t state_off, MetalBufferHandle w, std::size_t w_off,
                                        MetalBufferHandle bias, std::size_t bias_off, MetalBufferHandle y,
                                        std::size_t y_off, Conv1dDims dims) {
    ok(lssm_causal_conv1d_update_f16(impl_->ctx, x_new, x_off, state, state_off, w, w_off, bias, bias_off, y, y_off,
                                     cv(dims)));
}

void MetalOps::seed_conv_state_f16(MetalBufferHandle xBC, std::size_t xBC_off, MetalBufferHandle state,
                                   std::size_t state_off, uint32_t L, uint32_t D, uint32_t K) {
    ok(lssm_seed_conv_state_f16(impl_->ctx, xBC, xBC_off, state, state_off, L, D, K));
}

void MetalOps::inproj_fused_f16(MetalBufferHandle normed, std::size_t normed_off, MetalBufferHandle W_in,
                                std::size_t w_in_off, MetalBufferHandle W_conv, std::size_t w_conv_off,
                                MetalBufferHandle conv_b, std::size_t conv_b_off, MetalBufferHandle proj_z,
                                std::size_t z_off, MetalBufferHandle ssd_x, std::size_t x_off,
                                MetalBufferHandle ssd_B, std::size_t b_off, MetalBufferHandle ssd_C,
                                std::size_t c_off, MetalBufferHandle proj_dt, std::size_t dt_off,
                                MetalBufferHandle proj_xBC, std::size_t xBC_off, FusedInProjDims dims) {
    ok(lssm_inproj_fused_f16(impl_->ctx, normed, normed_off, W_in, w_in_off, W_conv, w_conv_off, conv_b, conv_b_off,
                             proj_z, z_off, ssd_x, x_off, ssd_B, b_off, ssd_C, c_off, proj_dt, dt_off, proj_xBC,
                             xBC_off, cv(dims)));
}

void MetalOps::ssd_chunked_f16(MetalBufferHandle X, std::size_t X_off, MetalBufferHandle B, std::size_t B_off,
                               MetalBufferHandle C, std::size_t C_off, MetalBufferHandle dt_raw, std::size_t dt_off,
                               MetalBufferHandle dt_bias, std::size_t db_off, MetalBufferHandle A_log,
                               std::size_t A_off, MetalBufferHandle D_skip, std::size_t D_off, MetalBufferHandle Y,
                               std::size_t Y_off, MetalBufferHandle state_io, std::size_t S_off, SSDDims dims) {
    ok(lssm_ssd_chunked_f16(impl_->ctx, X, X_off, B, B_off, C, C_off, dt_raw, dt_off, dt_bias, db_off, A_log, A_off,
                            D_skip, D_off, Y, Y_off, state_io, S_off, cv(dims)));
}

void MetalOps::ssd_step_f16(MetalBufferHandle x, std::size_t x_off, MetalBufferHandle B, std::size_t B_off,
                            MetalBufferHandle C, std::size_t C_off, MetalBufferHandle dt_raw, std::size_t dt_off,
                            MetalBufferHandle dt_bias, std::size_t db_off, MetalBufferHandle A_log, std::size_t A_off,
                            MetalBufferHandle D_skip, std::size_t D_off, MetalBufferHandle state, std::size_t S_off,
                            MetalBufferHandle y, std::size_t y_off, SSDStepDims dims) {
    ok(lssm_ssd_step_f16(impl_->ctx, x, x_off, B, B_off, C, C_off, dt_raw, dt_off, dt_bias, db_off, A_log, A_off,
                         D_skip, D_off, state, S_off, y, y_off, cv(dims)));
}

// ---- DeviceBuffer ------------------------------------------------------------
DeviceBuffer::DeviceBuffer(MetalOps& ops, std::size_t nbytes) : ops_(ops), nbytes_(nbytes) {
    ok(lssm_alloc(ops_.impl()->ctx, nbytes ? nbytes : 1, &ptr_));
}

DeviceBuffer::~DeviceBuffer() {
    if (ptr_) lssm_free(ops_.impl()->ctx, ptr_);
}

void DeviceBuffer::upload(const void* src, std::size_t nbytes, std::size_t off) {
    if (off + nbytes > nbytes_) throw std::runtime_error("DeviceBuffer::upload: range exceeds the buffer");
    ok(lssm_upload(ops_.impl()->ctx, ptr_, off, src, nbytes));
}

void DeviceBuffer::download(void* dst, std::size_t nbytes, std::size_t off) const {
    if (off + nbytes > nbytes_) throw std::runtime_error("DeviceBuffer::download: range exceeds the buffer");
    ok(lssm_download(ops_.impl()->ctx, dst, ptr_, off, nbytes));
}

void DeviceBuffer::zero() { ok(lssm_memset(ops_.impl()->ctx, ptr_, 0, 0, nbytes_)); }

}  // namespace lite_ssm
