#pragma once
// lite_ssm_b200/ops.hpp — drop-in replacement for lite-ssm's `lite_ssm::MetalOps`
// (include/lite_ssm/ops.hpp:57-244 of the reference) on B200.
//
// Same namespace, class name, dims structs and method signatures, so the reference's
// model code (src/model/*.cpp) compiles against it unchanged. Every method forwards to
// the C ABI of liblssm_cuda.so (include/lssm_cuda.h) and, like the Metal backend,
// throws std::runtime_error on bad dims or a device error, with the C ABI's error text.
//
// Buffers: a MetalBufferHandle is a device pointer (from DeviceBuffer below, or any
// cudaMalloc'd base); offsets are byte offsets from it, as in the reference. There is
// no unified memory on an x86 host with a B200, so host data moves with
// DeviceBuffer::upload / download instead of writing through `contents()`.
//
// Threading: one MetalOps per host thread (it owns a CUDA stream), as the reference
// uses one MetalOps per thread. Outside a batch every op waits for completion;
// between begin_batch() and commit_and_wait() ops are only enqueued.

#include <cstddef>
#include <cstdint>
#include <memory>
#include <string>
#include <string_view>

namespace lite_ssm {

using MetalBufferHandle = void*;

struct LinearDims     { uint32_t M; uint32_t N; uint32_t K; };
struct RMSNormDims    { uint32_t rows; uint32_t dim; float eps; };
struct RMSLinearDims  { uint32_t N; uint32_t K; float eps; };
struct Conv1dDims     { uint32_t B; uint32_t L; uint32_t D; uint32_t K; };

struct SSDDims {
    uint32_t L;
    uint32_t H;
    uint32_t P;
    uint32_t N;
    uint32_t n_groups;
    uint32_t chunk_size;
    float    dt_min;
    float    dt_max;
    uint32_t has_D;        // 0/1
};

struct SSDStepDims {
    uint32_t H;
    uint32_t P;
    uint32_t N;
    uint32_t n_groups;
    float    dt_min;
    float    dt_max;
    uint32_t has_D;
};

class MetalOps {
public:
    MetalOps();                      // device 0, a stream of its own
    explicit MetalOps(int device);
    ~MetalOps();
    MetalOps(const MetalOps&)            = delete;
    MetalOps& operator=(const MetalOps&) = delete;

    // True when the CUDA kernels are present for this GPU (the metallib probe of the reference).
    bool metallib_loaded() const;
    // True if the backend implements the named kernel (names of tests/test_metal_ops.cpp:31-49).
    bool has_pipeline(std::string_view name);
    // Path of the loaded kernel library (liblssm_cuda.so).
    const std::string& metallib_path() const;

    void begin_batch();
    void commit_and_wait();
    bool batch_active() const;

    void rmsnorm_f16(MetalBufferHandle x, std::size_t x_off,
                     MetalBufferHandle w, std::size_t w_off,
                     MetalBufferHandle y, std::size_t y_off,
                     RMSNormDims dims);

    void linear_f16_gemv(MetalBufferHandle x, std::size_t x_off,
                         MetalBufferHandle w, std::size_t w_off,
                         MetalBufferHandle y, std::size_t y_off,
                         LinearDims dims);

    void linear_silu_f16_gemv(MetalBufferHandle x, std::size_t x_off,
                              MetalBufferHandle w, std::size_t w_off,
                              MetalBufferHandle y, std::size_t y_off,
                              LinearDims dims);

    void rmsnorm_linear_f16_gemv(MetalBufferHandle x,      std::size_t x_off,
                                 MetalBufferHandle w_norm, std::size_t w_norm_off,
                                 MetalBufferHandle w,      std::size_t w_off,
                                 MetalBufferHandle y,      std::size_t y_off,
                                 RMSLinearDims dims);

    void linear_f16_gemm(MetalBufferHandle x, std::size_t x_off,
                         MetalBufferHandle w, std::size_t w_off,
                         MetalBufferHandle y, std::size_t y_off,
                         LinearDims dims);

    void linear_silu_f16_gemm(MetalBufferHandle x, std::size_t x_off,
                              MetalBufferHandle w, std::size_t w_off,
                              MetalBufferHandle y, std::size_t y_off,
                              LinearDims dims);

    void linear_int4_gemv(MetalBufferHandle x,       std::size_t x_off,
                          MetalBufferHandle w,       std::size_t w_packed_off,
                          MetalBufferHandle w_scl,   std::size_t w_scales_off,
                          MetalBufferHandle y,       std::size_t y_off,
                          LinearDims dims);

    void linear_int4_gemm(MetalBufferHandle x,       std::size_t x_off,
                          MetalBufferHandle w,       std::size_t w_packed_off,
                          MetalBufferHandle w_scl,   std::size_t w_scales_off,
                          MetalBufferHandle y,       std::size_t y_off,
                          LinearDims dims);

    void silu_f16(MetalBufferHandle x, std::size_t x_off,
                  MetalBufferHandle y, std::size_t y_off,
                  uint32_t n);

    void add_inplace_f16(MetalBufferHandle y, std::size_t y_off,
                         MetalBufferHandle x, std::size_t x_off,
                         uint32_t n);

    void split_silu_xBC_f16(MetalBufferHandle xBC,   std::size_t xBC_off,
                            MetalBufferHandle x_out, std::size_t x_off,
                            MetalBufferHandle B_out, std::size_t B_off,
                            MetalBufferHandle C_out, std::size_t C_off,
                            uint32_t L, uint32_t d_inner, uint32_t d_state,
                            uint32_t n_groups);

    void silu_gated_f16(MetalBufferHandle x,    std::size_t x_off,
                        MetalBufferHandle gate, std::size_t gate_off,
                        MetalBufferHandle y,    std::size_t y_off,
                        uint32_t n);

    void causal_conv1d_f16(MetalBufferHandle x,    std::size_t x_off,
                           MetalBufferHandle w,    std::size_t w_off,
                           MetalBufferHandle bias, std::size_t bias_off,
                           MetalBufferHandle y,    std::size_t y_off,
                           Conv1dDims dims);

    void causal_conv1d_update_f16(MetalBufferHandle x_new, std::size_t x_off,
                                  MetalBufferHandle state, std::size_t state_off,
                                  MetalBufferHandle w,     std::size_t w_off,
                                  MetalBufferHandle bias,  std::size_t bias_off,
                                  MetalBufferHandle y,     std::size_t y_off,
                                  Conv1dDims dims);

    void seed_conv_state_f16(MetalBufferHandle xBC,   std::size_t xBC_off,
                             MetalBufferHandle state, std::size_t state_off,
                             uint32_t L, uint32_t D, uint32_t K);

    struct FusedInProjDims {
        uint32_t L;
        uint32_t d_model;
        uint32_t d_inner;
        uint32_t d_state;
        uint32_t n_groups;
        uint32_t n_heads;
        uint32_t d_conv;
        uint32_t proj_dim;     // d_inner + xBC_dim + n_heads
    };
    void inproj_fused_f16(MetalBufferHandle normed,   std::size_t normed_off,
                          MetalBufferHandle W_in,     std::size_t w_in_off,
                          MetalBufferHandle W_conv,   std::size_t w_conv_off,
                          MetalBufferHandle conv_b,   std::size_t conv_b_off,
                          MetalBufferHandle proj_z,   std::size_t z_off,
                          MetalBufferHandle ssd_x,    std::size_t x_off,
                          MetalBufferHandle ssd_B,    std::size_t b_off,
                          MetalBufferHandle ssd_C,    std::size_t c_off,
                          MetalBufferHandle proj_dt,  std::size_t dt_off,
                          MetalBufferHandle proj_xBC, std::size_t xBC_off,
                          FusedInProjDims dims);

    void ssd_chunked_f16(MetalBufferHandle X,        std::size_t X_off,
                         MetalBufferHandle B,        std::size_t B_off,
                         MetalBufferHandle C,        std::size_t C_off,
                         MetalBufferHandle dt_raw,   std::size_t dt_off,
                         MetalBufferHandle dt_bias,  std::size_t db_off,
                         MetalBufferHandle A_log,    std::size_t A_off,
                         MetalBufferHandle D_skip,   std::size_t D_off,
                         MetalBufferHandle Y,        std::size_t Y_off,
                         MetalBufferHandle state_io, std::size_t S_off,
                         SSDDims dims);

    void ssd_step_f16(MetalBufferHandle x,        std::size_t x_off,
                      MetalBufferHandle B,        std::size_t B_off,
                      MetalBufferHandle C,        std::size_t C_off,
                      MetalBufferHandle dt_raw,   std::size_t dt_off,
                      MetalBufferHandle dt_bias,  std::size_t db_off,
                      MetalBufferHandle A_log,    std::size_t A_off,
                      MetalBufferHandle D_skip,   std::size_t D_off,
                      MetalBufferHandle state,    std::size_t S_off,
                      MetalBufferHandle y,        std::size_t y_off,
                      SSDStepDims dims);

    struct Impl;
    Impl* impl() const { return impl_.get(); }

private:
    std::unique_ptr<Impl> impl_;
};

// Device allocation used as a MetalBufferHandle (stands in for the reference's
// DeviceBuffer / UnifiedBuffer, include/lite_ssm/allocator.hpp): device memory, moved to
// and from the host with explicit copies on the owning MetalOps' stream.
class DeviceBuffer {
public:
    DeviceBuffer(MetalOps& ops, std::size_t nbytes);
    ~DeviceBuffer();
    DeviceBuffer(const DeviceBuffer&)            = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;

    MetalBufferHandle metal_buffer() const { return ptr_; }
    std::size_t size() const { return nbytes_; }
    void upload(const void* src, std::size_t nbytes, std::size_t off = 0);
    void download(void* dst, std::size_t nbytes, std::size_t off = 0) const;
    void zero();

private:
    MetalOps& ops_;
    void* ptr_ = nullptr;
    std::size_t nbytes_ = 0;
};

}  // namespace lite_ssm
