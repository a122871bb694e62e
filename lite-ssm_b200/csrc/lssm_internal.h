// lssm_internal.h — host-side plumbing shared by the C-ABI translation units:
// the context object, thread-local error reporting, status macros and the
// launcher declarations each kernel file exports to the C-ABI layer.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>
#include <vector>

#include "lssm_cuda.h"

struct lssm_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    bool owns_stream = false;
    bool batch_active = false;
    int sm_count = 148;
    // Device-side error word for bounded waits inside kernels (0 = ok).
    int* d_error = nullptr;
    // Graph batching: when set, begin_batch starts a stream capture and
    // commit_and_wait instantiates, launches and keeps the captured graph.
    bool capture_batches = false;
    bool capturing = false;
    cudaGraphExec_t last_graph = nullptr;
    // Device scratch of the ops that need one (INT4 GEMM split-K partials or dequantised
    // weights, the fused in_proj tile), on this context's device. It grows by allocating
    // a larger block; a superseded block that `last_graph` may still reference is kept in
    // `scratch_retired` until that graph is replaced or the context is destroyed.
    void* scratch = nullptr;
    size_t scratch_size = 0;
    std::vector<void*> scratch_retired;
};

namespace lssm {

void set_error(const char* fmt, ...);
lssm_status fail(lssm_status st, const char* fmt, ...);
lssm_status cuda_fail(cudaError_t e, const char* what);

// Called after every op launch: checks the launch, and outside a batch waits for
// completion (the one-shot semantics of src/backend/metal/ops.mm:131-148).
lssm_status finish_op(lssm_ctx* ctx, const char* name);

inline const uint8_t* bp(const void* p, size_t off) { return static_cast<const uint8_t*>(p) + off; }
inline uint8_t* bp(void* p, size_t off) { return static_cast<uint8_t*>(p) + off; }
inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// ---- launchers (kernel files) ------------------------------------------------
// All take device pointers that already include byte offsets; they enqueue on `s`
// and return cudaGetLastError().
cudaError_t launch_rmsnorm_f16(const void* x, const void* w, void* y, uint32_t rows, uint32_t dim, float eps,
                               cudaStream_t s);
cudaError_t launch_silu_f16(const void* x, void* y, uint32_t n, cudaStream_t s);
cudaError_t launch_add_inplace_f16(void* y, const void* x, uint32_t n, cudaStream_t s);
cudaError_t launch_silu_gated_f16(const void* z, const void* g, void* y, uint32_t n, cudaStream_t s);
cudaError_t launch_split_silu_xBC_f16(const void* xBC, void* xo, void* Bo, void* Co, uint32_t L, uint32_t d_inner,
                                      uint32_t d_state, uint32_t n_groups, cudaStream_t s);
cudaError_t launch_causal_conv1d_f16(const void* x, const void* w, const void* bias, void* y, uint32_t B,
                                     uint32_t L, uint32_t D, uint32_t K, cudaStream_t s);
cudaError_t launch_causal_conv1d_update_f16(const void* x_new, void* state, const void* w, const void* bias,
                                            void* y, uint32_t B, uint32_t D, uint32_t K, cudaStream_t s);
cudaError_t launch_seed_conv_state_f16(const void* xBC, void* state, uint32_t L, uint32_t D, uint32_t K,
                                       cudaStream_t s);
// Batched variant used by the engine: xBC (B, L, D) -> state (B, D, K).
cudaError_t launch_seed_conv_state_batched(const void* xBC, void* state, uint32_t B, uint32_t L, uint32_t D,
                                           uint32_t K, cudaStream_t s);

// GEMV family (M <= 8 activation rows). epilogue: 0 store, 1 silu.
cudaError_t launch_gemv_f16(const void* x, const void* w, void* y, uint32_t M, uint32_t N, uint32_t K,
                            const void* norm_w, float eps, int epilogue, cudaStream_t s);
cudaError_t launch_gemv_int4(const void* x, const void* packed, const void* scales, void* y, uint32_t M,
                             uint32_t N, uint32_t K, cudaStream_t s);

// GEMM (M rows of activations). Y[M,N] = X[M,K] W[N,K]^T; epilogue 0 store, 1 silu.
cudaError_t launch_gemm_f16(const void* x, const void* w, void* y, uint32_t M, uint32_t N, uint32_t K,
                            int epilogue, cudaStream_t s);
// INT4 weights dequantised (rounded to fp16, like shaders/linear.metal:538) into
// `scratch` (N*K halves, caller-owned) and multiplied with the fp16 GEMM.
cudaError_t launch_int4_dequant_f16(const void* packed, const void* scales, void* out, uint32_t N, uint32_t K,
                                    cudaStream_t s);
// INT4 GEMM with the dequantisation fused into the tcgen05 pipeline (k_gemm_i4.cu), same
// fp16 rounding of each weight; cudaErrorNotSupported when K % 256 or alignment rule it out.
// cuTensorMapEncodeTiled through the runtime's driver entry point (nullptr if unavailable).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();
// One-time per-device setup of the GEMV kernels (shared-memory limits), from context creation.
void gemv_init();
cudaError_t launch_gemm_i4(const void* x, const void* packed, const void* scales, void* y, uint32_t M, uint32_t N,
                           uint32_t K, int epilogue, cudaStream_t s, float* ws = nullptr, size_t ws_bytes = 0,
                           int* launches = nullptr);

cudaError_t launch_ssd_step(const void* x, const void* B, const void* C, const void* dt_raw, const void* dt_bias,
                            const void* A_log, const void* D, float* state, void* y, uint32_t batch, uint32_t H,
                            uint32_t P, uint32_t N, uint32_t G, float dt_min, float dt_max, uint32_t has_D,
                            cudaStream_t s);

struct SsdArgs {
    const void* X; const void* B; const void* C; const void* dt_raw;
    const void* dt_bias; const void* A_log; const void* D;
    void* Y; float* state;
    uint32_t batch, L, H, P, N, G, chunk;
    float dt_min, dt_max;
    uint32_t has_D;
    uint32_t x_dtype, dt_dtype, param_dtype, y_dtype;
    // Element strides (in elements) for X/Y rows, B/C rows and dt rows; 0 = dense default.
    uint64_t x_row_stride, bc_row_stride, dt_row_stride, y_row_stride;
    // Optional gate (model prefill): when z is set (fp16, rows of z_row_stride, y_dtype f16),
    // Y receives the gated half(silu(z) * half(y)) instead of y (mamba2_block.cpp:231-234).
    const void* z = nullptr;
    uint64_t z_row_stride = 0;
    // Optional scratch of the chunk-parallel scan (carried-state ring + counters,
    // ssd_chunked_cp_scratch bytes); without it the sequential tensor-core scan runs.
    void* ws = nullptr;
    size_t ws_bytes = 0;
    int sm_count = 0;
};
cudaError_t launch_ssd_chunked(const SsdArgs& a, cudaStream_t s);
size_t ssd_chunked_cp_scratch(uint32_t batch, uint32_t H);
cudaError_t launch_ssd_chunked_cp(const SsdArgs& s, void* ws, size_t ws_bytes, int sm_count, cudaStream_t st);
// out[r][c] = half(silu(z[r * z_stride + c]) * y[r][c]) over rows x d (y and out dense; may alias).
cudaError_t launch_gate(const void* z, uint64_t z_stride, const void* y, void* out, uint32_t rows, uint32_t d,
                        cudaStream_t s);

// ssd_step over `batch` sequences with per-sequence strides (elements). When z is set
// the output is the gated value half(silu(z) * half(y)) instead of y.
struct StepArgs {
    const __half* x; const __half* B; const __half* C; const __half* dt_raw;
    const __half* dt_bias; const __half* A_log; const __half* D;
    float* state; __half* y; const __half* z;
    uint32_t batch, H, P, N, G;
    float dt_min, dt_max;
    uint32_t has_D;
    uint64_t x_bs, bc_bs, dt_bs, y_bs, z_bs;
};
cudaError_t launch_ssd_step_ex(const StepArgs& a, cudaStream_t s);

// ---- persistent decode kernel (k_decode_persist.cu) -------------------------
struct PLayer {
    const uint8_t* in_w;       // in_proj packed (proj x dm/2); scales at in_w + proj*dm/2
    const uint8_t* out_w;      // out_proj packed (dm x di/2); scales at out_w + dm*di/2
    const __half* conv_w; const __half* conv_b;
    const __half* dt_bias; const __half* A_log; const __half* D;
    const __half* norm_w; const __half* mixer_norm_w;
    __half* conv_state;        // (B, xd, dconv)
    float* ssd_state;          // (B, H, P, N)
};

struct PParams {
    const PLayer* layers; uint32_t n_layer;
    const __half* embed; const __half* norm_f; const __half* lm_head;
    // in_proj outputs for the ssd phase as exchange words [B][proj], each {fp16 bits, 32-bit
    // epoch} in one 64-bit store (z, x / B / C after conv + SiLU, dt), so data and readiness
    // travel together and a reader polls only the words it needs. Layer l of step t carries
    // epoch epoch0 + t * n_layer + l.
    uint64_t* mb_in;
    uint32_t epoch0;
    float* opart;                            // out_proj partial sums [chunk][seq][d_model] fp32
    __half* gated;
    __half* logits;
    float* part_val; uint32_t* part_idx;     // (gridDim, B)
    uint32_t* cur; uint32_t* history; uint32_t hist_stride; uint32_t n_steps;
    uint32_t* bar; int* err;
    uint32_t B, dm, di, xd, proj, H, P, N, G, dconv, V;
    const void* maps;                        // CUtensorMap[4 * n_layer + 1] in device memory
    uint32_t seg_in, seg_out, seg_lm;        // 128-byte segments per streamed chunk (odd)
    // Optional phase trace of the first step: per CTA, TRACE_PER_LAYER %globaltimer
    // stamps per layer then TRACE_LM stamps for lm_head (null = off).
    uint64_t* trace;
};
constexpr uint32_t TRACE_PER_LAYER = 10, TRACE_LM = 6;
cudaError_t launch_decode_persist(const PParams& prm, int sm_count, cudaStream_t s);
// Host helpers: the shape limits of the persistent kernel and its tensor maps.
struct PersistShape { uint32_t n_layer, B, dm, di, xd, proj, H, P, N, G, dconv, V, sm_count; };
// Returns "" when the kernel can run this shape (and fills the chunk segments), else why not.
const char* decode_persist_plan(const PersistShape& sh, uint32_t* seg_in, uint32_t* seg_out, uint32_t* seg_lm);
size_t decode_persist_maps_bytes(uint32_t n_layer);
// Encodes the 4 * n_layer + 1 tensor maps into host memory `out` (decode_persist_maps_bytes).
bool decode_persist_encode_maps(void* out, const PLayer* layers, const void* lm_head, const PersistShape& sh,
                                uint32_t seg_in, uint32_t seg_out, uint32_t seg_lm);

// ---- head tensor parallelism (comm_nccl.cu, k_tp.cu) -------------------------
lssm_status comm_allreduce_f32(lssm_comm* c, float* buf, size_t n, cudaStream_t s);
lssm_status comm_allgather(lssm_comm* c, const void* src, void* dst, size_t bytes, cudaStream_t s);
int comm_rank(const lssm_comm* c);
int comm_world(const lssm_comm* c);
cudaError_t launch_rowsumsq(const void* x, uint64_t stride, uint32_t rows, uint32_t dim, float* out, cudaStream_t s);
cudaError_t launch_rmsnorm_total(const void* x, uint64_t stride, const void* w, const float* sumsq, uint32_t rows,
                                 uint32_t dim, uint32_t dim_total, float eps, void* y, cudaStream_t s);
cudaError_t launch_residual_f32(void* hidden, const float* part, uint64_t n, cudaStream_t s);
// Peer exchange of the tensor-parallel decode (comm_nccl.cu / k_tp.cu).
constexpr int P2P_MAX_RANKS = 8;
constexpr uint32_t P2P_BLOCKS = 64;       // CTAs (slices of 1024 floats) per exchange
struct P2PPeers {
    uint64_t* recv[P2P_MAX_RANKS];        // rank r's receive area [2][world][cap] words, as mapped here
};
lssm_status comm_p2p_setup(lssm_comm* c, size_t floats);
lssm_status comm_agree(lssm_comm* c, bool ok_local, bool* ok_all);
bool comm_p2p(const lssm_comm* c, size_t floats);
lssm_status comm_p2p_allreduce(lssm_comm* c, const float* part, size_t n, float* out, __half* hidden,
                               cudaStream_t s);
cudaError_t launch_p2p_allreduce(const P2PPeers& peers, const uint64_t* recv_local, uint32_t* epochs, int rank,
                                 int world, size_t cap, const float* part, uint32_t n, float* out, __half* hidden,
                                 uint64_t spin_ns, cudaStream_t s);
uint32_t argmax_chunks(uint32_t Vr);
cudaError_t launch_argmax_chunks(const void* logits, uint32_t ld, uint32_t B, uint32_t Vr, uint32_t v_off, uint2* cpair,
                                 uint32_t* ticket, uint2* out, cudaStream_t s);
cudaError_t launch_argmax_merge(const uint2* pairs, uint32_t world, uint32_t B, uint32_t* cur, uint32_t* history,
                                uint32_t hist_stride, uint32_t* step, const void* embed, void* hidden, uint32_t d_model,
                                cudaStream_t s);

}  // namespace lssm
