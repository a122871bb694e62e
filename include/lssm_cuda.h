/*
 * lssm_cuda.h — C ABI of the B200 (sm_100a) backend for lite-ssm's Mamba-2 hot path.
 *
 * Every entry point takes plain pointers, sizes and POD structs: no C++ or torch
 * types cross this boundary, so any FFI (ctypes, cgo, JNI, a C++ shim) can bind it.
 *
 * Drop-in mapping. lite-ssm's engine calls its compute backend through the
 * concrete class `lite_ssm::MetalOps` (include/lite_ssm/ops.hpp:57-244). Each op
 * there takes `(MetalBufferHandle buf, size_t byte_off)` pairs plus a POD dims
 * struct. Here `buf` is a device base pointer (from lssm_alloc or any cudaMalloc)
 * and the kernel reads `buf + byte_off`; the dims structs are field-for-field the
 * same as ops.hpp:30-55. Each op cites the MetalOps method it replaces.
 *
 * Synchronisation mirrors MetalOps (src/backend/metal/ops.mm:82-149): outside a
 * batch every op runs to completion before returning (one-shot semantics); between
 * lssm_begin_batch and lssm_commit_and_wait ops are only enqueued on the context's
 * stream and commit waits for all of them.
 *
 * Errors: every call returns an lssm_status; the message of the last failure on
 * the calling thread is available from lssm_last_error(). Where MetalOps throws
 * std::runtime_error for bad dims (ops.mm:179-181, 207-212, 323-324, 347), the
 * same condition returns LSSM_ERR_INVALID_ARGUMENT with the same wording.
 *
 * Threading: one lssm_ctx per host thread (as one MetalOps per thread). Device
 * weights may be shared read-only across contexts.
 */
#ifndef LSSM_CUDA_H
#define LSSM_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum lssm_status {
    LSSM_OK = 0,
    LSSM_ERR_INVALID_ARGUMENT = 1,
    LSSM_ERR_CUDA = 2,
    LSSM_ERR_STATE = 3,
    LSSM_ERR_FORMAT = 4,
    LSSM_ERR_NOT_FOUND = 5,
    LSSM_ERR_OUT_OF_MEMORY = 6,
    LSSM_ERR_TIMEOUT = 7
} lssm_status;

typedef struct lssm_ctx lssm_ctx;

/* ---- dims: field-for-field include/lite_ssm/ops.hpp:30-55 ---------------- */
typedef struct { uint32_t M, N, K; } lssm_linear_dims;                 /* LinearDims    ops.hpp:30 */
typedef struct { uint32_t rows, dim; float eps; } lssm_rmsnorm_dims;  /* RMSNormDims   ops.hpp:31 */
typedef struct { uint32_t N, K; float eps; } lssm_rmslinear_dims;     /* RMSLinearDims ops.hpp:32 */
typedef struct { uint32_t B, L, D, K; } lssm_conv1d_dims;             /* Conv1dDims    ops.hpp:33 */
typedef struct {                                                       /* SSDDims       ops.hpp:35-45 */
    uint32_t L, H, P, N, n_groups, chunk_size;
    float dt_min, dt_max;
    uint32_t has_D;
} lssm_ssd_dims;
typedef struct {                                                       /* SSDStepDims   ops.hpp:47-55 */
    uint32_t H, P, N, n_groups;
    float dt_min, dt_max;
    uint32_t has_D;
} lssm_ssd_step_dims;
typedef struct {                                                       /* MetalOps::FusedInProjDims ops.hpp:193-202 */
    uint32_t L, d_model, d_inner, d_state, n_groups, n_heads, d_conv, proj_dim;
} lssm_fused_inproj_dims;

/* ---- context, errors, kernel registry ---------------------------------- */
/* Replaces the lazy MTLDevice/MTLCommandQueue (src/backend/metal/metal_context.mm:30-105). */
lssm_status lssm_ctx_create(int device, lssm_ctx** out);
lssm_status lssm_ctx_destroy(lssm_ctx* ctx);
/* Use an external cudaStream_t (passed as void*) instead of the context's own stream. */
lssm_status lssm_ctx_set_stream(lssm_ctx* ctx, void* cuda_stream);
void* lssm_ctx_stream(lssm_ctx* ctx);
const char* lssm_last_error(void);
/* MetalOps::metallib_loaded (ops.hpp:64): 1 when the sm_100a code is loadable on the current device. */
int lssm_backend_loaded(void);
/* MetalOps::has_pipeline (ops.hpp:68): 1 if `name` is one of the kernels tests/test_metal_ops.cpp:31-49 lists. */
int lssm_has_kernel(const char* name);
const char* lssm_version(void);

/* ---- batching: MetalOps::begin_batch/commit_and_wait/batch_active (ops.hpp:91-93) */
lssm_status lssm_begin_batch(lssm_ctx* ctx);
lssm_status lssm_commit_and_wait(lssm_ctx* ctx);
int lssm_batch_active(lssm_ctx* ctx);
/* Graph batching (no reference counterpart; the Metal analogue is re-encoding a command
 * buffer): when enabled, begin_batch captures the ops into a CUDA graph and commit_and_wait
 * instantiates, runs and keeps it; lssm_replay_batch re-launches the kept graph `times` times
 * on the context stream without waiting (same buffers and offsets as when captured). */
lssm_status lssm_ctx_set_graph_batching(lssm_ctx* ctx, int enable);
lssm_status lssm_replay_batch(lssm_ctx* ctx, uint32_t times);

/* ---- device memory: replaces DeviceBuffer / UnifiedBuffer (include/lite_ssm/allocator.hpp:21-103)
 * There is no unified memory between an x86 host and a B200, so weights are copied
 * to HBM once and activations live in device buffers. */
lssm_status lssm_alloc(lssm_ctx* ctx, size_t nbytes, void** dptr);
lssm_status lssm_free(lssm_ctx* ctx, void* dptr);
lssm_status lssm_upload(lssm_ctx* ctx, void* dst, size_t dst_off, const void* host_src, size_t nbytes);
lssm_status lssm_download(lssm_ctx* ctx, void* host_dst, const void* src, size_t src_off, size_t nbytes);
/* DeviceBuffer::zero (src/backend/metal/metal_buffer.mm:141-143) as a device memset. */
lssm_status lssm_memset(lssm_ctx* ctx, void* dst, size_t dst_off, int value, size_t nbytes);

/* ---- ops: one per MetalOps method ------------------------------------- */
lssm_status lssm_rmsnorm_f16(lssm_ctx* ctx, const void* x, size_t x_off, const void* w, size_t w_off,
                             void* y, size_t y_off, lssm_rmsnorm_dims dims);            /* ops.hpp:99-102 */
lssm_status lssm_linear_f16_gemv(lssm_ctx* ctx, const void* x, size_t x_off, const void* w, size_t w_off,
                                 void* y, size_t y_off, lssm_linear_dims dims);         /* ops.hpp:104-107 */
lssm_status lssm_linear_silu_f16_gemv(lssm_ctx* ctx, const void* x, size_t x_off, const void* w,
                                      size_t w_off, void* y, size_t y_off,
                                      lssm_linear_dims dims);                           /* ops.hpp:109-112 */
lssm_status lssm_rmsnorm_linear_f16_gemv(lssm_ctx* ctx, const void* x, size_t x_off, const void* w_norm,
                                         size_t w_norm_off, const void* w, size_t w_off, void* y,
                                         size_t y_off, lssm_rmslinear_dims dims);       /* ops.hpp:114-118 */
lssm_status lssm_linear_f16_gemm(lssm_ctx* ctx, const void* x, size_t x_off, const void* w, size_t w_off,
                                 void* y, size_t y_off, lssm_linear_dims dims);         /* ops.hpp:120-123 */
lssm_status lssm_linear_silu_f16_gemm(lssm_ctx* ctx, const void* x, size_t x_off, const void* w,
                                      size_t w_off, void* y, size_t y_off,
                                      lssm_linear_dims dims);                           /* ops.hpp:125-128 */
lssm_status lssm_linear_int4_gemv(lssm_ctx* ctx, const void* x, size_t x_off, const void* w,
                                  size_t w_packed_off, const void* w_scl, size_t w_scales_off, void* y,
                                  size_t y_off, lssm_linear_dims dims);                 /* ops.hpp:135-139 */
/* The INT4 GEMM uses the context's device scratch (one block per context, on its device). For
 * M <= 128 it holds the split-K fp32 partials (8*M*N*4 bytes reserved); when the fused kernel
 * cannot take the shape, it holds the dequantised fp16 weight (N*K*2 bytes). The scratch grows by
 * allocating a larger block. Growth is refused inside a captured batch (LSSM_ERR_STATE): under
 * graph batching, first make one call of the same or a larger shape outside the batch. A block
 * that the kept graph of lssm_replay_batch may use is freed only when that graph is replaced
 * or the context destroyed, so replays never touch freed memory. */
lssm_status lssm_linear_int4_gemm(lssm_ctx* ctx, const void* x, size_t x_off, const void* w,
                                  size_t w_packed_off, const void* w_scl, size_t w_scales_off, void* y,
                                  size_t y_off, lssm_linear_dims dims);                 /* ops.hpp:141-145 */
/* Introspection (no reference counterpart, no device needed): the launch plan the INT4 GEMM
 * takes for (M, N, K) on `sms` SMs with `ws_bytes` of scratch (16-byte aligned operands and
 * K % 256 == 0 assumed). Returns 1 and the N tile / K split count when the fused kernel
 * takes the shape, 0 when it dequantises and runs the fp16 GEMM instead. Splitting K needs
 * room for the fp32 partials of at least two splits: ws_bytes >= 2*M*N*4; below that the
 * plan has one split. */
int lssm_plan_int4_gemm(uint32_t M, uint32_t N, uint32_t K, int sms, size_t ws_bytes, uint32_t* bn,
                        uint32_t* splits);
/* The work unit of CTA-tile `tile` in a fused INT4 GEMM launch of m_tiles x n_tiles x splits
 * units over nk 64-wide K blocks, computed by the same function the kernel uses:
 * out[5] = {m tile, n tile, split, first K block, end K block}. */
void lssm_int4_gemm_unit(uint32_t tile, uint32_t m_tiles, uint32_t n_tiles, uint32_t splits, uint32_t nk,
                         uint32_t* out);
/* The in_proj work of the persistent decode kernel for CTA s of G, computed by the function the
 * kernel uses: out[4] = {first channel unit (8 d_inner channels), units, first B / C / dt tile,
 * B / C / dt tiles (tile k = first + i * G)}. A CTA holding a B / C / dt tile is charged two units. */
void lssm_persist_in_deal(uint32_t s, uint32_t G, uint32_t d_inner, uint32_t n_spec, uint32_t* out);
/* The N tile (128, 144, 160, 192, 240 or 256 columns) the fp16 tensor-core GEMM (lssm_linear_f16_gemm,
 * and the INT4 GEMM's dequantise-then-GEMM path) picks for an M x N output on `sms` SMs, computed by the
 * launcher's own function: the fill of the last persistent wave weighed by the shared-memory operand rate. */
int lssm_plan_gemm_f16(uint32_t M, uint32_t N, int sms);
/* Batched-decode extensions (no MetalOps counterpart): the GEMVs above take one activation
 * row (dims.M == 1, the checks of ops.mm:207-212 and :323-324); these take 1 <= dims.M <= 8 rows
 * (the sequences of one decode step, row-major (M, K) in, (M, N) out) and read the weights once
 * for all rows. Same errors otherwise. */
lssm_status lssm_linear_f16_gemv_rows(lssm_ctx* ctx, const void* x, size_t x_off, const void* w, size_t w_off,
                                      void* y, size_t y_off, lssm_linear_dims dims);
lssm_status lssm_linear_int4_gemv_rows(lssm_ctx* ctx, const void* x, size_t x_off, const void* w,
                                       size_t w_packed_off, const void* w_scl, size_t w_scales_off, void* y,
                                       size_t y_off, lssm_linear_dims dims);
lssm_status lssm_silu_f16(lssm_ctx* ctx, const void* x, size_t x_off, void* y, size_t y_off,
                          uint32_t n);                                                  /* ops.hpp:147-149 */
lssm_status lssm_add_inplace_f16(lssm_ctx* ctx, void* y, size_t y_off, const void* x, size_t x_off,
                                 uint32_t n);                                           /* ops.hpp:151-153 */
lssm_status lssm_split_silu_xBC_f16(lssm_ctx* ctx, const void* xBC, size_t xBC_off, void* x_out,
                                    size_t x_off, void* B_out, size_t B_off, void* C_out, size_t C_off,
                                    uint32_t L, uint32_t d_inner, uint32_t d_state,
                                    uint32_t n_groups);                                 /* ops.hpp:158-163 */
lssm_status lssm_silu_gated_f16(lssm_ctx* ctx, const void* x, size_t x_off, const void* gate,
                                size_t gate_off, void* y, size_t y_off, uint32_t n);    /* ops.hpp:165-168 */
lssm_status lssm_causal_conv1d_f16(lssm_ctx* ctx, const void* x, size_t x_off, const void* w, size_t w_off,
                                   const void* bias, size_t bias_off, void* y, size_t y_off,
                                   lssm_conv1d_dims dims);                              /* ops.hpp:170-174 */
lssm_status lssm_causal_conv1d_update_f16(lssm_ctx* ctx, const void* x_new, size_t x_off, void* state,
                                          size_t state_off, const void* w, size_t w_off, const void* bias,
                                          size_t bias_off, void* y, size_t y_off,
                                          lssm_conv1d_dims dims);                       /* ops.hpp:176-181 */
lssm_status lssm_seed_conv_state_f16(lssm_ctx* ctx, const void* xBC, size_t xBC_off, void* state,
                                     size_t state_off, uint32_t L, uint32_t D, uint32_t K); /* ops.hpp:186-188 */
lssm_status lssm_inproj_fused_f16(lssm_ctx* ctx, const void* normed, size_t normed_off, const void* W_in,
                                  size_t w_in_off, const void* W_conv, size_t w_conv_off, const void* conv_b,
                                  size_t conv_b_off, void* proj_z, size_t z_off, void* ssd_x, size_t x_off,
                                  void* ssd_B, size_t b_off, void* ssd_C, size_t c_off, void* proj_dt,
                                  size_t dt_off, void* proj_xBC, size_t xBC_off,
                                  lssm_fused_inproj_dims dims);                         /* ops.hpp:203-214 */
/* Same op and arguments as lssm_inproj_fused_f16, for callers that cannot allocate device
 * memory at call time (a framework allocator that owns the whole memory budget, a serving
 * loop where cudaMalloc/cudaFree would block or synchronise the device, a process that must
 * not hit out-of-memory once running). It allocates nothing: its scratch (the fp32 matmul
 * tile, L * proj_dim * 4 bytes) lives in a 4 MiB static device array that every GPU loading
 * this library keeps until exit; larger requests return LSSM_ERR_INVALID_ARGUMENT. The array's
 * device address is looked up on the first call on each device, so make that first call
 * before any stream capture. All calls share the array: calls that overlap on the GPU race and
 * must be serialised by the caller. No counterpart in the reference (its in_proj kernel keeps
 * the tile in threadgroup memory, shaders/fused.metal:71-76). */
lssm_status lssm_inproj_fused_f16_noalloc(lssm_ctx* ctx, const void* normed, size_t normed_off, const void* W_in,
                                          size_t w_in_off, const void* W_conv, size_t w_conv_off,
                                          const void* conv_b, size_t conv_b_off, void* proj_z, size_t z_off,
                                          void* ssd_x, size_t x_off, void* ssd_B, size_t b_off, void* ssd_C,
                                          size_t c_off, void* proj_dt, size_t dt_off, void* proj_xBC,
                                          size_t xBC_off, lssm_fused_inproj_dims dims);
lssm_status lssm_ssd_chunked_f16(lssm_ctx* ctx, const void* X, size_t X_off, const void* B, size_t B_off,
                                 const void* C, size_t C_off, const void* dt_raw, size_t dt_off,
                                 const void* dt_bias, size_t db_off, const void* A_log, size_t A_off,
                                 const void* D_skip, size_t D_off, void* Y, size_t Y_off, void* state_io,
                                 size_t S_off, lssm_ssd_dims dims);                     /* ops.hpp:216-225 */
lssm_status lssm_ssd_step_f16(lssm_ctx* ctx, const void* x, size_t x_off, const void* B, size_t B_off,
                              const void* C, size_t C_off, const void* dt_raw, size_t dt_off,
                              const void* dt_bias, size_t db_off, const void* A_log, size_t A_off,
                              const void* D_skip, size_t D_off, void* state, size_t S_off, void* y,
                              size_t y_off, lssm_ssd_step_dims dims);                   /* ops.hpp:227-236 */

/* ---- batched SSD (the SSD-op configuration; no reference counterpart takes a batch,
 *      the reference kernel is ssd_chunked_f16 at shaders/ssd_chunked.metal:82-297) ----
 * X (batch, L, H, P), B/C (batch, L, G, N), dt_raw (batch, L, H), dt_bias/A_log/D (H),
 * state_io (batch, H, P, N) fp32 in/out, Y (batch, L, H, P). */
typedef enum lssm_dtype { LSSM_DT_F16 = 0, LSSM_DT_BF16 = 1, LSSM_DT_F32 = 2 } lssm_dtype;
typedef struct {
    uint32_t batch, L, H, P, N, n_groups, chunk_size;
    float dt_min, dt_max;
    uint32_t has_D;
    uint32_t x_dtype;      /* X, B, C: LSSM_DT_F16 or LSSM_DT_BF16 */
    uint32_t dt_dtype;     /* dt_raw: F16, BF16 or F32 */
    uint32_t param_dtype;  /* dt_bias, A_log, D: F16 or F32 */
    uint32_t y_dtype;      /* Y: F16, BF16 or F32 */
} lssm_ssd_batched_dims;
lssm_status lssm_ssd_chunked_batched(lssm_ctx* ctx, const void* X, const void* B, const void* C,
                                     const void* dt_raw, const void* dt_bias, const void* A_log,
                                     const void* D_skip, void* Y, void* state_io, lssm_ssd_batched_dims dims);
/* Batched-decode extension of ssd_step (ops.hpp:227-236 takes one sequence): one decode token of
 * dims.batch sequences, fp16 x (batch, H*P), B / C (batch, n_groups*N), dt_raw (batch, H), fp16
 * dt_bias / A_log / D (H), fp32 state_io (batch, H, P, N) updated in place, fp16 y (batch, H*P).
 * Uses dims.batch, H, P, N, n_groups, dt_min, dt_max, has_D; the dtype fields are ignored. */
lssm_status lssm_ssd_step_batched(lssm_ctx* ctx, const void* x, const void* B, const void* C, const void* dt_raw,
                                  const void* dt_bias, const void* A_log, const void* D_skip, void* state_io,
                                  void* y, lssm_ssd_batched_dims dims);

/* ---- engine: .ssm model + session (the callers of the ops: the .cpp files of src/model and src/runtime) ---- */
typedef struct lssm_model lssm_model;
typedef struct lssm_session lssm_session;

typedef struct {                       /* Mamba2Config, include/lite_ssm/model.hpp:22-36 */
    uint32_t d_model, n_layer, d_state, d_conv, expand, vocab_size, n_heads, d_head, chunk_size,
        default_dtype, n_groups, norm_before_gate;
} lssm_hparams;

/* SSMFile(path) + upload of the payload arena to HBM (src/core/ssm_loader.cpp:48-139). */
lssm_status lssm_model_load(lssm_ctx* ctx, const char* path, lssm_model** out);
/* Same, from a .ssm image already in host memory. */
lssm_status lssm_model_load_bytes(lssm_ctx* ctx, const void* bytes, size_t nbytes, lssm_model** out);
/* Seeded random-init model written directly in HBM in the .ssm layout
 * (int4 = in_proj/out_proj packed as INT4_B32 like tools/export_mamba2.py:55-103). */
lssm_status lssm_model_synthesize(lssm_ctx* ctx, const lssm_hparams* hp, uint64_t seed, int int4,
                                  lssm_model** out);
/* Write the model's .ssm image (header + index + payloads) to `path`. */
lssm_status lssm_model_save(lssm_model* m, const char* path);
lssm_status lssm_model_config(const lssm_model* m, lssm_hparams* out);
size_t lssm_model_nbytes(const lssm_model* m);
/* Device base pointer of the .ssm image in HBM and a tensor's (offset, nbytes, dtype). */
const void* lssm_model_device_base(const lssm_model* m);
lssm_status lssm_model_tensor(const lssm_model* m, const char* name, uint64_t* offset, uint64_t* nbytes,
                              uint32_t* dtype);
lssm_status lssm_model_destroy(lssm_model* m);

/* Mamba2State + Mamba2Workspace (src/model/state.cpp:30-124) for `batch` independent
 * sequences (the reference supports batch 1 only, state.cpp:32-34). */
lssm_status lssm_session_create(lssm_ctx* ctx, lssm_model* m, uint32_t batch, uint32_t max_seq_len,
                                lssm_session** out);
lssm_status lssm_session_destroy(lssm_session* s);
/* Mamba2State::reset (state.cpp:49-51). */
lssm_status lssm_session_reset(lssm_session* s);
/* Prefill `L` tokens per sequence (tokens: batch x L, host) and return the greedy
 * next token per sequence (host, batch entries). Mamba2Model::forward_prefill +
 * compute_logits + sample_greedy (mamba2_block.cpp:296-315, mamba2_model.cpp:144-175,
 * sampler.cpp:13-21). */
lssm_status lssm_prefill(lssm_session* s, const uint32_t* tokens, uint32_t L, uint32_t* next_tokens);
/* Greedy decode: feed `first` (batch entries, host), run `n_steps` decode steps and
 * write batch x n_steps generated ids (host). Mamba2Model::forward_step loop
 * (inference.cpp:55-67) with on-device argmax and embedding gather. */
lssm_status lssm_decode(lssm_session* s, const uint32_t* first, uint32_t n_steps, uint32_t* out_tokens);
/* generate() (src/runtime/inference.cpp:14-70), greedy, for batch sequences of equal
 * prompt length: out has batch x max_new ids. eos = 0xFFFFFFFF disables early stop. */
lssm_status lssm_generate(lssm_session* s, const uint32_t* prompt, uint32_t L, uint32_t max_new,
                          uint32_t eos, uint32_t* out_tokens, uint32_t* n_out);
/* fp32 copy of the logits of the last position computed (batch x vocab, host). */
lssm_status lssm_session_logits(lssm_session* s, float* out);
/* Device timing of the last prefill / decode call (CUDA events on the session stream), ms. */
lssm_status lssm_session_timing(lssm_session* s, float* prefill_ms, float* decode_ms);
/* Kernel launches issued by the last prefill and by the last lssm_decode call (all its
 * steps: 1 when the persistent decode kernel ran them). */
lssm_status lssm_session_launches(lssm_session* s, uint64_t* prefill, uint64_t* decode);
/* Engine knobs (no reference counterpart; the reference has one decode path):
 *   "persistent" 1 = run lssm_decode as one persistent cooperative kernel when the model
 *                qualifies (batch <= 2, INT4_B32 in/out_proj, fp16 lm_head, d_state 128,
 *                d_model and d_inner multiples of 256) (default 1);
 *   "cuda_graph" 1 = otherwise capture each decode step in a CUDA graph (default 1);
 *   "trace"      1 = record per-phase %globaltimer stamps of the persistent kernel's first
 *                step (read with lssm_session_trace). */
lssm_status lssm_session_set_option(lssm_session* s, const char* key, int64_t value);
/* ---- multi-GPU: head tensor parallelism (no reference counterpart: the reference is
 * single-device) ----------------------------------------------------------------------
 * One rank per GPU. Every rank loads (or synthesises) the same model; a TP session
 * copies this rank's shard: in_proj rows of its heads / groups ([z | x | B | C | dt]),
 * its conv channels and head parameters, the matching mixer-norm slice, the out_proj
 * columns of its d_inner slice (K split) and a vocab slice of lm_head. Per layer two
 * sum-all-reduces run on the context stream: the per-token sum of squares of the gated
 * activations (the gated RMSNorm spans the full d_inner, mamba2_block.cpp:235-238) and
 * the fp32 out_proj partials, rounded to fp16 once before the residual add. lm_head
 * argmax merges the ranks' (value, index) pairs with the first-max rule. Requires
 * n_heads and n_groups divisible by the world size. Session creation is collective too.
 * Decode steps run both all-reduces over a peer-memory exchange (CUDA IPC mappings of
 * every rank's receive area, peer stores + release/acquire flags over NVLink, the residual
 * add fused in) when all ranks are on distinct GPUs with peer access, else over NCCL;
 * session option "tp_p2p" = 0 forces NCCL (set it alike on every rank). */
#define LSSM_COMM_ID_BYTES 128
typedef struct lssm_comm lssm_comm;
/* NCCL unique id (LSSM_COMM_ID_BYTES bytes) made on one rank; the caller shares it. */
lssm_status lssm_comm_unique_id(uint8_t* out);
lssm_status lssm_comm_init(lssm_ctx* ctx, int rank, int world, const uint8_t* id, lssm_comm** out);
lssm_status lssm_comm_destroy(lssm_comm* c);
int lssm_comm_rank(const lssm_comm* c);
/* Sum-all-reduce of n fp32 device values in place across the ranks (collective, one-shot):
 * the peer exchange for n <= 65536 when every rank can use it, else NCCL. */
lssm_status lssm_comm_allreduce_f32(lssm_comm* c, float* buf, size_t n);
int lssm_comm_world(const lssm_comm* c);
/* A session over this rank's shard of `m` (see above). lssm_prefill / lssm_decode /
 * lssm_generate / lssm_session_logits are then collective: every rank calls them with the
 * same tokens. */
lssm_status lssm_session_create_tp(lssm_ctx* ctx, lssm_model* m, lssm_comm* comm, uint32_t batch,
                                   uint32_t max_seq_len, lssm_session** out);

/* Failure-path check of the peer exchange on one GPU: runs the exchange kernel against
 * local buffers with a flag no rank sets, so its bounded wait (spin_ns) runs out. Returns
 * LSSM_ERR_TIMEOUT and leaves the context usable. */
lssm_status lssm_p2p_wait_selftest(lssm_ctx* ctx, uint64_t spin_ns);

/* Phase trace of the last persistent decode: sm_count x (n_layer * 10 + 6) u64 words.
 * Per layer: [0] layer start, [1] in_proj RMSNorm staged, [2] in_proj + conv done,
 * [3] ssd inputs ready (the B / C / dt rows other SMs publish), [4] ssd_step done, [5] after
 * grid barrier, [6] out_proj RMSNorm
 * staged, [7] out_proj done, [8] producer's first in_proj copy issued, [9] ns the CTA's
 * first consumer warp waited on its weight ring during in_proj. Then lm_head: [0] norm staged, [1] logits +
 * partial argmax done, [2] after grid barrier, [3] token chosen, [4] ns waited on the
 * weight ring, [5] producer's first lm_head copy issued. With out = NULL only
 * *n_out is set. */
lssm_status lssm_session_trace(lssm_session* s, uint64_t* out, uint64_t cap, uint64_t* n_out);

/* ---- host-only .ssm helpers (no device needed) ---------------------------
 * Plan the header + tensor index of a Mamba2ForCausalLM .ssm file exactly as
 * tools/ssm_format.py:316-340 plan_layout does (int4 != 0: in_proj / out_proj as
 * INT4_B32, tools/export_mamba2.py:55-65). Writes the bytes to `out` when `cap` is
 * large enough and returns their count; data_offset / total_bytes may be null. */
size_t lssm_plan_layout(const lssm_hparams* hp, int int4, void* out, size_t cap, uint64_t* data_offset,
                        uint64_t* total_bytes);
/* Validate an .ssm image's header and index like SSMFile's constructor
 * (src/core/ssm_loader.cpp:48-139). Returns 0 on success; otherwise copies the
 * loader's message into err. */
int lssm_parse_header(const void* bytes, size_t nbytes, lssm_hparams* hp, uint32_t* n_tensors, char* err,
                      size_t err_cap);

#ifdef __cplusplus
}
#endif

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#endif /* LSSM_CUDA_H */
