// engine.cu — the model driver above the ops: .ssm loading to HBM, seeded synthetic
// models, sessions (recurrent state + workspace for `batch` sequences), prefill,
// CUDA-graph decode and greedy generation. Restates the sequence of
// src/model/mamba2_block.cpp:51-327, src/model/mamba2_model.cpp:62-211 and
// src/runtime/inference.cpp:14-70 with B200-first changes:
//   * the weights image is copied to HBM once (no unified memory on x86 + B200);
//   * in_proj is ONE GEMM/GEMV over all [z | xBC | dt] rows (the reference runs three
//     row slices of the same weight, mamba2_block.cpp:150-152: identical products);
//   * decode fuses RMSNorm into the GEMV prologue, conv-update + SiLU + split into one
//     kernel, the mixer gate into ssd_step, the residual add into the out_proj
//     epilogue, and argmax + next embedding gather into one kernel; the whole decode
//     step is captured once in a CUDA graph and replayed per token, with the greedy
//     token staying on the device (only the generated ids come back at the end).
#include <cuda_fp16.h>

#include <cmath>
#include <cstring>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <fstream>
#include <memory>
#include <sstream>

#include "device_util.cuh"
#include "lssm_internal.h"
#include "ssm_format.h"
#include "synth_rng.h"

namespace lssm {

cudaError_t launch_gemv_int4_ex(const void* x, const void* packed, const void* scales, void* y, uint32_t M,
                                uint32_t N, uint32_t K, const void* norm_w, float eps, int epilogue, cudaStream_t s);
cudaError_t launch_embed_gather(const uint32_t* tokens, const void* embed, void* hidden, uint32_t rows,
                                uint32_t d_model, uint32_t vocab, int* err, cudaStream_t s);
cudaError_t launch_conv_silu_split(const void* xbc, uint64_t in_stride, const void* w, const void* bias, void* xo,
                                   void* bo, void* co, uint32_t B, uint32_t L, uint32_t d_inner, uint32_t GN,
                                   uint32_t K, cudaStream_t s);
cudaError_t launch_conv_update_silu_split(const void* xbc, uint64_t in_stride, void* state, const void* w,
                                          const void* bias, void* xo, void* bo, void* co, uint32_t B, uint32_t d_inner,
                                          uint32_t GN, uint32_t K, cudaStream_t s);
cudaError_t launch_seed_strided(const void* xbc, uint64_t in_stride, void* state, uint32_t B, uint32_t L, uint32_t D,
                                uint32_t K, cudaStream_t s);
cudaError_t launch_synth_f16(void* out, uint64_t n, uint64_t seed, uint64_t stream, float amp, cudaStream_t s);
cudaError_t launch_synth_int4(void* out, uint32_t N, uint32_t K, uint64_t seed, uint64_t stream, float amp,
                              cudaStream_t s);

int* tc_error_word();

// ---------------------------------------------------------------------------
//  .ssm parse / plan
// ---------------------------------------------------------------------------
std::string ssm_parse(const uint8_t* base, size_t size, SsmImage* out) {
    if (size < sizeof(SsmHeader))
        return "SSMFile: file too small to contain a header (" + std::to_string(size) + " bytes)";
    SsmHeader h;
    std::memcpy(&h, base, sizeof(h));
    if (std::memcmp(h.magic, "LSSM", 4) != 0) return "SSMFile: bad magic; not a .ssm file";
    if (h.version != SSM_VERSION) return "SSMFile: unsupported version " + std::to_string(h.version);
    if (h.header_size != sizeof(SsmHeader)) return "SSMFile: header_size mismatch";
    if (h.index_offset < sizeof(SsmHeader) || h.index_offset > size || h.data_offset < h.index_offset ||
        h.data_offset > size)
        return "SSMFile: index/data offsets out of range";
    if (h.n_groups == 0) h.n_groups = 1;   // pre-group files (ssm_loader.cpp:40)
    out->hdr = h;
    out->order.clear();
    out->by_name.clear();
    size_t cur = h.index_offset;
    for (uint32_t i = 0; i < h.n_tensors; ++i) {
        if (cur + sizeof(SsmIndexPrefix) > size) return "SSMFile: out-of-bounds read while parsing tensor index prefix";
        SsmIndexPrefix p;
        std::memcpy(&p, base + cur, sizeof(p));
        cur += sizeof(p);
        if (p.rank == 0 || p.rank > 4)
            return "SSMFile: tensor " + std::to_string(i) + " has unsupported rank " + std::to_string(p.rank);
        if (cur + 8ull * p.rank > size) return "SSMFile: out-of-bounds read while parsing tensor shape";
        TensorRec t;
        t.dtype = p.dtype;
        t.rank = p.rank;
        t.offset = p.offset;
        t.nbytes = p.nbytes;
        std::memcpy(t.shape, base + cur, 8ull * p.rank);
        cur += 8ull * p.rank;
        if (cur + p.name_len > size) return "SSMFile: out-of-bounds read while parsing tensor name";
        t.name.assign(reinterpret_cast<const char*>(base + cur), p.name_len);
        cur += p.name_len;
        const size_t raw = sizeof(p) + 8ull * p.rank + p.name_len;
        cur += align_up(raw, 8) - raw;
        if (t.offset + t.nbytes > size) return "SSMFile: payload for '" + t.name + "' overflows file";
        if (p.dtype > DT_INT4_B32) return "SSMFile: '" + t.name + "' has unknown dtype";
        const size_t expect = packed_nbytes(t.dtype, t.numel());
        if (expect != t.nbytes)
            return "SSMFile: '" + t.name + "' nbytes=" + std::to_string(t.nbytes) + " but expected packed=" +
                   std::to_string(expect);
        if (out->by_name.count(t.name)) return "SSMFile: duplicate tensor name in index";
        out->by_name[t.name] = out->order.size();
        out->order.push_back(std::move(t));
        if (cur > h.data_offset) return "SSMFile: index walk overran data_offset";
    }
    return "";
}

std::vector<uint8_t> ssm_plan(const SsmHeader& hp, std::vector<TensorRec>& tensors, uint64_t* data_offset) {
    size_t index_size = 0;
    for (auto& t : tensors) index_size += align_up(sizeof(SsmIndexPrefix) + 8ull * t.rank + t.name.size(), 8);
    const uint64_t index_offset = sizeof(SsmHeader);
    const uint64_t doff = align_up(index_offset + index_size, SSM_ALIGN);
    uint64_t cursor = doff;
    for (auto& t : tensors) {
        t.nbytes = packed_nbytes(t.dtype, t.numel());
        t.offset = cursor;
        cursor = align_up(cursor + t.nbytes, SSM_ALIGN);
    }
    SsmHeader h = hp;
    std::memcpy(h.magic, "LSSM", 4);
    h.version = SSM_VERSION;
    h.header_size = sizeof(SsmHeader);
    h.n_tensors = (uint32_t)tensors.size();
    h.index_offset = index_offset;
    h.data_offset = doff;
    std::memset(h.reserved, 0, sizeof(h.reserved));
    std::vector<uint8_t> out(sizeof(SsmHeader) + index_size, 0);
    std::memcpy(out.data(), &h, sizeof(h));
    size_t pos = sizeof(SsmHeader);
    for (auto& t : tensors) {
        SsmIndexPrefix p{(uint32_t)t.name.size(), t.rank, t.dtype, 0, t.offset, t.nbytes};
        std::memcpy(out.data() + pos, &p, sizeof(p));
        pos += sizeof(p);
        std::memcpy(out.data() + pos, t.shape, 8ull * t.rank);
        pos += 8ull * t.rank;
        std::memcpy(out.data() + pos, t.name.data(), t.name.size());
        pos += t.name.size();
        pos = align_up(pos, 8);
    }
    *data_offset = doff;
    return out;
}

}  // namespace lssm

using namespace lssm;

// ---------------------------------------------------------------------------
//  Model
// ---------------------------------------------------------------------------
struct LayerW {
    const TensorRec *norm, *in_proj, *conv_w, *conv_b, *dt_bias, *A_log, *D, *mixer_norm, *out_proj;
};

struct lssm_model {
    lssm_ctx* ctx = nullptr;
    SsmImage img;
    std::vector<uint8_t> head;       // header + index bytes (for save)
    uint8_t* d_base = nullptr;       // whole .ssm image in HBM (file offsets valid)
    size_t nbytes = 0;
    std::vector<LayerW> layers;
    const TensorRec *embed = nullptr, *norm_f = nullptr, *lm_head = nullptr;
    uint32_t d_inner = 0, xbc = 0, proj = 0, GN = 0;
};

static lssm_status bind_model(lssm_model* m) {
    auto& im = m->img;
    auto& h = im.hdr;
    auto need = [&](const std::string& n, const TensorRec** out) -> lssm_status {
        *out = im.find(n);
        if (!*out) return fail(LSSM_ERR_NOT_FOUND, "Mamba2Model: missing tensor '%s'", n.c_str());
        return LSSM_OK;
    };
    if (lssm_status st = need("backbone.embeddings.weight", &m->embed)) return st;
    if (lssm_status st = need("backbone.norm_f.weight", &m->norm_f)) return st;
    m->lm_head = im.find("lm_head.weight");
    if (!m->lm_head) m->lm_head = m->embed;
    m->d_inner = h.expand * h.d_model;
    m->GN = h.n_groups * h.d_state;
    m->xbc = m->d_inner + 2 * m->GN;
    m->proj = m->d_inner + m->xbc + h.n_heads;
    if (h.n_heads * h.d_head != m->d_inner)
        return fail(LSSM_ERR_FORMAT, "Mamba2Model: n_heads * d_head != expand * d_model");
    if (h.n_heads % h.n_groups != 0) return fail(LSSM_ERR_FORMAT, "Mamba2Model: n_heads not divisible by n_groups");
    m->layers.resize(h.n_layer);
    for (uint32_t i = 0; i < h.n_layer; ++i) {
        const std::string p = "backbone.layers." + std::to_string(i) + ".";
        LayerW& L = m->layers[i];
        if (lssm_status st = need(p + "norm.weight", &L.norm)) return st;
        if (lssm_status st = need(p + "mixer.in_proj.weight", &L.in_proj)) return st;
        if (lssm_status st = need(p + "mixer.conv1d.weight", &L.conv_w)) return st;
        if (lssm_status st = need(p + "mixer.conv1d.bias", &L.conv_b)) return st;
        if (lssm_status st = need(p + "mixer.dt_bias", &L.dt_bias)) return st;
        if (lssm_status st = need(p + "mixer.A_log", &L.A_log)) return st;
        if (lssm_status st = need(p + "mixer.D", &L.D)) return st;
        if (lssm_status st = need(p + "mixer.norm.weight", &L.mixer_norm)) return st;
        if (lssm_status st = need(p + "mixer.out_proj.weight", &L.out_proj)) return st;
        if (L.in_proj->shape[0] != m->proj)
            return fail(LSSM_ERR_FORMAT, "Mamba2Model: in_proj output dim mismatch vs config (got %llu, expected %u)",
                        (unsigned long long)L.in_proj->shape[0], m->proj);
        if (L.conv_w->shape[0] != m->xbc) return fail(LSSM_ERR_FORMAT, "Mamba2Model: conv1d weight dim mismatch vs config");
        for (const TensorRec* t : {L.norm, L.conv_w, L.conv_b, L.dt_bias, L.A_log, L.D, L.mixer_norm})
            if (t->dtype != DT_F16)
                return fail(LSSM_ERR_FORMAT, "Mamba2Model: '%s' must be f16 (got dtype %u)", t->name.c_str(), t->dtype);
        for (const TensorRec* t : {L.in_proj, L.out_proj})
            if (t->dtype != DT_F16 && t->dtype != DT_INT4_B32)
                return fail(LSSM_ERR_FORMAT, "Mamba2Model: '%s' must be f16 or int4_b32", t->name.c_str());
    }
    if (m->embed->dtype != DT_F16 || m->norm_f->dtype != DT_F16)
        return fail(LSSM_ERR_FORMAT, "Mamba2Model: embeddings / norm_f must be f16");
    if (m->lm_head->dtype != DT_F16 && m->lm_head->dtype != DT_INT4_B32)
        return fail(LSSM_ERR_FORMAT, "Mamba2Model: lm_head must be f16 or int4_b32");
    return LSSM_OK;
}

static lssm_status upload_image(lssm_ctx* ctx, lssm_model* m, const uint8_t* bytes, size_t n) {
    cudaError_t e = cudaMalloc(&m->d_base, n);
    if (e != cudaSuccess) return cuda_fail(e, "lssm_model_load: weights arena");
    m->nbytes = n;
    // Stage through two pinned 64 MiB buffers so the copy runs at PCIe speed and the host
    // copy of one piece overlaps the device copy of the previous one.
    const size_t piece = 64ull << 20;
    void* pinned[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    bool staged = true;
    for (int i = 0; i < 2; ++i) {
        staged = staged && cudaMallocHost(&pinned[i], piece) == cudaSuccess &&
                 cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming) == cudaSuccess;
    }
    cudaGetLastError();
    size_t k = 0;
    for (size_t off = 0; off < n && e == cudaSuccess; off += piece, ++k) {
        const size_t len = std::min(piece, n - off);
        if (staged) {
            const int b = (int)(k & 1);
            if (k >= 2) e = cudaEventSynchronize(done[b]);   // the copy that last used this buffer
            if (e != cudaSuccess) break;
            std::memcpy(pinned[b], bytes + off, len);
            e = cudaMemcpyAsync(m->d_base + off, pinned[b], len, cudaMemcpyHostToDevice, ctx->stream);
            if (e == cudaSuccess) e = cudaEventRecord(done[b], ctx->stream);
        } else {
            e = cudaMemcpy(m->d_base + off, bytes + off, len, cudaMemcpyHostToDevice);
        }
    }
    const cudaError_t es = cudaStreamSynchronize(ctx->stream);
    if (e == cudaSuccess) e = es;
    for (int i = 0; i < 2; ++i) {
        if (done[i]) cudaEventDestroy(done[i]);
        if (pinned[i]) cudaFreeHost(pinned[i]);
    }
    if (e != cudaSuccess) return cuda_fail(e, "lssm_model_load: upload");
    return LSSM_OK;
}

extern "C" lssm_status lssm_model_load_bytes(lssm_ctx* ctx, const void* bytes, size_t nbytes, lssm_model** out) {
    if (!ctx || !bytes || !out) return fail(LSSM_ERR_INVALID_ARGUMENT, "lssm_model_load_bytes: null argument");
    cudaSetDevice(ctx->device);
    *out = nullptr;
    std::unique_ptr<lssm_model> m(new lssm_model());
    m->ctx = ctx;
    const uint8_t* b = static_cast<const uint8_t*>(bytes);
    std::string err = ssm_parse(b, nbytes, &m->img);
    if (!err.empty()) return fail(LSSM_ERR_FORMAT, "%s", err.c_str());
    m->head.assign(b, b + m->img.hdr.data_offset);
    if (lssm_status st = bind_model(m.get())) return st;
    if (lssm_status st = upload_image(ctx, m.get(), b, nbytes)) return st;
    *out = m.release();
    return LSSM_OK;
}

// The file is mapped read-only as MmapFile does (src/core/allocator.cpp:31-64, same open /
// empty-file errors), parsed and validated in place, and streamed to HBM from the mapping,
// with no host copy of the whole image. If mapping fails, the file is read instead.
extern "C" lssm_status lssm_model_load(lssm_ctx* ctx, const char* path, lssm_model** out) {
    if (!ctx || !path || !out) return fail(LSSM_ERR_INVALID_ARGUMENT, "lssm_model_load: null argument");
    const int fd = ::open(path, O_RDONLY);
    if (fd < 0) return fail(LSSM_ERR_INVALID_ARGUMENT, "MmapFile: cannot open '%s'", path);
    struct stat st {};
    if (::fstat(fd, &st) != 0) {
        ::close(fd);
        return fail(LSSM_ERR_INVALID_ARGUMENT, "MmapFile: cannot stat '%s'", path);
    }
    const size_t n = (size_t)st.st_size;
    if (n == 0) {
        ::close(fd);
        return fail(LSSM_ERR_FORMAT, "MmapFile: empty or invalid file '%s'", path);
    }
    void* map = ::mmap(nullptr, n, PROT_READ, MAP_PRIVATE, fd, 0);
    if (map == MAP_FAILED) {
        std::vector<uint8_t> buf(n);
        size_t got = 0;
        while (got < n) {
            const ssize_t r = ::read(fd, buf.data() + got, n - got);
            if (r <= 0) break;
            got += (size_t)r;
        }
        ::close(fd);
        if (got < n) return fail(LSSM_ERR_FORMAT, "cannot read '%s'", path);
        return lssm_model_load_bytes(ctx, buf.data(), n, out);
    }
    ::close(fd);
    ::madvise(map, n, MADV_SEQUENTIAL);
    const lssm_status stt = lssm_model_load_bytes(ctx, map, n, out);
    ::munmap(map, n);
    return stt;
}

// Tensor list of a Mamba2ForCausalLM state_dict, in its order (the order the
// reference exporter writes, tools/export_mamba2.py:162-195).
static std::vector<TensorRec> mamba2_tensor_list(const lssm_hparams& hp, int int4) {
    std::vector<TensorRec> v;
    auto add = [&](const std::string& n, uint32_t dt, std::initializer_list<uint64_t> shp) {
        TensorRec t;
        t.name = n;
        t.dtype = dt;
        t.rank = (uint32_t)shp.size();
        int i = 0;
        for (auto s : shp) t.shape[i++] = s;
        v.push_back(t);
    };
    const uint64_t di = (uint64_t)hp.expand * hp.d_model, G = hp.n_groups ? hp.n_groups : 1;
    const uint64_t xd = di + 2 * G * hp.d_state, proj = di + xd + hp.n_heads;
    const uint32_t lin = int4 ? DT_INT4_B32 : DT_F16;
    add("backbone.embeddings.weight", DT_F16, {hp.vocab_size, hp.d_model});
    for (uint32_t i = 0; i < hp.n_layer; ++i) {
        const std::string p = "backbone.layers." + std::to_string(i) + ".";
        add(p + "norm.weight", DT_F16, {hp.d_model});
        add(p + "mixer.dt_bias", DT_F16, {hp.n_heads});
        add(p + "mixer.A_log", DT_F16, {hp.n_heads});
        add(p + "mixer.D", DT_F16, {hp.n_heads});
        add(p + "mixer.conv1d.weight", DT_F16, {xd, 1, hp.d_conv});
        add(p + "mixer.conv1d.bias", DT_F16, {xd});
        add(p + "mixer.in_proj.weight", (hp.d_model % 32 == 0) ? lin : DT_F16, {proj, hp.d_model});
        add(p + "mixer.norm.weight", DT_F16, {di});
        add(p + "mixer.out_proj.weight", (di % 32 == 0) ? lin : DT_F16, {hp.d_model, di});
    }
    add("backbone.norm_f.weight", DT_F16, {hp.d_model});
    add("lm_head.weight", DT_F16, {hp.vocab_size, hp.d_model});
    return v;
}

static uint16_t host_f2h(float f) {
    __half h = __float2half_rn(f);
    return *reinterpret_cast<uint16_t*>(&h);
}

// Small per-head / per-channel vectors are made on the host in double precision and
// rounded once to fp16 (identical on every machine with the same libm).
//   A_log  = log(1 + 15 u)            (A = -exp(A_log) in [-16, -1])
//   dt_bias = dt + log(-expm1(-dt)),  dt = exp(log(1e-3) + u log(100))  (inverse softplus)
//   D = 0.5 + u;   norm weights = 0.9 + 0.2 u
static void host_vector(const std::string& kind, uint64_t seed, uint64_t stream, uint64_t n, uint16_t* out) {
    for (uint64_t i = 0; i < n; ++i) {
        const double u = 0.5 * ((double)synth_value(seed, stream, i, 1.0f) + 1.0);
        double v;
        if (kind == "A_log") v = std::log(1.0 + 15.0 * u);
        else if (kind == "dt_bias") {
            const double dt = std::exp(std::log(1e-3) + u * std::log(100.0));
            v = dt + std::log(-std::expm1(-dt));
        } else if (kind == "D") v = 0.5 + u;
        else v = 0.9 + 0.2 * u;   // norm weights
        out[i] = host_f2h((float)v);
    }
}

extern "C" lssm_status lssm_model_synthesize(lssm_ctx* ctx, const lssm_hparams* hpp, uint64_t seed, int int4,
                                             lssm_model** out) {
    if (!ctx || !hpp || !out) return fail(LSSM_ERR_INVALID_ARGUMENT, "lssm_model_synthesize: null argument");
    cudaSetDevice(ctx->device);
    *out = nullptr;
    lssm_hparams hp = *hpp;
    if (hp.n_groups == 0) hp.n_groups = 1;
    if (!hp.d_model || !hp.n_layer || !hp.d_state || !hp.d_conv || !hp.expand || !hp.vocab_size || !hp.n_heads ||
        !hp.d_head)
        return fail(LSSM_ERR_INVALID_ARGUMENT, "lssm_model_synthesize: zero hyperparameter");
    std::unique_ptr<lssm_model> m(new lssm_model());
    m->ctx = ctx;
    std::vector<TensorRec> ts = mamba2_tensor_list(hp, int4);
    SsmHeader h{};
    h.d_model = hp.d_model; h.n_layer = hp.n_layer; h.d_state = hp.d_state; h.d_conv = hp.d_conv;
    h.expand = hp.expand; h.vocab_size = hp.vocab_size; h.n_heads = hp.n_heads; h.d_head = hp.d_head;
    h.chunk_size = hp.chunk_size ? hp.chunk_size : 256; h.default_dtype = DT_F16; h.n_groups = hp.n_groups;
    h.norm_before_gate = hp.norm_before_gate;
    uint64_t doff = 0;
    m->head = ssm_plan(h, ts, &doff);
    const size_t total = align_up(ts.back().offset + ts.back().nbytes, SSM_ALIGN);
    std::string err = ssm_parse(m->head.data(), m->head.size(), &m->img);
    // The header alone is shorter than the payload offsets; re-parse against the full size.
    {
        std::vector<uint8_t> probe(m->head);
        SsmImage im;
        im.hdr = *reinterpret_cast<const SsmHeader*>(probe.data());
        for (size_t i = 0; i < ts.size(); ++i) { im.by_name[ts[i].name] = i; im.order.push_back(ts[i]); }
        m->img = std::move(im);
    }
    (void)err;
    if (lssm_status st = bind_model(m.get())) return st;
    cudaError_t e = cudaMalloc(&m->d_base, total);
    if (e != cudaSuccess) return cuda_fail(e, "lssm_model_synthesize: weights arena");
    m->nbytes = total;
    e = cudaMemsetAsync(m->d_base, 0, total, ctx->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->d_base, m->head.data(), m->head.size(), cudaMemcpyHostToDevice, ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "lssm_model_synthesize");
    const double inv_sqrt3 = 1.7320508075688772;
    std::vector<uint16_t> hv;
    for (size_t i = 0; i < ts.size(); ++i) {
        const TensorRec& t = m->img.order[i];
        const uint64_t stream = i + 1;
        uint8_t* dst = m->d_base + t.offset;
        const std::string& n = t.name;
        auto ends = [&](const char* s) { return n.size() >= strlen(s) && n.compare(n.size() - strlen(s), strlen(s), s) == 0; };
        if (ends("embeddings.weight") || n == "lm_head.weight") {
            // lm_head is tied to the embeddings (same stream => same values)
            const uint64_t st = (n == "lm_head.weight") ? 1 : stream;
            e = launch_synth_f16(dst, t.numel(), seed, st, (float)(0.5 * inv_sqrt3), ctx->stream);
        } else if (ends("in_proj.weight") || ends("out_proj.weight")) {
            const float amp = (float)(inv_sqrt3 / std::sqrt((double)t.shape[1]));
            if (t.dtype == DT_INT4_B32)
                e = launch_synth_int4(dst, (uint32_t)t.shape[0], (uint32_t)t.shape[1], seed, stream, amp, ctx->stream);
            else
                e = launch_synth_f16(dst, t.numel(), seed, stream, amp, ctx->stream);
        } else if (ends("conv1d.weight") || ends("conv1d.bias")) {
            e = launch_synth_f16(dst, t.numel(), seed, stream, 0.5f, ctx->stream);
        } else {
            hv.resize(t.numel());
            const char* kind = ends("A_log") ? "A_log" : ends("dt_bias") ? "dt_bias" : ends(".D") ? "D" : "norm";
            host_vector(kind, seed, stream, t.numel(), hv.data());
            e = cudaMemcpyAsync(dst, hv.data(), t.nbytes, cudaMemcpyHostToDevice, ctx->stream);
            if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
        }
        if (e != cudaSuccess) return cuda_fail(e, "lssm_model_synthesize: fill");
    }
    e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "lssm_model_synthesize");
    *out = m.release();
    return LSSM_OK;
}

extern "C" lssm_status lssm_model_save(lssm_model* m, const char* path) {
    if (!m || !path) return fail(LSSM_ERR_INVALID_ARGUMENT, "lssm_model_save: null argument");
    cudaSetDevice(m->ctx->device);
    std::vector<uint8_t> host(m->nbytes);
    cudaError_t e = cudaMemcpy(host.data(), m->d_base, m->nbytes, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(e, "lssm_model_save");
    std::memcpy(host.data(), m->head.data(), m->head.size());
    std::ofstream f(path, std::ios::binary);
    if (!f) return fail(LSSM_ERR_INVALID_ARGUMENT, "lssm_model_save: cannot open '%s'", path);
    f.write(reinterpret_cast<const char*>(host.data()), (std::streamsize)host.size());
    return f ? LSSM_OK : fail(LSSM_ERR_INVALID_ARGUMENT, "lssm_model_save: write failed");
}

extern "C" lssm_status lssm_model_config(const lssm_model* m, lssm_hparams* o) {
    if (!m || !o) return fail(LSSM_ERR_INVALID_ARGUMENT, "lssm_model_config: null argument");
    const SsmHeader& h = m->img.hdr;
    *o = lssm_hparams{h.d_model, h.n_layer, h.d_state, h.d_conv, h.expand, h.vocab_size, h.n_heads, h.d_head,
                      h.chunk_size, h.default_dtype, h.n_groups, h.norm_before_gate};
    return LSSM_OK;
}

extern "C" size_t lssm_model_nbytes(const lssm_model* m) { return m ? m->nbytes : 0; }
extern "C" const void* lssm_model_device_base(const lssm_model* m) { return m ? m->d_base : nullptr; }

extern "C" lssm_status lssm_model_tensor(const lssm_model* m, const char* name, uint64_t* offset, uint64_t* nbytes,
                                         uint32_t* dtype) {
    if (!m || !name) return fail(LSSM_ERR_INVALID_ARGUMENT, "lssm_model_tensor: null argument");
    const TensorRec* t = m->img.find(name);
    if (!t) return fail(LSSM_ERR_NOT_FOUND, "SSMFile: no tensor named '%s'", name);
    if (offset) *offset = t->offset;
    if (nbytes) *nbytes = t->nbytes;
    if (dtype) *dtype = t->dtype;
    return LSSM_OK;
}

extern "C" lssm_status lssm_model_destroy(lssm_model* m) {
    if (!m) return LSSM_OK;
    cudaSetDevice(m->ctx->device);
    cudaStreamSynchronize(m->ctx->stream);
    if (m->d_base) cudaFree(m->d_base);
    delete m;
    return LSSM_OK;
}

// Host-only planner export (format tests run it without a GPU).
extern "C" size_t lssm_plan_layout(const lssm_hparams* hp, int int4, void* out, size_t cap, uint64_t* data_offset,
                                   uint64_t* total_bytes) {
    std::vector<TensorRec> ts = mamba2_tensor_list(*hp, int4);
    SsmHeader h{};
    h.d_model = hp->d_model; h.n_layer = hp->n_layer; h.d_state = hp->d_state; h.d_conv = hp->d_conv;
    h.expand = hp->expand; h.vocab_size = hp->vocab_size; h.n_heads = hp->n_heads; h.d_head = hp->d_head;
    h.chunk_size = hp->chunk_size; h.default_dtype = DT_F16; h.n_groups = hp->n_groups ? hp->n_groups : 1;
    h.norm_before_gate = hp->norm_before_gate;
    uint64_t doff = 0;
    std::vector<uint8_t> b = ssm_plan(h, ts, &doff);
    if (data_offset) *data_offset = doff;
    if (total_bytes) *total_bytes = align_up(ts.back().offset + ts.back().nbytes, SSM_ALIGN);
    if (out && cap >= b.size()) std::memcpy(out, b.data(), b.size());
    return b.size();
}

// Host-only parser export: returns 0 and fills hparams on success, else copies the
// loader's message into `err` (the same messages as src/core/ssm_loader.cpp).
extern "C" int lssm_parse_header(const void* bytes, size_t n, lssm_hparams* hp, uint32_t* n_tensors, char* err,
                                 size_t err_cap) {
    SsmImage im;
    std::string e = ssm_parse(static_cast<const uint8_t*>(bytes), n, &im);
    if (!e.empty()) {
        if (err && err_cap) { std::strncpy(err, e.c_str(), err_cap - 1); err[err_cap - 1] = 0; }
        return 1;
    }
    const SsmHeader& h = im.hdr;
    if (hp) *hp = lssm_hparams{h.d_model, h.n_layer, h.d_state, h.d_conv, h.expand, h.vocab_size, h.n_heads,
                               h.d_head, h.chunk_size, h.default_dtype, h.n_groups, h.norm_before_gate};
    if (n_tensors) *n_tensors = h.n_tensors;
    return 0;
}

// ---------------------------------------------------------------------------
//  Session
// ---------------------------------------------------------------------------
// Weights one layer reads: into the model image (one GPU) or this rank's shard (TP).
struct LayerRef {
    const uint8_t* in_w; uint32_t in_dt;
    const uint8_t* out_w; uint32_t out_dt;
    const __half *conv_w, *conv_b, *dt_bias, *A_log, *D, *norm, *mixer_norm;
};

struct lssm_session {
    lssm_ctx* ctx = nullptr;
    lssm_model* m = nullptr;
    uint32_t batch = 0, max_L = 0;
    // state
    uint8_t* conv = nullptr;   // per layer (batch, xbc, d_conv) fp16
    float* ssd = nullptr;      // per layer (batch, H, P, N) fp32
    size_t conv_layer = 0, ssd_layer = 0;   // elements per layer
    // workspace (rows = batch * max_L)
    __half *hidden = nullptr, *normed = nullptr, *proj = nullptr, *xs = nullptr, *Bs = nullptr, *Cs = nullptr,
           *ys = nullptr, *gated = nullptr, *mixn = nullptr, *logits = nullptr, *lastrows = nullptr;
    __half* wscratch = nullptr;   // dequantised INT4 weight for the prefill GEMM
    size_t wscratch_elems = 0;
    uint32_t *d_tokens = nullptr, *d_cur = nullptr, *d_hist = nullptr, *d_step = nullptr;
    uint32_t hist_cap = 0;
    int* d_err = nullptr;
    cudaEvent_t ev[4] = {};
    float prefill_ms = 0.0f, decode_ms = 0.0f;
    uint64_t nl = 0;                          // kernel launches issued (running count)
    uint64_t prefill_launches = 0, decode_step_launches = 0, decode_launches = 0;
    bool use_graph = true;
    cudaGraphExec_t graph = nullptr;
    bool logits_valid = false;
    // persistent decode kernel (one launch for all decode steps) when the model allows it
    bool persist_ok = false, use_persist = true;
    PLayer* d_players = nullptr;
    float* d_part_val = nullptr;
    uint32_t* d_part_idx = nullptr;
    uint32_t* d_bar = nullptr;
    uint32_t seg_in = 0, seg_out = 0, seg_lm = 0;
    void* d_maps = nullptr;        // CUtensorMap[4 * n_layer + 1]
    float* d_opart = nullptr;      // out_proj partial-sum slots of the persistent kernel
    // persistent kernel's exchange words between SMs ({payload, epoch} u64; see PParams) and the
    // epoch of the next launch (every launch uses epochs never used before on these words)
    uint64_t* d_mb = nullptr;
    size_t mb_words = 0;
    uint32_t epoch_next = 1;
    const char* persist_why = "";  // why the persistent kernel is not used ("" = it is)
    uint64_t* d_trace = nullptr;   // phase stamps of the persistent kernel's first step
    bool trace_on = false;
    // Weights and local dims: the model's for one GPU, this rank's shard for TP.
    std::vector<LayerRef> lw;
    const uint8_t* lm_w = nullptr; uint32_t lm_dt = 0;
    const __half* embed = nullptr; const __half* norm_f = nullptr;
    uint32_t di = 0, xd = 0, proj_dim = 0, GN = 0, H = 0, G = 0, V = 0, v_off = 0, v_max = 0;
    // head tensor parallelism
    lssm_comm* comm = nullptr;
    int tp_rank = 0, tp_world = 1;
    bool use_p2p = true;            // decode all-reduces over the peer exchange when it is set up
    uint8_t* d_shard = nullptr;
    float *d_sumsq = nullptr, *d_part32 = nullptr;
    __half* d_gather = nullptr;    // all ranks' logits, for lssm_session_logits
    // greedy pick: per-chunk (value, index) pairs, per-row tickets, per-rank row pairs
    uint2 *d_cpair = nullptr, *d_pair = nullptr;
    uint32_t* d_ticket = nullptr;
};

static lssm_status s_alloc(void** p, size_t n, const char* what) {
    cudaError_t e = cudaMalloc(p, n ? n : 16);
    if (e != cudaSuccess) return cuda_fail(e, what);
    return LSSM_OK;
}

extern "C" lssm_status lssm_session_destroy(lssm_session* s) {
    if (!s) return LSSM_OK;
    cudaSetDevice(s->ctx->device);
    cudaStreamSynchronize(s->ctx->stream);
    if (s->graph) cudaGraphExecDestroy(s->graph);
    void* ps[] = {s->conv, s->ssd, s->hidden, s->normed, s->proj, s->xs, s->Bs, s->Cs, s->ys, s->gated, s->mixn,
                  s->logits, s->lastrows, s->wscratch, s->d_tokens, s->d_cur, s->d_hist, s->d_step, s->d_err,
                  s->d_players, s->d_part_val, s->d_part_idx, s->d_bar, s->d_trace, s->d_maps, s->d_opart, s->d_mb,
                  s->d_shard, s->d_sumsq, s->d_part32, s->d_gather, s->d_cpair, s->d_pair, s->d_ticket};
    for (void* p : ps)
        if (p) cudaFree(p);
    for (auto& e : s->ev)
        if (e) cudaEventDestroy(e);
    delete s;
    return LSSM_OK;
}

static size_t trace_words(const lssm_session* s) {
    return (size_t)s->m->img.hdr.n_layer * TRACE_PER_LAYER + TRACE_LM;
}

// Decide whether the persistent decode kernel can run this model/batch (its shape plan,
// INT4_B32 in/out_proj, fp16 lm_head, 16-byte aligned weights) and build its per-layer
// pointer table and tensor maps. Anything else keeps the per-op graph path (the reason
// is kept in persist_why).
static lssm_status setup_persistent(lssm_session* s) {
    lssm_model* m = s->m;
    const SsmHeader& h = m->img.hdr;
    s->persist_ok = false;
    s->persist_why = "";
    if (!tc_error_word()) { s->persist_why = "no device error word"; return LSSM_OK; }
    PersistShape sh{h.n_layer, s->batch, h.d_model, m->d_inner, m->xbc, m->proj, h.n_heads, h.d_head,
                    h.d_state, h.n_groups, h.d_conv, h.vocab_size, (uint32_t)s->ctx->sm_count};
    const char* why = decode_persist_plan(sh, &s->seg_in, &s->seg_out, &s->seg_lm);
    if (*why) { s->persist_why = why; return LSSM_OK; }
    if (m->lm_head->dtype != DT_F16) { s->persist_why = "lm_head is not fp16"; return LSSM_OK; }
    auto al = [&](const TensorRec* t) { return ((uintptr_t)(m->d_base + t->offset) % 16) == 0; };
    if (!al(m->embed) || !al(m->norm_f) || !al(m->lm_head)) { s->persist_why = "unaligned tensor"; return LSSM_OK; }
    for (auto& L : m->layers) {
        if (L.in_proj->dtype != DT_INT4_B32 || L.out_proj->dtype != DT_INT4_B32) {
            s->persist_why = "in_proj / out_proj not int4_b32";
            return LSSM_OK;
        }
        if (!al(L.in_proj) || !al(L.out_proj) || !al(L.norm) || !al(L.mixer_norm)) {
            s->persist_why = "unaligned tensor";
            return LSSM_OK;
        }
    }
    std::vector<PLayer> pl(h.n_layer);
    for (uint32_t l = 0; l < h.n_layer; ++l) {
        const LayerW& L = m->layers[l];
        auto hp = [&](const TensorRec* t) { return reinterpret_cast<const __half*>(m->d_base + t->offset); };
        pl[l].in_w = m->d_base + L.in_proj->offset;
        pl[l].out_w = m->d_base + L.out_proj->offset;
        pl[l].conv_w = hp(L.conv_w);
        pl[l].conv_b = hp(L.conv_b);
        pl[l].dt_bias = hp(L.dt_bias);
        pl[l].A_log = hp(L.A_log);
        pl[l].D = hp(L.D);
        pl[l].norm_w = hp(L.norm);
        pl[l].mixer_norm_w = hp(L.mixer_norm);
        pl[l].conv_state = reinterpret_cast<__half*>(s->conv) + s->conv_layer * l;
        pl[l].ssd_state = s->ssd + s->ssd_layer * l;
    }
    std::vector<uint8_t> maps(decode_persist_maps_bytes(h.n_layer));
    if (!decode_persist_encode_maps(maps.data(), pl.data(), m->d_base + m->lm_head->offset, sh, s->seg_in, s->seg_out,
                                    s->seg_lm)) {
        s->persist_why = "tensor map encoding failed";
        return LSSM_OK;
    }
    lssm_status st;
    if ((st = s_alloc(reinterpret_cast<void**>(&s->d_players), pl.size() * sizeof(PLayer), "session: layer table")))
        return st;
    if ((st = s_alloc(&s->d_maps, maps.size(), "session: tensor maps"))) return st;
    const size_t nchC = m->d_inner / (s->seg_out * 256);
    if ((st = s_alloc(reinterpret_cast<void**>(&s->d_opart), nchC * s->batch * h.d_model * 4, "session: out_proj slots")))
        return st;
    // exchange words of the in_proj outputs [B][proj]
    s->mb_words = (size_t)s->batch * m->proj;
    if ((st = s_alloc(reinterpret_cast<void**>(&s->d_mb), s->mb_words * 8, "session: exchange words"))) return st;
    if (cudaMemset(s->d_mb, 0, s->mb_words * 8) != cudaSuccess) return fail(LSSM_ERR_CUDA, "session: exchange words");
    s->epoch_next = 1;
    const size_t parts = (size_t)s->ctx->sm_count * s->batch;
    if ((st = s_alloc(reinterpret_cast<void**>(&s->d_part_val), parts * 4, "session: argmax partials"))) return st;
    if ((st = s_alloc(reinterpret_cast<void**>(&s->d_part_idx), parts * 4, "session: argmax partials"))) return st;
    if ((st = s_alloc(reinterpret_cast<void**>(&s->d_bar), 16, "session: grid barrier"))) return st;
    cudaError_t e = cudaMemcpy(s->d_players, pl.data(), pl.size() * sizeof(PLayer), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(s->d_maps, maps.data(), maps.size(), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(e, "session: persistent decode tables upload");
    s->persist_ok = true;
    return LSSM_OK;
}

static PParams persist_params(lssm_session* s, uint32_t n_steps) {
    lssm_model* m = s->m;
    const SsmHeader& h = m->img.hdr;
    auto hp = [&](const TensorRec* t) { return reinterpret_cast<const __half*>(m->d_base + t->offset); };
    PParams p{};
    p.layers = s->d_players;
    p.n_layer = h.n_layer;
    p.embed = hp(m->embed);
    p.norm_f = hp(m->norm_f);
    p.lm_head = hp(m->lm_head);
    p.mb_in = s->d_mb;
    p.epoch0 = s->epoch_next;
    p.opart = s->d_opart;
    p.gated = s->gated;
    p.logits = s->logits;
    p.part_val = s->d_part_val; p.part_idx = s->d_part_idx;
    p.cur = s->d_cur; p.history = s->d_hist; p.hist_stride = s->hist_cap; p.n_steps = n_steps;
    p.bar = s->d_bar; p.err = tc_error_word();
    p.B = s->batch; p.dm = h.d_model; p.di = m->d_inner; p.xd = m->xbc; p.proj = m->proj;
    p.H = h.n_heads; p.P = h.d_head; p.N = h.d_state; p.G = h.n_groups; p.dconv = h.d_conv; p.V = h.vocab_size;
    p.maps = s->d_maps;
    p.seg_in = s->seg_in; p.seg_out = s->seg_out; p.seg_lm = s->seg_lm;
    p.trace = s->trace_on ? s->d_trace : nullptr;
    return p;
}

// One GPU: every layer reads the model image.
static void bind_model_refs(lssm_session* s) {
    lssm_model* m = s->m;
    const SsmHeader& h = m->img.hdr;
    auto hp = [&](const TensorRec* t) { return reinterpret_cast<const __half*>(m->d_base + t->offset); };
    s->lw.resize(h.n_layer);
    for (uint32_t l = 0; l < h.n_layer; ++l) {
        const LayerW& L = m->layers[l];
        s->lw[l] = {m->d_base + L.in_proj->offset, L.in_proj->dtype, m->d_base + L.out_proj->offset, L.out_proj->dtype,
                    hp(L.conv_w), hp(L.conv_b), hp(L.dt_bias), hp(L.A_log), hp(L.D), hp(L.norm), hp(L.mixer_norm)};
    }
    s->lm_w = m->d_base + m->lm_head->offset;
    s->lm_dt = m->lm_head->dtype;
    s->embed = hp(m->embed);
    s->norm_f = hp(m->norm_f);
    s->di = m->d_inner; s->xd = m->xbc; s->proj_dim = m->proj; s->GN = m->GN;
    s->H = h.n_heads; s->G = h.n_groups; s->V = h.vocab_size; s->v_off = 0; s->v_max = h.vocab_size;
}

static size_t lin_bytes(uint32_t dt, size_t N, size_t K) { return dt == DT_INT4_B32 ? N * K / 2 + N * K / 32 * 2 : N * K * 2; }
static size_t al256(size_t x) { return (x + 255) & ~(size_t)255; }

// Head tensor parallelism: copy this rank's shard of every layer out of the model image
// (rows of its heads / groups for in_proj and conv, its d_inner columns of out_proj,
// its vocab rows of lm_head) into one device buffer; norms and embeddings stay shared.
static lssm_status build_tp_shard(lssm_session* s) {
    lssm_model* m = s->m;
    const SsmHeader& h = m->img.hdr;
    const uint32_t T = (uint32_t)s->tp_world, r = (uint32_t)s->tp_rank;
    const uint32_t dm = h.d_model, di = m->d_inner, GN = m->GN, xd = m->xbc, P = h.d_head, N = h.d_state;
    const uint32_t dc = h.d_conv;
    if (h.n_heads % T || h.n_groups % T)
        return fail(LSSM_ERR_INVALID_ARGUMENT, "tensor parallel: n_heads (%u) and n_groups (%u) must divide by %u ranks",
                    h.n_heads, h.n_groups, T);
    const uint32_t Hr = h.n_heads / T, Gr = h.n_groups / T, dir = Hr * P, GNr = Gr * N, xdr = dir + 2 * GNr;
    const uint32_t projr = dir + xdr + Hr;
    if (dir % 32) return fail(LSSM_ERR_INVALID_ARGUMENT, "tensor parallel: d_inner slice %u is not a multiple of 32", dir);
    const uint32_t vmax = (h.vocab_size + T - 1) / T, voff = std::min(h.vocab_size, r * vmax);
    const uint32_t Vr = std::min(vmax, h.vocab_size - voff);
    // sizes
    size_t total = 0;
    std::vector<size_t> off_in(h.n_layer), off_out(h.n_layer), off_cw(h.n_layer), off_cb(h.n_layer), off_dtb(h.n_layer),
        off_al(h.n_layer), off_D(h.n_layer), off_mn(h.n_layer);
    for (uint32_t l = 0; l < h.n_layer; ++l) {
        const LayerW& L = m->layers[l];
        off_in[l] = total; total += al256(lin_bytes(L.in_proj->dtype, projr, dm));
        off_out[l] = total; total += al256(lin_bytes(L.out_proj->dtype, dm, dir));
        off_cw[l] = total; total += al256((size_t)xdr * dc * 2);
        off_cb[l] = total; total += al256((size_t)xdr * 2);
        off_dtb[l] = total; total += al256((size_t)Hr * 2);
        off_al[l] = total; total += al256((size_t)Hr * 2);
        off_D[l] = total; total += al256((size_t)Hr * 2);
        off_mn[l] = total; total += al256((size_t)dir * 2);
    }
    const size_t off_lm = total;
    total += al256(lin_bytes(m->lm_head->dtype, Vr, dm));
    if (lssm_status st = s_alloc(reinterpret_cast<void**>(&s->d_shard), total, "tensor parallel: shard")) return st;
    cudaStream_t st = s->ctx->stream;
    uint8_t* base = s->d_shard;
    const uint8_t* img = m->d_base;
    auto cp = [&](void* dst, const void* src, size_t n) -> cudaError_t {
        return n ? cudaMemcpyAsync(dst, src, n, cudaMemcpyDeviceToDevice, st) : cudaSuccess;
    };
    // row segments (model row, rows) of this rank's in_proj rows: [z | x | B | C | dt]
    const uint32_t seg_src[5] = {r * dir, di + r * dir, 2 * di + r * GNr, 2 * di + GN + r * GNr, di + xd + r * Hr};
    const uint32_t seg_n[5] = {dir, dir, GNr, GNr, Hr};
    // channel segments of the conv weights / bias: [x | B | C]
    const uint32_t ch_src[3] = {r * dir, di + r * GNr, di + GN + r * GNr};
    const uint32_t ch_n[3] = {dir, GNr, GNr};
    s->lw.resize(h.n_layer);
    cudaError_t e = cudaSuccess;
    auto hp = [&](const TensorRec* t) { return reinterpret_cast<const __half*>(img + t->offset); };
    for (uint32_t l = 0; l < h.n_layer && e == cudaSuccess; ++l) {
        const LayerW& L = m->layers[l];
        // in_proj rows
        const uint8_t* src = img + L.in_proj->offset;
        uint8_t* dst = base + off_in[l];
        if (L.in_proj->dtype == DT_INT4_B32) {
            const size_t rb = dm / 2, sb = dm / 32 * 2;
            const uint8_t* ssc = src + (size_t)m->proj * rb;
            uint8_t* dsc = dst + (size_t)projr * rb;
            for (uint32_t sg = 0, row = 0; sg < 5; row += seg_n[sg], ++sg) {
                if (e == cudaSuccess) e = cp(dst + (size_t)row * rb, src + (size_t)seg_src[sg] * rb, (size_t)seg_n[sg] * rb);
                if (e == cudaSuccess) e = cp(dsc + (size_t)row * sb, ssc + (size_t)seg_src[sg] * sb, (size_t)seg_n[sg] * sb);
            }
        } else {
            const size_t rb = (size_t)dm * 2;
            for (uint32_t sg = 0, row = 0; sg < 5; row += seg_n[sg], ++sg)
                if (e == cudaSuccess) e = cp(dst + (size_t)row * rb, src + (size_t)seg_src[sg] * rb, (size_t)seg_n[sg] * rb);
        }
        // out_proj columns [r * dir, (r + 1) * dir) of every row (K split)
        const uint8_t* osrc = img + L.out_proj->offset;
        uint8_t* odst = base + off_out[l];
        if (L.out_proj->dtype == DT_INT4_B32) {
            if (e == cudaSuccess)
                e = cudaMemcpy2DAsync(odst, dir / 2, osrc + (size_t)r * dir / 2, di / 2, dir / 2, dm,
                                      cudaMemcpyDeviceToDevice, st);
            if (e == cudaSuccess)
                e = cudaMemcpy2DAsync(odst + (size_t)dm * dir / 2, dir / 32 * 2, osrc + (size_t)dm * di / 2 + (size_t)r * dir / 32 * 2,
                                      di / 32 * 2, dir / 32 * 2, dm, cudaMemcpyDeviceToDevice, st);
        } else if (e == cudaSuccess) {
            e = cudaMemcpy2DAsync(odst, (size_t)dir * 2, osrc + (size_t)r * dir * 2, (size_t)di * 2, (size_t)dir * 2, dm,
                                  cudaMemcpyDeviceToDevice, st);
        }
        // conv weights / bias channels, head parameters, mixer-norm slice
        for (uint32_t sg = 0, ch = 0; sg < 3; ch += ch_n[sg], ++sg) {
            if (e == cudaSuccess)
                e = cp(base + off_cw[l] + (size_t)ch * dc * 2, img + L.conv_w->offset + (size_t)ch_src[sg] * dc * 2,
                       (size_t)ch_n[sg] * dc * 2);
            if (e == cudaSuccess)
                e = cp(base + off_cb[l] + (size_t)ch * 2, img + L.conv_b->offset + (size_t)ch_src[sg] * 2, (size_t)ch_n[sg] * 2);
        }
        if (e == cudaSuccess) e = cp(base + off_dtb[l], img + L.dt_bias->offset + (size_t)r * Hr * 2, (size_t)Hr * 2);
        if (e == cudaSuccess) e = cp(base + off_al[l], img + L.A_log->offset + (size_t)r * Hr * 2, (size_t)Hr * 2);
        if (e == cudaSuccess) e = cp(base + off_D[l], img + L.D->offset + (size_t)r * Hr * 2, (size_t)Hr * 2);
        if (e == cudaSuccess) e = cp(base + off_mn[l], img + L.mixer_norm->offset + (size_t)r * dir * 2, (size_t)dir * 2);
        auto bh = [&](size_t o) { return reinterpret_cast<const __half*>(base + o); };
        s->lw[l] = {base + off_in[l], L.in_proj->dtype, base + off_out[l], L.out_proj->dtype, bh(off_cw[l]),
                    bh(off_cb[l]), bh(off_dtb[l]), bh(off_al[l]), bh(off_D[l]), hp(L.norm), bh(off_mn[l])};
    }
    // lm_head vocab rows [voff, voff + Vr)
    if (e == cudaSuccess) {
        const uint8_t* lsrc = img + m->lm_head->offset;
        if (m->lm_head->dtype == DT_INT4_B32) {
            const size_t rb = dm / 2, sb = dm / 32 * 2;
            e = cp(base + off_lm, lsrc + (size_t)voff * rb, (size_t)Vr * rb);
            if (e == cudaSuccess)
                e = cp(base + off_lm + (size_t)Vr * rb, lsrc + (size_t)h.vocab_size * rb + (size_t)voff * sb, (size_t)Vr * sb);
        } else {
            e = cp(base + off_lm, lsrc + (size_t)voff * dm * 2, (size_t)Vr * dm * 2);
        }
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(e, "tensor parallel: shard copies");
    s->lm_w = base + off_lm;
    s->lm_dt = m->lm_head->dtype;
    s->embed = hp(m->embed);
    s->norm_f = hp(m->norm_f);
    s->di = dir; s->xd = xdr; s->proj_dim = projr; s->GN = GNr; s->H = Hr; s->G = Gr;
    s->V = Vr; s->v_off = voff; s->v_max = vmax;
    return LSSM_OK;
}

// Shard, buffers and options of a new session (no collective steps).
static lssm_status session_alloc(lssm_session* s, uint32_t batch, uint32_t max_L) {
    lssm_model* m = s->m;
    lssm_ctx* ctx = s->ctx;
    const SsmHeader& h = m->img.hdr;
    lssm_status st;
    if (s->comm) {
        if ((st = build_tp_shard(s))) return st;
    } else {
        bind_model_refs(s);
    }
    const size_t rows = (size_t)batch * max_L;
    s->conv_layer = (size_t)batch * s->xd * h.d_conv;
    s->ssd_layer = (size_t)batch * s->H * h.d_head * h.d_state;
#define SA(ptr, n, what) if ((st = s_alloc(reinterpret_cast<void**>(&ptr), n, what))) return st
    SA(s->conv, s->conv_layer * h.n_layer * 2, "session: conv state");
    SA(s->ssd, s->ssd_layer * h.n_layer * 4, "session: ssd state");
    SA(s->hidden, rows * h.d_model * 2, "session: hidden");
    // normed holds the RMSNorm output of either linear's input (d_model for in_proj,
    // d_inner for out_proj), so it is sized for the wider of the two.
    SA(s->normed, rows * std::max<size_t>(h.d_model, s->di) * 2, "session: normed");
    SA(s->proj, rows * s->proj_dim * 2, "session: proj");
    SA(s->xs, rows * s->di * 2, "session: x");
    SA(s->Bs, rows * s->GN * 2, "session: B");
    SA(s->Cs, rows * s->GN * 2, "session: C");
    SA(s->ys, rows * s->di * 2, "session: y");
    SA(s->gated, rows * s->di * 2, "session: gated");
    SA(s->mixn, rows * s->di * 2, "session: mixer norm");
    SA(s->logits, (size_t)batch * s->v_max * 2, "session: logits");
    SA(s->lastrows, (size_t)batch * h.d_model * 2, "session: last rows");
    SA(s->d_tokens, rows * 4, "session: tokens");
    SA(s->d_cur, (size_t)batch * 4, "session: current tokens");
    SA(s->d_step, 16, "session: step");
    SA(s->d_err, 16, "session: error word");
    if (s->comm) {
        SA(s->d_sumsq, rows * 4, "session: TP sum of squares");
        SA(s->d_part32, rows * h.d_model * 4, "session: TP out_proj partials");
    }
    SA(s->d_cpair, (size_t)batch * argmax_chunks(s->V) * sizeof(uint2), "session: argmax chunk pairs");
    SA(s->d_pair, (size_t)s->tp_world * batch * sizeof(uint2), "session: argmax row pairs");
    SA(s->d_ticket, (size_t)batch * 4, "session: argmax tickets");
    cudaMemsetAsync(s->d_ticket, 0, (size_t)batch * 4, ctx->stream);
    bool any_int4 = false;
    size_t wmax = 0;
    for (auto& L : s->lw) {
        if (L.in_dt == DT_INT4_B32) { any_int4 = true; wmax = std::max<size_t>(wmax, (size_t)s->proj_dim * h.d_model); }
        if (L.out_dt == DT_INT4_B32) { any_int4 = true; wmax = std::max<size_t>(wmax, (size_t)h.d_model * s->di); }
    }
    if (s->lm_dt == DT_INT4_B32) { any_int4 = true; wmax = std::max<size_t>(wmax, (size_t)s->V * h.d_model); }
    // dequant scratch of the INT4 prefill GEMMs; also the carried-state ring of the
    // chunk-parallel SSD scan, which runs while no GEMM uses it
    size_t wbytes = any_int4 ? wmax * 2 : 0;
    if (h.d_head == 64 && h.d_state == 128) wbytes = std::max(wbytes, ssd_chunked_cp_scratch(batch, s->H));
    if (wbytes) {
        SA(s->wscratch, wbytes, "session: dequant / scan scratch");
        s->wscratch_elems = wbytes / 2;
    }
#undef SA
    for (auto& e : s->ev) cudaEventCreate(&e);
    cudaMemsetAsync(s->d_err, 0, 16, ctx->stream);
    if (!s->comm && (st = setup_persistent(s))) return st;
    if (s->comm) s->persist_why = "tensor-parallel session";
    return LSSM_OK;
}

// Under tensor parallelism session creation is collective: every rank allocates, the ranks
// agree on the outcome (so one rank's failure fails all of them instead of leaving the others
// waiting), then set up the peer exchange of the decode all-reduces together.
static lssm_status session_create_impl(lssm_ctx* ctx, lssm_model* m, lssm_comm* comm, uint32_t batch, uint32_t max_L,
                                       lssm_session** out) {
    if (!ctx || !m || !out) return fail(LSSM_ERR_INVALID_ARGUMENT, "lssm_session_create: null argument");
    if (batch == 0 || max_L == 0) return fail(LSSM_ERR_INVALID_ARGUMENT, "lssm_session_create: batch and max_seq_len must be >= 1");
    cudaSetDevice(ctx->device);
    *out = nullptr;
    std::unique_ptr<lssm_session, lssm_status (*)(lssm_session*)> s(new lssm_session(), lssm_session_destroy);
    s->ctx = ctx;
    s->m = m;
    s->batch = batch;
    s->max_L = max_L;
    s->comm = comm;
    s->tp_rank = comm_rank(comm);
    s->tp_world = comm_world(comm);
    lssm_status st = session_alloc(s.get(), batch, max_L);
    if (comm) {
        const std::string why = st ? lssm_last_error() : std::string();
        bool all = false;
        if (lssm_status cst = comm_agree(comm, st == LSSM_OK, &all)) return cst;
        if (!all) {
            if (st) return fail(st, "%s", why.c_str());
            return fail(LSSM_ERR_CUDA, "lssm_session_create_tp: another rank failed to create its session");
        }
        // the peer exchange of the decode all-reduces (batch x d_model floats)
        if ((st = comm_p2p_setup(comm, (size_t)batch * m->img.hdr.d_model))) return st;
    } else if (st) {
        return st;
    }
    if ((st = lssm_session_reset(s.get()))) return st;
    *out = s.release();
    return LSSM_OK;
}

extern "C" lssm_status lssm_session_create(lssm_ctx* ctx, lssm_model* m, uint32_t batch, uint32_t max_L,
                                           lssm_session** out) {
    return session_create_impl(ctx, m, nullptr, batch, max_L, out);
}

extern "C" lssm_status lssm_session_create_tp(lssm_ctx* ctx, lssm_model* m, lssm_comm* comm, uint32_t batch,
                                              uint32_t max_L, lssm_session** out) {
    if (!comm) return fail(LSSM_ERR_INVALID_ARGUMENT, "lssm_session_create_tp: null communicator");
    return session_create_impl(ctx, m, comm, batch, max_L, out);
}

extern "C" lssm_status lssm_session_reset(lssm_session* s) {
    if (!s) return fail(LSSM_ERR_INVALID_ARGUMENT, "lssm_session_reset: null session");
    cudaSetDevice(s->ctx->device);
    const SsmHeader& h = s->m->img.hdr;
    cudaError_t e = cudaMemsetAsync(s->conv, 0, s->conv_layer * h.n_layer * 2, s->ctx->stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(s->ssd, 0, s->ssd_layer * h.n_layer * 4, s->ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s->ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "Mamba2State::reset");
    s->logits_valid = false;
    return LSSM_OK;
}

extern "C" lssm_status lssm_session_set_option(lssm_session* s, const char* key, int64_t value) {
    if (!s || !key) return fail(LSSM_ERR_INVALID_ARGUMENT, "lssm_session_set_option: null argument");
    if (std::strcmp(key, "persistent") == 0) {
        s->use_persist = value != 0;
        return LSSM_OK;
    }
    if (std::strcmp(key, "trace") == 0) {
        s->trace_on = value != 0;
        if (s->trace_on && !s->d_trace && s->persist_ok) {
            const size_t n = (size_t)s->ctx->sm_count * trace_words(s);
            if (lssm_status st = s_alloc(reinterpret_cast<void**>(&s->d_trace), n * 8, "session: trace")) return st;
            cudaMemset(s->d_trace, 0, n * 8);
        }
        return LSSM_OK;
    }
    if (std::strcmp(key, "cuda_graph") == 0) {
        s->use_graph = value != 0;
        if (s->graph) { cudaGraphExecDestroy(s->graph); s->graph = nullptr; }
        return LSSM_OK;
    }
    if (std::strcmp(key, "tp_p2p") == 0) {   // set alike on every rank
        s->use_p2p = value != 0;
        if (s->graph) { cudaGraphExecDestroy(s->graph); s->graph = nullptr; }
        return LSSM_OK;
    }
    return fail(LSSM_ERR_INVALID_ARGUMENT, "lssm_session_set_option: unknown key '%s'", key);
}

#define CU(expr)                                                  \
    do {                                                          \
        cudaError_t _e = (expr);                                  \
        if (_e != cudaSuccess) return cuda_fail(_e, #expr);       \
    } while (0)

static inline const void* W(const lssm_model* m, const TensorRec* t) { return m->d_base + t->offset; }

// Linear over `rows` activation rows with weight `wp` (f16 or INT4_B32, .ssm layout): Y = X W^T.
// rows <= 8 uses the GEMV kernels (optionally with fused RMSNorm / residual), otherwise
// the tensor-core GEMM (INT4: fused dequant for small M, else dequantised to scratch).
// epilogue: 0 store fp16, 1 SiLU, 2 residual add into y, 3 store fp32 (y is float*).
static lssm_status linear(lssm_session* s, const uint8_t* wp, uint32_t dtype, const __half* x, void* y, uint32_t rows,
                          uint32_t N, uint32_t K, const __half* prenorm, int epilogue, cudaStream_t st) {
    if (rows <= 8) {
        if (dtype == DT_INT4_B32)
            CU(launch_gemv_int4_ex(x, wp, wp + (size_t)N * K / 2, y, rows, N, K, prenorm, 1e-5f, epilogue, st));
        else
            CU(launch_gemv_f16(x, wp, y, rows, N, K, prenorm, 1e-5f, epilogue, st));
        s->nl += 1;
        return LSSM_OK;
    }
    const __half* xin = x;
    if (prenorm) {
        CU(launch_rmsnorm_f16(x, prenorm, s->normed, rows, K, 1e-5f, st));
        s->nl += 1;
        xin = s->normed;
    }
    // the GEMMs apply the residual (epilogue 2) in place on y
    const void* wf = wp;
    if (dtype == DT_INT4_B32) {
        // fused dequant GEMM when the operands allow it; else dequantise to scratch + GEMM
        const void* sc = wp + (size_t)N * K / 2;
        // the dequant scratch is idle on this path: it holds the split-K partials
        int launched = 0;
        const cudaError_t e = launch_gemm_i4(xin, wp, sc, y, rows, N, K, epilogue, st,
                                             reinterpret_cast<float*>(s->wscratch), s->wscratch_elems * 2, &launched);
        if (e == cudaSuccess) {
            s->nl += launched;
            return LSSM_OK;
        }
        if (e != cudaErrorNotSupported) return cuda_fail(e, "linear: fused INT4 GEMM");
        cudaGetLastError();
        CU(launch_int4_dequant_f16(wp, sc, s->wscratch, N, K, st));
        s->nl += 1;
        wf = s->wscratch;
    }
    CU(launch_gemm_f16(xin, wf, y, rows, N, K, epilogue, st));
    s->nl += 1;
    return LSSM_OK;
}

// One Mamba-2 block over rows = batch * L activation rows (decode: L == 1), on this
// session's weights and local dims (a rank's shard under tensor parallelism).
static lssm_status run_block(lssm_session* s, uint32_t layer, uint32_t L, bool decode, cudaStream_t st) {
    lssm_model* m = s->m;
    const SsmHeader& h = m->img.hdr;
    const LayerRef& lw = s->lw[layer];
    const uint32_t B = s->batch, rows = B * L, dm = h.d_model, di = s->di, GN = s->GN, xd = s->xd, proj = s->proj_dim,
                   H = s->H, P = h.d_head, N = h.d_state, Kc = h.d_conv;
    __half* conv = reinterpret_cast<__half*>(s->conv) + s->conv_layer * layer;
    float* ssd = s->ssd + s->ssd_layer * layer;
    lssm_status r;
    // 1+2. RMSNorm + in_proj over [z | xBC | dt]
    if ((r = linear(s, lw.in_w, lw.in_dt, s->hidden, s->proj, rows, proj, dm, lw.norm, 0, st))) return r;
    const __half* zc = s->proj;
    const __half* xbc = s->proj + di;
    const __half* dtc = s->proj + di + xd;
    if (decode) {
        // 3+4. conv update + SiLU + split
        CU(launch_conv_update_silu_split(xbc, proj, conv, lw.conv_w, lw.conv_b, s->xs, s->Bs, s->Cs, B, di, GN, Kc, st));
        // 5+6. ssd_step with the fused gate -> gated
        StepArgs a{};
        a.x = s->xs; a.B = s->Bs; a.C = s->Cs; a.dt_raw = dtc;
        a.dt_bias = lw.dt_bias; a.A_log = lw.A_log; a.D = lw.D;
        a.state = ssd; a.y = s->gated; a.z = zc;
        a.batch = B; a.H = H; a.P = P; a.N = N; a.G = s->G;
        a.dt_min = 1e-6f; a.dt_max = 1e6f; a.has_D = 1;
        a.x_bs = di; a.bc_bs = GN; a.dt_bs = proj; a.y_bs = di; a.z_bs = proj;
        CU(launch_ssd_step_ex(a, st));
        s->nl += 2;
    } else {
        CU(launch_conv_silu_split(xbc, proj, lw.conv_w, lw.conv_b, s->xs, s->Bs, s->Cs, B, L, di, GN, Kc, st));
        SsdArgs a{};
        a.X = s->xs; a.B = s->Bs; a.C = s->Cs; a.dt_raw = dtc;
        a.dt_bias = lw.dt_bias; a.A_log = lw.A_log; a.D = lw.D;
        a.Y = s->gated; a.state = ssd;   // gated output: the gate is applied in the scan's epilogue
        a.z = zc; a.z_row_stride = proj;
        a.batch = B; a.L = L; a.H = H; a.P = P; a.N = N; a.G = s->G; a.chunk = h.chunk_size;
        a.dt_min = 1e-6f; a.dt_max = 1e6f; a.has_D = 1;
        a.x_dtype = 0; a.dt_dtype = 0; a.param_dtype = 0; a.y_dtype = 0;
        a.x_row_stride = di; a.bc_row_stride = GN; a.dt_row_stride = proj; a.y_row_stride = di;
        // the chunk-parallel scan keeps its carried states in the dequant scratch, idle between
        // the in_proj and out_proj GEMMs
        a.ws_bytes = ssd_chunked_cp_scratch(B, H);
        if (s->wscratch && s->wscratch_elems * 2 >= a.ws_bytes) a.ws = s->wscratch;
        a.sm_count = s->ctx->sm_count;
        CU(launch_ssd_chunked(a, st));
        s->nl += 2;
    }
    // 7+8+9. gated RMSNorm + out_proj + residual add into hidden
    if (s->comm && decode && s->use_p2p && comm_p2p(s->comm, (size_t)rows * dm)) {
        // decode: the same two all-reduces over the peer exchange, the second one adding the
        // rounded sum to the residual in the same kernel
        CU(launch_rowsumsq(s->gated, di, rows, di, s->d_sumsq, st));
        if ((r = comm_p2p_allreduce(s->comm, s->d_sumsq, rows, s->d_sumsq, nullptr, st))) return r;
        CU(launch_rmsnorm_total(s->gated, di, lw.mixer_norm, s->d_sumsq, rows, di, m->d_inner, 1e-5f, s->mixn, st));
        if ((r = linear(s, lw.out_w, lw.out_dt, s->mixn, s->d_part32, rows, dm, di, nullptr, 3, st))) return r;
        if ((r = comm_p2p_allreduce(s->comm, s->d_part32, (size_t)rows * dm, nullptr, s->hidden, st))) return r;
        s->nl += 4;
    } else if (s->comm) {
        // the gated RMSNorm spans the full d_inner: all-reduce each row's sum of squares; the
        // out_proj partials of this rank's d_inner columns are summed in fp32 across the ranks
        // and rounded to fp16 once before the residual add
        CU(launch_rowsumsq(s->gated, di, rows, di, s->d_sumsq, st));
        if ((r = comm_allreduce_f32(s->comm, s->d_sumsq, rows, st))) return r;
        CU(launch_rmsnorm_total(s->gated, di, lw.mixer_norm, s->d_sumsq, rows, di, m->d_inner, 1e-5f, s->mixn, st));
        if ((r = linear(s, lw.out_w, lw.out_dt, s->mixn, s->d_part32, rows, dm, di, nullptr, 3, st))) return r;
        if ((r = comm_allreduce_f32(s->comm, s->d_part32, (size_t)rows * dm, st))) return r;
        CU(launch_residual_f32(s->hidden, s->d_part32, (uint64_t)rows * dm, st));
        s->nl += 3;
    } else if ((r = linear(s, lw.out_w, lw.out_dt, s->gated, s->hidden, rows, dm, di, lw.mixer_norm, 2, st))) {
        return r;
    }
    // 10. seed conv state from pre-conv xBC after a prefill
    if (!decode) {
        CU(launch_seed_strided(xbc, proj, conv, B, L, xd, Kc, st));
        s->nl += 1;
    }
    return LSSM_OK;
}

// norm_f + lm_head over `x` (batch rows, contiguous) -> logits, then the greedy token:
// d_cur; with `decode`, also history[step] and hidden = embed(next) for the next step.
// Under tensor parallelism the logits are this rank's vocab slice and the ranks merge
// their (value, index) first-max pairs.
static lssm_status pick_tokens(lssm_session* s, const __half* x, bool decode, cudaStream_t st) {
    lssm_model* m = s->m;
    const SsmHeader& h = m->img.hdr;
    // one call for all rows: the GEMV kernels for <= 8 rows, else the tensor-core GEMM, so
    // the lm_head weights are read once per step whatever the batch
    if (lssm_status r = linear(s, s->lm_w, s->lm_dt, x, s->logits, s->batch, s->V, h.d_model, s->norm_f, 0, st)) return r;
    uint32_t* hist = decode ? s->d_hist : nullptr;
    uint32_t* step = decode ? s->d_step : nullptr;
    const __half* emb = decode ? s->embed : nullptr;
    __half* hid = decode ? s->hidden : nullptr;
    const size_t B = s->batch, rk = (size_t)s->tp_rank;
    CU(launch_argmax_chunks(s->logits, s->V, s->batch, s->V, s->v_off, s->d_cpair, s->d_ticket, s->d_pair + rk * B, st));
    if (s->comm)
        if (lssm_status r = comm_allgather(s->comm, s->d_pair + rk * B, s->d_pair, B * sizeof(uint2), st)) return r;
    CU(launch_argmax_merge(s->d_pair, (uint32_t)s->tp_world, s->batch, s->d_cur, hist, s->hist_cap, step, emb, hid,
                           h.d_model, st));
    s->nl += decode ? 3 : 2;
    return LSSM_OK;
}

static lssm_status check_err(lssm_session* s, const char* what) {
    int herr = 0;
    CU(cudaMemcpy(&herr, s->d_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (herr == 2) {
        cudaMemset(s->d_err, 0, sizeof(int));
        return fail(LSSM_ERR_INVALID_ARGUMENT, "Mamba2Model::embed: token_id out of range (%s)", what);
    }
    int* tw = tc_error_word();
    if (tw) {
        CU(cudaMemcpy(&herr, tw, sizeof(int), cudaMemcpyDeviceToHost));
        if (herr) {
            cudaMemset(tw, 0, sizeof(int));
            return fail(LSSM_ERR_TIMEOUT, "%s: a bounded device wait timed out", what);
        }
    }
    return LSSM_OK;
}

extern "C" lssm_status lssm_prefill(lssm_session* s, const uint32_t* tokens, uint32_t L, uint32_t* next_tokens) {
    if (!s || !tokens) return fail(LSSM_ERR_INVALID_ARGUMENT, "lssm_prefill: null argument");
    if (L == 0) return fail(LSSM_ERR_INVALID_ARGUMENT, "forward_prefill: L must be >= 1");
    if (L > s->max_L) return fail(LSSM_ERR_INVALID_ARGUMENT, "forward_prefill: L exceeds workspace max_seq_len");
    cudaSetDevice(s->ctx->device);
    cudaStream_t st = s->ctx->stream;
    lssm_model* m = s->m;
    const SsmHeader& h = m->img.hdr;
    const uint32_t rows = s->batch * L;
    CU(cudaMemcpyAsync(s->d_tokens, tokens, (size_t)rows * 4, cudaMemcpyHostToDevice, st));
    const uint64_t nl0 = s->nl;
    CU(cudaEventRecord(s->ev[0], st));   // device timing starts with the tokens resident in HBM
    CU(launch_embed_gather(s->d_tokens, W(m, m->embed), s->hidden, rows, h.d_model, h.vocab_size, s->d_err, st));
    s->nl += 1;
    for (uint32_t l = 0; l < h.n_layer; ++l)
        if (lssm_status r = run_block(s, l, L, false, st)) return r;
    // last row of each sequence -> contiguous (batch, d_model)
    CU(cudaMemcpy2DAsync(s->lastrows, (size_t)h.d_model * 2, s->hidden + (size_t)(L - 1) * h.d_model,
                         (size_t)L * h.d_model * 2, (size_t)h.d_model * 2, s->batch, cudaMemcpyDeviceToDevice, st));
    if (lssm_status r = pick_tokens(s, s->lastrows, false, st)) return r;
    s->prefill_launches = s->nl - nl0;
    CU(cudaEventRecord(s->ev[1], st));
    if (next_tokens) CU(cudaMemcpyAsync(next_tokens, s->d_cur, (size_t)s->batch * 4, cudaMemcpyDeviceToHost, st));
    CU(cudaStreamSynchronize(st));
    cudaEventElapsedTime(&s->prefill_ms, s->ev[0], s->ev[1]);
    s->logits_valid = true;
    return check_err(s, "prefill");
}

// One decode step on the device: input = s->hidden rows (already embedded), output:
// logits, d_cur, history[step] and hidden = embed(next) for the following step.
static lssm_status decode_step_body(lssm_session* s, cudaStream_t st) {
    lssm_model* m = s->m;
    const SsmHeader& h = m->img.hdr;
    for (uint32_t l = 0; l < h.n_layer; ++l)
        if (lssm_status r = run_block(s, l, 1, true, st)) return r;
    return pick_tokens(s, s->hidden, true, st);
}

extern "C" lssm_status lssm_decode(lssm_session* s, const uint32_t* first, uint32_t n_steps, uint32_t* out_tokens) {
    if (!s || !first) return fail(LSSM_ERR_INVALID_ARGUMENT, "lssm_decode: null argument");
    cudaSetDevice(s->ctx->device);
    cudaStream_t st = s->ctx->stream;
    lssm_model* m = s->m;
    const SsmHeader& h = m->img.hdr;
    if (n_steps == 0) return LSSM_OK;
    if (n_steps > s->hist_cap) {
        if (s->d_hist) cudaFree(s->d_hist);
        s->d_hist = nullptr;
        if (s->graph) { cudaGraphExecDestroy(s->graph); s->graph = nullptr; }
        CU(cudaMalloc(&s->d_hist, (size_t)s->batch * n_steps * 4));
        s->hist_cap = n_steps;
    }
    CU(cudaMemcpyAsync(s->d_cur, first, (size_t)s->batch * 4, cudaMemcpyHostToDevice, st));
    CU(cudaMemsetAsync(s->d_step, 0, 4, st));
    if (s->persist_ok && s->use_persist) {
        // one cooperative launch runs all n_steps tokens (embedding gather included);
        // the kernel reads embedding rows directly, so the ids are range-checked here
        for (uint32_t b = 0; b < s->batch; ++b)
            if (first[b] >= h.vocab_size)
                return fail(LSSM_ERR_INVALID_ARGUMENT, "Mamba2Model::embed: token_id out of range (decode)");
        CU(cudaMemsetAsync(s->d_bar, 0, 4, st));
        // epochs [epoch_next, epoch_next + n_steps * n_layer) tag this launch's exchange words;
        // before the 32-bit tag would wrap, the words are cleared and the count restarts at 1
        const uint64_t span = (uint64_t)n_steps * h.n_layer;
        if ((uint64_t)s->epoch_next + span >= 0xFFFFFFF0ull) {
            if (span >= 0xFFFFFFF0ull) return fail(LSSM_ERR_INVALID_ARGUMENT, "decode: too many steps for one launch");
            CU(cudaMemsetAsync(s->d_mb, 0, s->mb_words * 8, st));
            s->epoch_next = 1;
        }
        PParams pp = persist_params(s, n_steps);
        s->epoch_next += (uint32_t)span;
        CU(cudaEventRecord(s->ev[2], st));
        CU(launch_decode_persist(pp, s->ctx->sm_count, st));
        CU(cudaEventRecord(s->ev[3], st));
        s->decode_launches = 1;
        if (out_tokens)
            CU(cudaMemcpy2DAsync(out_tokens, (size_t)n_steps * 4, s->d_hist, (size_t)s->hist_cap * 4, (size_t)n_steps * 4,
                                 s->batch, cudaMemcpyDeviceToHost, st));
        CU(cudaStreamSynchronize(st));
        cudaEventElapsedTime(&s->decode_ms, s->ev[2], s->ev[3]);
        s->logits_valid = true;
        return check_err(s, "decode");
    }
    CU(launch_embed_gather(s->d_cur, W(m, m->embed), s->hidden, s->batch, h.d_model, h.vocab_size, s->d_err, st));
    if (s->use_graph && !s->graph) {
        cudaGraph_t g;
        CU(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        const uint64_t nl0 = s->nl;
        lssm_status r = decode_step_body(s, st);
        s->decode_step_launches = s->nl - nl0;
        cudaError_t e = cudaStreamEndCapture(st, &g);
        if (r) { if (e == cudaSuccess) cudaGraphDestroy(g); return r; }
        if (e != cudaSuccess) return cuda_fail(e, "decode graph capture");
        e = cudaGraphInstantiate(&s->graph, g, 0);
        cudaGraphDestroy(g);
        if (e != cudaSuccess) { s->graph = nullptr; return cuda_fail(e, "decode graph instantiate"); }
    }
    CU(cudaEventRecord(s->ev[2], st));
    for (uint32_t i = 0; i < n_steps; ++i) {
        if (s->graph) CU(cudaGraphLaunch(s->graph, st));
        else {
            const uint64_t nl0 = s->nl;
            if (lssm_status r = decode_step_body(s, st)) return r;
            s->decode_step_launches = s->nl - nl0;
        }
    }
    CU(cudaEventRecord(s->ev[3], st));
    s->decode_launches = 1 + (uint64_t)n_steps * s->decode_step_launches;
    if (out_tokens) {
        // history is (batch, hist_cap); copy the first n_steps of each row
        CU(cudaMemcpy2DAsync(out_tokens, (size_t)n_steps * 4, s->d_hist, (size_t)s->hist_cap * 4, (size_t)n_steps * 4,
                             s->batch, cudaMemcpyDeviceToHost, st));
    }
    CU(cudaStreamSynchronize(st));
    cudaEventElapsedTime(&s->decode_ms, s->ev[2], s->ev[3]);
    s->logits_valid = true;
    return check_err(s, "decode");
}

extern "C" lssm_status lssm_generate(lssm_session* s, const uint32_t* prompt, uint32_t L, uint32_t max_new,
                                     uint32_t eos, uint32_t* out, uint32_t* n_out) {
    if (!s || !prompt || !out) return fail(LSSM_ERR_INVALID_ARGUMENT, "lssm_generate: null argument");
    if (max_new == 0) { if (n_out) *n_out = 0; return LSSM_OK; }
    lssm_status r = lssm_session_reset(s);
    if (r) return r;
    std::vector<uint32_t> first(s->batch);
    if ((r = lssm_prefill(s, prompt, L, first.data()))) return r;
    std::vector<uint32_t> rest((size_t)s->batch * (max_new - 1));
    if (max_new > 1 && (r = lssm_decode(s, first.data(), max_new - 1, rest.data()))) return r;
    uint32_t produced = max_new;
    for (uint32_t b = 0; b < s->batch; ++b) {
        out[(size_t)b * max_new] = first[b];
        for (uint32_t i = 1; i < max_new; ++i) out[(size_t)b * max_new + i] = rest[(size_t)b * (max_new - 1) + i - 1];
    }
    if (eos != 0xFFFFFFFFu && s->batch == 1) {   // inference.cpp:56 stops after emitting eos
        for (uint32_t i = 0; i < max_new; ++i)
            if (out[i] == eos) { produced = i + 1; break; }
    }
    if (n_out) *n_out = produced;
    return LSSM_OK;
}

extern "C" lssm_status lssm_session_logits(lssm_session* s, float* out) {
    if (!s || !out) return fail(LSSM_ERR_INVALID_ARGUMENT, "lssm_session_logits: null argument");
    if (!s->logits_valid) return fail(LSSM_ERR_STATE, "lssm_session_logits: no logits computed yet");
    const SsmHeader& h = s->m->img.hdr;
    auto f = [](uint16_t v) { return __half2float(*reinterpret_cast<__half*>(&v)); };
    if (s->comm) {
        // collective: gather every rank's vocab slice (batch x v_max each, rank-major)
        const size_t per = (size_t)s->batch * s->v_max, W = (size_t)s->tp_world;
        if (!s->d_gather) {
            if (lssm_status st = s_alloc(reinterpret_cast<void**>(&s->d_gather), per * W * 2, "session: logits gather"))
                return st;
        }
        if (lssm_status st = comm_allgather(s->comm, s->logits, s->d_gather, per * 2, s->ctx->stream)) return st;
        std::vector<uint16_t> tmp(per * W);
        CU(cudaStreamSynchronize(s->ctx->stream));
        CU(cudaMemcpy(tmp.data(), s->d_gather, per * W * 2, cudaMemcpyDeviceToHost));
        for (size_t r = 0; r < W; ++r) {
            const size_t voff = std::min<size_t>(h.vocab_size, r * s->v_max);
            const size_t vr = std::min<size_t>(s->v_max, h.vocab_size - voff);
            for (size_t b = 0; b < s->batch; ++b)
                for (size_t j = 0; j < vr; ++j) out[b * h.vocab_size + voff + j] = f(tmp[r * per + b * vr + j]);
        }
        return LSSM_OK;
    }
    const size_t n = (size_t)s->batch * h.vocab_size;
    std::vector<uint16_t> tmp(n);
    CU(cudaMemcpy(tmp.data(), s->logits, n * 2, cudaMemcpyDeviceToHost));
    for (size_t i = 0; i < n; ++i) out[i] = f(tmp[i]);
    return LSSM_OK;
}

extern "C" lssm_status lssm_session_trace(lssm_session* s, uint64_t* out, uint64_t cap, uint64_t* n_out) {
    if (!s || !n_out) return fail(LSSM_ERR_INVALID_ARGUMENT, "lssm_session_trace: null argument");
    *n_out = 0;
    if (!s->persist_ok)
        return fail(LSSM_ERR_STATE, "lssm_session_trace: the persistent decode kernel does not run this session (%s)",
                    s->persist_why);
    if (!s->d_trace) return fail(LSSM_ERR_STATE, "lssm_session_trace: tracing is off");
    const size_t n = (size_t)s->ctx->sm_count * trace_words(s);
    *n_out = n;
    if (!out) return LSSM_OK;
    if (cap < n) return fail(LSSM_ERR_INVALID_ARGUMENT, "lssm_session_trace: buffer holds %llu words, %zu needed",
                             (unsigned long long)cap, n);
    CU(cudaMemcpy(out, s->d_trace, n * 8, cudaMemcpyDeviceToHost));
    return LSSM_OK;
}

extern "C" lssm_status lssm_session_launches(lssm_session* s, uint64_t* prefill, uint64_t* decode_step) {
    if (!s) return fail(LSSM_ERR_INVALID_ARGUMENT, "lssm_session_launches: null session");
    if (prefill) *prefill = s->prefill_launches;
    if (decode_step) *decode_step = s->decode_launches;
    return LSSM_OK;
}

extern "C" lssm_status lssm_session_timing(lssm_session* s, float* prefill_ms, float* decode_ms) {
    if (!s) return fail(LSSM_ERR_INVALID_ARGUMENT, "lssm_session_timing: null session");
    if (prefill_ms) *prefill_ms = s->prefill_ms;
    if (decode_ms) *decode_ms = s->decode_ms;
    return LSSM_OK;
}
