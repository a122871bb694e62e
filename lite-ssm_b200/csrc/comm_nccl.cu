// comm_nccl.cu — communicator of the head-tensor-parallel path (one rank per GPU, NVLink /
// NVSwitch): NCCL for setup and large messages, and a peer-memory exchange for the small
// per-layer all-reduces of decode.
//
// NCCL is opened at run time (dlopen "libnccl.so.2"): a process that already loaded NCCL
// (torch.distributed) shares that copy, otherwise the system library is used, and the
// kernel library itself keeps no link-time NCCL dependency. The unique id is made on one
// rank (lssm_comm_unique_id) and handed to the others by the caller (torch.distributed
// broadcast, a file, ...). Collectives run on the context's stream, so they order with the
// engine's kernels and can be captured in the decode CUDA graph.
//
// Peer exchange (comm_p2p_setup, collective): every rank allocates a receive area
// [2 parities][world][cap] of 8-byte words (value + epoch) and maps every peer's area
// through CUDA IPC (plain peer stores over NVLink, point to point). It is enabled only
// when all ranks sit on distinct GPUs with peer access: the exchange kernels poll for words
// that other ranks' kernels write, which must never share one GPU.
#include <dlfcn.h>
#include <nccl.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "lssm_internal.h"

struct lssm_comm {
    lssm_ctx* ctx = nullptr;
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1;
    // peer exchange
    bool p2p = false;
    size_t cap = 0;                       // floats per (parity, source rank)
    uint64_t* recv = nullptr;             // local [2][world][cap] words (epoch << 32 | value)
    uint32_t* epochs = nullptr;           // local [P2P_BLOCKS] call counters
    lssm::P2PPeers peers{};               // every rank's receive area as mapped here
};

namespace lssm {

int* tc_error_word();

namespace {

struct NcclApi {
    void* lib = nullptr;
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
    std::string error;
};

NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            api.error = std::string("cannot open libnccl.so.2: ") + dlerror();
            return;
        }
        api.lib = h;
        api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
        api.CommInitRank = reinterpret_cast<decltype(api.CommInitRank)>(dlsym(h, "ncclCommInitRank"));
        api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
        api.AllReduce = reinterpret_cast<decltype(api.AllReduce)>(dlsym(h, "ncclAllReduce"));
        api.AllGather = reinterpret_cast<decltype(api.AllGather)>(dlsym(h, "ncclAllGather"));
        api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(dlsym(h, "ncclGetErrorString"));
        if (!api.GetUniqueId || !api.CommInitRank || !api.CommDestroy || !api.AllReduce || !api.AllGather ||
            !api.GetErrorString)
            api.error = "libnccl.so.2 lacks a required entry point";
    });
    return api;
}

lssm_status nccl_fail(ncclResult_t r, const char* what) {
    return fail(LSSM_ERR_CUDA, "%s: NCCL error %d (%s)", what, (int)r, nccl().GetErrorString(r));
}

}  // namespace

// Sum-all-reduce in place (fp32) on the communicator's context stream.
lssm_status comm_allreduce_f32(lssm_comm* c, float* buf, size_t n, cudaStream_t s) {
    if (!c || c->world == 1 || !n) return LSSM_OK;
    const ncclResult_t r = nccl().AllReduce(buf, buf, n, ncclFloat32, ncclSum, c->comm, s);
    return r == ncclSuccess ? LSSM_OK : nccl_fail(r, "ncclAllReduce");
}

// All-gather of `bytes` bytes per rank: dst holds world * bytes, rank-major.
lssm_status comm_allgather(lssm_comm* c, const void* src, void* dst, size_t bytes, cudaStream_t s) {
    if (!c || c->world == 1) {
        if (src != dst && bytes) {
            const cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, s);
            if (e != cudaSuccess) return cuda_fail(e, "all-gather (one rank)");
        }
        return LSSM_OK;
    }
    const ncclResult_t r = nccl().AllGather(src, dst, bytes, ncclUint8, c->comm, s);
    return r == ncclSuccess ? LSSM_OK : nccl_fail(r, "ncclAllGather");
}

// Whether every rank passes ok_local (collective; NCCL float min on 0 / 1).
lssm_status comm_agree(lssm_comm* c, bool ok_local, bool* ok_all) {
    *ok_all = ok_local;
    if (!c || c->world == 1) return LSSM_OK;
    float* d = nullptr;
    if (cudaMalloc(&d, sizeof(float)) != cudaSuccess) return fail(LSSM_ERR_OUT_OF_MEMORY, "comm: flag");
    const float h = ok_local ? 1.0f : 0.0f;
    cudaStream_t s = c->ctx->stream;
    cudaMemcpyAsync(d, &h, sizeof(float), cudaMemcpyHostToDevice, s);
    const ncclResult_t r = nccl().AllReduce(d, d, 1, ncclFloat32, ncclMin, c->comm, s);
    float out = 0.0f;
    cudaMemcpyAsync(&out, d, sizeof(float), cudaMemcpyDeviceToHost, s);
    const cudaError_t e = cudaStreamSynchronize(s);
    cudaFree(d);
    if (r != ncclSuccess) return nccl_fail(r, "ncclAllReduce (agree)");
    if (e != cudaSuccess) return cuda_fail(e, "comm: agree");
    *ok_all = out > 0.5f;
    return LSSM_OK;
}

// All-gather of a small host blob (bytes per rank) through NCCL; out holds world * bytes.
static lssm_status host_allgather(lssm_comm* c, const void* in, size_t bytes, void* out) {
    uint8_t* d = nullptr;
    if (cudaMalloc(&d, bytes * (c->world + 1)) != cudaSuccess) return fail(LSSM_ERR_OUT_OF_MEMORY, "comm: gather");
    cudaStream_t s = c->ctx->stream;
    cudaMemcpyAsync(d + bytes * c->world, in, bytes, cudaMemcpyHostToDevice, s);
    const ncclResult_t r = nccl().AllGather(d + bytes * c->world, d, bytes, ncclUint8, c->comm, s);
    cudaMemcpyAsync(out, d, bytes * c->world, cudaMemcpyDeviceToHost, s);
    const cudaError_t e = cudaStreamSynchronize(s);
    cudaFree(d);
    if (r != ncclSuccess) return nccl_fail(r, "ncclAllGather (setup)");
    if (e != cudaSuccess) return cuda_fail(e, "comm: gather");
    return LSSM_OK;
}

static void p2p_release(lssm_comm* c) {
    for (int r = 0; r < c->world && r < P2P_MAX_RANKS; ++r) {
        if (r == c->rank) continue;
        if (c->peers.recv[r]) cudaIpcCloseMemHandle(c->peers.recv[r]);
    }
    c->peers = P2PPeers{};
    if (c->recv) cudaFree(c->recv);
    if (c->epochs) cudaFree(c->epochs);
    c->recv = nullptr;
    c->epochs = nullptr;
    c->p2p = false;
    c->cap = 0;
}

// Collective: set up (or grow to `floats`) the peer exchange. Leaves c->p2p false, on every
// rank alike, when any rank cannot take part; the callers then use NCCL.
lssm_status comm_p2p_setup(lssm_comm* c, size_t floats) {
    if (!c || c->world == 1) return LSSM_OK;
    if (c->p2p && c->cap >= floats) return LSSM_OK;
    cudaSetDevice(c->ctx->device);
    if (c->p2p) {   // grow: every rank is here too (same session shapes in the same order)
        cudaStreamSynchronize(c->ctx->stream);
        p2p_release(c);
    }
    const int W = c->world;
    bool ok = W <= P2P_MAX_RANKS && !std::getenv("LSSM_TP_NO_P2P");
    // distinct devices with peer access between every pair
    char bus[32] = {0};
    if (cudaDeviceGetPCIBusId(bus, sizeof(bus), c->ctx->device) != cudaSuccess) ok = false;
    std::vector<char> all_bus((size_t)W * sizeof(bus));
    if (lssm_status st = host_allgather(c, bus, sizeof(bus), all_bus.data())) return st;
    for (int r = 0; r < W && ok; ++r) {
        if (r == c->rank) continue;
        if (std::strncmp(&all_bus[(size_t)r * sizeof(bus)], bus, sizeof(bus)) == 0) { ok = false; break; }
        int peer_dev = -1, can = 0;
        if (cudaDeviceGetByPCIBusId(&peer_dev, &all_bus[(size_t)r * sizeof(bus)]) != cudaSuccess ||
            cudaDeviceCanAccessPeer(&can, c->ctx->device, peer_dev) != cudaSuccess || !can)
            ok = false;
    }
    cudaGetLastError();
    // local area: recv [2][W][cap] words
    const size_t cap = (floats + 1023) / 1024 * 1024;
    const size_t total = 2 * (size_t)W * cap * sizeof(uint64_t);
    cudaIpcMemHandle_t mine{};
    if (ok) {
        if (cudaMalloc(&c->recv, total) != cudaSuccess || cudaMalloc(&c->epochs, P2P_BLOCKS * sizeof(uint32_t)) != cudaSuccess ||
            cudaMemset(c->recv, 0, total) != cudaSuccess || cudaMemset(c->epochs, 0, P2P_BLOCKS * sizeof(uint32_t)) != cudaSuccess ||
            cudaIpcGetMemHandle(&mine, c->recv) != cudaSuccess)
            ok = false;
        cudaDeviceSynchronize();
    }
    cudaGetLastError();
    bool all = false;
    if (lssm_status st = comm_agree(c, ok, &all)) return st;
    if (!all) {
        p2p_release(c);
        return LSSM_OK;
    }
    std::vector<cudaIpcMemHandle_t> handles(W);
    if (lssm_status st = host_allgather(c, &mine, sizeof(mine), handles.data())) return st;
    bool opened = true;
    for (int r = 0; r < W; ++r) {
        void* base = nullptr;
        if (r == c->rank) {
            base = c->recv;
        } else if (cudaIpcOpenMemHandle(&base, handles[r], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            opened = false;
            base = nullptr;
        }
        c->peers.recv[r] = static_cast<uint64_t*>(base);
    }
    cudaGetLastError();
    if (lssm_status st = comm_agree(c, opened, &all)) return st;
    if (!all) {
        p2p_release(c);
        return LSSM_OK;
    }
    c->cap = cap;
    c->p2p = true;
    return LSSM_OK;
}

bool comm_p2p(const lssm_comm* c, size_t floats) { return c && c->p2p && floats <= c->cap; }

// Sum-all-reduce of n fp32 over the peer exchange. Residual form (hidden != nullptr):
// hidden[i] = half(hidden[i] + half(sum)); else out[i] = sum (out may alias part).
lssm_status comm_p2p_allreduce(lssm_comm* c, const float* part, size_t n, float* out, __half* hidden,
                               cudaStream_t s) {
    const cudaError_t e = launch_p2p_allreduce(c->peers, c->recv, c->epochs, c->rank, c->world, c->cap, part,
                                               (uint32_t)n, out, hidden, 2000000000ull, s);
    return e == cudaSuccess ? LSSM_OK : cuda_fail(e, "peer all-reduce");
}

int comm_rank(const lssm_comm* c) { return c ? c->rank : 0; }
int comm_world(const lssm_comm* c) { return c ? c->world : 1; }

}  // namespace lssm

using namespace lssm;

extern "C" lssm_status lssm_comm_unique_id(uint8_t* out) {
    if (!out) return fail(LSSM_ERR_INVALID_ARGUMENT, "lssm_comm_unique_id: null argument");
    NcclApi& api = nccl();
    if (!api.error.empty()) return fail(LSSM_ERR_NOT_FOUND, "lssm_comm_unique_id: %s", api.error.c_str());
    ncclUniqueId id;
    const ncclResult_t r = api.GetUniqueId(&id);
    if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
    static_assert(sizeof(ncclUniqueId) == LSSM_COMM_ID_BYTES, "NCCL unique id size");
    std::memcpy(out, &id, sizeof(id));
    return LSSM_OK;
}

extern "C" lssm_status lssm_comm_init(lssm_ctx* ctx, int rank, int world, const uint8_t* id, lssm_comm** out) {
    if (!ctx || !id || !out) return fail(LSSM_ERR_INVALID_ARGUMENT, "lssm_comm_init: null argument");
    if (world < 1 || rank < 0 || rank >= world)
        return fail(LSSM_ERR_INVALID_ARGUMENT, "lssm_comm_init: rank %d outside world %d", rank, world);
    *out = nullptr;
    auto* c = new lssm_comm();
    c->ctx = ctx;
    c->rank = rank;
    c->world = world;
    if (world > 1) {
        NcclApi& api = nccl();
        if (!api.error.empty()) {
            delete c;
            return fail(LSSM_ERR_NOT_FOUND, "lssm_comm_init: %s", api.error.c_str());
        }
        cudaSetDevice(ctx->device);
        ncclUniqueId uid;
        std::memcpy(&uid, id, sizeof(uid));
        const ncclResult_t r = api.CommInitRank(&c->comm, world, uid, rank);
        if (r != ncclSuccess) {
            delete c;
            return nccl_fail(r, "ncclCommInitRank");
        }
    }
    *out = c;
    return LSSM_OK;
}

extern "C" lssm_status lssm_comm_destroy(lssm_comm* c) {
    if (!c) return LSSM_OK;
    cudaSetDevice(c->ctx->device);
    cudaStreamSynchronize(c->ctx->stream);
    if (c->p2p) {
        // no rank may unmap or free while another still exchanges: agree first (collective)
        bool all = false;
        comm_agree(c, true, &all);
        p2p_release(c);
    }
    if (c->comm) nccl().CommDestroy(c->comm);
    delete c;
    return LSSM_OK;
}

// Sum-all-reduce of n fp32 in place across the ranks, on the context stream, then a
// synchronize (one-shot, like the ops outside a batch). Collective. Decode-sized buffers
// (n <= 65536) go over the peer exchange when every rank can use it, larger ones over NCCL.
extern "C" lssm_status lssm_comm_allreduce_f32(lssm_comm* c, float* buf, size_t n) {
    if (!c || (!buf && n)) return fail(LSSM_ERR_INVALID_ARGUMENT, "lssm_comm_allreduce_f32: null argument");
    cudaSetDevice(c->ctx->device);
    lssm_status st = LSSM_OK;
    if (n <= (size_t)1024 * P2P_BLOCKS && c->world > 1 && !(st = comm_p2p_setup(c, n)) && comm_p2p(c, n))
        st = comm_p2p_allreduce(c, buf, n, buf, nullptr, c->ctx->stream);
    else if (!st)
        st = comm_allreduce_f32(c, buf, n, c->ctx->stream);
    if (st) return st;
    const cudaError_t e = cudaStreamSynchronize(c->ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "lssm_comm_allreduce_f32");
    int* ew = tc_error_word();
    int h = 0;
    cudaMemcpy(&h, ew, sizeof(int), cudaMemcpyDeviceToHost);
    if (h) {
        cudaMemset(ew, 0, sizeof(int));
        return fail(LSSM_ERR_TIMEOUT, "lssm_comm_allreduce_f32: a bounded wait timed out");
    }
    return LSSM_OK;
}

extern "C" int lssm_comm_rank(const lssm_comm* c) { return comm_rank(c); }
extern "C" int lssm_comm_world(const lssm_comm* c) { return comm_world(c); }

// Bounded-wait check of the peer exchange on one GPU: the exchange kernel runs as rank 0 of
// 2 against local buffers only (its "peer" areas are this rank's own), so its wait for
// rank 1's flag can only run out. Returns LSSM_ERR_TIMEOUT when the kernel gave up and
// reported it, and leaves the context usable.
extern "C" lssm_status lssm_p2p_wait_selftest(lssm_ctx* ctx, uint64_t spin_ns) {
    if (!ctx) return fail(LSSM_ERR_INVALID_ARGUMENT, "lssm_p2p_wait_selftest: null context");
    cudaSetDevice(ctx->device);
    const size_t cap = 1024;
    uint64_t* words = nullptr;   // recv [2][2][cap]
    float* part = nullptr;       // part / out [cap]
    uint32_t* epochs = nullptr;
    if (cudaMalloc(&words, 4 * cap * sizeof(uint64_t)) != cudaSuccess || cudaMalloc(&part, cap * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&epochs, P2P_BLOCKS * sizeof(uint32_t)) != cudaSuccess) {
        if (words) cudaFree(words);
        if (part) cudaFree(part);
        return fail(LSSM_ERR_OUT_OF_MEMORY, "lssm_p2p_wait_selftest: buffers");
    }
    cudaMemset(words, 0, 4 * cap * sizeof(uint64_t));
    cudaMemset(part, 0, cap * sizeof(float));
    cudaMemset(epochs, 0, P2P_BLOCKS * sizeof(uint32_t));
    P2PPeers peers{};
    peers.recv[0] = peers.recv[1] = words;   // "rank 1" is this GPU's own area: nothing writes its words
    cudaError_t e = launch_p2p_allreduce(peers, words, epochs, 0, 2, cap, part, 1024, part, nullptr, spin_ns,
                                         ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    cudaFree(words);
    cudaFree(part);
    cudaFree(epochs);
    if (e != cudaSuccess) return cuda_fail(e, "lssm_p2p_wait_selftest");
    int* ew = tc_error_word();
    int h = 0;
    cudaMemcpy(&h, ew, sizeof(int), cudaMemcpyDeviceToHost);
    if (!h) return LSSM_OK;
    cudaMemset(ew, 0, sizeof(int));
    return fail(LSSM_ERR_TIMEOUT, "peer exchange: a bounded wait timed out");
}
