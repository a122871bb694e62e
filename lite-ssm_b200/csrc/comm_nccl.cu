// comm_nccl.cu — NCCL communicator for the head-tensor-parallel path (one rank per GPU,
// NVLink / NVSwitch). NCCL is opened at run time (dlopen "libnccl.so.2"): a process that
// already loaded NCCL (torch.distributed) shares that copy, otherwise the system library
// is used, and the kernel library itself keeps no link-time NCCL dependency.
//
// The unique id is made on one rank (lssm_comm_unique_id) and handed to the others by
// the caller (torch.distributed broadcast, a file, ...). Collectives run on the
// context's stream, so they order with the engine's kernels and can be captured in the
// decode CUDA graph.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "lssm_internal.h"

struct lssm_comm {
    lssm_ctx* ctx = nullptr;
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1;
};

namespace lssm {

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
    if (c->comm) nccl().CommDestroy(c->comm);
    delete c;
    return LSSM_OK;
}

extern "C" int lssm_comm_rank(const lssm_comm* c) { return comm_rank(c); }
extern "C" int lssm_comm_world(const lssm_comm* c) { return comm_world(c); }
