// Tensor-parallel communicator: NCCL over NVLink / NVSwitch, bound at run
// time (dlopen of libnccl.so.2), so the library loads and serves single-GPU
// work where NCCL is absent.  One communicator per rank (one process or host
// thread per GPU); the host distributes the unique id (ifr_comm_unique_id on
// rank 0) by any means it has, e.g. torch.distributed or Julia's Distributed.
//
// Used by the tensor-parallel model (config 5): an in-place sum all-reduce of
// the residual stream after the row-parallel projections, and an all-gather
// of per-rank argmax candidates of the vocab-parallel lm_head.
#include "../../include/inferno_b200.h"
#include "comm.h"

#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

int ifr_fail(int code, const char *fmt, ...);
int ifr_ctx_device(const ifr_ctx *c);

namespace {

struct NcclApi {
    void *lib = nullptr;
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char *(*err)(ncclResult_t) = nullptr;
    bool ok = false;
};

NcclApi &api() {
    static NcclApi a;
    static std::once_flag once;
    std::call_once(once, [] {
        const char *names[] = {"libnccl.so.2", "libnccl.so"};
        for (const char *n : names)
            if ((a.lib = dlopen(n, RTLD_NOW | RTLD_GLOBAL))) break;
        if (!a.lib) return;
        a.get_unique_id = (decltype(a.get_unique_id))dlsym(a.lib, "ncclGetUniqueId");
        a.init_rank = (decltype(a.init_rank))dlsym(a.lib, "ncclCommInitRank");
        a.destroy = (decltype(a.destroy))dlsym(a.lib, "ncclCommDestroy");
        a.all_reduce = (decltype(a.all_reduce))dlsym(a.lib, "ncclAllReduce");
        a.all_gather = (decltype(a.all_gather))dlsym(a.lib, "ncclAllGather");
        a.err = (decltype(a.err))dlsym(a.lib, "ncclGetErrorString");
        a.ok = a.get_unique_id && a.init_rank && a.destroy && a.all_reduce && a.all_gather && a.err;
    });
    return a;
}

int nccl_fail(ncclResult_t r, const char *what) {
    return ifr_fail(IFR_ERR_CUDA, "%s: %s", what, api().err ? api().err(r) : "NCCL error");
}

}  // namespace

struct ifr_comm {
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1, device = 0;
};

int comm_rank(const ifr_comm *c) { return c ? c->rank : 0; }
int comm_world(const ifr_comm *c) { return c ? c->world : 1; }

int comm_allreduce_sum(ifr_comm *c, float *buf, size_t n, cudaStream_t s) {
    if (!c || c->world == 1) return IFR_OK;
    ncclResult_t r = api().all_reduce(buf, buf, n, ncclFloat32, ncclSum, c->comm, s);
    return r == ncclSuccess ? IFR_OK : nccl_fail(r, "ncclAllReduce");
}

int comm_allgather_bytes(ifr_comm *c, const void *send, void *recv, size_t bytes, cudaStream_t s) {
    if (!c || c->world == 1) {
        if (send != recv && cudaMemcpyAsync(recv, send, bytes, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
            return ifr_fail(IFR_ERR_CUDA, "allgather copy");
        return IFR_OK;
    }
    ncclResult_t r = api().all_gather(send, recv, bytes, ncclUint8, c->comm, s);
    return r == ncclSuccess ? IFR_OK : nccl_fail(r, "ncclAllGather");
}

extern "C" {

int ifr_comm_available(void) { return api().ok ? 1 : 0; }

int ifr_comm_unique_id(uint8_t *out) {
    if (!out) return ifr_fail(IFR_ERR_ARG, "NULL argument");
    if (!api().ok) return ifr_fail(IFR_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) is not available");
    ncclUniqueId id;
    ncclResult_t r = api().get_unique_id(&id);
    if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
    memcpy(out, id.internal, IFR_COMM_ID_BYTES);
    return IFR_OK;
}

int ifr_comm_create(ifr_ctx *ctx, int rank, int world, const uint8_t *id, ifr_comm **out) {
    if (!ctx || !out || (world > 1 && !id)) return ifr_fail(IFR_ERR_ARG, "NULL argument");
    if (world < 1 || rank < 0 || rank >= world) return ifr_fail(IFR_ERR_ARG, "rank %d of world %d", rank, world);
    ifr_comm *c = new ifr_comm();
    c->rank = rank;
    c->world = world;
    c->device = ifr_ctx_device(ctx);
    if (world > 1) {
        if (!api().ok) {
            delete c;
            return ifr_fail(IFR_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) is not available");
        }
        ncclUniqueId uid;
        memcpy(uid.internal, id, IFR_COMM_ID_BYTES);
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(c->device);
        ncclResult_t r = api().init_rank(&c->comm, world, uid, rank);
        cudaSetDevice(prev);
        if (r != ncclSuccess) {
            delete c;
            return nccl_fail(r, "ncclCommInitRank");
        }
    }
    *out = c;
    return IFR_OK;
}

int ifr_comm_destroy(ifr_comm *c) {
    if (!c) return IFR_OK;
    if (c->comm) api().destroy(c->comm);
    delete c;
    return IFR_OK;
}

}  // extern "C"
