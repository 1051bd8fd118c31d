// NCCL communicator for data parallelism.  rtensor has no data-parallel mode
// (crates/rtensor/README.md:123 lists it as absent); this is the new exchange
// step of the B200 design: every rank holds a full replica, takes its slice of
// the global batch, and dW/db are summed over ranks with ncclAllReduce before
// the identical optimiser step runs everywhere.
//
// NCCL is resolved at run time (dlopen) instead of at link time: a process
// that already holds a libnccl.so.2 (PyTorch ships its own) keeps using that
// one, and processes that never form a communicator never load NCCL at all.
// RT_NCCL_LIB overrides the library path.
#include <dlfcn.h>
#include <nccl.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "internal.h"

namespace {

struct NcclApi {
    bool loaded = false;
    std::string error;
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*ReduceScatter)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                                  cudaStream_t) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
    // optional (NCCL >= 2.18): a second communicator over the same ranks
    ncclResult_t (*CommSplit)(ncclComm_t, int, int, ncclComm_t*, ncclConfig_t*) = nullptr;
};

NcclApi& nccl_api() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        const char* env = getenv("RT_NCCL_LIB");
        void* h = nullptr;
        if (env && *env) h = dlopen(env, RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            api.error = std::string("cannot load libnccl.so.2: ") + dlerror();
            return;
        }
        api.GetUniqueId = (decltype(api.GetUniqueId))dlsym(h, "ncclGetUniqueId");
        api.CommInitRank = (decltype(api.CommInitRank))dlsym(h, "ncclCommInitRank");
        api.CommDestroy = (decltype(api.CommDestroy))dlsym(h, "ncclCommDestroy");
        api.AllReduce = (decltype(api.AllReduce))dlsym(h, "ncclAllReduce");
        api.ReduceScatter = (decltype(api.ReduceScatter))dlsym(h, "ncclReduceScatter");
        api.AllGather = (decltype(api.AllGather))dlsym(h, "ncclAllGather");
        api.GetErrorString = (decltype(api.GetErrorString))dlsym(h, "ncclGetErrorString");
        api.CommSplit = (decltype(api.CommSplit))dlsym(h, "ncclCommSplit");
        if (!api.GetUniqueId || !api.CommInitRank || !api.CommDestroy || !api.AllReduce || !api.ReduceScatter ||
            !api.AllGather || !api.GetErrorString) {
            api.error = "libnccl.so.2 lacks a required symbol";
            return;
        }
        api.loaded = true;
    });
    return api;
}

int need_nccl() {
    NcclApi& a = nccl_api();
    if (!a.loaded) return rt::fail(RT_ERR_NCCL, "%s", a.error.c_str());
    return RT_OK;
}

}  // namespace

struct rt_comm {
    rt_ctx* ctx = nullptr;
    ncclComm_t nccl = nullptr;
    ncclComm_t nccl2 = nullptr;  // second communicator (comm_open_second), its own queue of collectives
    int rank = 0, world = 1;
    // device staging for the IPC handles comm_share_buffer all-gathers
    // (allocated with the communicator, so that call allocates nothing
    // before its collective)
    uint8_t* handles = nullptr;
};

namespace rt {

int comm_allreduce(rt_comm* comm, float* buf, int64_t count, cudaStream_t st) {
    if (!comm || count == 0) return RT_OK;
    NcclApi& A = nccl_api();
    ncclResult_t r = A.AllReduce(buf, buf, (size_t)count, ncclFloat32, ncclSum, comm->nccl, st);
    if (r != ncclSuccess) return fail(RT_ERR_NCCL, "ncclAllReduce failed: %s", A.GetErrorString(r));
    return RT_OK;
}

int comm_rank(const rt_comm* comm) { return comm ? comm->rank : 0; }

// Opens the second communicator over the same ranks (ncclCommSplit, one
// color): collectives issued on it queue separately from the first's, so the
// sharded optimiser's weight all-gathers do not wait behind gradient
// reduce-scatters or hold them up.  Collective: every rank calls it.  Returns
// false (and the caller keeps one queue) when NCCL has no ncclCommSplit.
bool comm_open_second(rt_comm* comm, int* status) {
    *status = RT_OK;
    if (!comm) return false;
    if (comm->nccl2) return true;
    NcclApi& A = nccl_api();
    if (!A.CommSplit) return false;
    ncclResult_t r = A.CommSplit(comm->nccl, 0, comm->rank, &comm->nccl2, nullptr);
    if (r != ncclSuccess) {
        comm->nccl2 = nullptr;
        *status = fail(RT_ERR_NCCL, "ncclCommSplit failed: %s", A.GetErrorString(r));
        return false;
    }
    return true;
}
int comm_world(const rt_comm* comm) { return comm ? comm->world : 1; }

// In place: buf holds world * count elements; rank r's slice
// [r * count, (r + 1) * count) receives the sum of that slice over the ranks.
int comm_reduce_scatter(rt_comm* comm, float* buf, int64_t count, cudaStream_t st) {
    if (!comm || count == 0) return RT_OK;
    NcclApi& A = nccl_api();
    ncclResult_t r = A.ReduceScatter(buf, buf + (int64_t)comm->rank * count, (size_t)count, ncclFloat32, ncclSum,
                                     comm->nccl, st);
    if (r != ncclSuccess) return fail(RT_ERR_NCCL, "ncclReduceScatter failed: %s", A.GetErrorString(r));
    return RT_OK;
}

// In place: rank r's slice [r * count, (r + 1) * count) of buf is copied to
// the same slice of every rank's buf (elem_bytes 2 for bf16, 4 for f32).
int comm_all_gather(rt_comm* comm, void* buf, int64_t count, int elem_bytes, cudaStream_t st, bool second) {
    if (!comm || count == 0) return RT_OK;
    NcclApi& A = nccl_api();
    char* b = static_cast<char*>(buf);
    ncclComm_t nc = second && comm->nccl2 ? comm->nccl2 : comm->nccl;
    ncclResult_t r = A.AllGather(b + (int64_t)comm->rank * count * elem_bytes, b, (size_t)count,
                                 elem_bytes == 2 ? ncclBfloat16 : ncclFloat32, nc, st);
    if (r != ncclSuccess) return fail(RT_ERR_NCCL, "ncclAllGather failed: %s", A.GetErrorString(r));
    return RT_OK;
}

int comm_allreduce_bf16(rt_comm* comm, __nv_bfloat16* buf, int64_t count, cudaStream_t st) {
    if (!comm || count == 0) return RT_OK;
    NcclApi& A = nccl_api();
    ncclResult_t r = A.AllReduce(buf, buf, (size_t)count, ncclBfloat16, ncclSum, comm->nccl, st);
    if (r != ncclSuccess) return fail(RT_ERR_NCCL, "ncclAllReduce (bf16) failed: %s", A.GetErrorString(r));
    return RT_OK;
}

// Maps a local device allocation (the base of a cudaMalloc block) of every
// rank into this process: peers[q] = rank q's block (peers[rank] = local).
// The CUDA IPC handles travel by an in-place ncclAllGather.  Collective.
// Fails (RT_ERR_UNSUPPORTED) when a peer's block cannot be mapped; the
// caller then keeps NCCL for that exchange.
int comm_share_buffer(rt_comm* comm, void* local, void** peers) {
    RT_CHECK(comm && local && peers && comm->world <= kMaxPeers, "comm_share_buffer: bad arguments");
    NcclApi& A = nccl_api();
    cudaStream_t st = comm->ctx->stream;
    const int W = comm->world;
    // Every rank reaches the all-gather whatever happens before it, so that
    // a local failure cannot leave the other ranks waiting in the collective.
    cudaIpcMemHandle_t mine;
    std::memset(&mine, 0, sizeof(mine));
    int rc = RT_OK;
    if (cudaIpcGetMemHandle(&mine, local) != cudaSuccess) rc = fail(RT_ERR_UNSUPPORTED, "cudaIpcGetMemHandle failed");
    uint8_t* dev = comm->handles;
    std::vector<cudaIpcMemHandle_t> all(W);
    if (cudaMemcpyAsync(dev + sizeof(mine) * comm->rank, &mine, sizeof(mine), cudaMemcpyHostToDevice, st) !=
        cudaSuccess && rc == RT_OK)
        rc = fail(RT_ERR_CUDA, "comm_share_buffer: handle upload failed");
    ncclResult_t r = A.AllGather(dev + sizeof(mine) * comm->rank, dev, sizeof(mine), ncclUint8, comm->nccl, st);
    if (r != ncclSuccess && rc == RT_OK) rc = fail(RT_ERR_NCCL, "ncclAllGather (IPC handles) failed: %s", A.GetErrorString(r));
    if ((cudaMemcpyAsync(all.data(), dev, sizeof(mine) * W, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
         cudaStreamSynchronize(st) != cudaSuccess) && rc == RT_OK)
        rc = fail(RT_ERR_CUDA, "comm_share_buffer: handle download failed");
    RT_TRY(rc);
    for (int q = 0; q < W; ++q) peers[q] = nullptr;
    peers[comm->rank] = local;
    for (int q = 0; q < W; ++q) {
        if (q == comm->rank) continue;
        cudaError_t e = cudaIpcOpenMemHandle(&peers[q], all[q], cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            peers[q] = nullptr;
            comm_unshare_buffer(comm, peers);
            return fail(RT_ERR_UNSUPPORTED, "cannot map rank %d's buffer: %s", q, cudaGetErrorString(e));
        }
    }
    return RT_OK;
}

// Closes the mappings comm_share_buffer opened (not the local block).
void comm_unshare_buffer(rt_comm* comm, void** peers) {
    if (!comm || !peers) return;
    for (int q = 0; q < comm->world; ++q)
        if (q != comm->rank && peers[q]) {
            cudaIpcCloseMemHandle(peers[q]);
            peers[q] = nullptr;
        }
}

// True on every rank when `mine` is true on every rank (an in-place
// ncclAllReduce(min) of one int on `scratch`, synchronised).  Collective.
bool comm_all_true(rt_comm* comm, bool mine, float* scratch, int* status) {
    *status = RT_OK;
    NcclApi& A = nccl_api();
    cudaStream_t st = comm->ctx->stream;
    int v = mine ? 1 : 0;
    int* dv = reinterpret_cast<int*>(scratch);
    if (cudaMemcpyAsync(dv, &v, sizeof(v), cudaMemcpyHostToDevice, st) != cudaSuccess) {
        *status = fail(RT_ERR_CUDA, "comm_all_true: upload failed");
        v = 0;
    }
    ncclResult_t r = A.AllReduce(dv, dv, 1, ncclInt32, ncclMin, comm->nccl, st);
    if (r != ncclSuccess) {
        *status = fail(RT_ERR_NCCL, "ncclAllReduce (agreement) failed: %s", A.GetErrorString(r));
        return false;
    }
    if (cudaMemcpyAsync(&v, dv, sizeof(v), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess) {
        *status = fail(RT_ERR_CUDA, "comm_all_true: download failed");
        return false;
    }
    return v == 1;
}

// A barrier in stream order: a one-float ncclAllReduce on `scratch`.  Work
// enqueued on `st` after it runs once every rank has reached it, so device
// writes that each rank finished before its barrier (peer-memory stores and
// copies included) are in place.  `second` issues it on the second
// communicator (its own queue of collectives).
int comm_barrier(rt_comm* comm, float* scratch, cudaStream_t st, bool second) {
    NcclApi& A = nccl_api();
    ncclComm_t nc = second && comm->nccl2 ? comm->nccl2 : comm->nccl;
    ncclResult_t r = A.AllReduce(scratch, scratch, 1, ncclFloat32, ncclSum, nc, st);
    if (r != ncclSuccess) return fail(RT_ERR_NCCL, "ncclAllReduce (barrier) failed: %s", A.GetErrorString(r));
    return RT_OK;
}

}  // namespace rt

using namespace rt;

extern "C" {

int rt_comm_unique_id(unsigned char id[128]) {
    RT_CHECK(id, "id buffer is NULL");
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
    RT_TRY(need_nccl());
    NcclApi& A = nccl_api();
    ncclUniqueId u;
    ncclResult_t r = A.GetUniqueId(&u);
    if (r != ncclSuccess) return fail(RT_ERR_NCCL, "ncclGetUniqueId failed: %s", A.GetErrorString(r));
    memcpy(id, &u, 128);
    return RT_OK;
}

int rt_comm_init(rt_ctx* ctx, int rank, int world, const unsigned char id[128], rt_comm** out) {
    RT_CHECK(ctx && id && out, "rt_comm_init: bad arguments");
    RT_CHECK(world >= 1 && rank >= 0 && rank < world, "rt_comm_init: rank %d / world %d", rank, world);
    RT_TRY(need_nccl());
    NcclApi& A = nccl_api();
    RT_CUDA(cudaSetDevice(ctx->device));
    ncclUniqueId u;
    memcpy(&u, id, 128);
    rt_comm* c = new rt_comm;
    c->ctx = ctx;
    c->rank = rank;
    c->world = world;
    if (cudaMalloc(&c->handles, sizeof(cudaIpcMemHandle_t) * (size_t)world) != cudaSuccess) {
        delete c;
        return fail(RT_ERR_OOM, "rt_comm_init: handle staging allocation failed");
    }
    ncclResult_t r = A.CommInitRank(&c->nccl, world, u, rank);
    if (r != ncclSuccess) {
        cudaFree(c->handles);
        delete c;
        return fail(RT_ERR_NCCL, "ncclCommInitRank(rank %d of %d) failed: %s", rank, world, A.GetErrorString(r));
    }
    *out = c;
    return RT_OK;
}

int rt_comm_destroy(rt_comm* c) {
    if (!c) return RT_OK;
    if (c->nccl2) nccl_api().CommDestroy(c->nccl2);
    if (c->nccl) nccl_api().CommDestroy(c->nccl);
    if (c->handles) cudaFree(c->handles);
    delete c;
    return RT_OK;
}

int rt_comm_allreduce_f32(rt_comm* c, float* buf, int64_t count) {
    RT_CHECK(c && buf && count >= 0, "rt_comm_allreduce_f32: bad arguments");
    return comm_allreduce(c, buf, count, c->ctx->stream);
}

}  // extern "C"
