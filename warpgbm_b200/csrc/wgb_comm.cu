// Native tree loop and its NCCL communicator (sm_100a library, host code).
//
// wgb_grow_tree runs the whole per-tree sequence of the level-wise engine
// -- residuals, quantisation, and per level the histogram build, its
// reduction over ranks, the split search and the partition -- as stream
// work issued from C++, so no Python runs inside a tree.  For a row-sharded
// fit it sums the per-level histograms with its own NCCL communicator
// (ncclAllReduce on the engine's stream; int64 SUM, so the reduction order
// is irrelevant and every rank picks the same splits).
//
// NCCL is not linked: the library resolves the few entry points it needs
// with dlsym from the libnccl.so.2 that the process has already loaded
// (torch's), so it shares that library instance instead of bringing its own.
#include <dlfcn.h>

#include <cstring>

#include "wgb_common.cuh"

namespace wgb {

// NCCL's C interface, as far as used here (nccl.h: ncclUniqueId is 128
// bytes passed by value; ncclInt64 = 4, ncclFloat32 = 7; ncclSum = 0,
// ncclMax = 2; ncclSuccess = 0).
struct NcclUid {
    char internal[128];
};
using nccl_get_uid_t = int (*)(NcclUid *);
using nccl_init_rank_t = int (*)(void **, int, NcclUid, int);
using nccl_all_reduce_t = int (*)(const void *, void *, size_t, int, int, void *, cudaStream_t);
using nccl_reduce_scatter_t = int (*)(const void *, void *, size_t, int, int, void *, cudaStream_t);
using nccl_all_gather_t = int (*)(const void *, void *, size_t, int, void *, cudaStream_t);
using nccl_destroy_t = int (*)(void *);
using nccl_err_t = const char *(*)(int);
constexpr int NCCL_INT32 = 2, NCCL_INT64 = 4, NCCL_FLOAT32 = 7, NCCL_SUM = 0, NCCL_MAX = 2;

struct NcclApi {
    bool ok = false;
    nccl_get_uid_t get_uid = nullptr;
    nccl_init_rank_t init_rank = nullptr;
    nccl_all_reduce_t all_reduce = nullptr;
    nccl_reduce_scatter_t reduce_scatter = nullptr;
    nccl_all_gather_t all_gather = nullptr;
    nccl_destroy_t destroy = nullptr;
    nccl_err_t err = nullptr;
};

static NcclApi &nccl() {
    static NcclApi api = [] {
        NcclApi a;
        // the instance already in the process (torch's), else the soname
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return a;
        a.get_uid = reinterpret_cast<nccl_get_uid_t>(dlsym(h, "ncclGetUniqueId"));
        a.init_rank = reinterpret_cast<nccl_init_rank_t>(dlsym(h, "ncclCommInitRank"));
        a.all_reduce = reinterpret_cast<nccl_all_reduce_t>(dlsym(h, "ncclAllReduce"));
        a.reduce_scatter = reinterpret_cast<nccl_reduce_scatter_t>(dlsym(h, "ncclReduceScatter"));
        a.all_gather = reinterpret_cast<nccl_all_gather_t>(dlsym(h, "ncclAllGather"));
        a.destroy = reinterpret_cast<nccl_destroy_t>(dlsym(h, "ncclCommDestroy"));
        a.err = reinterpret_cast<nccl_err_t>(dlsym(h, "ncclGetErrorString"));
        a.ok = a.get_uid && a.init_rank && a.all_reduce && a.reduce_scatter && a.all_gather && a.destroy && a.err;
        return a;
    }();
    return api;
}

}  // namespace wgb

struct wgb_comm {
    void *nccl_comm;
    int rank, world;
};

using namespace wgb;

#define WGB_NCCL(call)                                                                    \
    do {                                                                                  \
        const int r_ = (call);                                                            \
        if (r_ != 0) {                                                                    \
            set_error("%s failed: %s", #call, nccl().err ? nccl().err(r_) : "NCCL error"); \
            return WGB_ERR_CUDA;                                                          \
        }                                                                                 \
    } while (0)

extern "C" {

int wgb_comm_unique_id(uint8_t *id) {
    WGB_CHECK_ARG(id != nullptr, "id is NULL");
    WGB_CHECK_ARG(nccl().ok, "libnccl.so.2 is not loaded in this process (import torch first)");
    NcclUid u;
    WGB_NCCL(nccl().get_uid(&u));
    std::memcpy(id, u.internal, sizeof(u.internal));
    return WGB_OK;
}

int wgb_comm_init(int32_t rank, int32_t world, const uint8_t *id, wgb_comm **out) {
    WGB_CHECK_ARG(out != nullptr && id != nullptr, "NULL argument");
    WGB_CHECK_ARG(world >= 1 && rank >= 0 && rank < world, "rank %d / world %d out of range", rank, world);
    WGB_CHECK_ARG(nccl().ok, "libnccl.so.2 is not loaded in this process (import torch first)");
    NcclUid u;
    std::memcpy(u.internal, id, sizeof(u.internal));
    void *c = nullptr;
    WGB_NCCL(nccl().init_rank(&c, world, u, rank));
    *out = new wgb_comm{c, rank, world};
    return WGB_OK;
}

int wgb_comm_destroy(wgb_comm *comm) {
    if (!comm) return WGB_OK;
    const int r = nccl().destroy(comm->nccl_comm);
    delete comm;
    if (r != 0) {
        set_error("ncclCommDestroy failed: %s", nccl().err(r));
        return WGB_ERR_CUDA;
    }
    return WGB_OK;
}

int wgb_comm_allreduce(wgb_comm *comm, void *buf, int64_t count, int32_t kind, void *stream) {
    WGB_CHECK_ARG(comm != nullptr && (buf != nullptr || count == 0) && count >= 0, "bad all-reduce arguments");
    WGB_CHECK_ARG(kind == 0 || kind == 1, "kind: 0 = int64 sum, 1 = float32 max");
    if (count == 0 || comm->world == 1) return WGB_OK;
    WGB_NCCL(nccl().all_reduce(buf, buf, (size_t)count, kind == 0 ? NCCL_INT64 : NCCL_FLOAT32,
                               kind == 0 ? NCCL_SUM : NCCL_MAX, comm->nccl_comm, as_stream(stream)));
    return WGB_OK;
}

int wgb_comm_reduce_scatter(wgb_comm *comm, const int64_t *send, int64_t *recv, int64_t recvcount, void *stream) {
    WGB_CHECK_ARG(comm != nullptr && send != nullptr && recv != nullptr && recvcount >= 0,
                  "bad reduce-scatter arguments");
    if (recvcount == 0) return WGB_OK;
    if (comm->world == 1) {
        WGB_CUDA(cudaMemcpyAsync(recv, send, sizeof(int64_t) * recvcount, cudaMemcpyDeviceToDevice,
                                 as_stream(stream)));
        return WGB_OK;
    }
    WGB_NCCL(nccl().reduce_scatter(send, recv, (size_t)recvcount, NCCL_INT64, NCCL_SUM, comm->nccl_comm,
                                   as_stream(stream)));
    return WGB_OK;
}

int wgb_comm_allgather_i32(wgb_comm *comm, int32_t *buf, int64_t count, void *stream) {
    WGB_CHECK_ARG(comm != nullptr && (buf != nullptr || count == 0) && count >= 0, "bad all-gather arguments");
    if (count == 0 || comm->world == 1) return WGB_OK;
    WGB_NCCL(nccl().all_gather(buf + (long long)comm->rank * count, buf, (size_t)count, NCCL_INT32,
                               comm->nccl_comm, as_stream(stream)));
    return WGB_OK;
}

int wgb_grow_tree(const wgb_ws *ws, wgb_comm *comm, void *stream) {
    int rc;
#define WGB_STEP(expr)      \
    if ((rc = (expr)) != 0) \
    return rc
    WGB_STEP(wgb_tree_reset(ws, stream));
    WGB_STEP(wgb_tree_residual(ws, stream));
    const int nt = ws->ntree > 1 ? ws->ntree : 1;
    if (comm) WGB_STEP(wgb_comm_allreduce(comm, ws->maxabs, nt, 1, stream));
    WGB_STEP(wgb_tree_quantize(ws, stream));
    WGB_STEP(wgb_tree_subset(ws, stream));
    WGB_STEP(wgb_tree_root(ws, stream));
    const bool sliced = ws->nslice > 1;
    WGB_CHECK_ARG(!sliced || (comm && comm->world == ws->nslice && comm->rank == ws->slice),
                  "a feature-sliced fit needs the communicator of its nslice ranks");
    // slot size of the pool (ks positions per slot when sliced)
    const long long P = 2ll * ws->E * (sliced ? ws->ks : ws->k) * (ws->B + 1) + 2;
    for (int d = 0; d < ws->D; ++d) {
        WGB_STEP(wgb_level_hist(ws, d, stream));
        int first, count;
        wgb_level_slots(ws, d, &first, &count);
        if (sliced) {
            // every rank gets the global sums of its slice of the level's slots
            WGB_STEP(wgb_comm_reduce_scatter(comm, ws->hstage, ws->hg + (long long)first * P, (long long)count * P,
                                             stream));
        } else if (comm) {
            WGB_STEP(wgb_comm_allreduce(comm, ws->hg + (long long)first * P, (long long)count * P, 0, stream));
        }
        WGB_STEP(wgb_level_split(ws, d, stream));
        if (sliced) {
            // every rank's best split per node, then the same choice on all ranks
            WGB_STEP(wgb_comm_allgather_i32(comm, ws->win, (long long)(nt << d) * ws->win_words, stream));
            WGB_STEP(wgb_level_pick(ws, d, stream));
        }
        WGB_STEP(wgb_level_partition(ws, d, stream));
    }
    WGB_STEP(wgb_tree_finish(ws, stream));
#undef WGB_STEP
    return WGB_OK;
}

}  // extern "C"
