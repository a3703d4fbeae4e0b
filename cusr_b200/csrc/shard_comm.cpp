// shard_comm.cpp — dlopen'ed NCCL, non-blocking communicator with deadlines (see shard_comm.h).
#include "shard_comm.h"

#include <dlfcn.h>

#include <chrono>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <thread>

#include "../../include/cusr_co.h"

namespace cusr {
namespace {

struct NcclApi {
    bool ok = false;
    ncclResult_t (*getUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*commInitRankConfig)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *) = nullptr;
    ncclResult_t (*allReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*commGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
    ncclResult_t (*commAbort)(ncclComm_t) = nullptr;
    const char *(*getErrorString)(ncclResult_t) = nullptr;
};

NcclApi &api() {
    static NcclApi a;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            fprintf(stderr, "[cusr_b200] sample-sharded mode needs NCCL: %s\n", dlerror());
            return;
        }
#define CUSR_SYM(field, name) a.field = reinterpret_cast<decltype(a.field)>(dlsym(h, name))
        CUSR_SYM(getUniqueId, "ncclGetUniqueId");
        CUSR_SYM(commInitRankConfig, "ncclCommInitRankConfig");
        CUSR_SYM(allReduce, "ncclAllReduce");
        CUSR_SYM(commGetAsyncError, "ncclCommGetAsyncError");
        CUSR_SYM(commAbort, "ncclCommAbort");
        CUSR_SYM(getErrorString, "ncclGetErrorString");
#undef CUSR_SYM
        a.ok = a.getUniqueId && a.commInitRankConfig && a.allReduce && a.commGetAsyncError &&
               a.commAbort && a.getErrorString;
        if (!a.ok) fprintf(stderr, "[cusr_b200] libnccl lacks a required symbol\n");
    });
    return a;
}

double now_s() {
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

int fail(ShardComm &sc, const char *what, ncclResult_t r) {
    NcclApi &a = api();
    fprintf(stderr, "[cusr_b200] rank %d: %s: %s\n", sc.rank, what,
            a.getErrorString ? a.getErrorString(r) : "nccl error");
    if (sc.comm && a.commAbort) a.commAbort(sc.comm);
    sc.comm = nullptr;
    sc.failed = true;
    return CO_ERR_CUDA;
}

// Poll a non-blocking communicator until its last operation left the in-progress state.
int settle(ShardComm &sc, const char *what) {
    NcclApi &a = api();
    const double t0 = now_s();
    for (;;) {
        ncclResult_t st = ncclSuccess;
        ncclResult_t r = a.commGetAsyncError(sc.comm, &st);
        if (r != ncclSuccess) return fail(sc, what, r);
        if (st == ncclSuccess) return CO_OK;
        if (st != ncclInProgress) return fail(sc, what, st);
        if (now_s() - t0 > sc.timeout_s) {
            fprintf(stderr, "[cusr_b200] rank %d: %s timed out after %.0f s\n", sc.rank, what,
                    sc.timeout_s);
            return fail(sc, what, ncclInProgress);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

}  // namespace

int shard_unique_id(unsigned char out[NCCL_UNIQUE_ID_BYTES]) {
    NcclApi &a = api();
    if (!a.ok) return CO_ERR_CUDA;
    ncclUniqueId id;
    if (a.getUniqueId(&id) != ncclSuccess) return CO_ERR_CUDA;
    std::memcpy(out, id.internal, NCCL_UNIQUE_ID_BYTES);
    return CO_OK;
}

int shard_init(ShardComm &sc, const unsigned char id[NCCL_UNIQUE_ID_BYTES], int nranks, int rank,
               double timeout_s) {
    NcclApi &a = api();
    if (!a.ok) return CO_ERR_CUDA;
    if (nranks < 1 || rank < 0 || rank >= nranks) return CO_ERR_NULLARG;
    shard_destroy(sc);
    sc.nranks = nranks;
    sc.rank = rank;
    sc.timeout_s = timeout_s > 0 ? timeout_s : 120.0;
    sc.failed = false;
    ncclUniqueId uid;
    std::memcpy(uid.internal, id, NCCL_UNIQUE_ID_BYTES);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclResult_t r = a.commInitRankConfig(&sc.comm, nranks, uid, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) return fail(sc, "ncclCommInitRankConfig", r);
    return settle(sc, "communicator init");
}

int shard_allreduce(ShardComm &sc, void *buf, size_t count, bool fp64, cudaStream_t stream) {
    NcclApi &a = api();
    if (!sc.comm) return CO_ERR_CUDA;
    ncclResult_t r = a.allReduce(buf, buf, count, fp64 ? ncclFloat64 : ncclFloat32, ncclSum,
                                 sc.comm, stream);
    if (r != ncclSuccess && r != ncclInProgress) return fail(sc, "ncclAllReduce", r);
    return settle(sc, "all-reduce enqueue");
}

int shard_wait_event(ShardComm &sc, cudaEvent_t ev) {
    NcclApi &a = api();
    const double t0 = now_s();
    for (;;) {
        cudaError_t e = cudaEventQuery(ev);
        if (e == cudaSuccess) return CO_OK;
        if (e != cudaErrorNotReady) {
            fprintf(stderr, "[cusr_b200] rank %d: %s\n", sc.rank, cudaGetErrorString(e));
            return CO_ERR_CUDA;
        }
        if (sc.comm) {
            ncclResult_t st = ncclSuccess;
            if (a.commGetAsyncError(sc.comm, &st) != ncclSuccess ||
                (st != ncclSuccess && st != ncclInProgress))
                return fail(sc, "all-reduce", st);
        }
        if (now_s() - t0 > sc.timeout_s) {
            fprintf(stderr, "[cusr_b200] rank %d: waiting for peers timed out after %.0f s\n",
                    sc.rank, sc.timeout_s);
            return fail(sc, "peer wait", ncclInProgress);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

// Teardown aborts rather than destroys: abort is local (no exchange with peers that may already
// be gone) and every operation of this module has completed by the time a call returns.
void shard_destroy(ShardComm &sc) {
    NcclApi &a = api();
    if (sc.comm && a.ok) a.commAbort(sc.comm);
    sc.comm = nullptr;
}

}  // namespace cusr
