// nccl.cu -- the one collective of the multi-GPU path: a one-time broadcast
// of the fp32 weight slab from rank 0 over NVLink (NCCL). NCCL is opened at
// run time so that single-GPU users never need it.
//
// The communicator is created non-blocking and every wait on it is bounded
// (TCG_NCCL_TIMEOUT seconds, default 300): a rank that never joins makes the
// others return an error from tcg_vit_upload_bcast, after ncclCommAbort, in
// place of hanging in ncclCommInitRank.
#include "tcg_common.cuh"
#include "tcg_internal.h"

#include <dlfcn.h>
#include <nccl.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <unistd.h>

namespace tcg {
namespace {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId *);
    ncclResult_t (*comm_init_rank_config)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *);
    ncclResult_t (*broadcast)(const void *, void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*get_async_error)(ncclComm_t, ncclResult_t *);
    ncclResult_t (*comm_abort)(ncclComm_t);
    ncclResult_t (*comm_finalize)(ncclComm_t);
    ncclResult_t (*comm_destroy)(ncclComm_t);
    const char *(*error_string)(ncclResult_t);
    bool ok;
};

NcclApi *nccl()
{
    static NcclApi api;
    static bool tried = false;
    if (tried) return api.ok ? &api : nullptr;
    tried = true;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return nullptr;
    api.get_unique_id = (decltype(api.get_unique_id))dlsym(h, "ncclGetUniqueId");
    api.comm_init_rank_config = (decltype(api.comm_init_rank_config))dlsym(h, "ncclCommInitRankConfig");
    api.broadcast = (decltype(api.broadcast))dlsym(h, "ncclBroadcast");
    api.get_async_error = (decltype(api.get_async_error))dlsym(h, "ncclCommGetAsyncError");
    api.comm_abort = (decltype(api.comm_abort))dlsym(h, "ncclCommAbort");
    api.comm_finalize = (decltype(api.comm_finalize))dlsym(h, "ncclCommFinalize");
    api.comm_destroy = (decltype(api.comm_destroy))dlsym(h, "ncclCommDestroy");
    api.error_string = (decltype(api.error_string))dlsym(h, "ncclGetErrorString");
    api.ok = api.get_unique_id && api.comm_init_rank_config && api.broadcast && api.get_async_error &&
             api.comm_abort && api.comm_finalize && api.comm_destroy && api.error_string;
    return api.ok ? &api : nullptr;
}

double now_s()
{
    timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return (double)t.tv_sec + 1e-9 * (double)t.tv_nsec;
}

double timeout_s()
{
    const char *e = getenv("TCG_NCCL_TIMEOUT");
    const double v = e ? atof(e) : 0.0;
    return v > 0.0 ? v : 300.0;
}

// Polls a non-blocking communicator until its pending operation finishes.
bool settle(NcclApi *api, ncclComm_t comm, double deadline, const char *what)
{
    for (;;) {
        ncclResult_t st = ncclSuccess;
        const ncclResult_t r = api->get_async_error(comm, &st);
        if (r != ncclSuccess) return fail("%s: ncclCommGetAsyncError: %s", what, api->error_string(r));
        if (st == ncclSuccess) return true;
        if (st != ncclInProgress) return fail("%s: %s", what, api->error_string(st));
        if (now_s() > deadline) return fail("%s: the other ranks did not answer within %.0f s", what, timeout_s());
        usleep(500);
    }
}

}  // namespace

bool broadcast_once(void *buf, size_t count_floats, int rank, int nranks, const unsigned char id[128], void *buf2,
                    size_t count2)
{
    NcclApi *api = nccl();
    if (!api) return fail("NCCL (libnccl.so.2) is not available");
    if (nranks < 1 || rank < 0 || rank >= nranks) return fail("bad rank %d of %d", rank, nranks);
    if (nranks == 1) return true;
    const double deadline = now_s() + timeout_s();
    ncclUniqueId uid;
    memcpy(uid.internal, id, sizeof uid.internal);
    ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
    config.blocking = 0;
    ncclComm_t comm = nullptr;
    ncclResult_t r = api->comm_init_rank_config(&comm, nranks, uid, rank, &config);
    if (r != ncclSuccess && r != ncclInProgress)
        return fail("ncclCommInitRankConfig(rank %d of %d): %s", rank, nranks, api->error_string(r));
    bool ok = settle(api, comm, deadline, "ncclCommInitRank");
    if (ok) {
        r = api->broadcast(buf, buf, count_floats, ncclFloat32, 0, comm, ctx().cur);
        ok = (r == ncclSuccess || r == ncclInProgress) ? settle(api, comm, deadline, "ncclBroadcast")
                                                       : fail("ncclBroadcast: %s", api->error_string(r));
    }
    if (ok && buf2 && count2) {   // a second buffer over the same communicator, in stream order
        r = api->broadcast(buf2, buf2, count2, ncclFloat32, 0, comm, ctx().cur);
        ok = (r == ncclSuccess || r == ncclInProgress) ? settle(api, comm, deadline, "ncclBroadcast")
                                                       : fail("ncclBroadcast: %s", api->error_string(r));
    }
    // the broadcast is enqueued on this thread's stream; wait for it with the same bound
    cudaError_t ce = cudaSuccess;
    while (ok) {
        ce = cudaStreamQuery(ctx().cur);
        if (ce != cudaErrorNotReady) break;
        if (now_s() > deadline) {
            ok = fail("ncclBroadcast: not complete within %.0f s", timeout_s());
            break;
        }
        usleep(200);
    }
    if (ok && ce != cudaSuccess) ok = fail("ncclBroadcast: %s", cudaGetErrorString(ce));
    if (ok) {
        r = api->comm_finalize(comm);
        ok = (r == ncclSuccess || r == ncclInProgress) ? settle(api, comm, deadline, "ncclCommFinalize")
                                                       : fail("ncclCommFinalize: %s", api->error_string(r));
    }
    if (ok) {
        api->comm_destroy(comm);
    } else if (comm) {
        api->comm_abort(comm);    // ends the init or the collective on this rank
        cudaGetLastError();
    }
    return ok;
}

}  // namespace tcg

extern "C" bool tcg_nccl_unique_id(unsigned char id[128])
{
    tcg::NcclApi *api = tcg::nccl();
    if (!api) return tcg::fail("NCCL (libnccl.so.2) is not available");
    ncclUniqueId uid;
    const ncclResult_t r = api->get_unique_id(&uid);
    if (r != ncclSuccess) return tcg::fail("ncclGetUniqueId: %s", api->error_string(r));
    memcpy(id, uid.internal, sizeof uid.internal);
    return true;
}
