// nccl.cu -- the one collective of the multi-GPU path: a one-time broadcast
// of the fp32 weight slab from rank 0 over NVLink (NCCL). NCCL is opened at
// run time so that single-GPU users never need it.
#include "tcg_common.cuh"
#include "tcg_internal.h"

#include <dlfcn.h>
#include <nccl.h>
#include <string.h>

namespace tcg {
namespace {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId *);
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int);
    ncclResult_t (*broadcast)(const void *, void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
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
    api.comm_init_rank = (decltype(api.comm_init_rank))dlsym(h, "ncclCommInitRank");
    api.broadcast = (decltype(api.broadcast))dlsym(h, "ncclBroadcast");
    api.comm_destroy = (decltype(api.comm_destroy))dlsym(h, "ncclCommDestroy");
    api.error_string = (decltype(api.error_string))dlsym(h, "ncclGetErrorString");
    api.ok = api.get_unique_id && api.comm_init_rank && api.broadcast && api.comm_destroy && api.error_string;
    return api.ok ? &api : nullptr;
}

}  // namespace

bool broadcast_once(void *buf, size_t count_floats, int rank, int nranks, const unsigned char id[128])
{
    NcclApi *api = nccl();
    if (!api) return fail("NCCL (libnccl.so.2) is not available");
    if (nranks < 1 || rank < 0 || rank >= nranks) return fail("bad rank %d of %d", rank, nranks);
    if (nranks == 1) return true;
    ncclUniqueId uid;
    memcpy(uid.internal, id, sizeof uid.internal);
    ncclComm_t comm = nullptr;
    ncclResult_t r = api->comm_init_rank(&comm, nranks, uid, rank);
    if (r != ncclSuccess) return fail("ncclCommInitRank(rank %d of %d): %s", rank, nranks, api->error_string(r));
    r = api->broadcast(buf, buf, count_floats, ncclFloat32, 0, comm, ctx().cur);
    const cudaError_t ce = cudaStreamSynchronize(ctx().cur);
    api->comm_destroy(comm);
    if (r != ncclSuccess) return fail("ncclBroadcast: %s", api->error_string(r));
    TCG_CUDA(ce);
    return true;
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
