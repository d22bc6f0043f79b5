// NCCL, loaded at run time (dlopen "libnccl.so.2") only when a tensor-parallel
// engine is created, so single-GPU use never depends on it.  In a process that
// already imported torch the loader returns torch's own libnccl.so.2.
#include <dlfcn.h>
#include <nccl.h>

#include <cstdio>
#include <mutex>

#include "alb_common.cuh"
#include "alb_nccl.h"

namespace alb {

struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*AllReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
    const char * (*GetErrorString)(ncclResult_t) = nullptr;
    bool ok = false;
};

static NcclApi & api() {
    static NcclApi a;
    static std::once_flag once;
    std::call_once(once, [] {
        void * h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
#define ALB_SYM(field, name) a.field = reinterpret_cast<decltype(a.field)>(dlsym(h, name))
        ALB_SYM(GetUniqueId, "ncclGetUniqueId");
        ALB_SYM(CommInitRank, "ncclCommInitRank");
        ALB_SYM(AllReduce, "ncclAllReduce");
        ALB_SYM(AllGather, "ncclAllGather");
        ALB_SYM(CommDestroy, "ncclCommDestroy");
        ALB_SYM(CommAbort, "ncclCommAbort");
        ALB_SYM(CommGetAsyncError, "ncclCommGetAsyncError");
        ALB_SYM(GetErrorString, "ncclGetErrorString");
#undef ALB_SYM
        a.ok = a.GetUniqueId && a.CommInitRank && a.AllReduce && a.AllGather && a.CommDestroy && a.CommAbort && a.GetErrorString;
    });
    return a;
}

static int nccl_fail(ncclResult_t r, const char * what) {
    char buf[256];
    snprintf(buf, sizeof(buf), "%s: %s", what, api().GetErrorString ? api().GetErrorString(r) : "nccl error");
    alb_set_last_error_msg(buf);
    return ALB_ERR_NCCL;
}

int nccl_unique_id(void * out128) {
    if (!api().ok) { alb_set_last_error_msg("libnccl.so.2 not loadable"); return ALB_ERR_UNSUPPORTED; }
    ncclUniqueId id;
    const ncclResult_t r = api().GetUniqueId(&id);
    if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
    static_assert(sizeof(ncclUniqueId) == 128, "unique id size");
    memcpy(out128, &id, 128);
    return ALB_OK;
}

int nccl_init(void ** comm, int rank, int size, const void * id128) {
    if (!api().ok) { alb_set_last_error_msg("libnccl.so.2 not loadable"); return ALB_ERR_UNSUPPORTED; }
    ncclUniqueId id;
    memcpy(&id, id128, 128);
    ncclComm_t c = nullptr;
    const ncclResult_t r = api().CommInitRank(&c, size, id, rank);
    if (r != ncclSuccess) return nccl_fail(r, "ncclCommInitRank");
    *comm = c;
    return ALB_OK;
}

int nccl_allgather_f32(void * comm, const float * src, float * dst, size_t count, cudaStream_t st) {
    const ncclResult_t r = api().AllGather(src, dst, count, ncclFloat32, static_cast<ncclComm_t>(comm), st);
    if (r != ncclSuccess) return nccl_fail(r, "ncclAllGather");
    return ALB_OK;
}

int nccl_allreduce(void * comm, const void * src, void * dst, size_t count, int dtype, int op, cudaStream_t st) {
    const ncclDataType_t dt = dtype == 0 ? ncclFloat32 : ncclUint64;
    const ncclRedOp_t ro = op == 0 ? ncclSum : ncclMax;
    const ncclResult_t r = api().AllReduce(src, dst, count, dt, ro, static_cast<ncclComm_t>(comm), st);
    if (r != ncclSuccess) return nccl_fail(r, "ncclAllReduce");
    return ALB_OK;
}

int nccl_async_error(void * comm) {
    if (!comm || !api().CommGetAsyncError) return ALB_OK;
    ncclResult_t e = ncclSuccess;
    api().CommGetAsyncError(static_cast<ncclComm_t>(comm), &e);
    return e == ncclSuccess || e == ncclInProgress ? ALB_OK : nccl_fail(e, "nccl async error");
}

void nccl_destroy(void * comm, bool abort) {
    if (!comm || !api().ok) return;
    if (abort) api().CommAbort(static_cast<ncclComm_t>(comm));
    else api().CommDestroy(static_cast<ncclComm_t>(comm));
}

}  // namespace alb
