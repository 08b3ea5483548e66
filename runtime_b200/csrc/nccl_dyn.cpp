// NCCL, loaded when first asked for (the LM-head row split over GPUs is the
// library's only collective).  The library does not link NCCL: a process
// that never splits a head needs no NCCL at all, and one that has loaded
// PyTorch's NCCL (same soname) shares that copy.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "backend_internal.h"
#include "mf_common.cuh"

namespace mf {
namespace {

struct NcclApi {
    bool tried = false;
    bool ok = false;
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    const char *(*error_string)(ncclResult_t) = nullptr;
};

NcclApi &api() {
    static NcclApi a;
    static std::mutex mu;
    std::lock_guard<std::mutex> lock(mu);
    if (a.tried) return a;
    a.tried = true;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return a;
    a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    a.comm_init_rank = reinterpret_cast<decltype(a.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    a.all_gather = reinterpret_cast<decltype(a.all_gather)>(dlsym(h, "ncclAllGather"));
    a.comm_destroy = reinterpret_cast<decltype(a.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    a.error_string = reinterpret_cast<decltype(a.error_string)>(dlsym(h, "ncclGetErrorString"));
    a.ok = a.get_unique_id && a.comm_init_rank && a.all_gather && a.comm_destroy;
    return a;
}

int32_t nccl_fail(ncclResult_t r) {
    (void)r;
    return fail(MF_BACKEND_FAILURE, "NCCL call failed");
}

}  // namespace

int32_t nccl_unique_id(uint8_t *out, size_t capacity) {
    NcclApi &a = api();
    if (!a.ok) return fail(MF_UNSUPPORTED, "NCCL is not available to this process");
    if (capacity < sizeof(ncclUniqueId)) return fail(MF_INVALID_ARGUMENT, "NCCL unique id needs 128 bytes");
    ncclUniqueId id;
    ncclResult_t r = a.get_unique_id(&id);
    if (r != ncclSuccess) return nccl_fail(r);
    memcpy(out, &id, sizeof(id));
    return MF_OK;
}

int32_t nccl_comm_init(void **comm, const uint8_t *id_bytes, int rank, int world) {
    NcclApi &a = api();
    if (!a.ok) return fail(MF_UNSUPPORTED, "NCCL is not available to this process");
    ncclUniqueId id;
    memcpy(&id, id_bytes, sizeof(id));
    ncclComm_t c = nullptr;
    ncclResult_t r = a.comm_init_rank(&c, world, id, rank);
    if (r != ncclSuccess) return nccl_fail(r);
    *comm = c;
    return MF_OK;
}

int32_t nccl_all_gather_f32(const float *send, float *recv, size_t count, void *comm, cudaStream_t stream) {
    NcclApi &a = api();
    if (!a.ok || !comm) return fail(MF_UNSUPPORTED, "NCCL communicator missing");
    ncclResult_t r = a.all_gather(send, recv, count, ncclFloat32, static_cast<ncclComm_t>(comm), stream);
    if (r != ncclSuccess) return nccl_fail(r);
    return MF_OK;
}

void nccl_comm_destroy(void *comm) {
    NcclApi &a = api();
    if (a.ok && comm) a.comm_destroy(static_cast<ncclComm_t>(comm));
}

}  // namespace mf
