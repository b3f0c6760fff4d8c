// nccl_gather.cpp — the head all-gather of KV-head sharding over NCCL, for
// C/C++ hosts that shard across GPUs without torch (the fused peer-store
// gather in decode.cu is the other tier). NCCL is opened at run time
// (libnccl.so.2, or $GKV_NCCL_LIB), so the library itself still loads on a
// machine without NCCL; only these entry points then report the error.
#include <dlfcn.h>
#include <nccl.h>

#include <cstdlib>
#include <mutex>

#include "../../include/genllm_kv.h"
#include "kernels.h"

namespace {

struct Nccl {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
    bool ok = false;
};

const Nccl& nccl() {
    static Nccl n;
    static std::once_flag once;
    std::call_once(once, [] {
        const char* path = getenv("GKV_NCCL_LIB");
        void* h = dlopen(path && path[0] ? path : "libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (!h) return;
        n.get_unique_id = reinterpret_cast<decltype(n.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
        n.comm_init_rank = reinterpret_cast<decltype(n.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
        n.comm_destroy = reinterpret_cast<decltype(n.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
        n.all_gather = reinterpret_cast<decltype(n.all_gather)>(dlsym(h, "ncclAllGather"));
        n.error_string = reinterpret_cast<decltype(n.error_string)>(dlsym(h, "ncclGetErrorString"));
        n.ok = n.get_unique_id && n.comm_init_rank && n.comm_destroy && n.all_gather && n.error_string;
    });
    return n;
}

int fail(int status, const char* what) {
    gkv::set_last_error(what);
    return status;
}

int nccl_fail(ncclResult_t r) { return fail(GKV_ERR_CUDA, nccl().error_string(r)); }

}  // namespace

extern "C" {

int gkv_nccl_unique_id(void* id) {
    if (!id) return fail(GKV_ERR_INVALID, "null id");
    if (!nccl().ok) return fail(GKV_ERR_UNSUPPORTED, "NCCL not found (libnccl.so.2 / GKV_NCCL_LIB)");
    const ncclResult_t r = nccl().get_unique_id(static_cast<ncclUniqueId*>(id));
    return r == ncclSuccess ? GKV_OK : nccl_fail(r);
}

int gkv_nccl_comm_create(int device, int world, int rank, const void* id, void** comm) {
    if (!id || !comm || world < 1 || rank < 0 || rank >= world) return fail(GKV_ERR_INVALID, "bad arguments");
    if (!nccl().ok) return fail(GKV_ERR_UNSUPPORTED, "NCCL not found (libnccl.so.2 / GKV_NCCL_LIB)");
    if (cudaSetDevice(device) != cudaSuccess) return fail(GKV_ERR_CUDA, "cannot select the device");
    ncclUniqueId u;
    static_assert(sizeof(u) == 128, "NCCL unique id size");
    __builtin_memcpy(&u, id, sizeof(u));
    ncclComm_t c = nullptr;
    const ncclResult_t r = nccl().comm_init_rank(&c, world, u, rank);
    if (r != ncclSuccess) return nccl_fail(r);
    *comm = c;
    return GKV_OK;
}

int gkv_nccl_comm_destroy(void* comm) {
    if (!comm) return GKV_OK;
    if (!nccl().ok) return fail(GKV_ERR_UNSUPPORTED, "NCCL not found");
    const ncclResult_t r = nccl().comm_destroy(static_cast<ncclComm_t>(comm));
    return r == ncclSuccess ? GKV_OK : nccl_fail(r);
}

int gkv_allgather_heads(void* comm, const void* local, void* full, size_t bytes_per_rank, gkv_stream_t stream) {
    if (!comm || !local || !full || bytes_per_rank == 0) return fail(GKV_ERR_INVALID, "bad arguments");
    if (!nccl().ok) return fail(GKV_ERR_UNSUPPORTED, "NCCL not found");
    const ncclResult_t r = nccl().all_gather(local, full, bytes_per_rank, ncclUint8, static_cast<ncclComm_t>(comm),
                                             reinterpret_cast<cudaStream_t>(stream));
    return r == ncclSuccess ? GKV_OK : nccl_fail(r);
}

}  // extern "C"
