// tb_nccl.cu -- run-time bound NCCL entry points (see tb_nccl.h).
#include "tb_nccl.h"

#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

namespace tb {
namespace {

struct NcclApi {
    bool ok = false;
    std::string why;
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
};

const NcclApi& api() {
    static NcclApi a;
    static std::once_flag once;
    std::call_once(once, [] {
        // An already-loaded libnccl.so.2 (e.g. the one torch.distributed uses)
        // is returned as is; otherwise the loader search path decides.
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            a.why = std::string("cannot load libnccl.so.2: ") + dlerror();
            return;
        }
        a.get_unique_id = (decltype(a.get_unique_id))dlsym(h, "ncclGetUniqueId");
        a.comm_init_rank = (decltype(a.comm_init_rank))dlsym(h, "ncclCommInitRank");
        a.comm_destroy = (decltype(a.comm_destroy))dlsym(h, "ncclCommDestroy");
        a.all_reduce = (decltype(a.all_reduce))dlsym(h, "ncclAllReduce");
        a.error_string = (decltype(a.error_string))dlsym(h, "ncclGetErrorString");
        a.ok = a.get_unique_id && a.comm_init_rank && a.comm_destroy && a.all_reduce && a.error_string;
        if (!a.ok) a.why = "libnccl.so.2 lacks an expected symbol";
    });
    return a;
}

}  // namespace

int nccl_unique_id(unsigned char* id, std::string& why) {
    const NcclApi& a = api();
    if (!a.ok) {
        why = a.why;
        return 1;
    }
    ncclUniqueId u;
    const ncclResult_t r = a.get_unique_id(&u);
    if (r != ncclSuccess) {
        why = std::string("ncclGetUniqueId: ") + a.error_string(r);
        return 1;
    }
    static_assert(sizeof(u) == kNcclIdBytes, "ncclUniqueId size");
    std::memcpy(id, &u, kNcclIdBytes);
    return 0;
}

int nccl_comm_init(void** comm, const unsigned char* id, int rank, int world, std::string& why) {
    const NcclApi& a = api();
    if (!a.ok) {
        why = a.why;
        return 1;
    }
    ncclUniqueId u;
    std::memcpy(&u, id, kNcclIdBytes);
    ncclComm_t c = nullptr;
    const ncclResult_t r = a.comm_init_rank(&c, world, u, rank);
    if (r != ncclSuccess) {
        why = std::string("ncclCommInitRank: ") + a.error_string(r);
        return 1;
    }
    *comm = c;
    return 0;
}

void nccl_comm_destroy(void* comm) {
    const NcclApi& a = api();
    if (a.ok && comm) a.comm_destroy((ncclComm_t)comm);
}

cudaError_t nccl_allreduce_sum_f32(void* comm, float* buf, size_t count, cudaStream_t st, std::string& why) {
    const NcclApi& a = api();
    if (!a.ok || !comm) {
        why = a.ok ? "no communicator" : a.why;
        return cudaErrorNotSupported;
    }
    const ncclResult_t r = a.all_reduce(buf, buf, count, ncclFloat32, ncclSum, (ncclComm_t)comm, st);
    if (r != ncclSuccess) {
        why = std::string("ncclAllReduce: ") + a.error_string(r);
        return cudaErrorUnknown;
    }
    return cudaSuccess;
}

}  // namespace tb
