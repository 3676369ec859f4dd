// tp.cu -- NCCL for the tensor-parallel verify forward, loaded at run time.
//
// The library does not link NCCL: libnccl.so.2 is opened on first use (an
// already-loaded copy, e.g. the one a host framework brought in, is reused),
// so single-GPU users need no NCCL and a host's own NCCL is not duplicated.
// Only the entry points below are used; their signatures are NCCL's public
// API (nccl.h).
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "kernels.h"

namespace mlxcat {

namespace {

struct NcclApi {
    bool ok = false;
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    const char *(*error_string)(ncclResult_t) = nullptr;
    ncclResult_t (*group_start)() = nullptr;
    ncclResult_t (*group_end)() = nullptr;
    ncclResult_t (*send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
};

NcclApi &api() {
    static NcclApi a;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
        a.comm_init_rank = reinterpret_cast<decltype(a.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
        a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(dlsym(h, "ncclAllReduce"));
        a.comm_destroy = reinterpret_cast<decltype(a.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
        a.error_string = reinterpret_cast<decltype(a.error_string)>(dlsym(h, "ncclGetErrorString"));
        a.group_start = reinterpret_cast<decltype(a.group_start)>(dlsym(h, "ncclGroupStart"));
        a.group_end = reinterpret_cast<decltype(a.group_end)>(dlsym(h, "ncclGroupEnd"));
        a.send = reinterpret_cast<decltype(a.send)>(dlsym(h, "ncclSend"));
        a.recv = reinterpret_cast<decltype(a.recv)>(dlsym(h, "ncclRecv"));
        a.ok = a.get_unique_id && a.comm_init_rank && a.all_reduce && a.comm_destroy && a.error_string &&
               a.group_start && a.group_end && a.send && a.recv;
    });
    return a;
}

const char *err_str(ncclResult_t r) { return api().error_string ? api().error_string(r) : "NCCL unavailable"; }

}  // namespace

bool tp_available() { return api().ok; }

const char *tp_unique_id(uint8_t *out) {
    if (!api().ok) return "libnccl.so.2 could not be loaded";
    static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id is 128 bytes");
    ncclUniqueId id;
    const ncclResult_t r = api().get_unique_id(&id);
    if (r != ncclSuccess) return err_str(r);
    memcpy(out, &id, sizeof id);
    return nullptr;
}

const char *tp_connect(void **comm, const uint8_t *id, int nranks, int rank) {
    if (!api().ok) return "libnccl.so.2 could not be loaded";
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof uid);
    ncclComm_t c = nullptr;
    const ncclResult_t r = api().comm_init_rank(&c, nranks, uid, rank);
    if (r != ncclSuccess) return err_str(r);
    // NCCL handles the CUDA errors of its own probing internally, but they stay
    // in the runtime's last-error slot, where the next kernel launch's
    // cudaGetLastError would report them as its own: clear it.
    (void)cudaGetLastError();
    *comm = c;
    return nullptr;
}

const char *tp_allreduce_sum(void *comm, float *buf, size_t n, cudaStream_t st) {
    const ncclResult_t r = api().all_reduce(buf, buf, n, ncclFloat32, ncclSum, static_cast<ncclComm_t>(comm), st);
    if (r != ncclSuccess) return err_str(r);
    (void)cudaGetLastError();   // as after ncclCommInitRank
    return nullptr;
}


void tp_destroy(void *comm) {
    if (comm && api().ok) api().comm_destroy(static_cast<ncclComm_t>(comm));
}

}  // namespace mlxcat
