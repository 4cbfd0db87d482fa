// mg_ep.cu -- expert parallelism: the NCCL plumbing.
//
// Experts are sharded contiguously over the ranks of one box (rank r holds
// experts [r E/G, (r+1) E/G)); tokens, attention, KV cache, router and trunk
// are replicated.  After a layer's routed experts ran, each rank holds the
// outputs of the (token, rank-slot) pairs routed to its own experts and zeros
// in every other slot; a sum all-reduce of that slot buffer therefore gives
// every rank the exact per-slot outputs (adding zeros is exact), and the
// combine that follows runs in the reference's order on identical data: the
// result is bit-identical to one GPU holding all experts.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, the copy already in the
// process when there is one), so a single-GPU process never needs it.
#include <dlfcn.h>
#include <nccl.h>

#include <mutex>

#include "mg_common.cuh"
#include "mg_ep.h"

namespace mg {

struct NcclApi {
    void *lib = nullptr;
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
    const char *(*error_string)(ncclResult_t) = nullptr;
};

static NcclApi g_nccl;
static std::mutex g_nccl_mu;

static int nccl_load() {
    std::lock_guard<std::mutex> lk(g_nccl_mu);
    if (g_nccl.lib) return MG_OK;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
        set_error("expert parallelism: cannot load libnccl.so.2 (%s)", dlerror());
        return MG_ERR_COMM;
    }
    NcclApi a;
    a.lib = h;
    a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    a.comm_init_rank = reinterpret_cast<decltype(a.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(dlsym(h, "ncclAllReduce"));
    a.comm_destroy = reinterpret_cast<decltype(a.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    a.comm_abort = reinterpret_cast<decltype(a.comm_abort)>(dlsym(h, "ncclCommAbort"));
    a.error_string = reinterpret_cast<decltype(a.error_string)>(dlsym(h, "ncclGetErrorString"));
    if (!a.get_unique_id || !a.comm_init_rank || !a.all_reduce || !a.comm_destroy || !a.comm_abort ||
        !a.error_string) {
        set_error("expert parallelism: libnccl.so.2 lacks a required symbol");
        return MG_ERR_COMM;
    }
    g_nccl = a;
    return MG_OK;
}

#define MG_NCCL(call)                                                                                  \
    do {                                                                                               \
        ncclResult_t _r = (call);                                                                      \
        if (_r != ncclSuccess) {                                                                       \
            ::mg::set_error("%s:%d %s: %s", __FILE__, __LINE__, #call, g_nccl.error_string(_r));      \
            return MG_ERR_COMM;                                                                        \
        }                                                                                              \
    } while (0)

int ep_unique_id(void *out) {
    MG_REQUIRE(out, MG_ERR_ARG, "ep_unique_id: null output");
    int rc = nccl_load();
    if (rc) return rc;
    ncclUniqueId id;
    MG_NCCL(g_nccl.get_unique_id(&id));
    memcpy(out, &id, sizeof(id));
    return MG_OK;
}

int ep_init(EpComm *c, int rank, int world, const void *id) {
    MG_REQUIRE(c && id && world >= 1 && rank >= 0 && rank < world, MG_ERR_ARG, "ep_init: bad arguments");
    c->rank = rank;
    c->world = world;
    c->comm = nullptr;
    if (world == 1) return MG_OK;
    int rc = nccl_load();
    if (rc) return rc;
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof(uid));
    ncclComm_t comm = nullptr;
    MG_NCCL(g_nccl.comm_init_rank(&comm, world, uid, rank));
    c->comm = comm;
    return MG_OK;
}

// in-place sum over the ranks (the per-slot expert outputs)
int ep_allreduce_sum(const EpComm &c, float *buf, size_t count, cudaStream_t st) {
    if (c.world <= 1 || count == 0) return MG_OK;
    MG_REQUIRE(c.comm, MG_ERR_STATE, "expert parallelism: no communicator");
    MG_NCCL(g_nccl.all_reduce(buf, buf, count, ncclFloat32, ncclSum, static_cast<ncclComm_t>(c.comm), st));
    return MG_OK;
}

void ep_destroy(EpComm *c) {
    if (c && c->comm) {
        g_nccl.comm_destroy(static_cast<ncclComm_t>(c->comm));
        c->comm = nullptr;
    }
}

}  // namespace mg
