// mg_ep.cu -- expert parallelism: the NCCL plumbing and the host watchdog.
//
// Experts are sharded contiguously over the ranks of one box (rank r holds
// experts [r E/G, (r+1) E/G)); every rank owns whole sequences (attention, KV
// cache, router and lm_head of its own tokens; the trunk weights are
// replicated).  Each MoE layer exchanges routed tokens with the ranks that hold
// their experts and sends the per-slot expert outputs back to the token's
// owner, which combines them in the reference's order (mg_ep_xchg.cu).  The
// data moves through buffers every rank maps into every other (CUDA IPC over
// NVLink): copy-engine puts in prefill, store-and-flag kernels in decode.
// NCCL carries only control: the communicator-id bootstrap, the all-gather
// of prefill counts and IPC handles, small all-reduces (agreements, barriers).
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, the copy already in the
// process when there is one), so a single-GPU process never needs it.
#include <dlfcn.h>
#include <nccl.h>
#include <time.h>
#include <unistd.h>

#include <cstdlib>
#include <mutex>
#include <vector>

#include "mg_common.cuh"
#include "mg_ep.h"

namespace mg {

struct NcclApi {
    void *lib = nullptr;
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
    ncclResult_t (*async_error)(ncclComm_t, ncclResult_t *) = nullptr;
    const char *(*error_string)(ncclResult_t) = nullptr;
};

static NcclApi g_nccl;
static std::mutex g_nccl_mu;

template <typename F>
static bool sym(void *h, F &fn, const char *name) {
    fn = reinterpret_cast<F>(dlsym(h, name));
    return fn != nullptr;
}

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
    bool ok = sym(h, a.get_unique_id, "ncclGetUniqueId") && sym(h, a.comm_init_rank, "ncclCommInitRank") &&
              sym(h, a.all_reduce, "ncclAllReduce") && sym(h, a.all_gather, "ncclAllGather") &&
              sym(h, a.comm_destroy, "ncclCommDestroy") &&
              sym(h, a.comm_abort, "ncclCommAbort") && sym(h, a.async_error, "ncclCommGetAsyncError") &&
              sym(h, a.error_string, "ncclGetErrorString");
    if (!ok) {
        set_error("expert parallelism: libnccl.so.2 lacks a required symbol");
        return MG_ERR_COMM;
    }
    g_nccl = a;
    return MG_OK;
}

// A failed NCCL call marks the communicator broken (it is aborted at the next
// wait or at teardown, never destroyed normally).
#define MG_NCCL(c, call)                                                                               \
    do {                                                                                               \
        ncclResult_t _r = (call);                                                                      \
        if (_r != ncclSuccess) {                                                                       \
            (c).broken = true;                                                                         \
            ::mg::set_error("%s:%d %s: %s", __FILE__, __LINE__, #call, g_nccl.error_string(_r));      \
            return MG_ERR_COMM;                                                                        \
        }                                                                                              \
    } while (0)

static ncclComm_t nc(const EpComm &c) { return static_cast<ncclComm_t>(c.comm); }

static int ep_ready(const EpComm &c) {
    MG_REQUIRE(c.comm, MG_ERR_STATE, "expert parallelism: no communicator");
    MG_REQUIRE(!c.broken, MG_ERR_COMM, "expert parallelism: the communicator was aborted after an earlier failure");
    return MG_OK;
}

int ep_unique_id(void *out) {
    MG_REQUIRE(out, MG_ERR_ARG, "ep_unique_id: null output");
    int rc = nccl_load();
    if (rc) return rc;
    ncclUniqueId id;
    ncclResult_t r = g_nccl.get_unique_id(&id);
    MG_REQUIRE(r == ncclSuccess, MG_ERR_COMM, "ncclGetUniqueId: %s", g_nccl.error_string(r));
    memcpy(out, &id, sizeof(id));
    return MG_OK;
}

int ep_init(EpComm *c, int rank, int world, const void *id) {
    MG_REQUIRE(c && id && world >= 1 && world <= EP_MAX_WORLD && rank >= 0 && rank < world, MG_ERR_ARG,
               "ep_init: bad arguments (rank %d of %d; at most %d ranks)", rank, world, EP_MAX_WORLD);
    c->rank = rank;
    c->world = world;
    c->comm = nullptr;
    c->broken = false;
    if (const char *t = getenv("MIDGE_EP_TIMEOUT_S")) c->timeout_s = atof(t) > 0 ? atof(t) : c->timeout_s;
    if (world == 1) return MG_OK;
    int rc = nccl_load();
    if (rc) return rc;
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof(uid));
    ncclComm_t comm = nullptr;
    MG_NCCL(*c, g_nccl.comm_init_rank(&comm, world, uid, rank));
    c->comm = comm;
    MG_CUDA(cudaMalloc(&c->d_ints, 64 * sizeof(int)));
    MG_CUDA(cudaHostAlloc(&c->h_ints, 64 * sizeof(int), cudaHostAllocDefault));
    return MG_OK;
}

void ep_destroy(EpComm *c) {
    if (!c) return;
    if (c->comm) {
        // a communicator whose peers may be gone or whose collective failed
        // is aborted (destroy could wait for them)
        if (c->broken) g_nccl.comm_abort(nc(*c));
        else g_nccl.comm_destroy(nc(*c));
        c->comm = nullptr;
    }
    if (c->d_ints) cudaFree(c->d_ints);
    if (c->h_ints) cudaFreeHost(c->h_ints);
    c->d_ints = nullptr;
    c->h_ints = nullptr;
}

int ep_allgather_ints(EpComm &c, const int *send, int *recv, size_t count, cudaStream_t st) {
    if (c.world <= 1) {
        if (count && send != recv) MG_CUDA(cudaMemcpyAsync(recv, send, count * 4, cudaMemcpyDeviceToDevice, st));
        return MG_OK;
    }
    TRY(ep_ready(c));
    MG_NCCL(c, g_nccl.all_gather(send, recv, count, ncclInt32, nc(c), st));
    return MG_OK;
}

int ep_allreduce_max_ints(EpComm &c, const int *v, int *out, int n, cudaStream_t st) {
    MG_REQUIRE(n >= 1 && n <= 8, MG_ERR_ARG, "allreduce_max_ints: n %d", n);
    if (c.world <= 1) {
        memcpy(out, v, (size_t)n * sizeof(int));
        return MG_OK;
    }
    TRY(ep_ready(c));
    memcpy(c.h_ints, v, (size_t)n * sizeof(int));
    MG_CUDA(cudaMemcpyAsync(c.d_ints, c.h_ints, (size_t)n * sizeof(int), cudaMemcpyHostToDevice, st));
    MG_NCCL(c, g_nccl.all_reduce(c.d_ints, c.d_ints, (size_t)n, ncclInt32, ncclMax, nc(c), st));
    MG_CUDA(cudaMemcpyAsync(c.h_ints, c.d_ints, (size_t)n * sizeof(int), cudaMemcpyDeviceToHost, st));
    TRY(ep_stream_wait(c, st));
    memcpy(out, c.h_ints, (size_t)n * sizeof(int));
    return MG_OK;
}

// ------------------------------------------------------ peer buffers
int ep_peer_alloc(EpComm &c, EpPeer &b, size_t bytes, cudaStream_t st) {
    MG_REQUIRE(bytes > 0, MG_ERR_ARG, "ep_peer_alloc: empty buffer");
    b.bytes = bytes;
    void *local = nullptr;
    MG_CUDA(cudaMalloc(&local, bytes));
    MG_CUDA(cudaMemset(local, 0, bytes));
    b.peer[c.rank] = local;
    if (c.world <= 1) return MG_OK;
    TRY(ep_ready(c));
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    const int G = c.world;
    cudaIpcMemHandle_t h;
    MG_CUDA(cudaIpcGetMemHandle(&h, local));
    int *dh = nullptr;
    MG_CUDA(cudaMalloc(&dh, (size_t)(G + 1) * 64));
    std::vector<cudaIpcMemHandle_t> all(G);
    int rc = MG_OK;
    if (cudaMemcpy(reinterpret_cast<uint8_t *>(dh) + (size_t)G * 64, &h, 64, cudaMemcpyHostToDevice) != cudaSuccess) {
        set_error("ep_peer_alloc: handle upload failed");
        rc = MG_ERR_CUDA;
    }
    if (rc == MG_OK) rc = ep_allgather_ints(c, dh + G * 16, dh, 16, st);
    if (rc == MG_OK) rc = ep_stream_wait(c, st);
    if (rc == MG_OK && cudaMemcpy(all.data(), dh, (size_t)G * 64, cudaMemcpyDeviceToHost) != cudaSuccess) {
        set_error("ep_peer_alloc: handle download failed");
        rc = MG_ERR_CUDA;
    }
    cudaFree(dh);
    for (int d = 0; d < G && rc == MG_OK; d++) {
        if (d == c.rank) continue;
        cudaError_t e = cudaIpcOpenMemHandle(&b.peer[d], all[d], cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            set_error("ep_peer_alloc: cudaIpcOpenMemHandle of rank %d: %s", d, cudaGetErrorString(e));
            rc = MG_ERR_CUDA;
        }
    }
    return rc;
}

void ep_peer_free(EpComm &c, EpPeer &b) {
    for (int d = 0; d < c.world && d < EP_MAX_WORLD; d++) {
        if (!b.peer[d]) continue;
        if (d == c.rank) cudaFree(b.peer[d]);
        else cudaIpcCloseMemHandle(b.peer[d]);
        b.peer[d] = nullptr;
    }
}

int ep_barrier(EpComm &c, cudaStream_t st) {
    if (c.world <= 1) return MG_OK;
    TRY(ep_ready(c));
    MG_NCCL(c, g_nccl.all_reduce(c.d_ints + 32, c.d_ints + 32, 1, ncclInt32, ncclSum, nc(c), st));
    return MG_OK;
}

int ep_put(EpComm &c, const float *src, const int64_t *src_off, const int64_t *cnt, EpPeer &dst,
           const int64_t *dst_off, cudaStream_t st) {
    for (int d = 0; d < c.world; d++) {
        if (!cnt[d]) continue;
        float *to = static_cast<float *>(dst.peer[d]) + dst_off[d];
        MG_REQUIRE(dst.peer[d] && (size_t)(dst_off[d] + cnt[d]) * 4 <= dst.bytes, MG_ERR_ARG,
                   "ep_put: block of %lld floats at %lld exceeds rank %d's buffer", (long long)cnt[d],
                   (long long)dst_off[d], d);
        MG_CUDA(cudaMemcpyAsync(to, src + src_off[d], (size_t)cnt[d] * 4, cudaMemcpyDeviceToDevice, st));
    }
    return MG_OK;
}

// ------------------------------------------------------------- watchdog
static double now_s() {
    timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + 1e-9 * ts.tv_nsec;
}

int ep_watchdog(int (*query)(void *), int (*async_error)(void *), void (*abort_comm)(void *), void *ctx,
                double timeout_s, int poll_us) {
    const double t0 = now_s();
    for (long it = 0;; it++) {
        const int q = query(ctx);
        if (q > 0) return MG_OK;
        if (q < 0) {
            abort_comm(ctx);
            set_error("expert parallelism: device error while waiting for a collective; communicator aborted");
            return MG_ERR_CUDA;
        }
        if (async_error(ctx)) {
            abort_comm(ctx);
            set_error("expert parallelism: the communicator reported an asynchronous error; aborted");
            return MG_ERR_COMM;
        }
        if (now_s() - t0 > timeout_s) {
            abort_comm(ctx);
            set_error("expert parallelism: a wait for the other ranks exceeded %.1f s; communicator aborted",
                      timeout_s);
            return MG_ERR_COMM;
        }
        if (poll_us > 0 && it > 64) usleep((useconds_t)poll_us);
    }
}

struct WaitCtx {
    EpComm *c;
    cudaStream_t st;
};

static int wd_query(void *p) {
    const cudaError_t e = cudaStreamQuery(static_cast<WaitCtx *>(p)->st);
    if (e == cudaSuccess) return 1;
    if (e == cudaErrorNotReady) return 0;
    return -1;
}

static int wd_async(void *p) {
    EpComm *c = static_cast<WaitCtx *>(p)->c;
    ncclResult_t r = ncclSuccess;
    if (g_nccl.async_error(nc(*c), &r) != ncclSuccess) return 1;
    return r != ncclSuccess && r != ncclInProgress;
}

static void wd_abort(void *p) {
    EpComm *c = static_cast<WaitCtx *>(p)->c;
    c->broken = true;
    if (c->comm) {
        g_nccl.comm_abort(nc(*c));
        c->comm = nullptr;
    }
}

int ep_stream_wait(EpComm &c, cudaStream_t st) {
    if (c.world <= 1 || !c.comm) {
        MG_CUDA(cudaStreamSynchronize(st));
        return MG_OK;
    }
    WaitCtx w{&c, st};
    return ep_watchdog(wd_query, wd_async, wd_abort, &w, c.timeout_s, 20);
}

}  // namespace mg

// ----------------------------------------------------- watchdog self-test
// The watchdog loop against fakes, on the CPU (no GPU and no NCCL needed).
namespace {
struct FakeWait {
    int scenario;
    long polls = 0;
    int aborted = 0;
};
int fake_query(void *p) {
    auto *f = static_cast<FakeWait *>(p);
    f->polls++;
    if (f->scenario == 0) return f->polls >= 100 ? 1 : 0;  // finishes after 100 polls
    if (f->scenario == 3) return f->polls >= 10 ? -1 : 0;  // device error
    return 0;                                               // never finishes
}
int fake_async(void *p) {
    auto *f = static_cast<FakeWait *>(p);
    return f->scenario == 2 && f->polls >= 50;  // the communicator fails after 50 polls
}
void fake_abort(void *p) { static_cast<FakeWait *>(p)->aborted++; }
}  // namespace

extern "C" int mg_ep_watchdog_selftest(int scenario, double timeout_s, int *aborted) {
    MG_REQUIRE(scenario >= 0 && scenario <= 3 && aborted, MG_ERR_ARG, "watchdog selftest: bad arguments");
    FakeWait f{scenario};
    const int rc = mg::ep_watchdog(fake_query, fake_async, fake_abort, &f, timeout_s, 100);
    *aborted = f.aborted;
    return rc;
}
