// mg_ep.h -- expert-parallel communicator (NCCL loaded at run time) and the
// host watchdog around its blocking waits.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace mg {

constexpr int EP_MAX_WORLD = 8;  // ranks of one box

struct EpComm {
    int rank = 0, world = 1;
    void *comm = nullptr;    // ncclComm_t
    bool broken = false;     // a collective failed or a wait timed out: the communicator was aborted
    double timeout_s = 600;  // host waits on a stream that holds collectives (MIDGE_EP_TIMEOUT_S)
    int *d_ints = nullptr;   // small device scratch for host-level agreements (allreduce of a few ints)
    int *h_ints = nullptr;   // pinned mirror
};

int ep_unique_id(void *out);  // 128 bytes
int ep_init(EpComm *c, int rank, int world, const void *id);
void ep_destroy(EpComm *c);

// Collectives on `st` (enqueued, asynchronous; graph-capturable).
int ep_allgather_ints(EpComm &c, const int *send, int *recv, size_t count, cudaStream_t st);

// Host agreement: out[i] = max over ranks of v[i] (n <= 8 ints); synchronous.
int ep_allreduce_max_ints(EpComm &c, const int *v, int *out, int n, cudaStream_t st);

// Wait for `st` to drain.  With one rank: cudaStreamSynchronize.  With
// several: poll the stream and the communicator's asynchronous error; on an
// error or after c.timeout_s the communicator is aborted (ncclCommAbort, which
// ends collectives that wait for a rank that will not come) and MG_ERR_COMM
// is returned; the model is then unusable for further collectives.
int ep_stream_wait(EpComm &c, cudaStream_t st);

// The watchdog loop itself, over callbacks (so that its logic runs on the CPU
// against fakes): query() returns 1 when the work is done, 0 while it runs,
// < 0 on a device error; async_error() returns nonzero once the communicator
// reports an error; abort_comm() is called once on error or timeout.
// Returns MG_OK, MG_ERR_COMM (error or timeout) or MG_ERR_CUDA.
int ep_watchdog(int (*query)(void *), int (*async_error)(void *), void (*abort_comm)(void *), void *ctx,
                double timeout_s, int poll_us);

// A buffer every rank allocates and maps into every other rank's process
// (CUDA IPC over NVLink): peer[d] is rank d's copy, peer[rank] the local one.
struct EpPeer {
    void *peer[EP_MAX_WORLD] = {};
    size_t bytes = 0;
};
int ep_peer_alloc(EpComm &c, EpPeer &b, size_t bytes, cudaStream_t st);
void ep_peer_free(EpComm &c, EpPeer &b);
// every rank's stream reaches this point before any passes it (a 1-int
// NCCL all-reduce): orders peer writes before the reads they feed
int ep_barrier(EpComm &c, cudaStream_t st);
// copy engine puts: to rank d, cnt[d] floats from src + src_off[d] into rank
// d's copy of dst at dst_off[d] (the own block is a local copy)
int ep_put(EpComm &c, const float *src, const int64_t *src_off, const int64_t *cnt, EpPeer &dst,
           const int64_t *dst_off, cudaStream_t st);

// contiguous expert shard of `rank`
inline void ep_range(int n_experts, int world, int rank, int *e0, int *n_local) {
    *n_local = n_experts / world;
    *e0 = rank * (*n_local);
}

}  // namespace mg
