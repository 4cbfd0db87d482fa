// mg_ep.h -- expert-parallel communicator (NCCL loaded at run time).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

namespace mg {

struct EpComm {
    int rank = 0, world = 1;
    void *comm = nullptr;  // ncclComm_t
};

int ep_unique_id(void *out);  // 128 bytes
int ep_init(EpComm *c, int rank, int world, const void *id);
int ep_allreduce_sum(const EpComm &c, float *buf, size_t count, cudaStream_t st);
void ep_destroy(EpComm *c);

// contiguous expert shard of `rank`
inline void ep_range(int n_experts, int world, int rank, int *e0, int *n_local) {
    *n_local = n_experts / world;
    *e0 = rank * (*n_local);
}

}  // namespace mg
