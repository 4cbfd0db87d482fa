// mg_selftest.cu -- the failure path of a bounded device wait, run on purpose.
//
// Every pipelined kernel of this library waits on mbarriers with a bounded
// number of polls; a wait that runs out writes the stream error word, the
// role stops, waits (with the full budget) for the copies it issued to land,
// frees TMEM, and the host turns the error word into MG_ERR_TIMEOUT.  This
// kernel exercises exactly that sequence on a wait that nothing satisfies:
// warp 1 allocates TMEM, warp 0 issues a bulk copy into shared memory that
// completes on one barrier, then waits `polls` times on a second barrier that
// never receives an arrival, records the timeout, drains its copy (full
// budget: the copy always lands) and the CTA frees TMEM and exits.  Nothing
// faults and nothing hangs; the context stays usable.
#include "mg_common.cuh"
#include "mg_kernels.h"
#include "mg_tc.cuh"

namespace mg {

constexpr int ST_ERR = 31;  // error word code of the self-test's timed-out wait

__global__ void k_wait_selftest(const uint8_t *src, int polls, int *err, int *drained) {
    __shared__ __align__(128) uint8_t buf[4096];
    __shared__ uint64_t landed, never;
    __shared__ uint32_t tmem;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        mbar_init(&landed, 1);
        mbar_init(&never, 1);
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(&tmem, 32);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0 && lane == 0) {
        mbar_arrive_expect_tx(&landed, 4096);
        bulk_g2s(buf, src, 4096, &landed);
        bool ok = true;
        for (int i = 0; i < polls && !(ok = mbar_try_wait(&never, 0)); i++) {
        }
        if (!ok) atomicCAS(err, 0, ST_ERR);
        // the copy this thread issued lands before the CTA may exit
        *drained = mbar_wait(&landed, 0) ? (int)buf[4095] + 1 : -1;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 32);
    }
}

int wait_selftest(int polls, int *drained_host) {
    MG_REQUIRE(polls >= 1 && polls <= (1 << 20) && drained_host, MG_ERR_ARG, "wait selftest: bad arguments");
    int *err = stream_error_word();
    MG_REQUIRE(err, MG_ERR_OOM, "wait selftest: no error word");
    uint8_t *src = nullptr;
    int *drained = nullptr;
    MG_CUDA(cudaMalloc(&src, 4096 + 16));
    drained = reinterpret_cast<int *>(src + 4096);
    MG_CUDA(cudaMemset(src, 0x2A, 4096));
    MG_CUDA(cudaMemset(drained, 0, 4));
    k_wait_selftest<<<1, 64>>>(src, polls, err, drained);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    int h = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&h, drained, 4, cudaMemcpyDeviceToHost);
    cudaFree(src);
    MG_REQUIRE(e == cudaSuccess, MG_ERR_CUDA, "wait selftest: %s", cudaGetErrorString(e));
    *drained_host = h;
    return stream_error_check();  // MG_ERR_TIMEOUT, error word cleared
}

}  // namespace mg

extern "C" int mg_wait_selftest(int polls, int *drained) { return mg::wait_selftest(polls, drained); }
