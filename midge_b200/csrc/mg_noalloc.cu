// mg_noalloc.cu -- mg_moe_ffn for callers that may not allocate device memory.
//
// Some callers cannot hand mg_moe_ffn a scratch buffer and must not trigger
// a device allocation on the call path: a host that runs its decode loop
// inside a memory budget fixed at start-up, code that runs while another
// component owns the device allocator, or a host binding with no device
// allocator of its own (a plain C / cgo caller).  For them the gate/up
// activations live in a fixed device array compiled into this library,
// sized for MG_NOALLOC_MAX_H floats (4 MiB).  Limits: n_tok <= 16, as for
// mg_moe_ffn (MG_ERR_ARG beyond), and n_tok * top_k * ffn <= 1,048,576
// (MG_ERR_RANGE beyond): 16 tokens fit at top-k 16 and ffn 4096.
//
// Set-up: the first call on a device, with that device current, looks up the
// array's device address (cudaGetSymbolAddress) and keeps it for the
// device's later calls.  That first call should therefore come before any
// stream capture.  Nothing in the array needs to start at zero: every
// element the down projection reads was written by the gate/up kernel of the
// same call.  The array is shared by all calls on a device, so calls that
// overlap in time on one device (other streams or host threads) race on it
// and must be serialised by the caller.
#include <mutex>

#include "mg_common.cuh"
#include "mg_kernels.h"

namespace mg {

static __device__ __align__(256) float g_noalloc_h[MG_NOALLOC_MAX_H];

constexpr int NOALLOC_MAX_DEV = 64;
static float *g_noalloc_ptr[NOALLOC_MAX_DEV];
static std::mutex g_noalloc_mu;

static int noalloc_scratch(float **out) {
    int dev = 0;
    MG_CUDA(cudaGetDevice(&dev));
    MG_REQUIRE(dev >= 0 && dev < NOALLOC_MAX_DEV, MG_ERR_ARG, "moe_ffn_noalloc: device %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void *p = nullptr;
        cudaError_t rc = cudaGetSymbolAddress(&p, g_noalloc_h);
        if (rc != cudaSuccess || !p) {
            set_error("moe_ffn_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(rc));
            return MG_ERR_CUDA;
        }
        g_noalloc_ptr[dev] = static_cast<float *>(p);
    }
    *out = g_noalloc_ptr[dev];
    return MG_OK;
}

}  // namespace mg

using namespace mg;

extern "C" int mg_moe_ffn_noalloc(const mg_expert_layout *L, const uint8_t *experts, int layer, int n_experts,
                                  const float *xb, int n_tok, int top_k, const int32_t *sel, const float *weights,
                                  int act_plain, float alpha, float limit, float *x, void *stream) {
    MG_REQUIRE(L && experts && layer >= 0 && n_tok >= 0 && top_k >= 0, MG_ERR_ARG, "moe_ffn_noalloc: bad arguments");
    MG_REQUIRE(n_tok <= MG_NOALLOC_MAX_TOK, MG_ERR_ARG, "moe_ffn_noalloc: n_tok = %d exceeds %d tokens per call", n_tok,
               MG_NOALLOC_MAX_TOK);
    const int64_t need = (int64_t)n_tok * top_k * L->ffn;
    MG_REQUIRE(need <= MG_NOALLOC_MAX_H, MG_ERR_RANGE,
               "moe_ffn_noalloc: n_tok*top_k*ffn = %lld exceeds the fixed scratch of %d floats", (long long)need,
               MG_NOALLOC_MAX_H);
    float *h = nullptr;
    int rc = noalloc_scratch(&h);
    if (rc) return rc;
    return mg_moe_ffn(L, experts, layer, n_experts, xb, n_tok, top_k, sel, weights, act_plain, alpha, limit, h, x,
                      stream);
}
