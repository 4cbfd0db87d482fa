// mg_abi.cu -- extern "C" entry points of libmidgecuda.so (kernel level) and
// the error state.  Model-level entry points live in mg_model.cu.
#include <cstdarg>
#include <cstdio>

#include "mg_common.cuh"
#include "mg_kernels.h"

namespace mg {

static thread_local char g_err[512] = "";

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

void *encode_tiled_fn() {
    static void *fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = p;
    }
    return fn;
}

// byte tensor {row bytes, rows [, experts, layers]}, box 128 B x box_rows, 128-byte swizzle, OOB -> 0
static int map_weights(CUtensorMap *map, const void *base, int rank, const cuuint64_t *dims, const cuuint64_t *strides,
                       int box_rows) {
    EncodeTiledFn fn = reinterpret_cast<EncodeTiledFn>(encode_tiled_fn());
    MG_REQUIRE(fn, MG_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    MG_REQUIRE((reinterpret_cast<uintptr_t>(base) & 15) == 0, MG_ERR_ARG, "weight map: base not 16-byte aligned");
    for (int i = 0; i < rank - 1; i++)
        MG_REQUIRE(strides[i] % 16 == 0, MG_ERR_ARG, "weight map: stride %llu not a multiple of 16",
                   (unsigned long long)strides[i]);
    cuuint32_t box[4] = {128, (cuuint32_t)box_rows, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, (cuuint32_t)rank, const_cast<void *>(base), dims, strides, box,
                    estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    MG_REQUIRE(r == CUDA_SUCCESS, MG_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return MG_OK;
}

int map_weights_2d(CUtensorMap *map, const void *base, int64_t rowbytes, int64_t rows, int box_rows) {
    cuuint64_t dims[2] = {(cuuint64_t)rowbytes, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)rowbytes};
    return map_weights(map, base, 2, dims, strides, box_rows);
}

int map_weights_4d(CUtensorMap *map, const void *base, int64_t rowbytes, int64_t rows, int64_t n_experts,
                   int64_t n_layers, int64_t expert_stride, int64_t layer_stride, int box_rows) {
    cuuint64_t dims[4] = {(cuuint64_t)rowbytes, (cuuint64_t)rows, (cuuint64_t)n_experts, (cuuint64_t)n_layers};
    cuuint64_t strides[3] = {(cuuint64_t)rowbytes, (cuuint64_t)expert_stride, (cuuint64_t)layer_stride};
    return map_weights(map, base, 4, dims, strides, box_rows);
}

int num_sms() {
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!cache[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

int ensure_smem_attr(const void *fn, size_t bytes) {
    if (bytes <= 48 * 1024) return MG_OK;
    struct Entry { const void *fn; int dev; size_t bytes; };
    static Entry table[512];
    static int n = 0;
    int dev = 0;
    MG_CUDA(cudaGetDevice(&dev));
    int slot = -1;
    for (int i = 0; i < n; i++)
        if (table[i].fn == fn && table[i].dev == dev) {
            if (table[i].bytes >= bytes) return MG_OK;
            slot = i;
        }
    // the dynamic limit excludes the kernel's static shared memory
    MG_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    if (slot >= 0) table[slot].bytes = bytes;
    else if (n < 512) table[n++] = {fn, dev, bytes};
    return MG_OK;
}

}  // namespace mg

using namespace mg;

extern "C" const char *mg_last_error(void) { return g_err; }
extern "C" int mg_version(void) { return 1; }

extern "C" int mg_gemv(int dt, int scale_fmt, const void *w, const void *scales, int64_t rows, int64_t cols,
                       const float *x, int64_t ldx, int n_tok, const float *bias, int accumulate, float *y, int64_t ldy,
                       void *stream) {
    return gemv(dt, scale_fmt, w, scales, rows, cols, x, ldx, n_tok, bias, accumulate, y, ldy, (cudaStream_t)stream);
}

extern "C" int mg_dequant_rows(int dt, int scale_fmt, const void *w, const void *scales, int64_t rows, int64_t cols,
                               const int32_t *ids, int n, float *out, void *stream) {
    return dequant_rows(dt, scale_fmt, w, scales, rows, cols, ids, n, out, (cudaStream_t)stream);
}

extern "C" int mg_scales_to_ue8m0(const uint16_t *f16, uint8_t *ue8m0, int64_t n, int *n_inexact, void *stream) {
    return scales_to_ue8m0(f16, ue8m0, n, n_inexact, (cudaStream_t)stream);
}

extern "C" int mg_rmsnorm(const float *x, const float *w, float *out, int64_t n, int n_rows, float eps, void *stream) {
    return rmsnorm(x, w, out, n, n_rows, eps, (cudaStream_t)stream);
}

extern "C" int mg_to_f16_ftz(const float *x, uint16_t *out, int64_t n, void *stream) {
    return to_f16_ftz(x, out, n, (cudaStream_t)stream);
}

extern "C" int mg_router_topk(const float *xb, int n_tok, const float *rw, const float *rb, int n_experts,
                              int64_t hidden, int top_k, int router_norm, int variant, float *logits, int32_t *sel,
                              float *weights, void *stream) {
    RouterArgs a{};
    a.x = xb;
    a.norm_w = nullptr;
    a.rw = rw;
    a.rb = rb;
    a.n_experts = n_experts;
    a.top_k = top_k;
    a.router_norm = router_norm;
    a.variant = variant;
    a.hidden = hidden;
    a.n_tok = n_tok;
    a.logits = logits;
    a.sel = sel;
    a.weights = weights;
    a.usage = nullptr;
    return router(a, (cudaStream_t)stream);
}

extern "C" int mg_sample_topp(const float *logits, int64_t ldl, int64_t V, int n_rows, float temp, float top_p,
                              uint64_t *rng, int32_t *out, float *probs, void *stream) {
    return sample_topp(logits, ldl, V, n_rows, temp, top_p, rng, out, probs, (cudaStream_t)stream);
}

// wt_expert_layout (engine/mten.h:136-150) with wt_sizes (engine/mten.h:101-109)
extern "C" int mg_expert_layout_init(mg_expert_layout *L, int dt, int64_t hidden, int64_t ffn, int64_t n_experts) {
    MG_REQUIRE(L && hidden > 0 && ffn > 0 && n_experts > 0, MG_ERR_ARG, "expert_layout: bad arguments");
    L->dt = dt == MG_MXFP4_E8 ? MG_MXFP4 : dt;
    L->scale_fmt = dt == MG_MXFP4_E8 ? MG_SCALE_UE8M0 : MG_SCALE_F16;
    L->hidden = hidden;
    L->ffn = ffn;
    const int64_t rows[3] = {ffn, ffn, hidden}, cols[3] = {hidden, hidden, ffn};
    auto a64 = [](int64_t v) { return (v + 63) & ~(int64_t)63; };
    int64_t o = 0;
    for (int m = 0; m < 3; m++) {
        int64_t db, sb;
        switch (dt) {
        case MG_F32: db = rows[m] * cols[m] * 4; sb = 0; break;
        case MG_Q8R: db = rows[m] * cols[m]; sb = rows[m] * 4; break;
        case MG_Q4G32:
        case MG_MXFP4:
        case MG_MXFP4_E8:
            MG_REQUIRE(cols[m] % 32 == 0, MG_ERR_SPEC, "expert_layout: 4-bit needs dims %% 32 == 0");
            db = rows[m] * cols[m] / 2;
            sb = rows[m] * (cols[m] / 32) * (dt == MG_MXFP4_E8 ? 1 : 2);
            break;
        default: set_error("expert_layout: bad dtype %d", dt); return MG_ERR_SPEC;
        }
        L->off[m][0] = o; o = a64(o + db);
        L->off[m][1] = o; o = a64(o + sb);
        L->off[m][2] = o; o = a64(o + rows[m] * 4);
    }
    L->expert_stride = a64(o);
    L->layer_stride = L->expert_stride * n_experts;
    return MG_OK;
}

extern "C" int mg_moe_ffn(const mg_expert_layout *L, const uint8_t *experts, int layer, int n_experts, const float *xb,
                          int n_tok, int top_k, const int32_t *sel, const float *weights, int act_plain, float alpha,
                          float limit, float *h_scratch, float *x, void *stream) {
    MG_REQUIRE(L && experts && layer >= 0, MG_ERR_ARG, "moe_ffn: bad arguments");
    MoeArgs a{};
    a.L = *L;
    a.experts_layer = experts + (int64_t)layer * L->layer_stride;
    a.n_experts = n_experts;
    a.xb = xb;
    a.n_tok = n_tok;
    a.top_k = top_k;
    a.sel = sel;
    a.weights = weights;
    a.act_plain = act_plain;
    a.alpha = alpha;
    a.limit = limit;
    a.h = h_scratch;
    a.x = x;
    a.ldx = L->hidden;
    return moe_decode(a, (cudaStream_t)stream);
}

// ------------------------------------------------------------ microbench
namespace mg {
__global__ void k_bench_fill(uint8_t *p, int64_t n, uint32_t seed) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        uint32_t h = (uint32_t)i * 2654435761u ^ seed;
        h ^= h >> 15;
        h *= 0x2c1b3c6du;
        p[i] = (uint8_t)(h >> 24);
    }
}
// scales of every copy: mxfp4 -> ue8m0 2^k, k in [-8,-4]; q4g32 -> f16 2^-4;
// q8r -> f32 1/127
__global__ void k_bench_scales(uint8_t *buf, int64_t per, int64_t soff, int64_t nsc, int copies, int dt) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nsc * copies;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t c = i / nsc, j = i - c * nsc;
        uint8_t *sp = buf + c * per + soff;
        if (dt == MG_MXFP4) sp[j] = (uint8_t)(127 - 8 + (int)(j % 5));
        else if (dt == MG_Q4G32) reinterpret_cast<uint16_t *>(sp)[j] = 0x2c00;
        else reinterpret_cast<float *>(sp)[j] = 1.0f / 127.0f;
    }
}
}  // namespace mg

extern "C" int mg_bench_gemv(int dt, int64_t rows, int64_t cols, int n_tok, double seconds, int device, double *gbps) {
    MG_REQUIRE(gbps && rows > 0 && cols > 0 && n_tok >= 1 && n_tok <= 256 &&
                   (dt == MG_MXFP4 || dt == MG_Q4G32 || dt == MG_Q8R),
               MG_ERR_ARG, "bench_gemv: bad arguments");
    MG_CUDA(cudaSetDevice(device));
    const int64_t db = dt == MG_Q8R ? rows * cols : rows * cols / 2;
    const int64_t nsc = dt == MG_Q8R ? rows : rows * (cols / 32);
    const int64_t sb_dev = dt == MG_Q8R ? rows * 4 : dt == MG_MXFP4 ? nsc : nsc * 2;  // bytes on the device
    const int64_t sb_file = dt == MG_Q8R ? rows * 4 : nsc * 2;                        // bytes in the container
    const int64_t soff = (db + 255) & ~255LL;
    const int64_t per = soff + ((sb_dev + 255) & ~255LL);
    int copies = (int)(512e6 / per) + 1;
    if (copies < 2) copies = 2;
    const int fmt = dt == MG_MXFP4 ? MG_SCALE_UE8M0 : MG_SCALE_F16;
    uint8_t *buf = nullptr;
    float *x = nullptr, *y = nullptr;
    cudaStream_t st = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    int rc = MG_OK;
    if (cudaMalloc(&buf, (size_t)per * copies) != cudaSuccess || cudaMalloc(&x, (size_t)n_tok * cols * 4) != cudaSuccess ||
        cudaMalloc(&y, (size_t)n_tok * rows * 4) != cudaSuccess ||
        cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess || cudaEventCreate(&e0) != cudaSuccess ||
        cudaEventCreate(&e1) != cudaSuccess) {
        set_error("bench_gemv: allocation failed");
        rc = MG_ERR_OOM;
    }
    float ms = 0.f;
    int64_t calls = 0;
    if (rc == MG_OK) {
        k_bench_fill<<<1184, 256, 0, st>>>(buf, per * copies, 7u);
        k_bench_scales<<<1184, 256, 0, st>>>(buf, per, soff, nsc, copies, dt);
        cudaMemsetAsync(x, 0, (size_t)n_tok * cols * 4, st);
        for (int c = 0; c < copies && rc == MG_OK; c++) {  // warm-up (also sets kernel attributes)
            uint8_t *w = buf + (int64_t)c * per;
            rc = gemv(dt, fmt, w, w + soff, rows, cols, x, cols, n_tok, nullptr, 0, y, rows, st);
        }
        // one pass over all copies captured as a graph, so the measurement is
        // the device time of back-to-back GEMVs, not the host launch rate
        cudaGraph_t g = nullptr;
        cudaGraphExec_t ge = nullptr;
        if (rc == MG_OK && cudaStreamSynchronize(st) == cudaSuccess &&
            cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
            for (int c = 0; c < copies && rc == MG_OK; c++) {
                uint8_t *w = buf + (int64_t)c * per;
                rc = gemv(dt, fmt, w, w + soff, rows, cols, x, cols, n_tok, nullptr, 0, y, rows, st);
            }
            if (cudaStreamEndCapture(st, &g) != cudaSuccess || rc != MG_OK ||
                cudaGraphInstantiate(&ge, g, 0) != cudaSuccess) {
                if (rc == MG_OK) { set_error("bench_gemv: graph capture failed"); rc = MG_ERR_CUDA; }
            }
        }
        while (rc == MG_OK && ms < seconds * 1e3) {
            cudaEventRecord(e0, st);
            cudaGraphLaunch(ge, st);
            cudaEventRecord(e1, st);
            if (cudaEventSynchronize(e1) != cudaSuccess) {
                set_error("bench_gemv: kernel failed");
                rc = MG_ERR_CUDA;
                break;
            }
            float t = 0.f;
            cudaEventElapsedTime(&t, e0, e1);
            ms += t;
            calls += copies;
        }
        if (ge) cudaGraphExecDestroy(ge);
        if (g) cudaGraphDestroy(g);
    }
    if (rc == MG_OK) *gbps = (double)calls * (db + sb_file) / (ms * 1e-3) / (1024.0 * 1024.0 * 1024.0);
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    cudaFree(buf);
    cudaFree(x);
    cudaFree(y);
    if (st) cudaStreamDestroy(st);
    return rc;
}
