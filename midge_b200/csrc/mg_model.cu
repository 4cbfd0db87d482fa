// mg_model.cu -- the model behind mg_model: HBM-resident trunk and experts,
// f16 KV cache, and the decode / expert-major prefill passes built from the
// kernels of mg_gemv.cu, mg_moe.cu and mg_attn.cu.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>

#include "mg_attn.h"
#include "mg_common.cuh"
#include "mg_kernels.h"
#include "mg_model.h"
#include "mg_ep_xchg.h"
#include "mg_prefill.h"

using mg::DevMat;

namespace mg {

// ----------------------------------------------------------- small kernels
// first maximum of each row (engine/midge.c:657-660: strict >, so ties keep
// the lowest index; a NaN never compares greater)
__global__ void k_argmax(const float *__restrict__ logits, int64_t V, int32_t *out) {
    __shared__ float sv[32];
    __shared__ int si[32];
    const float *l = logits + (int64_t)blockIdx.x * V;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int64_t i = threadIdx.x; i < V; i += blockDim.x) {
        float v = l[i];
        if (v > bv || (bi == 0x7fffffff && !(v != v))) { bv = v; bi = (int)i; }
    }
    for (int o = 16; o > 0; o >>= 1) {
        float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (lane == 0) { sv[w] = bv; si[w] = bi; }
    __syncthreads();
    if (w == 0) {
        int nw = blockDim.x >> 5;
        bv = lane < nw ? sv[lane] : -INFINITY;
        bi = lane < nw ? si[lane] : 0x7fffffff;
        for (int o = 16; o > 0; o >>= 1) {
            float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) {
            // the reference starts from element 0: a NaN there is never replaced
            float l0 = l[0];
            out[blockIdx.x] = (l0 != l0 || bi == 0x7fffffff) ? 0 : bi;
        }
    }
}

// Sliding layers after a prefill chunk: the last min(n, cap) tokens' f16 K/V
// go to their ring slots.
// Greedy chaining on the device: the argmax of the step just run becomes
// the next step's token (recorded in out[step]); positions advance by one.
// keys: the fused lm_head argmax (value << 32 | ~index, 0 = no finite
// maximum -> token 0); else amax holds the indices.
__global__ void k_advance(const unsigned long long *keys, const int32_t *amax, int n, int32_t *toks, int32_t *tok_pos,
                          int32_t *out, int32_t *step) {
    const int i = threadIdx.x;
    const int s = *step;
    if (i < n) {
        int32_t t;
        if (keys) {
            const unsigned long long k = keys[i];
            t = k ? (int32_t)(0xffffffffu - (uint32_t)(k & 0xffffffffull)) : 0;
        } else {
            t = amax[i];
        }
        toks[i] = t;
        tok_pos[i] += 1;
        out[(int64_t)s * n + i] = t;
    }
    __syncthreads();
    if (i == 0) *step = s + 1;
}

__global__ void k_ring_store(const uint16_t *__restrict__ tk, const uint16_t *__restrict__ tv, int n, int pos0,
                             int cap, int kv_dim, uint16_t *kc, uint16_t *vc) {
    int first = n > cap ? n - cap : 0;
    int t = first + blockIdx.x;
    if (t >= n) return;
    int slot = (pos0 + t) % cap;
    for (int i = threadIdx.x; i < kv_dim; i += blockDim.x) {
        kc[(int64_t)slot * kv_dim + i] = tk[(int64_t)t * kv_dim + i];
        vc[(int64_t)slot * kv_dim + i] = tv[(int64_t)t * kv_dim + i];
    }
}

// ---- seeded synthetic expert weights (benchmarks of shapes too big for a file)
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
__device__ __forceinline__ float gauss(uint64_t h) {  // Box-Muller from one hash
    float u1 = ((uint32_t)(h >> 40) + 1) * (1.0f / 16777217.0f);
    float u2 = (uint32_t)(h & 0xffffff) * (1.0f / 16777216.0f);
    return sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

// part: 0 = data, 1 = scales, 2 = bias of matrix `mat`, for every (layer, expert)
// le runs over the local blob (n_local experts per layer); the seed uses the
// global (layer, expert) index so that every rank of an expert-parallel run
// holds exactly its shard of the same model
__global__ void k_synth_part(uint8_t *base, int64_t expert_stride, int64_t n_le, int64_t off, int64_t bytes, int part,
                             int dt, int64_t rows, int64_t cols, uint64_t seed, int n_local, int e0, int n_experts) {
    for (int64_t le = blockIdx.y; le < n_le; le += gridDim.y) {
        uint8_t *p = base + le * expert_stride + off;
        const int64_t lg = (le / n_local) * n_experts + e0 + le % n_local;
        uint64_t s0 = mix64(seed ^ (uint64_t)(lg * 9 + part * 3 + off));
        if (part == 0) {
            for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8; i < bytes;
                 i += (int64_t)gridDim.x * blockDim.x * 8) {
                uint64_t h = mix64(s0 + (uint64_t)i);
                if (dt == MG_Q8R) {  // int8 uniform in [-127, 127]
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        uint32_t r = (uint32_t)((h >> (8 * j)) & 0xff);
                        int v = (int)((r * 255u) >> 8) - 127;  // 0..254 -> -127..127
                        if (i + j < bytes) p[i + j] = (uint8_t)(int8_t)v;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 8; j++)
                        if (i + j < bytes) p[i + j] = (uint8_t)(h >> (8 * j));
                }
            }
        } else if (part == 1) {
            if (dt == MG_Q8R) {  // f32 row scales: 2^round(log2(1/(127 sqrt(cols))))
                float s = exp2f(rintf(log2f(1.0f / (127.0f * sqrtf((float)cols)))));
                for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows; i += (int64_t)gridDim.x * blockDim.x)
                    reinterpret_cast<float *>(p)[i] = s;
            } else {  // f16 2^k, k uniform in [-8, -4]
                for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < bytes / 2;
                     i += (int64_t)gridDim.x * blockDim.x) {
                    uint64_t h = mix64(s0 + (uint64_t)i);
                    int k = -8 + (int)(h % 5);
                    reinterpret_cast<uint16_t *>(p)[i] = (uint16_t)((k + 15) << 10);
                }
            }
        } else {
            for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows; i += (int64_t)gridDim.x * blockDim.x)
                reinterpret_cast<float *>(p)[i] = 0.1f * gauss(mix64(s0 + (uint64_t)i));
        }
    }
}

// Re-express one layer's scale blobs: pass over (expert, mat) blobs into a
// temp, then copy back into the first half of each blob.
__global__ void k_layer_scales(uint8_t *layer, int64_t expert_stride, int n_experts, int64_t off0, int64_t n0,
                               int64_t off1, int64_t n1, int64_t off2, int64_t n2, uint8_t *tmp, int to_tmp,
                               int *bad) {
    int e = blockIdx.y;
    int64_t tot = n0 + n1 + n2;
    uint8_t *eb = layer + (int64_t)e * expert_stride;
    uint8_t *te = tmp + (int64_t)e * tot;
    int local_bad = 0;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < tot; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t off, j;
        if (i < n0) { off = off0; j = i; }
        else if (i < n0 + n1) { off = off1; j = i - n0; }
        else { off = off2; j = i - n0 - n1; }
        if (to_tmp) {
            uint32_t hb = reinterpret_cast<const uint16_t *>(eb + off)[j];
            uint32_t ex = (hb >> 10) & 31u, man = hb & 1023u;
            uint8_t u = 0;
            if (hb == 0) u = 0;
            else if (hb & 0x8000u) local_bad++;
            else if (ex == 0) { if (__popc(man) == 1) u = (uint8_t)(103 + (31 - __clz(man))); else local_bad++; }
            else if (ex == 31 || man != 0) local_bad++;
            else u = (uint8_t)(ex + 112);
            te[i] = u;
        } else {
            eb[off + j] = te[i];
        }
    }
    if (to_tmp && local_bad) atomicAdd(bad, local_bad);
}

// Check only: count scales that are not a zero or positive power of two.
__global__ void k_layer_scales_check(const uint8_t *base, int64_t expert_stride, int64_t n_le, int64_t off, int64_t n,
                                     int *bad) {
    int local_bad = 0;
    for (int64_t le = blockIdx.y; le < n_le; le += gridDim.y) {
        const uint16_t *s = reinterpret_cast<const uint16_t *>(base + le * expert_stride + off);
        for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
            uint32_t hb = s[i], ex = (hb >> 10) & 31u, man = hb & 1023u;
            bool ok = hb == 0 || (!(hb & 0x8000u) && ((ex == 0 && __popc(man) == 1) || (ex != 0 && ex != 31 && man == 0)));
            local_bad += !ok;
        }
    }
    if (local_bad) atomicAdd(bad, local_bad);
}

}  // namespace mg

// ===================================================================== model
using namespace mg;

template <typename T>
static int dalloc(mg_model *m, T **p, size_t bytes) {
    void *q = nullptr;
    cudaError_t e = cudaMalloc(&q, bytes ? bytes : 16);
    if (e != cudaSuccess) {
        set_error("cudaMalloc(%zu) failed: %s", bytes, cudaGetErrorString(e));
        return MG_ERR_OOM;
    }
    m->allocs.push_back(q);
    *p = reinterpret_cast<T *>(q);
    return MG_OK;
}



extern "C" int mg_model_create(const mg_spec *spec, int ctx, int max_seqs, int device, mg_model **out) {
    MG_REQUIRE(spec && out, MG_ERR_ARG, "model_create: null argument");
    *out = nullptr;
    const mg_spec &s = *spec;
    MG_REQUIRE(s.hidden > 0 && s.vocab > 0 && s.n_layers > 0 && s.ffn > 0 && s.n_experts > 0 && s.top_k > 0,
               MG_ERR_SPEC, "invalid spec");  // engine/midge.c:135-137
    MG_REQUIRE(s.top_k <= 16 && s.top_k <= s.n_experts, MG_ERR_SPEC, "top_k %d unsupported", s.top_k);
    MG_REQUIRE(s.n_heads > 0 && s.n_kv_heads > 0 && s.n_heads % s.n_kv_heads == 0 && s.head_dim > 0 &&
                   s.head_dim % 2 == 0,
               MG_ERR_SPEC, "invalid attention shape");
    MG_REQUIRE(ctx > 0 && max_seqs >= 1 && max_seqs <= 64, MG_ERR_ARG, "bad ctx %d / max_seqs %d", ctx, max_seqs);
    MG_CUDA(cudaSetDevice(device));
    mg_model *m = new mg_model();
    m->spec = s;
    m->layer_sliding.assign(s.layer_sliding, s.layer_sliding ? s.layer_sliding + s.n_layers : nullptr);
    if (!s.layer_sliding) m->layer_sliding.assign(s.n_layers, 0);
    m->spec.layer_sliding = m->layer_sliding.data();
    m->ctx = ctx;
    m->max_seqs = max_seqs;
    m->device = device;
    cudaError_t e = cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        delete m;
        set_error("stream create: %s", cudaGetErrorString(e));
        return MG_ERR_CUDA;
    }
    int L = s.n_layers;
    m->wq.resize(L); m->wk.resize(L); m->wv.resize(L); m->wo.resize(L); m->router_w.resize(L);
    for (auto *vec : {&m->bq, &m->bk, &m->bv, &m->bo, &m->router_b, &m->attn_norm, &m->mlp_norm, &m->sinks, &m->qn, &m->kn})
        vec->assign(L, nullptr);
    m->pos.assign(max_seqs, 0);
    m->e0 = 0;
    m->n_local = s.n_experts;
    const char *ng = getenv("MIDGE_NO_GRAPH");
    m->use_graphs = !(ng && *ng && *ng != '0');
    const char *ns = getenv("MIDGE_DECODE_KERNELS");
    m->use_stream = !(ns && !strcmp(ns, "tile"));
    const char *ak = getenv("MIDGE_ATTN_KERNELS");
    m->tc_attn = !(ak && !strcmp(ak, "scalar"));
    const char *mk = getenv("MIDGE_MOE_KERNELS");
    m->bs_moe = !(mk && !strcmp(mk, "mma"));  // where the format allows (set in ready)
    const char *pd = getenv("MIDGE_PDL");
    m->pdl = !(pd && !strcmp(pd, "0"));
    const char *as = getenv("MIDGE_ATTN_SPLIT");
    if (as && *as) {  // positions per decode-attention split: a multiple of 64, 64..1024
        int v = atoi(as);
        m->attn_split = v < 64 ? 64 : (v > 1024 ? 1024 : v / 64 * 64);
    }
    const char *pk = getenv("MIDGE_PREFILL_KERNELS");
    m->tc_prefill = !(pk && !strcmp(pk, "tile"));
    const char *pc = getenv("MIDGE_PREFILL_CHUNK");
    if (pc && *pc) {
        int v = atoi(pc);
        m->pf_chunk = v < DEC_MAX ? DEC_MAX : (v > 4096 ? 4096 : v);
    }
    *out = m;
    return MG_OK;
}

static int upload(mg_model *m, void **dst, const void *src, size_t bytes) {
    TRY(dalloc(m, dst, bytes));
    MG_CUDA(cudaMemcpy(*dst, src, bytes, cudaMemcpyHostToDevice));
    return MG_OK;
}

extern "C" int mg_model_set_dense(mg_model *m, const char *name, int dt, int64_t rows, int64_t cols, const void *data,
                                  const void *scales) {
    MG_REQUIRE(m && name && data && rows > 0, MG_ERR_ARG, "set_dense: bad arguments");
    MG_CUDA(cudaSetDevice(m->device));
    DevMat d;
    d.dt = dt;
    d.rows = rows;
    d.cols = cols;
    size_t db = 0, sb = 0;
    if (cols == 0) {
        MG_REQUIRE(dt == MG_F32, MG_ERR_SPEC, "tensor %s must be f32", name);  // engine/midge.c:196
        db = (size_t)rows * 4;
    } else {
        switch (dt) {
        case MG_F32: db = (size_t)rows * cols * 4; break;
        case MG_Q8R: db = (size_t)rows * cols; sb = (size_t)rows * 4; break;
        case MG_Q4G32:
        case MG_MXFP4:
            MG_REQUIRE(cols % 32 == 0, MG_ERR_SPEC, "tensor %s: cols %% 32 != 0", name);
            db = (size_t)rows * cols / 2;
            sb = (size_t)rows * (cols / 32) * 2;
            break;
        default: set_error("tensor %s: unknown dtype %d", name, dt); return MG_ERR_SPEC;
        }
        MG_REQUIRE(sb == 0 || scales, MG_ERR_ARG, "tensor %s: scales missing", name);
    }
    TRY(upload(m, &d.data, data, db));
    if (sb) TRY(upload(m, &d.scales, scales, sb));
    std::string n(name);
    if (n == "embed") { m->embed = d; return MG_OK; }
    if (n == "lm_head") { m->lm_head = d; return MG_OK; }
    if (n == "final_norm") { m->final_norm = (float *)d.data; return MG_OK; }
    int layer = -1;
    char rest[64] = {0};
    if (sscanf(name, "L%d.%63s", &layer, rest) != 2 || layer < 0 || layer >= m->spec.n_layers) {
        return MG_OK;  // unknown tensors are ignored, as the reference never looks them up
    }
    std::string r(rest);
    if (r == "attn.q") m->wq[layer] = d;
    else if (r == "attn.k") m->wk[layer] = d;
    else if (r == "attn.v") m->wv[layer] = d;
    else if (r == "attn.o") m->wo[layer] = d;
    else if (r == "router.w") {
        MG_REQUIRE(dt == MG_F32, MG_ERR_SPEC, "router %s must be f32", name);
        m->router_w[layer] = d;
    } else if (r == "attn.q_b") m->bq[layer] = (float *)d.data;
    else if (r == "attn.k_b") m->bk[layer] = (float *)d.data;
    else if (r == "attn.v_b") m->bv[layer] = (float *)d.data;
    else if (r == "attn.o_b") m->bo[layer] = (float *)d.data;
    else if (r == "router.b") m->router_b[layer] = (float *)d.data;
    else if (r == "attn.norm") m->attn_norm[layer] = (float *)d.data;
    else if (r == "mlp.norm") m->mlp_norm[layer] = (float *)d.data;
    else if (r == "attn.sinks") m->sinks[layer] = (float *)d.data;
    else if (r == "attn.q_norm") m->qn[layer] = (float *)d.data;
    else if (r == "attn.k_norm") m->kn[layer] = (float *)d.data;
    return MG_OK;
}

static int convert_expert_scales(mg_model *m) {
    mg_expert_layout &L = m->el;
    if (L.scale_fmt == MG_SCALE_UE8M0) return MG_OK;  // an "mxfp4e8" container: already ue8m0 bytes
    if (L.dt != MG_MXFP4 && L.dt != MG_Q4G32) return MG_OK;
    const char *keep = getenv("MIDGE_F16_SCALES");
    if (keep && *keep && *keep != '0') return MG_OK;
    int64_t ns[3];
    for (int mt = 0; mt < 3; mt++) {
        int64_t rows = mt == 2 ? L.hidden : L.ffn, cols = mt == 2 ? L.ffn : L.hidden;
        ns[mt] = rows * (cols / 32);
    }
    int *bad = nullptr;
    TRY(dalloc(m, &bad, sizeof(int)));
    MG_CUDA(cudaMemsetAsync(bad, 0, sizeof(int), m->st));
    int64_t n_le = (int64_t)m->spec.n_layers * m->n_local;
    for (int mt = 0; mt < 3; mt++) {
        dim3 g(64, (unsigned)(n_le < 4096 ? n_le : 4096));
        k_layer_scales_check<<<g, 256, 0, m->st>>>(m->experts, L.expert_stride, n_le, L.off[mt][1], ns[mt], bad);
        MG_CHECK_LAUNCH();
    }
    int h_bad = 0;
    MG_CUDA(cudaMemcpyAsync(&h_bad, bad, sizeof(int), cudaMemcpyDeviceToHost, m->st));
    MG_CUDA(cudaStreamSynchronize(m->st));
    if (h_bad) {
        fprintf(stderr, "# %d expert scales are not powers of two: keeping f16 scales\n", h_bad);
        return MG_OK;
    }
    int64_t per_expert = ns[0] + ns[1] + ns[2];
    uint8_t *tmp = nullptr;
    void *tmpv = nullptr;
    MG_CUDA(cudaMalloc(&tmpv, (size_t)per_expert * m->n_local));
    tmp = (uint8_t *)tmpv;
    for (int layer = 0; layer < m->spec.n_layers; layer++) {
        uint8_t *lb = m->experts + (int64_t)layer * L.layer_stride;
        dim3 g(32, m->n_local);
        for (int pass = 1; pass >= 0; pass--) {
            k_layer_scales<<<g, 256, 0, m->st>>>(lb, L.expert_stride, m->n_local, L.off[0][1], ns[0], L.off[1][1],
                                                 ns[1], L.off[2][1], ns[2], tmp, pass, bad);
        }
    }
    cudaError_t e = cudaGetLastError();
    cudaError_t e2 = cudaStreamSynchronize(m->st);
    cudaFree(tmpv);
    if (e != cudaSuccess || e2 != cudaSuccess) {
        set_error("scale re-expression failed: %s", cudaGetErrorString(e != cudaSuccess ? e : e2));
        return MG_ERR_CUDA;
    }
    L.scale_fmt = MG_SCALE_UE8M0;
    return MG_OK;
}

static int experts_alloc(mg_model *m, int dt) {
    const mg_spec &s = m->spec;
    TRY(mg_expert_layout_init(&m->el, dt, s.hidden, s.ffn, m->n_local));
    m->experts_bytes = (size_t)s.n_layers * m->el.layer_stride;
    MG_REQUIRE(!m->experts, MG_ERR_STATE, "experts already loaded");
    TRY(dalloc(m, &m->experts, m->experts_bytes));
    return MG_OK;
}

extern "C" int mg_ep_unique_id(void *id) { return ep_unique_id(id); }

extern "C" int mg_model_set_ep(mg_model *m, int rank, int world, const void *id) {
    MG_REQUIRE(m && !m->experts && !m->ready, MG_ERR_STATE, "set_ep: call after create, before the experts");
    MG_REQUIRE(world >= 1 && rank >= 0 && rank < world && (world == 1 || id), MG_ERR_ARG, "set_ep: bad arguments");
    MG_REQUIRE(m->spec.n_experts % world == 0, MG_ERR_SPEC, "set_ep: %d experts do not split over %d ranks",
               m->spec.n_experts, world);
    MG_CUDA(cudaSetDevice(m->device));
    TRY(ep_init(&m->ep, rank, world, id));
    ep_range(m->spec.n_experts, world, rank, &m->e0, &m->n_local);
    return MG_OK;
}

extern "C" int mg_model_set_experts(mg_model *m, int dt, const void *data, uint64_t bytes) {
    MG_REQUIRE(m && data, MG_ERR_ARG, "set_experts: bad arguments");
    MG_CUDA(cudaSetDevice(m->device));
    TRY(experts_alloc(m, dt));
    // the blob holds every expert; this rank uploads its shard of each layer
    const int64_t full_layer = m->el.expert_stride * m->spec.n_experts;
    const size_t full_bytes = (size_t)m->spec.n_layers * full_layer;
    MG_REQUIRE(bytes >= full_bytes, MG_ERR_SPEC, "experts.midge too small: need %zu data bytes",
               full_bytes);  // engine/midge.c:224-227
    const size_t seg = (size_t)m->el.layer_stride;  // local bytes per layer
    auto src_of = [&](size_t dst_off) {
        const size_t layer = dst_off / seg, in = dst_off % seg;
        return (size_t)layer * full_layer + (size_t)m->e0 * m->el.expert_stride + in;
    };
    // pinned double-buffered staging; the host copy into a stage overlaps the
    // DMA of the other
    const size_t CH = 64ull << 20;
    void *stage[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    int rc = MG_OK;
    for (int i = 0; i < 2 && rc == MG_OK; i++) {
        if (cudaHostAlloc(&stage[i], CH, cudaHostAllocDefault) != cudaSuccess ||
            cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming) != cudaSuccess) {
            set_error("pinned staging allocation failed");
            rc = MG_ERR_OOM;
        }
    }
    const uint8_t *src = (const uint8_t *)data;
    size_t off = 0;
    int b = 0;
    while (rc == MG_OK && off < m->experts_bytes) {
        size_t n = m->experts_bytes - off < CH ? m->experts_bytes - off : CH;
        if (n > seg - off % seg) n = seg - off % seg;  // a copy never crosses a layer of the local blob
        if (cudaEventSynchronize(done[b]) != cudaSuccess) { rc = MG_ERR_CUDA; break; }
        memcpy(stage[b], src + src_of(off), n);
        if (cudaMemcpyAsync(m->experts + off, stage[b], n, cudaMemcpyHostToDevice, m->st) != cudaSuccess ||
            cudaEventRecord(done[b], m->st) != cudaSuccess) {
            set_error("expert upload failed");
            rc = MG_ERR_CUDA;
            break;
        }
        off += n;
        b ^= 1;
    }
    cudaStreamSynchronize(m->st);
    for (int i = 0; i < 2; i++) {
        if (stage[i]) cudaFreeHost(stage[i]);
        if (done[i]) cudaEventDestroy(done[i]);
    }
    if (rc != MG_OK) return rc;
    return convert_expert_scales(m);
}

extern "C" int mg_model_synth_experts(mg_model *m, int dt, uint64_t seed) {
    MG_REQUIRE(m, MG_ERR_ARG, "synth_experts: null model");
    MG_REQUIRE(dt == MG_MXFP4 || dt == MG_Q8R || dt == MG_Q4G32, MG_ERR_ARG, "synth_experts: dtype %d unsupported", dt);
    MG_CUDA(cudaSetDevice(m->device));
    TRY(experts_alloc(m, dt));
    const mg_expert_layout &L = m->el;
    int64_t n_le = (int64_t)m->spec.n_layers * m->n_local;
    for (int mt = 0; mt < 3; mt++) {
        int64_t rows = mt == 2 ? L.hidden : L.ffn, cols = mt == 2 ? L.ffn : L.hidden;
        int64_t db = dt == MG_Q8R ? rows * cols : rows * cols / 2;
        int64_t sb = dt == MG_Q8R ? rows * 4 : rows * (cols / 32) * 2;
        int64_t bb = rows * 4;
        int64_t sizes[3] = {db, sb, bb};
        for (int part = 0; part < 3; part++) {
            dim3 g(16, (unsigned)(n_le < 8192 ? n_le : 8192));
            k_synth_part<<<g, 256, 0, m->st>>>(m->experts, L.expert_stride, n_le, L.off[mt][part], sizes[part], part, dt,
                                               rows, cols, seed + (uint64_t)mt * 7919u, m->n_local, m->e0,
                                               m->spec.n_experts);
            MG_CHECK_LAUNCH();
        }
    }
    MG_CUDA(cudaStreamSynchronize(m->st));
    return convert_expert_scales(m);
}

// YaRN rope tables in double precision, the arithmetic of engine/midge.c:141-176
static void rope_tables(const mg_spec &s, int ctx, std::vector<float> &co, std::vector<float> &si) {
    int hd = s.head_dim, half = hd / 2;
    std::vector<double> inv(half);
    double mscale = 1.0;
    for (int i = 0; i < half; i++) inv[i] = 1.0 / pow((double)s.rope_theta, (double)(2 * i) / hd);
    if (s.yarn) {
        double f = s.yarn_factor, base = s.rope_theta, orig = s.yarn_orig_ctx;
        double low = hd * log(orig / (s.yarn_beta_fast * 2.0 * M_PI)) / (2.0 * log(base));
        double high = hd * log(orig / (s.yarn_beta_slow * 2.0 * M_PI)) / (2.0 * log(base));
        if (s.yarn_truncate) { low = floor(low); high = ceil(high); }
        if (low < 0) low = 0;
        if (high > hd - 1) high = hd - 1;
        if (high == low) high = low + 0.001;
        for (int i = 0; i < half; i++) {
            double ramp = ((double)i - low) / (high - low);
            ramp = ramp < 0 ? 0 : ramp > 1 ? 1 : ramp;
            double keep = 1.0 - ramp;  // 1 keeps the unscaled (high-frequency) rate
            inv[i] = (inv[i] / f) * (1.0 - keep) + inv[i] * keep;
        }
        mscale = 0.1 * log(f) + 1.0;
    }
    co.resize((size_t)ctx * half);
    si.resize((size_t)ctx * half);
    for (int p = 0; p < ctx; p++)
        for (int i = 0; i < half; i++) {
            double a = (double)p * inv[i];
            co[(size_t)p * half + i] = (float)(cos(a) * mscale);
            si[(size_t)p * half + i] = (float)(sin(a) * mscale);
        }
}

static int prefill_prepare(mg_model *m);
static int rebase_prepare(mg_model *m);
static int ep_prepare(mg_model *m);

extern "C" int mg_model_ready(mg_model *m) {
    MG_REQUIRE(m, MG_ERR_ARG, "ready: null model");
    MG_CUDA(cudaSetDevice(m->device));
    const mg_spec &s = m->spec;
    // every tensor the reference requires (engine/midge.c:229-260)
    MG_REQUIRE(m->embed.data && m->lm_head.data && m->final_norm, MG_ERR_SPEC, "missing embed/lm_head/final_norm");
    MG_REQUIRE(m->experts, MG_ERR_SPEC, "experts not loaded");
    for (int l = 0; l < s.n_layers; l++) {
        MG_REQUIRE(m->wq[l].data && m->wk[l].data && m->wv[l].data && m->wo[l].data && m->router_w[l].data,
                   MG_ERR_SPEC, "missing tensor L%d.attn.{q,k,v,o} / router.w", l);
        MG_REQUIRE(m->bq[l] && m->bk[l] && m->bv[l] && m->bo[l] && m->router_b[l] && m->attn_norm[l] && m->mlp_norm[l],
                   MG_ERR_SPEC, "missing tensor L%d bias/norm", l);
        MG_REQUIRE(!s.sinks || m->sinks[l], MG_ERR_SPEC, "missing tensor L%d.attn.sinks", l);
        MG_REQUIRE(!s.qk_norm || (m->qn[l] && m->kn[l]), MG_ERR_SPEC, "missing tensor L%d.attn.q_norm/k_norm", l);
        MG_REQUIRE(m->router_w[l].rows == s.n_experts && m->router_w[l].cols == s.hidden, MG_ERR_SPEC,
                   "router L%d shape", l);
    }
    std::vector<float> co, si;
    rope_tables(s, m->ctx, co, si);
    TRY(upload(m, (void **)&m->rope_cos, co.data(), co.size() * 4));
    TRY(upload(m, (void **)&m->rope_sin, si.data(), si.size() * 4));
    const int kv_dim = s.n_kv_heads * s.head_dim, q_dim = s.n_heads * s.head_dim;
    m->kc.resize(s.n_layers);
    m->vc.resize(s.n_layers);
    m->cap.resize(s.n_layers);
    for (int l = 0; l < s.n_layers; l++) {  // engine/midge.c:268-273
        int c = m->layer_sliding[l] && s.sliding_window > 0 && s.sliding_window < m->ctx ? s.sliding_window : m->ctx;
        m->cap[l] = c;
        TRY(dalloc(m, &m->kc[l], (size_t)m->max_seqs * c * kv_dim * 2));
        TRY(dalloc(m, &m->vc[l], (size_t)m->max_seqs * c * kv_dim * 2));
        MG_CUDA(cudaMemset(m->kc[l], 0, (size_t)m->max_seqs * c * kv_dim * 2));
        MG_CUDA(cudaMemset(m->vc[l], 0, (size_t)m->max_seqs * c * kv_dim * 2));
    }
    if (m->pf_chunk > m->ctx) m->pf_chunk = m->ctx;  // a chunk never exceeds the context
    if (m->pf_chunk < DEC_MAX) m->pf_chunk = DEC_MAX;
    const int R = m->pf_chunk;
    m->rows_max = R;
    const int64_t H = s.hidden;
    TRY(dalloc(m, &m->x, (size_t)R * H * 4));
    TRY(dalloc(m, &m->xb, (size_t)R * H * 4));
    TRY(dalloc(m, &m->q, (size_t)R * q_dim * 4));
    TRY(dalloc(m, &m->k, (size_t)R * kv_dim * 4));
    TRY(dalloc(m, &m->v, (size_t)R * kv_dim * 4));
    TRY(dalloc(m, &m->ao, (size_t)R * q_dim * 4));
    TRY(dalloc(m, &m->h, (size_t)R * s.top_k * s.ffn * 4));
    TRY(dalloc(m, &m->logits, (size_t)DEC_MAX * s.vocab * 4));
    TRY(dalloc(m, &m->wts, (size_t)R * s.top_k * 4));
    TRY(dalloc(m, &m->sel, (size_t)R * s.top_k * 4));
    TRY(dalloc(m, &m->tok_pos, (size_t)R * 4));
    TRY(dalloc(m, &m->tok_seq, (size_t)R * 4));
    TRY(dalloc(m, &m->toks, (size_t)R * 4));
    TRY(dalloc(m, &m->amax, (size_t)DEC_MAX * 4));
    TRY(dalloc(m, &m->tmp_k, (size_t)R * kv_dim * 2));
    TRY(dalloc(m, &m->tmp_v, (size_t)R * kv_dim * 2));
    TRY(dalloc(m, &m->usage, (size_t)s.n_layers * s.n_experts * 4));
    MG_CUDA(cudaMemset(m->usage, 0, (size_t)s.n_layers * s.n_experts * 4));
    // streamed decode buffers.  K splits: about one unit (row tile x split)
    // per SM; a unit's fixed cost (the two warps' hand-over, epilogue and the
    // next unit's first wait, ~2 us measured at 8 tokens) outweighs its share
    // of the weight stream when a CTA takes several short units.
    const int qkv_dim = q_dim + 2 * kv_dim;
    const int tiles_qkv = (int)((q_dim + 127) / 128 + 2 * ((kv_dim + 127) / 128)), tiles_o = (int)((H + 127) / 128);
    m->ks_qkv = stream_ksplit(MG_Q8R, H, std::max(1, num_sms() / tiles_qkv));
    m->ks_o = stream_ksplit(MG_Q8R, q_dim, std::max(1, num_sms() / tiles_o));
    m->ks_down = moe_down_ksplit(m->el, 2);
    MG_CUDA(cudaHostAlloc(&m->h_err, sizeof(int), cudaHostAllocDefault));
    *m->h_err = 0;
    TRY(dalloc(m, &m->qkv, (size_t)DEC_MAX * qkv_dim * 4));
    TRY(dalloc(m, &m->qkv_part, (size_t)m->ks_qkv * DEC_MAX * qkv_dim * 4));
    TRY(dalloc(m, &m->o_part, (size_t)m->ks_o * DEC_MAX * H * 4));
    TRY(dalloc(m, &m->moe_y, (size_t)m->ks_down * DEC_MAX * s.top_k * H * 4));
    TRY(dalloc(m, &m->rlogits, (size_t)R * s.n_experts * 4));  // decode and prefill router logits
    TRY(dalloc(m, &m->rticket, 16));
    MG_CUDA(cudaMemset(m->rticket, 0, 16));
    TRY(dalloc(m, &m->xa, (size_t)DEC_MAX * H * 4));
    TRY(dalloc(m, &m->amax_keys, (size_t)DEC_MAX * 8));
    MG_CUDA(cudaHostAlloc(&m->h_keys, DEC_MAX * 8, cudaHostAllocDefault));
    TRY(stream_prepare());
    // TMA maps for the streamed decode (q8r trunk, any 4-bit/int8 experts)
    m->maps_ok = false;
    {
        bool q8 = m->lm_head.dt == MG_Q8R;
        for (int l = 0; l < s.n_layers; l++)
            q8 = q8 && m->wq[l].dt == MG_Q8R && m->wk[l].dt == MG_Q8R && m->wv[l].dt == MG_Q8R && m->wo[l].dt == MG_Q8R;
        const bool ex = m->el.dt == MG_MXFP4 || m->el.dt == MG_Q4G32 || m->el.dt == MG_Q8R;
        if (q8 && ex) {
            m->map_q.resize(s.n_layers); m->map_k.resize(s.n_layers); m->map_v.resize(s.n_layers); m->map_o.resize(s.n_layers);
            for (int l = 0; l < s.n_layers; l++) {
                TRY(map_weights_2d(&m->map_q[l], m->wq[l].data, m->wq[l].cols, m->wq[l].rows, 128));
                TRY(map_weights_2d(&m->map_k[l], m->wk[l].data, m->wk[l].cols, m->wk[l].rows, 128));
                TRY(map_weights_2d(&m->map_v[l], m->wv[l].data, m->wv[l].cols, m->wv[l].rows, 128));
                TRY(map_weights_2d(&m->map_o[l], m->wo[l].data, m->wo[l].cols, m->wo[l].rows, 128));
            }
            TRY(map_weights_2d(&m->map_lm, m->lm_head.data, m->lm_head.cols, m->lm_head.rows, 128));
            const mg_expert_layout &L = m->el;
            const int64_t rb_in = L.dt == MG_Q8R ? L.hidden : L.hidden / 2;
            const int64_t rb_dn = L.dt == MG_Q8R ? L.ffn : L.ffn / 2;
            TRY(map_weights_4d(&m->map_ex[0], m->experts + L.off[0][0], rb_in, L.ffn, m->n_local, s.n_layers,
                               L.expert_stride, L.layer_stride, 64));
            TRY(map_weights_4d(&m->map_ex[1], m->experts + L.off[1][0], rb_in, L.ffn, m->n_local, s.n_layers,
                               L.expert_stride, L.layer_stride, 64));
            TRY(map_weights_4d(&m->map_ex[2], m->experts + L.off[2][0], rb_dn, L.hidden, m->n_local, s.n_layers,
                               L.expert_stride, L.layer_stride, 128));
            m->maps_ok = true;
        }
    }
    // block-scaled decode MoE: activation limb buffers and their maps
    if (m->bs_moe && m->maps_ok && bsmoe_supported(m->el) && s.top_k <= 16) {
        BsBuffers &b = m->bs;
        b.kpad_h = bs_kpad(H);
        b.kpad_f = bs_kpad(m->el.ffn);
        b.slots_max = 8 * s.top_k;
        TRY(dalloc(m, &b.xl, bs_limb_bytes(8, b.kpad_h)));
        TRY(dalloc(m, &b.xsf, bs_word_bytes(8, b.kpad_h)));
        TRY(dalloc(m, &b.hl, bs_limb_bytes(b.slots_max, b.kpad_f)));
        TRY(dalloc(m, &b.hsf, bs_word_bytes(b.slots_max, b.kpad_f)));
        TRY(dalloc(m, &b.sync, bs_sync_bytes()));
        TRY(bs_buffers_init(b));
        // the experts' scales as the tensor core reads them (one atom copy)
        TRY(dalloc(m, &b.atoms, (size_t)s.n_layers * m->n_local * bs_atoms_bytes(m->el, b.kpad_h, b.kpad_f)));
        TRY(bs_atoms_build(b, m->el, m->experts, s.n_layers, m->n_local, m->st));
        // the block-scaled down pass runs whole rows per unit: one partial
        // plane (moe_y was sized for the streamed kernels' two)
        m->ks_down = 1;
    } else {
        m->bs_moe = false;
    }
    m->attn_max_splits = (m->ctx + m->attn_split - 1) / m->attn_split;
    TRY(dalloc(m, &m->attn_part, (size_t)DEC_MAX * s.n_heads * m->attn_max_splits * (s.head_dim + 2) * 4));
    MG_CUDA(cudaHostAlloc(&m->h_toks, R * 4, cudaHostAllocDefault));
    MG_CUDA(cudaHostAlloc(&m->h_pos, R * 4, cudaHostAllocDefault));
    MG_CUDA(cudaHostAlloc(&m->h_seq, R * 4, cudaHostAllocDefault));
    MG_CUDA(cudaHostAlloc(&m->h_amax, DEC_MAX * 4, cudaHostAllocDefault));
    if (m->ep.world > 1) {  // the collectives are placed in the streamed decode and tensor-core prefill
        MG_REQUIRE(m->maps_ok && m->use_stream, MG_ERR_SPEC,
                   "expert parallelism needs the streamed decode kernels (q8r trunk, 4-bit/int8 experts)");
    }
    TRY(dalloc(m, &m->samp_probs, (size_t)DEC_MAX * s.vocab * 4));
    TRY(dalloc(m, &m->samp_rng, (size_t)DEC_MAX * 8));
    TRY(dalloc(m, &m->samp_out, (size_t)DEC_MAX * 4));
    TRY(dalloc(m, &m->greedy_out, (size_t)GREEDY_MAX * DEC_MAX * 4));
    TRY(dalloc(m, &m->greedy_step, 16));
    TRY(rebase_prepare(m));
    TRY(prefill_prepare(m));
    MG_REQUIRE(m->ep.world == 1 || m->tc_prefill, MG_ERR_SPEC,
               "expert parallelism needs the tensor-core prefill (MXFP4 with power-of-two scales or q8r experts)");
    if (m->ep.world > 1) TRY(ep_prepare(m));
    m->ready = true;
    return MG_OK;
}

// Expert-parallel exchange buffers.  Decode: at most EP_DEC_TOK tokens per
// step over all ranks (the streamed MoE kernels' batch).  Prefill: a chunk of
// R local tokens goes to at most min(world, top_k) ranks per token; a rank
// receives at most every rank's chunk.
static int ep_prepare(mg_model *m) {
    const mg_spec &s = m->spec;
    const int G = m->ep.world, k = s.top_k, R = m->rows_max;
    const int64_t H = s.hidden;
    m->ep_rowf = ep_rowf(H, k);
    const int rowf = m->ep_rowf;
    EpComm &c = m->ep;
    cudaStream_t st = m->st;
    // buffers the other ranks write into (CUDA IPC over NVLink)
    TRY(ep_peer_alloc(c, m->epd_recv_p, (size_t)EP_DEC_TOK * rowf * 4, st));
    TRY(ep_peer_alloc(c, m->epd_y_p, (size_t)2 * DEC_MAX * k * H * 4, st));
    TRY(ep_peer_alloc(c, m->ep_flags_p, 256, st));
    m->epd_recv = static_cast<float *>(m->epd_recv_p.peer[c.rank]);
    m->moe_y = static_cast<float *>(m->epd_y_p.peer[c.rank]);  // the owner's slot outputs arrive here
    TRY(dalloc(m, &m->ep_seq, 16));
    MG_CUDA(cudaMemset(m->ep_seq, 0, 16));
    for (int d = 0; d < G; d++) {
        m->epd_peers.recv[d] = static_cast<float *>(m->epd_recv_p.peer[d]);
        m->epd_peers.y[d] = static_cast<float *>(m->epd_y_p.peer[d]);
        m->epd_peers.flag[d] = static_cast<uint32_t *>(m->ep_flags_p.peer[d]);
    }
    m->epd_peers.seq = m->ep_seq;
    m->epd_peers.err = stream_error_word();
    TRY(dalloc(m, &m->epd_xb, (size_t)EP_DEC_TOK * H * 4));
    TRY(dalloc(m, &m->epd_sel, (size_t)EP_DEC_TOK * k * 4));
    TRY(dalloc(m, &m->epd_y, (size_t)m->ks_down * EP_DEC_TOK * k * H * 4));
    const int per_tok = std::min(G, k);
    m->epp_cap_recv = (int64_t)G * R;
    TRY(dalloc(m, &m->epp_counts, (size_t)2 * G * 4));
    TRY(dalloc(m, &m->epp_all, (size_t)2 * G * G * 4));
    MG_CUDA(cudaHostAlloc(&m->epp_h_all, (size_t)2 * G * G * 4, cudaHostAllocDefault));
    m->host_allocs.push_back(m->epp_h_all);
    TRY(dalloc(m, &m->epp_send_row, (size_t)R * G * 4));
    TRY(dalloc(m, &m->epp_ret_pos, (size_t)R * k * 4));
    TRY(dalloc(m, &m->epp_send, (size_t)R * per_tok * rowf * 4));
    TRY(ep_peer_alloc(c, m->epp_recv_p, (size_t)m->epp_cap_recv * rowf * 4, st));
    m->epp_recv = static_cast<float *>(m->epp_recv_p.peer[c.rank]);
    TRY(dalloc(m, &m->epp_sel, (size_t)m->epp_cap_recv * k * 4));
    TRY(dalloc(m, &m->epp_ret_row, (size_t)m->epp_cap_recv * k * 4));
    TRY(dalloc(m, &m->epp_slot2, (size_t)m->epp_cap_recv * k * 4));
    TRY(dalloc(m, &m->epp_ret_send, (size_t)m->epp_cap_recv * k * H * 4));
    TRY(ep_peer_alloc(c, m->epp_ret_recv_p, (size_t)R * k * H * 4, st));
    m->epp_ret_recv = static_cast<float *>(m->epp_ret_recv_p.peer[c.rank]);
    const char *es = getenv("MIDGE_EP_STATS");
    m->ep_stats = es && *es == '1';
    if (m->ep_stats) {
        m->ep_ev.resize((size_t)s.n_layers * 5);
        for (auto &e : m->ep_ev) MG_CUDA(cudaEventCreate(&e));
    }
    return MG_OK;
}

// Tensor-core prefill of the routed experts: MXFP4 with ue8m0 scales (exact
// in f16 after a per-matrix rebase, checked here) or q8r, dims % 64.
static int prefill_prepare(mg_model *m) {
    const mg_spec &s = m->spec;
    const mg_expert_layout &L = m->el;
    const int R = m->rows_max, E = m->n_local;
    const bool fmt = (L.dt == MG_MXFP4 && L.scale_fmt == MG_SCALE_UE8M0) || L.dt == MG_Q8R;
    const int q_dim = s.n_heads * s.head_dim;
    // trunk projections on the tensor cores: q8r matrices, reduction dims % 64
    bool dense = m->tc_prefill && s.hidden % 64 == 0 && q_dim % 64 == 0;
    for (int l = 0; l < s.n_layers && dense; l++)
        dense = m->wq[l].dt == MG_Q8R && m->wk[l].dt == MG_Q8R && m->wv[l].dt == MG_Q8R && m->wo[l].dt == MG_Q8R;
    m->tc_dense = dense;
    if (!m->tc_prefill || !fmt || L.hidden % 64 || L.ffn % 64) m->tc_prefill = false;
    if (!m->tc_prefill && !m->tc_dense) return MG_OK;
    // expert parallel: the experts of this rank may receive every rank's slots
    const int64_t slots = (int64_t)R * s.top_k * m->ep.world;
    const int64_t xrow = std::max((int64_t)slots * L.hidden, (int64_t)R * std::max<int64_t>(s.hidden, q_dim));
    TRY(dalloc(m, &m->pf_xhi, (size_t)xrow * 2));
    TRY(dalloc(m, &m->pf_xlo, (size_t)xrow * 2));
    if (!m->tc_prefill) return MG_OK;
    TRY(dalloc(m, &m->pf_counts, (size_t)E * 4));
    TRY(dalloc(m, &m->pf_offs, (size_t)(E + 1) * 4));
    TRY(dalloc(m, &m->pf_cursor, (size_t)E * 4));
    TRY(dalloc(m, &m->pf_ntiles, 16));
    TRY(dalloc(m, &m->pf_pos, (size_t)slots * 4));
    TRY(dalloc(m, &m->pf_slot, (size_t)slots * 4));
    TRY(dalloc(m, (uint8_t **)&m->pf_tiles, (size_t)(slots / 128 + 1 + E) * sizeof(XgTile)));
    TRY(dalloc(m, &m->pf_hhi, (size_t)slots * L.ffn * 2));
    TRY(dalloc(m, &m->pf_hlo, (size_t)slots * L.ffn * 2));
    if (m->ep.world == 1) TRY(dalloc(m, &m->pf_y, (size_t)slots * L.hidden * 4));  // else the return buffer
    if (L.dt == MG_MXFP4 && !m->rebase_ok) {
        fprintf(stderr, "# expert matrices span more than 35 scale binades: tile prefill kernels\n");
        m->tc_prefill = false;
    }
    return MG_OK;
}

// Per-(layer, expert, matrix) rebase exponents of MXFP4 experts with ue8m0
// scales: e2m1 x 2^(code - 127 - k0) is exact in f16 for every matrix whose
// codes span at most 35 binades (the tensor-core kernels' weight operand).
static int rebase_prepare(mg_model *m) {
    const mg_spec &s = m->spec;
    const mg_expert_layout &L = m->el;
    m->rebase_ok = false;
    if (L.dt != MG_MXFP4 || L.scale_fmt != MG_SCALE_UE8M0) return MG_OK;
    const int E = m->n_local;
    TRY(dalloc(m, &m->pf_rebase, (size_t)s.n_layers * E * 3 * 4));
    MG_CUDA(cudaMemset(m->pf_rebase, 0, (size_t)s.n_layers * E * 3 * 4));
    int *inexact = nullptr;
    TRY(dalloc(m, &inexact, 4));
    MG_CUDA(cudaMemsetAsync(inexact, 0, 4, m->st));
    TRY(pf_rebase(m->experts, L, s.n_layers, E, m->pf_rebase, inexact, m->st));
    int h = 0;
    MG_CUDA(cudaMemcpyAsync(&h, inexact, 4, cudaMemcpyDeviceToHost, m->st));
    MG_CUDA(cudaStreamSynchronize(m->st));
    m->rebase_ok = h == 0;
    return MG_OK;
}

// ------------------------------------------------------------ forward passes
// y[n x w.rows] (=|+=) W x + bias for the n activation rows already split
// into m->pf_xhi / pf_xlo (tcgen05 dense GEMM)
static int dense_rows(mg_model *m, const DevMat &w, int n, const float *bias, int acc, float *y, int64_t ldy) {
    DenseGemm d{};
    d.w = w.data; d.scales = w.scales; d.bias = bias; d.rows = w.rows; d.cols = w.cols;
    d.x_hi = m->pf_xhi; d.x_lo = m->pf_xlo; d.n = n;
    d.y = y; d.ldy = ldy; d.accumulate = acc; d.err = stream_error_word();
    return dense_gemm(d, m->st);
}

static int gemv_rows(mg_model *m, const DevMat &w, const float *x, int64_t ldx, int n, const float *bias, int acc,
                     float *y, int64_t ldy) {
    for (int r0 = 0; r0 < n; r0 += 16) {
        int nn = n - r0 < 16 ? n - r0 : 16;
        TRY(gemv(w.dt, MG_SCALE_F16, w.data, w.scales, w.rows, w.cols, x + (int64_t)r0 * ldx, ldx, nn, bias, acc,
                 y + (int64_t)r0 * ldy, ldy, m->st));
    }
    return MG_OK;
}

static MoePrefill prefill_args(mg_model *m, int layer) {
    const mg_spec &s = m->spec;
    MoePrefill pf{};
    pf.L = m->el;
    pf.experts_layer = m->experts + (int64_t)layer * m->el.layer_stride;
    pf.rebase = m->pf_rebase ? m->pf_rebase + (int64_t)layer * m->n_local * 3 : nullptr;
    pf.top_k = s.top_k; pf.n_experts = s.n_experts; pf.e0 = m->e0; pf.n_local = m->n_local;
    pf.act_plain = s.act_plain; pf.alpha = s.alpha; pf.limit = s.limit;
    pf.counts = m->pf_counts; pf.offs = m->pf_offs; pf.cursor = m->pf_cursor; pf.ntiles = m->pf_ntiles;
    pf.pos_of_slot = m->pf_pos; pf.slot_of_pos = m->pf_slot; pf.tiles = (XgTile *)m->pf_tiles;
    pf.x_hi = m->pf_xhi; pf.x_lo = m->pf_xlo; pf.h_hi = m->pf_hhi; pf.h_lo = m->pf_hlo;
    pf.err = stream_error_word();
    return pf;
}

// Expert-parallel MoE block of a prefill chunk (engine/midge.c:595-611 with
// the experts spread over the ranks).  The n local tokens (0: this rank only
// serves its experts to the other ranks' tokens) are routed in m->sel / m->wts
// with their normed rows in m->xb.  One host agreement (the per-destination
// token and slot counts of every rank), then the dispatch of [row | ids] to
// the ranks holding the experts, the grouped GEMMs over the received tokens,
// the outputs back to the owners, and the combine in ascending expert order.
static int moe_prefill_ep(mg_model *m, int layer, int n) {
    const mg_spec &s = m->spec;
    EpComm &c = m->ep;
    const int G = c.world, me = c.rank, k = s.top_k, rowf = m->ep_rowf;
    const int64_t H = s.hidden;
    cudaStream_t st = m->st;
    cudaEvent_t *ev = m->ep_stats ? &m->ep_ev[(size_t)layer * 5] : nullptr;
    if (ev) MG_CUDA(cudaEventRecord(ev[0], st));
    TRY(ep_pf_plan(m->sel, n, k, G, m->n_local, s.n_experts, m->epp_counts, m->epp_send_row, m->epp_ret_pos, st));
    TRY(ep_allgather_ints(c, m->epp_counts, m->epp_all, (size_t)2 * G, st));
    MG_CUDA(cudaMemcpyAsync(m->epp_h_all, m->epp_all, (size_t)2 * G * G * 4, cudaMemcpyDeviceToHost, st));
    TRY(ep_stream_wait(c, st));
    const int *A = m->epp_h_all;  // A[r*2G + d]: tokens r -> d; A[r*2G + G + d]: slots r -> d
    // my blocks (offsets in my buffers) and where they land in the receiver's
    // buffers: rank d's receive buffer is source-major, its return buffer
    // expert-rank-major
    int64_t so[EP_MAX_WORLD], sc[EP_MAX_WORLD], dsto[EP_MAX_WORLD];
    int64_t bso[EP_MAX_WORLD], bsc[EP_MAX_WORLD], bdsto[EP_MAX_WORLD];
    int64_t a = 0, a2 = 0, n_recv = 0;
    for (int d = 0; d < G; d++) {
        sc[d] = (int64_t)A[me * 2 * G + d] * rowf; so[d] = a; a += sc[d];          // my tokens to d
        bsc[d] = (int64_t)A[d * 2 * G + G + me] * H; bso[d] = a2; a2 += bsc[d];    // outputs of d's slots, back
        n_recv += A[d * 2 * G + me];
        int64_t t = 0, u = 0;
        for (int q = 0; q < me; q++) {
            t += A[q * 2 * G + d];      // tokens ranks < me send to d
            u += A[d * 2 * G + G + q];  // d's slots on ranks < me
        }
        dsto[d] = t * rowf;
        bdsto[d] = u * H;
    }
    MG_REQUIRE(n_recv <= m->epp_cap_recv, MG_ERR_STATE, "expert parallel prefill: %lld tokens received (room for %lld)",
               (long long)n_recv, (long long)m->epp_cap_recv);
    if (ev) MG_CUDA(cudaEventRecord(ev[1], st));
    TRY(ep_pf_pack(m->xb, m->sel, n, k, G, H, rowf, m->epp_send_row, m->epp_send, st));
    TRY(ep_put(c, m->epp_send, so, sc, m->epp_recv_p, dsto, st));  // copy engines, NVLink
    TRY(ep_barrier(c, st));                                          // every rank's rows have landed
    if (ev) MG_CUDA(cudaEventRecord(ev[2], st));
    TRY(ep_pf_unpack_sel(m->epp_recv, (int)n_recv, k, H, rowf, m->epp_sel, st));
    TRY(ep_pf_retplan(m->epp_sel, (int)n_recv, k, m->e0, m->n_local, m->epp_ret_row, st));
    MoePrefill pf = prefill_args(m, layer);
    pf.n = (int)n_recv;
    pf.sel = m->epp_sel;
    pf.xb = m->epp_recv;
    pf.ldx = rowf;
    pf.out_row = m->epp_ret_row;
    pf.slot2 = m->epp_slot2;
    pf.y = m->epp_ret_send;
    TRY(moe_prefill_experts(pf, st));
    if (ev) MG_CUDA(cudaEventRecord(ev[3], st));
    TRY(ep_put(c, m->epp_ret_send, bso, bsc, m->epp_ret_recv_p, bdsto, st));
    TRY(ep_barrier(c, st));
    TRY(pf_combine(m->x, H, m->sel, m->wts, n, k, s.n_experts, m->epp_ret_recv, m->epp_ret_pos, st));
    if (ev) MG_CUDA(cudaEventRecord(ev[4], st));
    return MG_OK;
}

// after a synchronised prefill chunk: add the phase times of every layer
static void ep_stats_collect(mg_model *m) {
    if (!m->ep_stats) return;
    for (int l = 0; l < m->spec.n_layers; l++) {
        cudaEvent_t *ev = &m->ep_ev[(size_t)l * 5];
        for (int p = 0; p < 4; p++) {
            float ms = 0.f;
            if (cudaEventElapsedTime(&ms, ev[p], ev[p + 1]) == cudaSuccess) m->ep_ms[p] += ms;
        }
    }
    cudaGetLastError();
}

extern "C" int mg_model_ep_stats(mg_model *m, double *ms4) {
    MG_REQUIRE(m && ms4, MG_ERR_ARG, "ep_stats: bad arguments");
    for (int p = 0; p < 4; p++) ms4[p] = m->ep_ms[p];
    return MG_OK;
}

// The per-layer body shared by decode (n rows = sequences, one token each)
// and prefill (n rows = consecutive tokens of one sequence).
static int layer_pass(mg_model *m, int layer, int n, bool prefill, int seq, int pos0) {
    const mg_spec &s = m->spec;
    const int64_t H = s.hidden;
    const int hd = s.head_dim, q_dim = s.n_heads * hd, kv_dim = s.n_kv_heads * hd;
    cudaStream_t st = m->st;
    // attention (engine/midge.c:341-400)
    TRY(rmsnorm(m->x, m->attn_norm[layer], m->xb, H, n, s.norm_eps, st));
    const bool dense = prefill && m->tc_dense;
    if (dense) {
        TRY(split_rows(m->xb, H, n, H, m->pf_xhi, m->pf_xlo, st));
        TRY(dense_rows(m, m->wq[layer], n, m->bq[layer], 0, m->q, q_dim));
        TRY(dense_rows(m, m->wk[layer], n, m->bk[layer], 0, m->k, kv_dim));
        TRY(dense_rows(m, m->wv[layer], n, m->bv[layer], 0, m->v, kv_dim));
    } else {
        TRY(gemv_rows(m, m->wq[layer], m->xb, H, n, m->bq[layer], 0, m->q, q_dim));
        TRY(gemv_rows(m, m->wk[layer], m->xb, H, n, m->bk[layer], 0, m->k, kv_dim));
        TRY(gemv_rows(m, m->wv[layer], m->xb, H, n, m->bv[layer], 0, m->v, kv_dim));
    }
    const int cap = m->cap[layer];
    const bool sliding = cap < m->ctx;
    QkvPostArgs qa{};
    qa.q = m->q; qa.k = m->k; qa.v = m->v; qa.ldq = q_dim; qa.ldk = kv_dim;
    qa.n_heads = s.n_heads; qa.n_kv_heads = s.n_kv_heads; qa.head_dim = hd;
    qa.qn = s.qk_norm ? m->qn[layer] : nullptr; qa.kn = s.qk_norm ? m->kn[layer] : nullptr;
    qa.eps = s.norm_eps; qa.rope_cos = m->rope_cos; qa.rope_sin = m->rope_sin;
    qa.tok_pos = m->tok_pos; qa.tok_seq = m->tok_seq;
    qa.write_cache = prefill ? !sliding : 1;
    qa.kc = m->kc[layer]; qa.vc = m->vc[layer]; qa.cap = cap;
    qa.tmp_k = prefill ? m->tmp_k : nullptr; qa.tmp_v = prefill ? m->tmp_v : nullptr;
    TRY(qkv_post(qa, n, st));
    if (prefill) {
        AttnPrefillArgs pa{};
        pa.q = m->q; pa.ldq = q_dim; pa.tmp_k = m->tmp_k; pa.tmp_v = m->tmp_v;
        pa.kc = m->kc[layer]; pa.vc = m->vc[layer];
        pa.seq = seq; pa.pos0 = pos0; pa.n = n; pa.cap = cap;
        pa.n_heads = s.n_heads; pa.n_kv_heads = s.n_kv_heads; pa.head_dim = hd;
        pa.scale = s.attn_scale; pa.sinks = s.sinks ? m->sinks[layer] : nullptr;
        pa.out = m->ao; pa.ldo = q_dim; pa.use_tc = m->tc_attn;
        TRY(attn_prefill(pa, st));
        if (sliding) {
            int nst = n < cap ? n : cap;
            uint16_t *kcs = m->kc[layer] + (int64_t)seq * cap * kv_dim, *vcs = m->vc[layer] + (int64_t)seq * cap * kv_dim;
            k_ring_store<<<nst, 128, 0, st>>>(m->tmp_k, m->tmp_v, n, pos0, cap, kv_dim, kcs, vcs);
            MG_CHECK_LAUNCH();
        }
    } else {
        AttnDecodeArgs da{};
        da.q = m->q; da.ldq = q_dim; da.seq_ids = m->tok_seq; da.pos = m->tok_pos;
        da.kc = m->kc[layer]; da.vc = m->vc[layer]; da.cap = cap;
        da.n_heads = s.n_heads; da.n_kv_heads = s.n_kv_heads; da.head_dim = hd;
        da.scale = s.attn_scale; da.sinks = s.sinks ? m->sinks[layer] : nullptr;
        da.split_len = m->attn_split;
        da.max_splits = (cap + m->attn_split - 1) / m->attn_split;
        da.use_tc = m->tc_attn;
        da.partial = m->attn_part; da.out = m->ao; da.ldo = q_dim;
        TRY(attn_decode(da, n, st));
    }
    if (dense) {
        TRY(split_rows(m->ao, q_dim, n, q_dim, m->pf_xhi, m->pf_xlo, st));
        TRY(dense_rows(m, m->wo[layer], n, m->bo[layer], 1, m->x, H));
    } else {
        TRY(gemv_rows(m, m->wo[layer], m->ao, q_dim, n, m->bo[layer], 1, m->x, H));
    }
    // MoE (engine/midge.c:469-549; prefill routing engine/midge.c:404-434)
    RouterArgs ra{};
    ra.x = m->x; ra.norm_w = m->mlp_norm[layer]; ra.eps = s.norm_eps; ra.xb_out = m->xb;
    ra.rw = (const float *)m->router_w[layer].data; ra.rb = m->router_b[layer];
    ra.n_experts = s.n_experts; ra.top_k = s.top_k; ra.router_norm = s.router_norm; ra.variant = prefill ? 1 : 0;
    ra.hidden = H; ra.n_tok = n; ra.logits = nullptr; ra.sel = m->sel; ra.weights = m->wts;
    ra.usage = m->usage + (int64_t)layer * s.n_experts;
    if (prefill) TRY(router_batch(ra, m->rlogits, st));
    else TRY(router(ra, st));
    const uint8_t *lb = m->experts + (int64_t)layer * m->el.layer_stride;
    if (prefill && m->tc_prefill) {
        if (m->ep.world > 1) return moe_prefill_ep(m, layer, n);
        MoePrefill pf = prefill_args(m, layer);
        pf.n = n;
        pf.sel = m->sel; pf.w = m->wts; pf.xb = m->xb; pf.x = m->x; pf.y = m->pf_y;
        return moe_prefill(pf, st);
    }
    for (int r0 = 0; r0 < n; r0 += DEC_MAX) {
        int nn = n - r0 < DEC_MAX ? n - r0 : DEC_MAX;
        MoeArgs ma{};
        ma.L = m->el;
        ma.experts_layer = lb; ma.n_experts = s.n_experts;
        ma.xb = m->xb + (int64_t)r0 * H; ma.n_tok = nn; ma.top_k = s.top_k;
        ma.sel = m->sel + (int64_t)r0 * s.top_k; ma.weights = m->wts + (int64_t)r0 * s.top_k;
        ma.act_plain = s.act_plain; ma.alpha = s.alpha; ma.limit = s.limit;
        ma.h = m->h; ma.x = m->x + (int64_t)r0 * H; ma.ldx = H;
        TRY(moe_decode(ma, st));
    }
    return MG_OK;
}

static int logits_rows(mg_model *m, const float *x, int n) {
    const mg_spec &s = m->spec;
    TRY(rmsnorm(x, m->final_norm, m->xb, s.hidden, n, s.norm_eps, m->st));
    TRY(gemv_rows(m, m->lm_head, m->xb, s.hidden, n, nullptr, 0, m->logits, s.vocab));
    return MG_OK;
}

// Is the streamed decode path available for this model and batch?
static bool stream_ok(const mg_model *m, int n) {
    const mg_spec &s = m->spec;
    auto q8r_ok = [](const DevMat &d) { return d.dt == MG_Q8R && d.cols % 64 == 0; };
    bool trunk = true;
    for (int l = 0; l < s.n_layers; l++)
        trunk = trunk && q8r_ok(m->wq[l]) && q8r_ok(m->wk[l]) && q8r_ok(m->wv[l]) && q8r_ok(m->wo[l]);
    const bool ex = (m->el.dt == MG_MXFP4 || m->el.dt == MG_Q4G32 || (m->el.dt == MG_Q8R && s.hidden % 64 == 0 && s.ffn % 64 == 0)) &&
                    s.hidden % 32 == 0 && s.ffn % 32 == 0;
    return m->maps_ok && trunk && ex && q8r_ok(m->lm_head) && n <= 8 && n * s.top_k <= 128 && m->el.dt != MG_F32;
}

static MoeStreamArgs stream_moe_args(mg_model *m, int layer) {
    const mg_spec &s = m->spec;
    MoeStreamArgs ma{};
    ma.L = m->el; ma.experts_layer = m->experts + (int64_t)layer * m->el.layer_stride;
    ma.maps = m->map_ex; ma.layer = layer;
    ma.n_experts = m->n_local; ma.e0 = m->e0; ma.top_k = s.top_k;
    ma.act_plain = s.act_plain; ma.alpha = s.alpha; ma.limit = s.limit; ma.h = m->h;
    ma.down_ksplit = 2; ma.down_ksplit_out = m->ks_down;
    ma.bs = m->bs_moe ? &m->bs : nullptr;
    return ma;
}

// Expert-parallel routed experts of one decode layer: every rank's n_max rows
// [normed row | ids] are gathered (pads route nowhere), this rank's experts
// run over all of them (their outputs in the slots of local experts, zero in
// the others), and a sum reduce-scatter gives each owner its own tokens' slot
// outputs -- exactly one rank holds a nonzero value per slot, so the sum is
// exact and the owner's combine sees the one-GPU values.  n = 0: this rank has
// no tokens this step and only serves its experts.
static int ep_decode_moe(mg_model *m, int layer, int n) {
    const mg_spec &s = m->spec;
    EpComm &c = m->ep;
    const int G = c.world, k = s.top_k, nm = m->dec_nmax, n_all = G * nm, rowf = m->ep_rowf;
    const int64_t H = s.hidden;
    cudaStream_t st = m->st;
    TRY(ep_dec_dispatch(m->epd_peers, m->xb, m->sel, n, nm, H, k, rowf, c.rank, G, st));
    TRY(ep_dec_unpack(m->epd_recv, n_all, H, k, rowf, m->epd_xb, m->epd_sel, st));
    const int64_t plane_all = (int64_t)n_all * k * H, plane_loc = (int64_t)nm * k * H;
    MoeStreamArgs ma = stream_moe_args(m, layer);
    ma.n_tok = n_all; ma.sel = m->epd_sel; ma.xb = m->epd_xb; ma.y = m->epd_y;
    TRY(moe_stream(ma, st));
    return ep_dec_return(m->epd_peers, m->epd_y, m->epd_sel, nm, H, k, m->ks_down, plane_all, plane_loc, m->e0,
                         m->n_local, c.rank, G, st);
}

// One layer of the streamed decode: combine(previous MoE)+norm, QKV (K-split
// partials), RoPE/QK-norm/KV store, attention, O (partials folded into the
// residual by the router), router, streamed MoE.
static int layer_stream(mg_model *m, int layer, int n) {
    const mg_spec &s = m->spec;
    const int64_t H = s.hidden;
    const int hd = s.head_dim, q_dim = s.n_heads * hd, kv_dim = s.n_kv_heads * hd, qkv_dim = q_dim + 2 * kv_dim;
    cudaStream_t st = m->st;
    CombineNormArgs cn{};
    cn.x_in = layer > 0 ? m->xa : nullptr;
    cn.x = m->x; cn.y = layer > 0 ? m->moe_y : nullptr; cn.ksplit = m->ks_down;
    cn.sel = m->sel; cn.w = m->wts; cn.n_tok = n; cn.top_k = s.top_k; cn.n_experts = s.n_experts;
    cn.hidden = H; cn.nw = m->attn_norm[layer]; cn.eps = s.norm_eps; cn.xb = m->xb;
    if (m->ep.world > 1) cn.plane = (int64_t)m->dec_nmax * s.top_k * H;
    // programmatic after the MoE grid; not at layer 0, whose residual comes
    // from the embedding kernel just before
    cn.pdl = m->pdl && layer > 0 && m->ep.world == 1;
    TRY(combine_norm(cn, st));
    StreamGemvArgs g{};
    g.dt = MG_Q8R; g.scale_fmt = MG_SCALE_F16; g.nmat = 3; g.cols = H; g.x = m->xb; g.ldx = H; g.n_tok = n;
    g.ksplit = m->ks_qkv; g.part_stride = (int64_t)n * qkv_dim;  // effective split, computed at ready()
    const DevMat *mats[3] = {&m->wq[layer], &m->wk[layer], &m->wv[layer]};
    const float *bias[3] = {m->bq[layer], m->bk[layer], m->bv[layer]};
    const int64_t off[3] = {0, q_dim, q_dim + kv_dim};
    const CUtensorMap *maps[3] = {&m->map_q[layer], &m->map_k[layer], &m->map_v[layer]};
    for (int i = 0; i < 3; i++) {
        g.mat[i].map = maps[i];
        g.mat[i].w = mats[i]->data; g.mat[i].scales = mats[i]->scales; g.mat[i].bias = bias[i];
        g.mat[i].rows = mats[i]->rows; g.mat[i].y = m->qkv_part + off[i]; g.mat[i].ldy = qkv_dim;
    }
    TRY(stream_gemv(g, st));
    const int cap = m->cap[layer];
    QkvPostArgs qa{};
    qa.q = m->qkv; qa.k = m->qkv + q_dim; qa.v = m->qkv + q_dim + kv_dim; qa.ldq = qkv_dim; qa.ldk = qkv_dim;
    qa.n_heads = s.n_heads; qa.n_kv_heads = s.n_kv_heads; qa.head_dim = hd;
    qa.qn = s.qk_norm ? m->qn[layer] : nullptr; qa.kn = s.qk_norm ? m->kn[layer] : nullptr;
    qa.eps = s.norm_eps; qa.rope_cos = m->rope_cos; qa.rope_sin = m->rope_sin;
    qa.tok_pos = m->tok_pos; qa.tok_seq = m->tok_seq; qa.write_cache = 1;
    qa.kc = m->kc[layer]; qa.vc = m->vc[layer]; qa.cap = cap;
    // the K-split partial planes are summed inside (k_sum_parts order)
    qa.parts = m->qkv_part; qa.ks = m->ks_qkv; qa.plane = (int64_t)n * qkv_dim; qa.v_out = m->qkv + q_dim + kv_dim;
    qa.pdl = m->pdl;
    TRY(qkv_post_parts(qa, n, st));
    AttnDecodeArgs da{};
    da.q = m->qkv; da.ldq = qkv_dim; da.seq_ids = m->tok_seq; da.pos = m->tok_pos;
    da.kc = m->kc[layer]; da.vc = m->vc[layer]; da.cap = cap;
    da.n_heads = s.n_heads; da.n_kv_heads = s.n_kv_heads; da.head_dim = hd;
    da.scale = s.attn_scale; da.sinks = s.sinks ? m->sinks[layer] : nullptr;
    da.split_len = m->attn_split; da.max_splits = (cap + m->attn_split - 1) / m->attn_split;
    da.use_tc = m->tc_attn;
    da.partial = m->attn_part; da.out = m->ao; da.ldo = q_dim;
    da.pdl = m->pdl;
    TRY(attn_decode(da, n, st));
    StreamGemvArgs go{};
    go.dt = MG_Q8R; go.scale_fmt = MG_SCALE_F16; go.nmat = 1; go.cols = q_dim; go.x = m->ao; go.ldx = q_dim;
    go.n_tok = n; go.ksplit = m->ks_o; go.part_stride = (int64_t)n * H;
    go.mat[0].map = &m->map_o[layer];
    go.mat[0].w = m->wo[layer].data; go.mat[0].scales = m->wo[layer].scales; go.mat[0].bias = m->bo[layer];
    go.mat[0].rows = H; go.mat[0].y = m->o_part; go.mat[0].ldy = H;
    TRY(stream_gemv(go, st));
    RouterArgs ra{};
    ra.x = m->x; ra.norm_w = m->mlp_norm[layer]; ra.eps = s.norm_eps; ra.xb_out = m->xb;
    ra.rw = (const float *)m->router_w[layer].data; ra.rb = m->router_b[layer];
    ra.n_experts = s.n_experts; ra.top_k = s.top_k; ra.router_norm = s.router_norm; ra.variant = 0;
    ra.hidden = H; ra.n_tok = n; ra.logits = nullptr; ra.sel = m->sel; ra.weights = m->wts;
    ra.usage = m->usage + (int64_t)layer * s.n_experts;
    ra.x_parts = m->o_part; ra.x_parts_ks = m->ks_o; ra.x_parts_stride = (int64_t)n * H; ra.x_out = m->xa;
    ra.err = stream_error_word();
    ra.pdl = m->pdl;
    TRY(router_split(ra, m->rlogits, m->rticket, st));
    MoeStreamArgs ma{};
    ma.L = m->el; ma.experts_layer = m->experts + (int64_t)layer * m->el.layer_stride;
    ma.maps = m->map_ex; ma.layer = layer;
    ma.n_experts = m->n_local; ma.e0 = m->e0; ma.n_tok = n; ma.top_k = s.top_k; ma.sel = m->sel; ma.xb = m->xb;
    ma.act_plain = s.act_plain; ma.alpha = s.alpha; ma.limit = s.limit; ma.h = m->h; ma.y = m->moe_y;
    ma.down_ksplit = 2; ma.down_ksplit_out = m->ks_down;
    ma.bs = m->bs_moe ? &m->bs : nullptr;
    if (m->ep.world > 1) return ep_decode_moe(m, layer, n);
    return moe_stream(ma, st);
}

// embedding -> logits and argmax keys, device only (tokens/positions in m->toks / tok_pos)
static int decode_core_stream(mg_model *m, int n) {
    const mg_spec &s = m->spec;
    cudaStream_t st = m->st;
    if (n == 0) {  // expert parallel, no local sequence this step: serve the experts only
        for (int l = 0; l < s.n_layers; l++) TRY(ep_decode_moe(m, l, 0));
        return MG_OK;
    }
    TRY(dequant_rows(m->embed.dt, MG_SCALE_F16, m->embed.data, m->embed.scales, m->embed.rows, m->embed.cols, m->toks, n,
                     m->x, st));
    for (int l = 0; l < s.n_layers; l++) TRY(layer_stream(m, l, n));
    CombineNormArgs cn{};
    cn.x_in = m->xa;
    cn.x = m->x; cn.y = m->moe_y; cn.ksplit = m->ks_down; cn.sel = m->sel; cn.w = m->wts; cn.n_tok = n;
    cn.top_k = s.top_k; cn.n_experts = s.n_experts; cn.hidden = s.hidden; cn.nw = m->final_norm;
    cn.eps = s.norm_eps; cn.xb = m->xb;
    if (m->ep.world > 1) cn.plane = (int64_t)m->dec_nmax * s.top_k * s.hidden;
    cn.pdl = m->pdl && m->ep.world == 1;
    TRY(combine_norm(cn, st));
    StreamGemvArgs g{};
    g.dt = MG_Q8R; g.scale_fmt = MG_SCALE_F16; g.nmat = 1; g.cols = s.hidden; g.x = m->xb; g.ldx = s.hidden;
    g.n_tok = n; g.ksplit = 1; g.accumulate = 0;
    g.mat[0].map = &m->map_lm;
    g.mat[0].w = m->lm_head.data; g.mat[0].scales = m->lm_head.scales; g.mat[0].bias = nullptr;
    g.mat[0].rows = m->lm_head.rows; g.mat[0].y = m->logits; g.mat[0].ldy = s.vocab;
    g.amax = m->amax_keys;
    MG_CUDA(cudaMemsetAsync(m->amax_keys, 0, (size_t)n * 8, st));
    TRY(stream_gemv(g, st));
    return MG_OK;
}

// embedding -> logits and argmax (tile kernels), device only
static int decode_core_tile(mg_model *m, int n) {
    const mg_spec &s = m->spec;
    cudaStream_t st = m->st;
    TRY(dequant_rows(m->embed.dt, MG_SCALE_F16, m->embed.data, m->embed.scales, m->embed.rows, m->embed.cols, m->toks, n,
                     m->x, st));
    for (int l = 0; l < s.n_layers; l++) TRY(layer_pass(m, l, n, false, 0, 0));
    TRY(logits_rows(m, m->x, n));
    k_argmax<<<n, 1024, 0, st>>>(m->logits, s.vocab, m->amax);
    MG_CHECK_LAUNCH();
    return MG_OK;
}

// decode body for n sequences whose tokens/positions are already in the
// pinned staging arrays; everything stream-ordered (graph-capturable)
static int decode_body(mg_model *m, int n) {
    m->last_streamed = m->ep.world > 1 || (m->use_stream && stream_ok(m, n));
    cudaStream_t st = m->st;
    MG_CUDA(cudaMemcpyAsync(m->toks, m->h_toks, n * 4, cudaMemcpyHostToDevice, st));
    MG_CUDA(cudaMemcpyAsync(m->tok_pos, m->h_pos, n * 4, cudaMemcpyHostToDevice, st));
    MG_CUDA(cudaMemcpyAsync(m->tok_seq, m->h_seq, n * 4, cudaMemcpyHostToDevice, st));
    if (m->last_streamed) {
        TRY(decode_core_stream(m, n));
        MG_CUDA(cudaMemcpyAsync(m->h_keys, m->amax_keys, (size_t)n * 8, cudaMemcpyDeviceToHost, st));
        MG_CUDA(cudaMemcpyAsync(m->h_err, stream_error_word(), sizeof(int), cudaMemcpyDeviceToHost, st));
    } else {
        TRY(decode_core_tile(m, n));
        MG_CUDA(cudaMemcpyAsync(m->h_amax, m->amax, n * 4, cudaMemcpyDeviceToHost, st));
    }
    return MG_OK;
}

// one greedy step fed from the previous step's argmax, device only
static int decode_chain_body(mg_model *m, int n) {
    const bool streamed = m->ep.world > 1 || (m->use_stream && stream_ok(m, n));
    if (n > 0) {
        k_advance<<<1, 32, 0, m->st>>>(streamed ? m->amax_keys : nullptr, m->amax, n, m->toks, m->tok_pos,
                                       m->greedy_out, m->greedy_step);
        MG_CHECK_LAUNCH();
    }
    return streamed ? decode_core_stream(m, n) : decode_core_tile(m, n);
}

static int graph_kernels(cudaGraph_t g) {
    size_t nn = 0;
    if (cudaGraphGetNodes(g, nullptr, &nn) != cudaSuccess || nn == 0) return 0;
    std::vector<cudaGraphNode_t> nodes(nn);
    if (cudaGraphGetNodes(g, nodes.data(), &nn) != cudaSuccess) return 0;
    int k = 0;
    for (auto nd : nodes) {
        cudaGraphNodeType t;
        if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) k++;
    }
    return k;
}

// Run body(m, n) from a CUDA graph kept in tab[n].  The first run with this
// many sequences is eager (which also sets every kernel's launch attributes);
// the same stream-ordered body is then captured for the following runs
// (capture executes nothing).  Counts the kernels launched.
static int graph_run(mg_model *m, std::unordered_map<int, Graph> &tab, int n, int (*body)(mg_model *, int)) {
    if (!m->use_graphs) return body(m, n);  // eager-only runs are not counted
    const int key = n + 256 * (m->ep.world > 1 ? m->dec_nmax : 0);
    auto it = tab.find(key);
    if (it != tab.end()) {
        MG_CUDA(cudaGraphLaunch(it->second.exec, m->st));
        m->kernel_launches += (uint64_t)it->second.kernels;
        return MG_OK;
    }
    TRY(body(m, n));
    MG_CUDA(cudaStreamSynchronize(m->st));
    cudaGraph_t g = nullptr;
    MG_CUDA(cudaStreamBeginCapture(m->st, cudaStreamCaptureModeThreadLocal));
    int rc = body(m, n);
    cudaError_t ce = cudaStreamEndCapture(m->st, &g);
    if (rc != MG_OK) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    MG_REQUIRE(ce == cudaSuccess, MG_ERR_CUDA, "graph capture failed: %s", cudaGetErrorString(ce));
    Graph gr;
    gr.kernels = graph_kernels(g);
    cudaError_t ie = cudaGraphInstantiate(&gr.exec, g, 0);
    cudaGraphDestroy(g);
    MG_REQUIRE(ie == cudaSuccess, MG_ERR_CUDA, "graph instantiate failed: %s", cudaGetErrorString(ie));
    tab[key] = gr;
    m->kernel_launches += (uint64_t)gr.kernels;  // the eager run launched the same kernels
    return MG_OK;
}

static int run_decode(mg_model *m, int n) { return graph_run(m, m->dec_graphs, n, decode_body); }

// Expert parallel: every rank takes part in each decode step (n_seqs may be
// 0 on some ranks); the ranks agree on the tokens per rank of the step.
static int ep_decode_agree(mg_model *m, int n_seqs, int n_steps) {
    if (m->ep.world == 1) {
        m->dec_nmax = n_seqs;
        return MG_OK;
    }
    const int v[3] = {n_seqs, n_steps, -n_steps};
    int mx[3];
    TRY(ep_allreduce_max_ints(m->ep, v, mx, 3, m->st));
    MG_REQUIRE(mx[1] == -mx[2], MG_ERR_ARG, "expert parallel decode: the ranks asked for different step counts");
    MG_REQUIRE(mx[0] * m->ep.world <= EP_DEC_TOK, MG_ERR_ARG,
               "expert parallel decode: %d tokens per rank x %d ranks exceed %d per step", mx[0], m->ep.world,
               EP_DEC_TOK);
    MG_REQUIRE(m->use_stream && stream_ok(m, mx[0] * m->ep.world), MG_ERR_SPEC,
               "expert parallel decode needs the streamed kernels");
    m->dec_nmax = mx[0];
    return MG_OK;
}

extern "C" int mg_decode_step(mg_model *m, int n_seqs, const int32_t *seq_ids, const int32_t *toks, float *logits,
                              int32_t *argmax) {
    MG_REQUIRE(m && m->ready, MG_ERR_STATE, "decode: model not ready");
    const int n_min = m->ep.world > 1 ? 0 : 1;
    MG_REQUIRE(n_seqs >= n_min && n_seqs <= DEC_MAX && n_seqs <= m->max_seqs && (n_seqs == 0 || toks), MG_ERR_ARG,
               "decode: bad n_seqs %d", n_seqs);
    MG_CUDA(cudaSetDevice(m->device));
    const mg_spec &s = m->spec;
    for (int i = 0; i < n_seqs; i++) {
        int sq = seq_ids ? seq_ids[i] : i;
        MG_REQUIRE(sq >= 0 && sq < m->max_seqs, MG_ERR_ARG, "decode: sequence %d out of range", sq);
        for (int j = 0; j < i; j++) MG_REQUIRE((seq_ids ? seq_ids[j] : j) != sq, MG_ERR_ARG, "decode: duplicate sequence");
        MG_REQUIRE(m->pos[sq] < m->ctx, MG_ERR_RANGE, "context full (%d)", m->ctx);          // engine/midge.c:554
        MG_REQUIRE(toks[i] >= 0 && toks[i] < s.vocab, MG_ERR_RANGE, "token %d out of range", toks[i]);  // :555
        m->h_toks[i] = toks[i];
        m->h_pos[i] = m->pos[sq];
        m->h_seq[i] = sq;
    }
    TRY(ep_decode_agree(m, n_seqs, 1));
    if (m->dec_nmax == 0) return MG_OK;  // no rank decodes
    TRY(run_decode(m, n_seqs));
    if (logits && n_seqs)
        MG_CUDA(cudaMemcpyAsync(logits, m->logits, (size_t)n_seqs * s.vocab * 4, cudaMemcpyDeviceToHost, m->st));
    TRY(ep_stream_wait(m->ep, m->st));
    if (*m->h_err) {  // a bounded wait in a streamed kernel gave up
        *m->h_err = 0;
        return stream_error_check();
    }
    if (m->last_streamed)  // argmax came back packed as (ordered value << 32 | ~index); 0: no finite maximum
        for (int i = 0; i < n_seqs; i++)
            m->h_amax[i] = m->h_keys[i] ? (int32_t)(0xffffffffu - (uint32_t)(m->h_keys[i] & 0xffffffffull)) : 0;
    for (int i = 0; i < n_seqs; i++) m->pos[m->h_seq[i]]++;
    m->expert_loads += (uint64_t)n_seqs * s.top_k * s.n_layers;
    if (argmax) memcpy(argmax, m->h_amax, n_seqs * 4);
    return MG_OK;
}

extern "C" int mg_decode_greedy(mg_model *m, int n_seqs, const int32_t *seq_ids, const int32_t *toks, int n_steps,
                                int32_t *out_toks) {
    MG_REQUIRE(m && m->ready, MG_ERR_STATE, "greedy: model not ready");
    const int n_min = m->ep.world > 1 ? 0 : 1;
    MG_REQUIRE(n_seqs >= n_min && n_seqs <= DEC_MAX && n_seqs <= m->max_seqs && (n_seqs == 0 || (toks && out_toks)),
               MG_ERR_ARG, "greedy: bad arguments");
    MG_REQUIRE(n_steps >= 1 && n_steps <= GREEDY_MAX, MG_ERR_ARG, "greedy: n_steps %d not in [1, %d]", n_steps,
               GREEDY_MAX);
    MG_CUDA(cudaSetDevice(m->device));
    const mg_spec &s = m->spec;
    for (int i = 0; i < n_seqs; i++) {
        int sq = seq_ids ? seq_ids[i] : i;
        MG_REQUIRE(sq >= 0 && sq < m->max_seqs, MG_ERR_ARG, "greedy: sequence %d out of range", sq);
        for (int j = 0; j < i; j++) MG_REQUIRE((seq_ids ? seq_ids[j] : j) != sq, MG_ERR_ARG, "greedy: duplicate sequence");
        MG_REQUIRE(m->pos[sq] + n_steps <= m->ctx, MG_ERR_RANGE, "context full (%d)", m->ctx);
        MG_REQUIRE(toks[i] >= 0 && toks[i] < s.vocab, MG_ERR_RANGE, "token %d out of range", toks[i]);
        m->h_toks[i] = toks[i];
        m->h_pos[i] = m->pos[sq];
        m->h_seq[i] = sq;
    }
    cudaStream_t st = m->st;
    TRY(ep_decode_agree(m, n_seqs, n_steps));
    if (m->dec_nmax == 0) return MG_OK;  // no rank decodes
    MG_CUDA(cudaMemsetAsync(m->greedy_step, 0, 4, st));
    TRY(run_decode(m, n_seqs));
    for (int k = 1; k < n_steps; k++) TRY(graph_run(m, m->chain_graphs, n_seqs, decode_chain_body));
    const bool streamed = m->ep.world > 1 || (m->use_stream && stream_ok(m, n_seqs));
    if (n_seqs > 0) {
        k_advance<<<1, 32, 0, st>>>(streamed ? m->amax_keys : nullptr, m->amax, n_seqs, m->toks, m->tok_pos,
                                    m->greedy_out, m->greedy_step);
        MG_CHECK_LAUNCH();
        m->kernel_launches += 1;
        MG_CUDA(cudaMemcpyAsync(out_toks, m->greedy_out, (size_t)n_steps * n_seqs * 4, cudaMemcpyDeviceToHost, st));
    }
    TRY(ep_stream_wait(m->ep, st));
    *m->h_err = 0;
    TRY(stream_error_check());
    for (int i = 0; i < n_seqs; i++) m->pos[m->h_seq[i]] += n_steps;
    m->expert_loads += (uint64_t)n_seqs * s.top_k * s.n_layers * n_steps;
    return MG_OK;
}

extern "C" uint64_t mg_model_kernel_launches(const mg_model *m) { return m ? m->kernel_launches : 0; }

extern "C" int mg_model_moe_stream(mg_model *m, int layer, int n_tok, const int32_t *sel) {
    MG_REQUIRE(m && m->ready && sel && layer >= 0 && layer < m->spec.n_layers, MG_ERR_ARG, "moe_stream: bad arguments");
    MG_REQUIRE(m->use_stream && stream_ok(m, n_tok), MG_ERR_STATE, "moe_stream: the streamed kernels do not apply");
    MG_CUDA(cudaSetDevice(m->device));
    const mg_spec &s = m->spec;
    MoeStreamArgs ma{};
    ma.L = m->el; ma.experts_layer = m->experts + (int64_t)layer * m->el.layer_stride;
    ma.maps = m->map_ex; ma.layer = layer;
    ma.n_experts = m->n_local; ma.e0 = m->e0; ma.n_tok = n_tok; ma.top_k = s.top_k; ma.sel = sel; ma.xb = m->xb;
    ma.act_plain = s.act_plain; ma.alpha = s.alpha; ma.limit = s.limit; ma.h = m->h; ma.y = m->moe_y;
    ma.down_ksplit = 2; ma.down_ksplit_out = m->ks_down;
    ma.bs = m->bs_moe ? &m->bs : nullptr;
    return moe_stream(ma, m->st);
}

extern "C" int mg_forward(mg_model *m, int seq, int32_t token, float *logits, int32_t *argmax) {
    int32_t sq = seq;
    return mg_decode_step(m, 1, &sq, &token, logits, argmax);
}

extern "C" int mg_forward_batch(mg_model *m, int seq, const int32_t *toks, int n, int logits_mode, float *logits) {
    MG_REQUIRE(m && m->ready, MG_ERR_STATE, "forward_batch: model not ready");
    MG_REQUIRE(seq >= 0 && seq < m->max_seqs && n >= 0 && (n == 0 || toks), MG_ERR_ARG, "forward_batch: bad arguments");
    MG_REQUIRE(logits_mode >= 0 && logits_mode <= 2 && (logits_mode == 0 || logits || n == 0), MG_ERR_ARG,
               "forward_batch: bad logits mode");
    MG_CUDA(cudaSetDevice(m->device));
    const mg_spec &s = m->spec;
    for (int t = 0; t < n; t++) {  // engine/midge.c:580-583
        MG_REQUIRE(m->pos[seq] + t < m->ctx, MG_ERR_RANGE, "context full (%d)", m->ctx);
        MG_REQUIRE(toks[t] >= 0 && toks[t] < s.vocab, MG_ERR_RANGE, "token %d out of range", toks[t]);
    }
    int n_all = n;  // expert parallel: every rank runs as many chunks as the longest prompt needs
    if (m->ep.world > 1) {
        int mx = 0;
        TRY(ep_allreduce_max_ints(m->ep, &n, &mx, 1, m->st));
        n_all = mx;
    }
    for (int c0 = 0; c0 < n_all; c0 += m->pf_chunk) {
        int nc = n - c0 < m->pf_chunk ? n - c0 : m->pf_chunk;
        if (nc <= 0) {  // expert parallel, no local tokens in this chunk: serve the experts only
            for (int l = 0; l < s.n_layers; l++) TRY(moe_prefill_ep(m, l, 0));
            TRY(ep_stream_wait(m->ep, m->st));
            TRY(stream_error_check());
            ep_stats_collect(m);
            continue;
        }
        int pos0 = m->pos[seq];
        for (int t = 0; t < nc; t++) {
            m->h_toks[t] = toks[c0 + t];
            m->h_pos[t] = pos0 + t;
            m->h_seq[t] = seq;
        }
        cudaStream_t st = m->st;
        MG_CUDA(cudaMemcpyAsync(m->toks, m->h_toks, nc * 4, cudaMemcpyHostToDevice, st));
        MG_CUDA(cudaMemcpyAsync(m->tok_pos, m->h_pos, nc * 4, cudaMemcpyHostToDevice, st));
        MG_CUDA(cudaMemcpyAsync(m->tok_seq, m->h_seq, nc * 4, cudaMemcpyHostToDevice, st));
        TRY(dequant_rows(m->embed.dt, MG_SCALE_F16, m->embed.data, m->embed.scales, m->embed.rows, m->embed.cols, m->toks,
                         nc, m->x, st));
        for (int l = 0; l < s.n_layers; l++) TRY(layer_pass(m, l, nc, true, seq, pos0));
        const bool last_chunk = c0 + nc == n;
        if (logits_mode == 2) {
            for (int r0 = 0; r0 < nc; r0 += DEC_MAX) {
                int nn = nc - r0 < DEC_MAX ? nc - r0 : DEC_MAX;
                TRY(logits_rows(m, m->x + (int64_t)r0 * s.hidden, nn));
                MG_CUDA(cudaMemcpyAsync(logits + (int64_t)(c0 + r0) * s.vocab, m->logits, (size_t)nn * s.vocab * 4,
                                        cudaMemcpyDeviceToHost, st));
                if (last_chunk && r0 + nn == nc && nn > 1)  // the last position's logits stay in row 0
                    MG_CUDA(cudaMemcpyAsync(m->logits, m->logits + (int64_t)(nn - 1) * s.vocab, (size_t)s.vocab * 4,
                                            cudaMemcpyDeviceToDevice, st));
            }
        } else if (logits_mode == 1 && last_chunk) {
            TRY(logits_rows(m, m->x + (int64_t)(nc - 1) * s.hidden, 1));
            MG_CUDA(cudaMemcpyAsync(logits, m->logits, (size_t)s.vocab * 4, cudaMemcpyDeviceToHost, st));
        }
        TRY(ep_stream_wait(m->ep, st));
        if (m->tc_prefill || m->tc_dense) TRY(stream_error_check());
        if (m->ep.world > 1) ep_stats_collect(m);
        m->pos[seq] += nc;
        m->expert_loads += (uint64_t)nc * s.top_k * s.n_layers;
    }
    return MG_OK;
}

extern "C" int mg_model_sample(mg_model *m, int n_rows, float temp, float top_p, uint64_t *rng, int32_t *out) {
    MG_REQUIRE(m && m->ready && out && n_rows >= 1 && n_rows <= DEC_MAX && (temp <= 0.f || rng), MG_ERR_ARG,
               "sample: bad arguments");
    MG_CUDA(cudaSetDevice(m->device));
    cudaStream_t st = m->st;
    const int64_t V = m->spec.vocab;
    if (temp > 0.f) MG_CUDA(cudaMemcpyAsync(m->samp_rng, rng, (size_t)n_rows * 8, cudaMemcpyHostToDevice, st));
    TRY(sample_topp(m->logits, V, V, n_rows, temp, top_p, m->samp_rng, m->samp_out, m->samp_probs, st));
    MG_CUDA(cudaMemcpyAsync(m->h_amax, m->samp_out, (size_t)n_rows * 4, cudaMemcpyDeviceToHost, st));
    if (temp > 0.f) MG_CUDA(cudaMemcpyAsync(rng, m->samp_rng, (size_t)n_rows * 8, cudaMemcpyDeviceToHost, st));
    MG_CUDA(cudaStreamSynchronize(st));
    memcpy(out, m->h_amax, (size_t)n_rows * 4);
    return MG_OK;
}

extern "C" int mg_model_put_logits(mg_model *m, int row, const float *logits) {
    MG_REQUIRE(m && m->ready && logits && row >= 0 && row < DEC_MAX, MG_ERR_ARG, "put_logits: bad arguments");
    MG_CUDA(cudaSetDevice(m->device));
    MG_CUDA(cudaMemcpy(m->logits + (int64_t)row * m->spec.vocab, logits, (size_t)m->spec.vocab * 4,
                       cudaMemcpyHostToDevice));
    return MG_OK;
}

extern "C" int mg_model_logits(mg_model *m, int row, float *out) {
    MG_REQUIRE(m && m->ready && out && row >= 0 && row < DEC_MAX, MG_ERR_ARG, "logits: bad arguments");
    MG_CUDA(cudaSetDevice(m->device));
    MG_CUDA(cudaMemcpy(out, m->logits + (int64_t)row * m->spec.vocab, (size_t)m->spec.vocab * 4, cudaMemcpyDeviceToHost));
    return MG_OK;
}

extern "C" int mg_model_reset(mg_model *m, int seq) {
    MG_REQUIRE(m && seq >= 0 && seq < m->max_seqs, MG_ERR_ARG, "reset: bad sequence");
    m->pos[seq] = 0;
    return MG_OK;
}

extern "C" int mg_model_pos(const mg_model *m, int seq) {
    if (!m || seq < 0 || seq >= m->max_seqs) return MG_ERR_ARG;
    return m->pos[seq];
}

extern "C" int mg_model_get_usage(mg_model *m, uint32_t *usage) {
    MG_REQUIRE(m && m->ready && usage, MG_ERR_ARG, "get_usage: bad arguments");
    MG_CUDA(cudaSetDevice(m->device));
    MG_CUDA(cudaMemcpy(usage, m->usage, (size_t)m->spec.n_layers * m->spec.n_experts * 4, cudaMemcpyDeviceToHost));
    return MG_OK;
}

extern "C" int mg_model_set_usage(mg_model *m, const uint32_t *usage) {
    MG_REQUIRE(m && m->ready && usage, MG_ERR_ARG, "set_usage: bad arguments");
    MG_CUDA(cudaSetDevice(m->device));
    MG_CUDA(cudaMemcpy(m->usage, usage, (size_t)m->spec.n_layers * m->spec.n_experts * 4, cudaMemcpyHostToDevice));
    return MG_OK;
}

extern "C" uint64_t mg_model_expert_loads(const mg_model *m) { return m ? m->expert_loads : 0; }

extern "C" const uint8_t *mg_model_experts_device(const mg_model *m, mg_expert_layout *layout) {
    if (!m) return nullptr;
    if (layout) *layout = m->el;
    return m->experts;
}

extern "C" void *mg_model_stream(const mg_model *m) { return m ? (void *)m->st : nullptr; }

extern "C" int mg_model_free(mg_model *m) {
    if (!m) return MG_OK;
    cudaSetDevice(m->device);
    if (m->st) cudaStreamSynchronize(m->st);
    for (auto *tab : {&m->dec_graphs, &m->chain_graphs})  // graphs holding collectives go before the communicator
        for (auto &kv : *tab)
            if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
    for (mg::EpPeer *b : {&m->epd_recv_p, &m->epd_y_p, &m->ep_flags_p, &m->epp_recv_p, &m->epp_ret_recv_p})
        ep_peer_free(m->ep, *b);
    ep_destroy(&m->ep);
    for (void *p : m->allocs) cudaFree(p);
    for (void *p : m->host_allocs) cudaFreeHost(p);
    for (cudaEvent_t e : m->ep_ev) cudaEventDestroy(e);
    for (void *p : {(void *)m->h_toks, (void *)m->h_pos, (void *)m->h_seq, (void *)m->h_amax, (void *)m->h_err,
                    (void *)m->h_keys})
        if (p) cudaFreeHost(p);
    if (m->st) cudaStreamDestroy(m->st);
    delete m;
    return MG_OK;
}
