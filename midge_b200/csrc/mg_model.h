// mg_model.h -- device-resident model state behind the mg_model handle.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <string>
#include <unordered_map>
#include <vector>

#include "mg_bsmoe.h"
#include "mg_ep.h"
#include "mg_ep_xchg.h"
#include "midgecuda.h"

namespace mg {

struct DevMat {
    int dt = -1;
    int64_t rows = 0, cols = 0;
    void *data = nullptr;
    void *scales = nullptr;
};

constexpr int PF_CHUNK = 4096;  // default tokens per prefill pass through the layers (MIDGE_PREFILL_CHUNK)
constexpr int DEC_MAX = 16;     // sequences per decode step

constexpr int GREEDY_MAX = 4096;  // steps per mg_decode_greedy call
constexpr int EP_DEC_TOK = 8;     // expert parallel: tokens per decode step over all ranks

struct Graph {
    cudaGraphExec_t exec = nullptr;
    int kernels = 0;  // kernel nodes in the graph
};

}  // namespace mg

struct mg_model {
    mg_spec spec{};
    std::vector<int> layer_sliding;
    int ctx = 0, max_seqs = 0, device = 0;
    cudaStream_t st = nullptr;
    std::vector<void *> allocs;
    std::vector<void *> host_allocs;  // pinned host buffers freed with the model

    mg::DevMat embed, lm_head;
    float *final_norm = nullptr;
    std::vector<mg::DevMat> wq, wk, wv, wo, router_w;
    std::vector<float *> bq, bk, bv, bo, router_b, attn_norm, mlp_norm, sinks, qn, kn;

    mg_expert_layout el{};  // layout of the local blob: layer_stride = n_local experts
    int e0 = 0, n_local = 0;  // this rank's experts [e0, e0 + n_local) (expert parallelism)
    mg::EpComm ep;
    uint8_t *experts = nullptr;
    size_t experts_bytes = 0;

    std::vector<uint16_t *> kc, vc;
    std::vector<int> cap;
    float *rope_cos = nullptr, *rope_sin = nullptr;
    std::vector<int> pos;  // per sequence

    // work buffers
    int rows_max = 0;
    float *x = nullptr, *xb = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *ao = nullptr;
    float *h = nullptr, *logits = nullptr, *wts = nullptr, *attn_part = nullptr;
    int32_t *sel = nullptr, *tok_pos = nullptr, *tok_seq = nullptr, *toks = nullptr, *amax = nullptr;
    uint16_t *tmp_k = nullptr, *tmp_v = nullptr;
    uint32_t *usage = nullptr;
    // streamed decode: K-split partial planes and MoE down partials
    float *xa = nullptr;  // post-attention residual of the streamed decode
    float *qkv = nullptr, *qkv_part = nullptr, *o_part = nullptr, *moe_y = nullptr, *rlogits = nullptr;
    unsigned long long *amax_keys = nullptr, *h_keys = nullptr;
    unsigned *rticket = nullptr;  // last-block ticket of the decode router
    int ks_qkv = 1, ks_o = 1, ks_down = 1;
    // TMA maps of the streamed decode: per layer q, k, v, o; lm_head; experts
    std::vector<CUtensorMap> map_q, map_k, map_v, map_o;
    CUtensorMap map_lm;
    CUtensorMap map_ex[3];
    bool maps_ok = false;
    int attn_split = 64, attn_max_splits = 1;  // decode attention: positions per split (MIDGE_ATTN_SPLIT)

    // pinned host staging for per-step inputs/outputs
    int32_t *h_toks = nullptr, *h_pos = nullptr, *h_seq = nullptr, *h_amax = nullptr;
    int *h_err = nullptr;  // error word of the streamed kernels, copied back each step

    // tensor-core prefill of the routed experts (expert-major grouped GEMM)
    int pf_chunk = mg::PF_CHUNK;
    bool tc_prefill = false;
    bool tc_dense = false;  // trunk q/k/v/o of prefill on the tensor cores
    bool tc_attn = true;    // prefill attention on the tensor cores (MIDGE_ATTN_KERNELS=scalar: fp32 kernel)
    bool bs_moe = false;    // decode MoE on block-scaled tcgen05 MMAs (default for MXFP4 with ue8m0 scales;
                            // MIDGE_MOE_KERNELS=mma selects the mma.sync streamed kernels)
    mg::BsBuffers bs{};
    bool pdl = true;  // decode: programmatic launches of the small steps after the grids before them (MIDGE_PDL=0: off)
    bool rebase_ok = false; // pf_rebase holds exact f16 rebase exponents of every expert matrix
    int *pf_counts = nullptr, *pf_offs = nullptr, *pf_cursor = nullptr, *pf_ntiles = nullptr;
    int *pf_pos = nullptr, *pf_slot = nullptr, *pf_rebase = nullptr;
    void *pf_tiles = nullptr;  // mg::XgTile[]
    __half *pf_xhi = nullptr, *pf_xlo = nullptr, *pf_hhi = nullptr, *pf_hlo = nullptr;
    float *pf_y = nullptr;

    // device sampling (mg_model_sample): probabilities, generator states, picks
    float *samp_probs = nullptr;
    uint64_t *samp_rng = nullptr;
    int32_t *samp_out = nullptr;
    // expert parallelism (world > 1): token exchange buffers
    int ep_rowf = 0;       // floats per packed [normed row | top-k ids] row
    int dec_nmax = 0;      // decode: tokens per rank of the current step (max over the ranks)
    float *epd_recv = nullptr, *epd_xb = nullptr, *epd_y = nullptr;
    int32_t *epd_sel = nullptr;
    mg::EpPeer epd_recv_p, epd_y_p, ep_flags_p, epp_recv_p, epp_ret_recv_p;  // peer-mapped buffers
    mg::EpDecPeers epd_peers{};
    uint32_t *ep_seq = nullptr;  // decode hand-over epochs and tickets
    int64_t epp_cap_recv = 0;  // prefill: received tokens per layer and chunk, at most
    int *epp_counts = nullptr, *epp_all = nullptr, *epp_h_all = nullptr;
    int *epp_send_row = nullptr, *epp_ret_pos = nullptr, *epp_ret_row = nullptr, *epp_slot2 = nullptr;
    int32_t *epp_sel = nullptr;
    float *epp_send = nullptr, *epp_recv = nullptr, *epp_ret_send = nullptr, *epp_ret_recv = nullptr;

    // expert-parallel prefill phase timing (MIDGE_EP_STATS=1): per layer 5 events, summed per call
    bool ep_stats = false;
    std::vector<cudaEvent_t> ep_ev;
    double ep_ms[4] = {0, 0, 0, 0};  // plan + agreement, dispatch, expert GEMMs, return + combine

    std::unordered_map<int, mg::Graph> dec_graphs;    // keyed by n_seqs (and, expert-parallel, the step's n_max)
    std::unordered_map<int, mg::Graph> chain_graphs;  // device-fed greedy steps, keyed by n_seqs
    int32_t *greedy_out = nullptr, *greedy_step = nullptr;  // [GREEDY_MAX x DEC_MAX] tokens, step counter
    uint64_t kernel_launches = 0;  // kernels launched by the decode paths
    uint64_t expert_loads = 0;
    bool ready = false;
    bool use_graphs = true;
    bool use_stream = true;
    bool last_streamed = false;  // the last decode step took the streamed path  // streamed decode kernels (MIDGE_DECODE_KERNELS=tile selects the tile kernels)
};
