// mg_stream.cu -- launchers of the streamed (bulk-copy ring) decode GEMV.
#include "mg_kernels.h"
#include "mg_stream.cuh"

namespace mg {

// Error word of the streamed kernels (bounded mbarrier waits), one per device.
static int *sw_err_ptr() {
    static int *p[64] = {nullptr};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    if (!p[dev]) {
        if (cudaMalloc(&p[dev], sizeof(int)) != cudaSuccess) return nullptr;
        cudaMemset(p[dev], 0, sizeof(int));
    }
    return p[dev];
}

int stream_error_check() {
    int *e = sw_err_ptr();
    MG_REQUIRE(e, MG_ERR_CUDA, "stream: no error word");
    int h = 0;
    MG_CUDA(cudaMemcpy(&h, e, sizeof(int), cudaMemcpyDeviceToHost));
    if (h) {
        cudaMemset(e, 0, sizeof(int));
        set_error("streamed GEMV: a bounded wait timed out (code %d)", h);
        return MG_ERR_TIMEOUT;
    }
    return MG_OK;
}

int stream_prepare() { return sw_err_ptr() ? MG_OK : MG_ERR_OOM; }

template <int DT, int SC, int NT>
static int launch_stream_gemv(const StreamGemvArgs &a, cudaStream_t st) {
    using G = SwGeom<DT>;
    PolGemv<DT, SC> pol{};
    const int64_t rowbytes = DT == MG_Q8R ? a.cols : a.cols / 2;
    int64_t tiles = 0;
    for (int i = 0; i < a.nmat; i++) {
        pol.m[i].w = (const uint8_t *)a.mat[i].w;
        pol.m[i].sc = (const uint8_t *)a.mat[i].scales;
        pol.m[i].bias = a.mat[i].bias;
        pol.m[i].rows = a.mat[i].rows;
        pol.m[i].y = a.mat[i].y;
        pol.m[i].ldy = a.mat[i].ldy;
        pol.m[i].tile0 = tiles;
        tiles += (a.mat[i].rows + SW_ROWS - 1) / SW_ROWS;
    }
    pol.nmat = a.nmat;
    pol.cols = (int)a.cols;
    pol.ntiles = tiles;
    const int nsm = num_sms();
    int ks = a.ksplit > 0 ? a.ksplit : 1;
    const int64_t nseg = (rowbytes + G::SEGB - 1) / G::SEGB;
    if (ks > nseg) ks = (int)nseg;
    const int64_t segs_per_split = (nseg + ks - 1) / ks;
    ks = (int)((nseg + segs_per_split - 1) / segs_per_split);
    pol.ks_count = ks;
    pol.kbytes_per_split = segs_per_split * G::SEGB;
    pol.x = a.x;
    pol.ldx = a.ldx;
    pol.n_tok = a.n_tok;
    pol.accumulate = a.accumulate;
    pol.part_stride = a.part_stride;
    const size_t xs_bytes = (size_t)NT * 8 * (a.cols + XS_PAD) * 2;
    const size_t budget = 227 * 1024 - 1024;
    int nstages = (int)((budget - 128 - xs_bytes) / G::STAGE_BYTES);
    if (nstages > SW_MAX_STAGES) nstages = SW_MAX_STAGES;
    MG_REQUIRE(nstages >= 2, MG_ERR_ARG, "streamed gemv: %lld columns x %d tokens leave no room for a ring",
               (long long)a.cols, a.n_tok);
    const size_t smem = 128 + (size_t)nstages * G::STAGE_BYTES + xs_bytes;
    auto kfn = k_stream<DT, SC, NT, PolGemv<DT, SC>>;
    int rc = ensure_smem(kfn, smem);
    if (rc) return rc;
    int *err = sw_err_ptr();
    MG_REQUIRE(err, MG_ERR_OOM, "streamed gemv: no error word");
    const int64_t units = tiles * ks;
    const int grid = (int)(units < nsm ? units : nsm);
    kfn<<<grid, SW_THREADS, smem, st>>>(pol, nstages, err);
    MG_CHECK_LAUNCH();
    return MG_OK;
}

template <int DT, int SC>
static int stream_gemv_nt(const StreamGemvArgs &a, cudaStream_t st) {
    if (a.n_tok <= 4) return launch_stream_gemv<DT, SC, 1>(a, st);
    return launch_stream_gemv<DT, SC, 2>(a, st);
}

int stream_gemv(const StreamGemvArgs &a, cudaStream_t st) {
    MG_REQUIRE(a.nmat >= 1 && a.nmat <= 3 && a.x && a.n_tok >= 1 && a.n_tok <= 8 && a.cols > 0, MG_ERR_ARG,
               "streamed gemv: bad arguments");
    for (int i = 0; i < a.nmat; i++)
        MG_REQUIRE(a.mat[i].w && a.mat[i].y && a.mat[i].rows > 0 && (a.dt == MG_F32 || a.mat[i].scales), MG_ERR_ARG,
                   "streamed gemv: matrix %d incomplete", i);
    MG_REQUIRE(((reinterpret_cast<uintptr_t>(a.x) & 15) == 0) && (a.ldx % 4 == 0), MG_ERR_ARG,
               "streamed gemv: activations must be 16-byte aligned");
    switch (a.dt) {
    case MG_MXFP4:
        MG_REQUIRE(a.cols % 32 == 0, MG_ERR_ARG, "streamed gemv: cols %% 32");
        return a.scale_fmt == MG_SCALE_UE8M0 ? stream_gemv_nt<MG_MXFP4, MG_SCALE_UE8M0>(a, st)
                                             : stream_gemv_nt<MG_MXFP4, MG_SCALE_F16>(a, st);
    case MG_Q4G32:
        MG_REQUIRE(a.cols % 32 == 0, MG_ERR_ARG, "streamed gemv: cols %% 32");
        return a.scale_fmt == MG_SCALE_UE8M0 ? stream_gemv_nt<MG_Q4G32, MG_SCALE_UE8M0>(a, st)
                                             : stream_gemv_nt<MG_Q4G32, MG_SCALE_F16>(a, st);
    case MG_Q8R:
        MG_REQUIRE(a.cols % 64 == 0, MG_ERR_ARG, "streamed gemv: q8r cols %% 64");
        return stream_gemv_nt<MG_Q8R, MG_SCALE_F16>(a, st);
    }
    set_error("streamed gemv: dtype %d unsupported", a.dt);
    return MG_ERR_ARG;
}

}  // namespace mg
