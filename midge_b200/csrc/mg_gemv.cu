// mg_gemv.cu -- batched dequant-GEMV (decode), row dequant, scale re-expression,
// rmsnorm and the f16 flush conversion.
#include <cstdio>

#include "mg_gemv.cuh"
#include "mg_kernels.h"

namespace mg {

// ---------------------------------------------------------------- GEMV
// One block = 16*MT consecutive rows x all columns; 8 warps split the column
// chunks; partial sums meet in shared memory.  Epilogue: (q8r row scale),
// bias, store or accumulate.
template <int DT, int SC, int MT, int NT>
__global__ void __launch_bounds__(GEMV_THREADS) k_gemv(const uint8_t *__restrict__ w,
                                                       const uint8_t *__restrict__ scales, int64_t rows,
                                                       int cols, const float *__restrict__ x, int64_t ldx,
                                                       int n_tok, const float *__restrict__ bias,
                                                       int accumulate, float *__restrict__ y, int64_t ldy) {
    extern __shared__ __align__(16) unsigned char smem[];
    constexpr int ncol = NT * 8;
    const int xs_stride = cols + XS_PAD;
    __half *xs = reinterpret_cast<__half *>(smem);
    float *red = reinterpret_cast<float *>(smem + (size_t)ncol * xs_stride * 2);

    using Tile = GemvTile<DT, SC, MT, NT>;
    const int64_t ntiles = (rows + 16 * MT - 1) / (16 * MT);
    int c0, c1;
    warp_chunk_range(cols / Tile::CHUNK, c0, c1);
    if ((int64_t)blockIdx.x < ntiles) {
#pragma unroll
        for (int m = 0; m < MT; m++)
            prefetch_tile<DT, SC>(w, scales, (int64_t)blockIdx.x * 16 * MT + 16 * m, rows, cols, c0, c1);
    }
    stage_x<DT>(x, ldx, n_tok, cols, xs, xs_stride);
    __syncthreads();
    const int nt_active = (n_tok + 3) >> 2;

    // persistent over row tiles: the activations are staged once per block
    for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        const int64_t rbase = tile * 16 * MT;
        const int64_t nxt = tile + gridDim.x;
        if (nxt < ntiles) {
#pragma unroll
            for (int m = 0; m < MT; m++) prefetch_tile<DT, SC>(w, scales, nxt * 16 * MT + 16 * m, rows, cols, c0, c1);
        }
        const uint8_t *wp[MT];
        const uint8_t *sp[MT];
        int64_t r0[MT];
#pragma unroll
        for (int m = 0; m < MT; m++) { wp[m] = w; sp[m] = scales; r0[m] = rbase + 16 * m; }
        float acc[MT][NT][4];
#pragma unroll
        for (int m = 0; m < MT; m++)
#pragma unroll
            for (int nt = 0; nt < NT; nt++)
#pragma unroll
                for (int i = 0; i < 4; i++) acc[m][nt][i] = 0.f;
        Tile::run(wp, sp, r0, rows, cols, c0, c1, xs, xs_stride, nt_active, acc);
        gemv_block_reduce<MT, NT>(acc, red);
        for (int j = threadIdx.x; j < 16 * MT * n_tok; j += blockDim.x) {
            int tok = j / (16 * MT), rl = j - tok * 16 * MT;
            int64_t r = rbase + rl;
            if (r >= rows) continue;
            float v = gemv_out<NT>(red, rl >> 4, rl & 15, tok);
            if (DT == MG_Q8R) v = v * reinterpret_cast<const float *>(scales)[r];
            if (bias) v += bias[r];
            float *yp = y + (int64_t)tok * ldy + r;
            *yp = accumulate ? *yp + v : v;
        }
        __syncthreads();  // red is reused by the next tile
    }
}

// Plain FFMA GEMV for f32 weights (and q8r whose cols are not a multiple of
// 64): one warp per row, lanes stride the columns.
template <int DT>
__global__ void k_gemv_simple(const void *__restrict__ w, const float *__restrict__ scales, int64_t rows,
                              int cols, const float *__restrict__ x, int64_t ldx, int n_tok,
                              const float *__restrict__ bias, int accumulate, float *__restrict__ y,
                              int64_t ldy) {
    int lane = threadIdx.x & 31;
    int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= rows) return;
    for (int t = 0; t < n_tok; t++) {
        const float *xt = x + (int64_t)t * ldx;
        float a = 0.f;
        if (DT == MG_F32) {
            const float *wr = reinterpret_cast<const float *>(w) + r * cols;
            for (int c = lane; c < cols; c += 32) a = fmaf(wr[c], xt[c], a);
        } else {
            const int8_t *wr = reinterpret_cast<const int8_t *>(w) + r * cols;
            for (int c = lane; c < cols; c += 32) a = fmaf((float)wr[c], xt[c], a);
        }
        a = warp_sum(a);
        if (lane == 0) {
            if (DT == MG_Q8R) a *= scales[r];
            if (bias) a += bias[r];
            float *yp = y + (int64_t)t * ldy + r;
            *yp = accumulate ? *yp + a : a;
        }
    }
}

size_t gemv_smem_bytes(int cols, int mt, int nt) {
    return (size_t)nt * 8 * (cols + XS_PAD) * 2 + (size_t)GEMV_WARPS * mt * nt * 32 * 4 * 4;
}

template <int DT, int SC, int MT, int NT>
static int launch_gemv_t(const uint8_t *w, const uint8_t *s, int64_t rows, int cols, const float *x,
                         int64_t ldx, int n_tok, const float *bias, int acc, float *y, int64_t ldy,
                         cudaStream_t st) {
    size_t smem = gemv_smem_bytes(cols, MT, NT);
    auto kfn = k_gemv<DT, SC, MT, NT>;
    MG_REQUIRE(smem <= 200 * 1024, MG_ERR_ARG, "gemv: %d columns x %d tokens exceed shared memory", cols, n_tok);
    int rc = ensure_smem(kfn, smem);
    if (rc) return rc;
    int ntiles = ceil_div(rows, 16 * MT);
    int max_resident = 0;
    MG_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&max_resident, kfn, GEMV_THREADS, smem));
    int nsm = num_sms();
    int grid = max_resident > 0 && ntiles > max_resident * nsm ? max_resident * nsm : ntiles;
    kfn<<<grid, GEMV_THREADS, smem, st>>>(w, s, rows, cols, x, ldx, n_tok, bias, acc, y, ldy);
    MG_CHECK_LAUNCH();
    return MG_OK;
}

template <int DT, int SC>
static int launch_gemv_nt(const uint8_t *w, const uint8_t *s, int64_t rows, int cols, const float *x,
                          int64_t ldx, int n_tok, const float *bias, int acc, float *y, int64_t ldy,
                          cudaStream_t st) {
    // the staged activations must fit shared memory: split wide token sets
    int nt_fit = 4;
    while (nt_fit > 1 && gemv_smem_bytes(cols, 1, nt_fit) > 200 * 1024) nt_fit >>= 1;
    MG_REQUIRE(gemv_smem_bytes(cols, 1, 1) <= 200 * 1024, MG_ERR_ARG, "gemv: %d columns exceed shared memory", cols);
    if (n_tok > 4 * nt_fit) {
        int h = 4 * nt_fit;
        int rc = launch_gemv_nt<DT, SC>(w, s, rows, cols, x, ldx, h, bias, acc, y, ldy, st);
        if (rc) return rc;
        return launch_gemv_nt<DT, SC>(w, s, rows, cols, x + (int64_t)h * ldx, ldx, n_tok - h, bias, acc,
                                      y + (int64_t)h * ldy, ldy, st);
    }
    if (n_tok <= 4) return launch_gemv_t<DT, SC, 1, 1>(w, s, rows, cols, x, ldx, n_tok, bias, acc, y, ldy, st);
    if (n_tok <= 8) return launch_gemv_t<DT, SC, 1, 2>(w, s, rows, cols, x, ldx, n_tok, bias, acc, y, ldy, st);
    return launch_gemv_t<DT, SC, 1, 4>(w, s, rows, cols, x, ldx, n_tok, bias, acc, y, ldy, st);
}

int gemv(int dt, int scale_fmt, const void *w, const void *scales, int64_t rows, int64_t cols, const float *x,
         int64_t ldx, int n_tok, const float *bias, int accumulate, float *y, int64_t ldy, cudaStream_t st) {
    MG_REQUIRE(w && x && y && rows > 0 && cols > 0 && n_tok >= 1 && n_tok <= 256, MG_ERR_ARG,
               "gemv: bad arguments (rows=%lld cols=%lld n_tok=%d)", (long long)rows, (long long)cols, n_tok);
    MG_REQUIRE(cols < (1 << 30), MG_ERR_ARG, "gemv: cols too large");
    const uint8_t *wb = reinterpret_cast<const uint8_t *>(w), *sb = reinterpret_cast<const uint8_t *>(scales);
    int c = (int)cols;
    switch (dt) {
    case MG_MXFP4:
    case MG_Q4G32:
        MG_REQUIRE(cols % 32 == 0 && scales, MG_ERR_ARG, "gemv: 4-bit weights need cols %% 32 == 0 and scales");
        if (dt == MG_MXFP4)
            return scale_fmt == MG_SCALE_UE8M0
                       ? launch_gemv_nt<MG_MXFP4, MG_SCALE_UE8M0>(wb, sb, rows, c, x, ldx, n_tok, bias, accumulate, y, ldy, st)
                       : launch_gemv_nt<MG_MXFP4, MG_SCALE_F16>(wb, sb, rows, c, x, ldx, n_tok, bias, accumulate, y, ldy, st);
        return scale_fmt == MG_SCALE_UE8M0
                   ? launch_gemv_nt<MG_Q4G32, MG_SCALE_UE8M0>(wb, sb, rows, c, x, ldx, n_tok, bias, accumulate, y, ldy, st)
                   : launch_gemv_nt<MG_Q4G32, MG_SCALE_F16>(wb, sb, rows, c, x, ldx, n_tok, bias, accumulate, y, ldy, st);
    case MG_Q8R:
        MG_REQUIRE(scales, MG_ERR_ARG, "gemv: q8r needs row scales");
        if (cols % 64 == 0)
            return launch_gemv_nt<MG_Q8R, MG_SCALE_F16>(wb, sb, rows, c, x, ldx, n_tok, bias, accumulate, y, ldy, st);
        k_gemv_simple<MG_Q8R><<<ceil_div(rows, 8), 256, 0, st>>>(w, reinterpret_cast<const float *>(scales), rows, c,
                                                                  x, ldx, n_tok, bias, accumulate, y, ldy);
        MG_CHECK_LAUNCH();
        return MG_OK;
    case MG_F32:
        k_gemv_simple<MG_F32><<<ceil_div(rows, 8), 256, 0, st>>>(w, nullptr, rows, c, x, ldx, n_tok, bias,
                                                                  accumulate, y, ldy);
        MG_CHECK_LAUNCH();
        return MG_OK;
    }
    set_error("gemv: unknown dtype %d", dt);
    return MG_ERR_ARG;
}

// ------------------------------------------------------- row dequant
__global__ void k_dequant_rows(int dt, int scale_fmt, const uint8_t *__restrict__ w, const uint8_t *__restrict__ s,
                               int64_t rows, int64_t cols, const int32_t *__restrict__ ids, float *__restrict__ out) {
    int i = blockIdx.y;
    int64_t r = ids[i];
    float *o = out + (int64_t)i * cols;
    for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < cols; c += (int64_t)gridDim.x * blockDim.x) {
        if (r < 0 || r >= rows) { o[c] = 0.f; continue; }
        float v;
        if (dt == MG_F32) {
            v = reinterpret_cast<const float *>(w)[r * cols + c];
        } else if (dt == MG_Q8R) {
            v = (float)reinterpret_cast<const int8_t *>(w)[r * cols + c] * reinterpret_cast<const float *>(s)[r];
        } else {
            uint8_t b = w[r * (cols / 2) + c / 2];
            uint32_t code = (c & 1) ? (b >> 4) : (b & 15);
            int64_t gi = r * (cols / 32) + c / 32;
            float sc = scale_fmt == MG_SCALE_UE8M0 ? ue8m0_to_f32(s[gi]) : h2f(reinterpret_cast<const uint16_t *>(s)[gi]);
            float q;
            if (dt == MG_MXFP4) {
                // e2m1: sign, 2-bit exponent, 1-bit mantissa
                uint32_t e = (code >> 1) & 3, mb = code & 1;
                float mag = e == 0 ? 0.5f * (float)mb : ldexpf(1.0f + 0.5f * (float)mb, (int)e - 1);
                q = (code & 8) ? -mag : mag;
            } else {
                q = (float)((int)code - 8);
            }
            v = q * sc;
        }
        o[c] = v;
    }
}

int dequant_rows(int dt, int scale_fmt, const void *w, const void *scales, int64_t rows, int64_t cols,
                 const int32_t *ids, int n, float *out, cudaStream_t st) {
    MG_REQUIRE(w && ids && out && n >= 0 && rows > 0 && cols > 0, MG_ERR_ARG, "dequant_rows: bad arguments");
    if (n == 0) return MG_OK;
    dim3 grid((unsigned)ceil_div(cols, 256) < 64 ? ceil_div(cols, 256) : 64, n);
    k_dequant_rows<<<grid, 256, 0, st>>>(dt, scale_fmt, (const uint8_t *)w, (const uint8_t *)scales, rows, cols, ids, out);
    MG_CHECK_LAUNCH();
    return MG_OK;
}

// --------------------------------------------------- ue8m0 re-expression
__global__ void k_scales_ue8m0(const uint16_t *__restrict__ in, uint8_t *__restrict__ out, int64_t n, int *bad) {
    int local_bad = 0;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        uint32_t h = in[i];
        uint32_t ex = (h >> 10) & 31u, man = h & 1023u;
        uint8_t u = 0;
        if (h == 0) {
            u = 0;
        } else if (h & 0x8000u) {
            local_bad++;
        } else if (ex == 0) {  // subnormal: exact power of two iff one mantissa bit
            if (__popc(man) == 1) u = (uint8_t)(127 - 24 + (31 - __clz(man)));
            else local_bad++;
        } else if (ex == 31 || man != 0) {
            local_bad++;
        } else {
            u = (uint8_t)(ex - 15 + 127);
        }
        out[i] = u;
    }
    if (local_bad) atomicAdd(bad, local_bad);
}

int scales_to_ue8m0(const uint16_t *f16, uint8_t *ue8m0, int64_t n, int *n_inexact, cudaStream_t st) {
    MG_REQUIRE(f16 && ue8m0 && n_inexact && n >= 0, MG_ERR_ARG, "scales_to_ue8m0: bad arguments");
    if (n == 0) return MG_OK;
    int grid = ceil_div(n, 256);
    if (grid > 148 * 16) grid = 148 * 16;
    k_scales_ue8m0<<<grid, 256, 0, st>>>(f16, ue8m0, n, n_inexact);
    MG_CHECK_LAUNCH();
    return MG_OK;
}

// ------------------------------------------------------------- rmsnorm
__global__ void k_rmsnorm(const float *__restrict__ x, const float *__restrict__ w, float *__restrict__ out,
                          int64_t n, float eps) {
    __shared__ float scratch[32];
    const float *xr = x + (int64_t)blockIdx.x * n;
    float *orow = out + (int64_t)blockIdx.x * n;
    float ss = 0.f;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(xr[i], xr[i], ss);
    ss = block_sum(ss, scratch);
    float inv = 1.0f / sqrtf(ss / (float)n + eps);
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) orow[i] = xr[i] * inv * w[i];
}

int rmsnorm(const float *x, const float *w, float *out, int64_t n, int n_rows, float eps, cudaStream_t st) {
    MG_REQUIRE(x && w && out && n > 0 && n_rows >= 0, MG_ERR_ARG, "rmsnorm: bad arguments");
    if (n_rows == 0) return MG_OK;
    k_rmsnorm<<<n_rows, 256, 0, st>>>(x, w, out, n, eps);
    MG_CHECK_LAUNCH();
    return MG_OK;
}

__global__ void k_to_f16_ftz(const float *__restrict__ x, uint16_t *__restrict__ out, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = f2h_ftz(x[i]);
}

int to_f16_ftz(const float *x, uint16_t *out, int64_t n, cudaStream_t st) {
    MG_REQUIRE(x && out && n >= 0, MG_ERR_ARG, "to_f16_ftz: bad arguments");
    if (n == 0) return MG_OK;
    int grid = ceil_div(n, 256);
    if (grid > 148 * 8) grid = 148 * 8;
    k_to_f16_ftz<<<grid, 256, 0, st>>>(x, out, n);
    MG_CHECK_LAUNCH();
    return MG_OK;
}

}  // namespace mg
