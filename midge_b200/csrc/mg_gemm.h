// mg_gemm.h -- argument blocks of the tcgen05 expert-major GEMM (prefill).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "midgecuda.h"

namespace mg {

enum { XG_GATEUP = 0, XG_DOWN = 1, XG_DENSE = 2 };

struct XgTile {
    int e;      // expert (0 for a dense matrix)
    int row0;   // first row of the N tile within the expert's group
    int nrows;  // valid rows in the tile (<= 128)
};

struct XgArgs {
    mg_expert_layout L;
    const uint8_t *experts_layer;
    const uint8_t *dense_w, *dense_s;  // DENSE mode: one q8r matrix and its row scales
    const float *dense_bias;
    int64_t M, K;                      // output features, reduction length
    const XgTile *tiles;
    const int *ntiles;                 // device count of valid tiles
    const int *offs;                   // first expert-major row of each expert
    const int *slot_of_pos;            // DOWN: (token, rank) slot of each expert-major row: y is slot-major
    const int *rebase;                 // [E x 3] MXFP4 scale rebase exponents of this layer
    __half *out_hi, *out_lo;           // GATEUP output [P x M]
    float *y;                          // DOWN / DENSE output
    int64_t ldy;
    int accumulate;                    // DENSE: y += result
    int n_rows;                        // DENSE: activation rows (tile i = rows 128 i ..), no tile list
    int act_plain;
    float alpha, limit;
    int *err;
};

struct XgLaunch {
    XgArgs args;
    const __half *x_hi, *x_lo;  // activations [x_rows x K] f16
    int64_t x_rows;
    int max_tiles;
};

int xgemm(int mode, int dt, const XgLaunch &l, cudaStream_t st);

}  // namespace mg
