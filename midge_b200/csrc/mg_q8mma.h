// mg_q8mma.h -- decode-time int8-row GEMV (the q8r trunk: q, k, v, o) on
// tcgen05.mma.kind::i8; see mg_q8mma.cu.
#pragma once
#include <cuda.h>
#include <stdint.h>

#include "mg_kernels.h"

namespace mg {

// y = W x for q8r matrices (StreamGemvArgs with every matrix's TMA map set,
// scales = f32 per row, K % 16 == 0, no amax).
bool q8mma_supported(const StreamGemvArgs &a);
int q8mma_gemv(const StreamGemvArgs &a, cudaStream_t st);

}  // namespace mg
