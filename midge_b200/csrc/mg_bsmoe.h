// mg_bsmoe.h -- decode-time routed experts on block-scaled tcgen05 MMAs
// (MXFP4 experts with ue8m0 scales); see mg_bsmoe.cu.
#pragma once
#include <cuda.h>
#include <stdint.h>

#include "mg_kernels.h"

namespace mg {

// Device buffers and TMA maps of the block-scaled decode MoE, owned by the
// model.  Activation rows are held as 16 packed e2m1 limbs each
// ([row*16 + limb][kpad/2] bytes) with one ue8m0 code per limb and block of
// 32 values (scale words [row][kpad/128][16], byte kb % 4 = block kb).
// The experts' own ue8m0 scales are also held as the tensor core reads them:
// per (layer, local expert) the gate/up units' atoms [ffn/64 tiles][kpad_h/256
// stages][1024 B], then the down units' [ceil(hidden/128)][kpad_f/256][1024 B]
// (bs_atoms_build, once the experts are loaded).
struct BsBuffers {
    uint8_t *xl;           // [8 tokens * 16][kpad_h/2] packed e2m1 limbs
    uint32_t *xsf;         // [8 tokens][kpad_h/128][16] scale words
    uint8_t *hl;           // [slots_max * 16][kpad_f/2]
    uint32_t *hsf;         // [slots_max][kpad_f/128][16]
    int kpad_h, kpad_f, slots_max;
    uint8_t *atoms;        // expert scale atoms, atoms_expert bytes per (layer, local expert)
    int64_t atoms_expert;  // bytes per expert
    int atoms_dn;          // first down unit of an expert (the gate/up units come first)
    uint32_t *sync;        // bs_sync_bytes(), zero between launches: per token group, its gate/up tiles done
};

bool bsmoe_supported(const mg_expert_layout &L);
int bs_kpad(int64_t k);  // K rounded up to the 256-value stage
size_t bs_limb_bytes(int rows, int kpad);
size_t bs_word_bytes(int rows, int kpad);
int bs_buffers_init(BsBuffers &b);
size_t bs_sync_bytes();
size_t bs_atoms_bytes(const mg_expert_layout &L, int kpad_h, int kpad_f);  // per expert
int bs_atoms_build(BsBuffers &b, const mg_expert_layout &L, const uint8_t *experts, int n_layers, int n_local,
                   cudaStream_t st);
int moe_bs(const MoeStreamArgs &a, cudaStream_t st);

}  // namespace mg
