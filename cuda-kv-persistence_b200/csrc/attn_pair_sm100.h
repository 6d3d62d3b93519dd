// BF16 remapped attention on SM pairs (csrc/attn_pair_sm100.cu): the same
// contract as launch_attn_bf16 (attn_sm100.h), without the key-range split.
#pragma once

#include "attn_sm100.h"

namespace kvp {

// Shapes the pair kernel runs (head_dim 128; any tokens, frames, mode,
// window, flat tiling and KVMap).
bool attn_pair_supported(const AttnDesc& d);

// One cluster of two CTAs per 256 query rows of one head.  Same arguments,
// checks and outputs as launch_attn_bf16.
int launch_attn_bf16_pair(const LayerIO& io, const AttnDesc& d, int* d_status, cudaStream_t stream);

}  // namespace kvp
