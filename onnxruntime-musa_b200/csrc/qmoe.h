// QMoE weight handling: block-wise / per-row symmetric int4 and int8 expert
// weights (codes stored unsigned with zero point 2^(bits-1); int4 packs element
// 2i in the low nibble of byte i).
#pragma once

#include "../../include/moe_b200.h"
#include "moe_kernels.h"

namespace moe {

struct QmoeDequantOut {
  const void* w1;
  const void* w2;
  const void* w3;
};

// Workspace bytes for the dequantised weight copies (0 for MoE problems).
size_t qmoe_workspace_bytes(const moe_b200_problem& p);

// Dequantises fc1/fc2(/fc3) of every expert into `ws` in element type p.dtype.
int qmoe_dequantize(const moe_b200_problem& p, const moe_b200_tensors& t, uint8_t* ws,
                    const int32_t* expert_offsets, QmoeDequantOut* out, cudaStream_t s);

}  // namespace moe
