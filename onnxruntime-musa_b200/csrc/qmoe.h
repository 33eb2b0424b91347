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

// Rows of one expert's fc1 weights (2*inter for fused swiglu, else inter).
int64_t fc1_rows(const moe_b200_problem& p);

// True when this QMoE call takes the weight-streaming decode kernels.
bool qmoe_use_decode(const moe_b200_problem& p);

// True when a QMoE call beyond the decode sizes runs the tensor-core kernel that
// dequantises the packed weights in shared memory (no unpacked copy in HBM).
bool qmoe_use_fused(const moe_b200_problem& p);

// Workspace bytes of the QMoE path: fp32 partial sums (decode) or the dequantised
// weight copies (larger calls); 0 for MoE problems.
size_t qmoe_workspace_bytes(const moe_b200_problem& p);

// Decode path, in three steps: fc1 (+fc3) from the packed weights into `act` (token
// rows read from the layer input through `src`, the inverse permutation), fc2 into
// fp32 partial sums in `ws`, and the routing-weighted combine of the partials.
int qmoe_decode_fc1(const moe_b200_problem& p, const moe_b200_tensors& t, const int32_t* src,
                    void* act, const int32_t* offsets, uint8_t* ws, cudaStream_t s);
int qmoe_decode_fc2(const moe_b200_problem& p, const moe_b200_tensors& t, const void* act,
                    const int32_t* offsets, uint8_t* ws, cudaStream_t s);
int qmoe_decode_combine(const moe_b200_problem& p, const moe_b200_tensors& t, const uint8_t* ws,
                        const int32_t* offsets, const int32_t* pos, const float* w,
                        cudaStream_t s);

// Bytes of the dequantised fc1/fc2(/fc3) copies of every expert (element type p.dtype,
// each matrix 256-byte aligned).
size_t qmoe_dequantized_bytes(const moe_b200_problem& p);

// True when the dequantised copies hold exact codes (q - zero point) and the scale, one per
// output row, is left to the GEMM epilogue (fp16 QMoE with block_size 0).
bool qmoe_dequantized_exact(const moe_b200_problem& p);

// Dequantises fc1/fc2(/fc3) of every expert into `dst` (qmoe_dequantized_bytes(p) bytes).
int qmoe_dequantize_into(const moe_b200_problem& p, const moe_b200_tensors& t, uint8_t* dst,
                         QmoeDequantOut* out, cudaStream_t s);

// Compares, bit for bit, the dequantised copies `have` with what qmoe_dequantize_into would
// write for the weights in `t` (diff_dev: one device int of scratch); synchronises `s`.
int qmoe_dequantized_differs(const moe_b200_problem& p, const moe_b200_tensors& t,
                             const QmoeDequantOut& have, int* diff_dev, cudaStream_t s,
                             bool* differs);

// Dequantises fc1/fc2(/fc3) of every expert into `ws` in element type p.dtype.
int qmoe_dequantize(const moe_b200_problem& p, const moe_b200_tensors& t, uint8_t* ws,
                    const int32_t* expert_offsets, QmoeDequantOut* out, cudaStream_t s);

}  // namespace moe
