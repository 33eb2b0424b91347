// Launch interface of the QMoE weight-streaming (decode) kernels.
#pragma once

#include "moe_kernels.h"

namespace moe {

// Packed weights of all experts with the same row addressing as GemmOperandB: the
// stored row of output row n of expert e is e*n_rows + (n + n_off)*G + g.
struct QOperand {
  const uint8_t* q;        // codes, K*bits/8 bytes per stored row
  const __half* scales;    // [E*n_rows][nb] (nb = ceil(K/block_size), or 1 per row)
  int g, G, n_off, n_rows;
};

struct QDecodeArgs {
  const __half* x;            // activations: [rows, K] in expert order, or the layer input
  const int32_t* src_rows;    // if set, routed row p reads x row src_rows[p] / k
  int k;
  int64_t rows;
  int K;
  int N;
  int E;
  const int32_t* offsets;     // [E+1]
  int bits;                   // 4 or 8
  int block_size;             // 0 = one scale per row
  bool gated;
  QOperand b1, b3;
  ActParams ap;
  const void* bias1;          // fp16 bias, element (e, n) at e*bias_e_stride + n*bias_stride
  const void* bias3;
  int bias_stride;
  int64_t bias_e_stride;
  __half* out;                // [rows, ldo] activation output (fc1 without split), or
  float* out_partial;         // [splits][rows][ldo] fp32 partial sums without bias
                              // (gated: gate sums at [0, N), linear sums at [N, 2N))
  int64_t ldo;
  int splits;
};

// Rows of T*k up to which the decode kernels replace dequantise + tensor-core GEMM.
constexpr int64_t kQmoeDecodeMaxRows = 512;
constexpr int kQmoeMaxSplits = 8;
// Routed rows up to which QMoE prefill dequantises in shared memory inside the GEMM.
constexpr int64_t kQmoeFusedMaxRows = 16384;

bool qmoe_decode_supported(int dtype, int bits, int block_size, int64_t H, int64_t I);
cudaError_t launch_qmoe_decode(const QDecodeArgs& a, int max_experts_touched, cudaStream_t s);
// act = activation(sum of fc1 partials + bias), fp16 [rows, N].
cudaError_t launch_finalize_fc1(const QDecodeArgs& a, __half* act, cudaStream_t s);
// out[t] = sum_j w[t,j] * (sum of fc2 partials of row pos[t,j] + fc2 bias of its expert).
cudaError_t launch_combine_partials(const float* part, int splits, int64_t rows, const int32_t* pos,
                                    const float* w, int T, int k, int H, const int32_t* offsets,
                                    int E, const void* bias, void* out, cudaStream_t s);

}  // namespace moe
