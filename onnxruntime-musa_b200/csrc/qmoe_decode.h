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
  // int4 with exact codes (block_size 0 or a multiple of 128): if set, `x` holds the
  // activations arranged by launch_qdec_prep and xcorr[x row][chunk] the offset term, and
  // the MMA runs on the biased codes (1024 + q in the low nibble, 1024 + 16 q in the high
  // nibble) with no per-code arithmetic; the chunk sums subtract xcorr.
  const float* xcorr = nullptr;
};

// Rows of T*k up to which the decode kernels replace dequantise + tensor-core GEMM.
constexpr int64_t kQmoeDecodeMaxRows = 512;
constexpr int kQmoeMaxSplits = 8;
// Routed rows up to which QMoE prefill dequantises in shared memory inside the GEMM.
constexpr int64_t kQmoeFusedMaxRows = 16384;

bool qmoe_decode_supported(int dtype, int bits, int block_size, int64_t H, int64_t I);
// Activations for the biased-code int4 path: x [rows, K] -> xp [rows, K] (each group of 8,
// x0..x7, stored as (x0,x4)(x1/16,x5/16)(x2,x6)(x3/16,x7/16): the mma.sync B fragments of
// the decode kernel's k order, odd slots scaled to match the in-place high nibbles) and
// corr [rows, K/128] = per 128-wide chunk, 1032 * sum(even slots) + 1152 * sum(odd, scaled).
// x_from_previous: x is written by the kernel launched just before (the fc1 activations);
// false when x is the layer input, so the prep overlaps the routing kernel.
cudaError_t launch_qdec_prep(const __half* x, int64_t rows, int K, __half* xp, float* corr,
                             bool x_from_previous, cudaStream_t s);
cudaError_t launch_qmoe_decode(const QDecodeArgs& a, int max_experts_touched, cudaStream_t s);
// act = activation(sum of fc1 partials + bias), fp16 [rows, N].
cudaError_t launch_finalize_fc1(const QDecodeArgs& a, __half* act, cudaStream_t s);
// out[t] = sum_j w[t,j] * (sum of fc2 partials of row pos[t,j] + fc2 bias of its expert).
cudaError_t launch_combine_partials(const float* part, int splits, int64_t rows, const int32_t* pos,
                                    const float* w, int T, int k, int H, const int32_t* offsets,
                                    int E, const void* bias, void* out, cudaStream_t s);

}  // namespace moe
