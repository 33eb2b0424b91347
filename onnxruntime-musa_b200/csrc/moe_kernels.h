// Internal launch interface between the host planner (moe_api.cu) and the device
// kernels.  Not part of the public C ABI.
#pragma once

#include "common.cuh"

namespace moe {

// Element type ids (ONNX TensorProto codes, as in the C ABI).
constexpr int kDtF32 = 1;
constexpr int kDtU8 = 2;
constexpr int kDtF16 = 10;
constexpr int kDtBF16 = 16;

// Records `fmt` as this thread's last error message (read by moe_b200_last_error)
// and returns `code`.
int set_error(int code, const char* fmt, ...);
// Resets the runtime's last-error state at the start of a public entry point.  A failed
// runtime call elsewhere in the process (an allocation that ran out of memory, say) leaves
// a non-sticky error that the next cudaGetLastError() would report; without the reset a
// launch check of this library would blame its own launch for it.  Sticky errors (a
// faulted context) stay and are still reported.
inline void clear_stale_cuda_error() { (void)cudaGetLastError(); }

inline int dtype_bytes(int dt) { return dt == kDtF32 ? 4 : (dt == kDtU8 ? 1 : 2); }

// Routing chunk: rows handled by one CTA of the router / permutation kernels (the
// standalone stage entry points use kRouteChunk; a layer call sizes chunks to the GPU).
constexpr int kRouteThreads = 256;
// Routing mode passed as launch_route's `normalize`: 0 / 1 = softmax top-k without / with
// renormalisation over the k selected; kRouteSparseMixer = the sparse-mixer top-2.
constexpr int kRouteSparseMixer = 2;
constexpr float kSparseMixerJitterEps = 0.01f;
constexpr int kRouteChunk = 256;
inline int num_route_chunks(int64_t rows, int chunk = kRouteChunk) {
  return static_cast<int>((rows + chunk - 1) / chunk);
}
// Rows per routing chunk of a layer call: about one chunk per SM, 32..256 rows.
inline int layer_route_chunk(int64_t rows) {
  int64_t c = (rows + 147) / 148;
  c = (c + 31) / 32 * 32;
  return static_cast<int>(c < 32 ? 32 : (c > kRouteChunk ? kRouteChunk : c));
}
constexpr int kMaxExperts = 256;
constexpr int kMaxEpRanks = 8;   // expert-parallel ranks (GPUs of one node)
constexpr int kMaxK = 32;
// Routed rows (T*k) up to which routing and the dispatch plan run in one CTA.
constexpr int kSmallDispatchRows = 1024;
// Default row limit of the CTA-pair kernel's swapped tail tiles (multiple of 16, <= 240).
constexpr int kPairSwapMax = 128;

// Words of a layer call's status block (error word + GEMM tile counters) that the first
// kernel of the call zeroes (`clear`, nullable): no separate memset in the stream.
constexpr int kClearWords = 4;
cudaError_t launch_route(int dtype, const void* logits, int T, int E, int k, int normalize,
                         int32_t* idx, float* w, int32_t* chunk_counts, cudaStream_t s,
                         int chunk = kRouteChunk, int* clear = nullptr);
// Routing + offsets + permutation of a call with T*k <= kSmallDispatchRows, one CTA
// (no GEMM tile prefixes: for the decode kernels only).
cudaError_t launch_small_dispatch(int dtype, const void* logits, int T, int E, int k,
                                  int normalize, int32_t* idx, float* w, int32_t* offsets,
                                  int32_t* pos, int32_t* src, cudaStream_t s,
                                  int* clear = nullptr);
cudaError_t launch_histogram(const int32_t* idx, int T, int k, int E, int32_t* chunk_counts,
                             int* err, cudaStream_t s, int chunk = kRouteChunk);
cudaError_t launch_plan(const int32_t* idx, int T, int k, int E, const int32_t* chunk_counts,
                        int32_t* chunk_base, int32_t* offsets, int32_t* tiles128,
                        int32_t* tiles64, int32_t* tiles256, int32_t* pos, int32_t* src,
                        cudaStream_t s, int chunk = kRouteChunk);
cudaError_t launch_gather(const void* x, int64_t row_bytes, int k, const int32_t* src,
                          int64_t rows, void* xp, cudaStream_t s);
// out[r] = sum over k of a[r, k] (fp16 rows, fp32 sum in a fixed order).
cudaError_t launch_row_sums(const void* a, int64_t rows, int K, float* out, cudaStream_t s);
cudaError_t launch_fill_f32(float* dst, float value, int64_t n, cudaStream_t s,
                            int* clear = nullptr);
cudaError_t launch_combine(int dtype, const void* y, const int32_t* pos, const float* w,
                           int T, int k, int H, void* out, cudaStream_t s);
// Residual add + RMS normalisation + router MatMul of the rows feeding an MoE node
// (norm_router.cu); H % 8 == 0, 16-byte aligned rows.
size_t norm_router_smem_bytes(int dtype, int64_t H);
cudaError_t launch_norm_router(int dtype, const void* x, const void* skip, const float* gamma,
                               float eps, const void* wr, int64_t rows, int H, int E,
                               void* residual_out, void* normed, void* logits, cudaStream_t s);

// One grouped GEMM pass over all experts:
//   out[r, n] = epilogue( sum_k A[r, k] * B1[e(r), n, k] [, sum_k A[r, k] * B3[e(r), n, k]] )
// for every permuted row r of expert e (rows offsets[e] .. offsets[e+1]).
// B matrices are addressed as [E][Nrows][G][K] with element (e, n, g, k) at
//   b + e*b_e_stride + (n*G + g)*K + k, so an interleaved fused fc1 (G=2) selects its
// gate (g=0) and linear (g=1) rows by g; a split fc1 selects halves by n offset.
struct GemmOperandB {
  const void* ptr;     // weights of all experts
  int g;               // interleave selector (0 or 1)
  int G;               // interleave factor (1 or 2)
  int n_off;           // row offset (split fc1: I for the linear half)
  int n_rows;          // rows of one expert's matrix (as stored: N*G + ...)
  const void* scales = nullptr;  // packed (QMoE) operand: fp16 scales per stored row/block
};

struct GemmArgs {
  int dtype;                   // element type of A, B and out
  const void* a;               // [R, K] permuted activations
  int64_t rows;                // R
  int K;
  int N;                       // output columns
  bool gated;                  // two B operands combined by act_gated
  GemmOperandB b1, b3;         // b3 used when gated
  const int32_t* offsets;      // [E+1]
  const int32_t* tiles128;     // [E+1] prefix of ceil(count/128)
  const int32_t* tiles64;      // [E+1] prefix of ceil(count/64)
  const int32_t* tiles256;     // [E+1] prefix of ceil(count/256)
  int E;
  const void* bias1;           // element (e, n) at bias1[e*bias_e_stride + n*bias_stride]
  const void* bias3;
  int bias_stride;
  int64_t bias_e_stride;
  ActParams ap;                // plain: act applied to (acc + bias1); kIdentity for fc2
  void* out;                   // [R, N]
  int64_t ldo;
  int* err;
  int qbits = 0;               // 4 / 8: B operands are packed codes (b*.scales set)
  int qblock = 0;              // scale block along K (0 = one scale per row)
  int test_stall = 0;          // test hook: tensor-core producers issue nothing
  // CTA-pair kernel: the last tile of an expert with at most this many rows runs with the
  // operands swapped (weights as M = 256, its rows as N = rows rounded up to 16); 0 = never.
  int swap_max = kPairSwapMax;
  // CTA-pair kernel: a zeroed int from which CTA pairs claim tiles in order (dynamic
  // schedule); nullptr = static round-robin.
  int* tile_counter = nullptr;
  // Packed operands with one scale per row (qblock 0): 0 = scale in the converters,
  // 1 = exact codes with the scale applied in the epilogue, 2 = biased codes (1024 + q) with
  // the epilogue subtracting (1024 + zp) * rowsum[row] before scaling (rowsum: fp32 sums of
  // the A rows over K; without it mode 2 runs as 1).
  int qepi = 0;
  const float* rowsum = nullptr;
  // Tensor-core kernels: output row remap for the expert-parallel return (row p of
  // segment q, seg_start[q] <= p < seg_start[q+1], is stored at row seg_dst[q] + p -
  // seg_start[q] of out_peers[q % remap_world]); seg_start == nullptr: rows of `out`.
  const int32_t* seg_start = nullptr;
  const int32_t* seg_dst = nullptr;
  int nseg = 0;
  int remap_world = 1;
  void* out_peers[kMaxEpRanks] = {};
  // Gathered A (fc1): row p of A is row gather_src[p] / gather_k of gather_x
  // ([gather_x_rows, K]).  The CTA-pair tensor-core kernel reads those rows straight
  // from gather_x with TMA gather4 loads; every other kernel gets them from a gather
  // pass into `a` first (launch_gemm_tc_gathered).
  const void* gather_x = nullptr;
  const int32_t* gather_src = nullptr;
  int gather_k = 1;
  int64_t gather_x_rows = 0;
  // fc2 with the routing-weighted combine fused into the epilogue (plain, ungated GEMM on
  // the single-device path): after storing its part of an output row (permuted row p,
  // token comb_src[p] / comb_k) in `out`, the epilogue counts one arrival per (token,
  // 32-column segment) in comb_cnt (zeroed, [tokens, N / 32]); the arrival that completes
  // the k rows of a segment sums them in slot order, w[t,j] * Y[pos[t,j]], into
  // comb_out[t] (fp32 accumulation, the order of the separate combine kernel).
  unsigned* comb_cnt = nullptr;
  const int32_t* comb_src = nullptr;
  const int32_t* comb_pos = nullptr;
  const float* comb_w = nullptr;
  void* comb_out = nullptr;
  int comb_k = 1;
};

cudaError_t launch_gemm_simt(const GemmArgs& g, cudaStream_t s);
// tcgen05 path; requires dtype f16/bf16, K % 8 == 0.
bool tc_supported(const GemmArgs& g);
// mode: 0 = choose, 1 = single-CTA kernel, 2 = CTA-pair (cta_group::2) kernel.
cudaError_t launch_gemm_tc(const GemmArgs& g, int num_sms, int mode, cudaStream_t s);
// True when launch_gemm_tc(g, mode) runs the CTA-pair kernel with A rows gathered by TMA
// (g.gather_src set, operands aligned for the gather map).
bool tc_pair_gathers(const GemmArgs& g, int mode);
// CTA-pair kernel with int4/int8 B operands dequantised in shared memory (fp16 only).
bool tc_q_supported(const GemmArgs& g);
cudaError_t launch_gemm_tc_q(const GemmArgs& g, int num_sms, cudaStream_t s);

}  // namespace moe
