// Grouped GEMM on the FFMA pipe (fp32 accumulate) with the MoE epilogues.
// This is the product path for fp32 MoE (fp32 tolerances rule out TF32 tensor
// cores) and for fp16/bf16 shapes the TMA path cannot address (K % 8 != 0).
// Reference analog: the library GEMM + GemmPostKernel bias/activation pass
// (musa/ep/src/kernels/math/matmul.cc:239-332, gemm_post_kernels.mu:27-53).
#include "moe_kernels.h"

namespace moe {

namespace {

constexpr int SB_M = 64, SB_N = 64, SB_K = 16, SB_THREADS = 256;

template <typename T>
__device__ __forceinline__ const T* b_row(const GemmOperandB& b, int e, int n, int K) {
  const T* base = static_cast<const T*>(b.ptr);
  return base + static_cast<int64_t>(e) * b.n_rows * K +
         (static_cast<int64_t>(n + b.n_off) * b.G + b.g) * K;
}

template <typename T>
__device__ __forceinline__ float bias_at(const void* bias, int e, int n, const GemmArgs& g) {
  if (bias == nullptr) return 0.f;
  return to_f(static_cast<const T*>(bias)[e * g.bias_e_stride +
                                          static_cast<int64_t>(n) * g.bias_stride]);
}

template <typename T, bool kGated>
__global__ void __launch_bounds__(SB_THREADS) simt_gemm_kernel(const GemmArgs g) {
  constexpr int NB = kGated ? 2 : 1;
  __shared__ __align__(16) float As[SB_K][SB_M + 4];
  __shared__ __align__(16) float Bs[NB][SB_K][SB_N + 4];

  const int tile = blockIdx.x;
  if (tile >= g.tiles64[g.E]) return;
  int lo = 0, hi = g.E - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (g.tiles64[mid] <= tile) lo = mid; else hi = mid - 1;
  }
  const int e = lo;
  const int row0 = g.offsets[e] + (tile - g.tiles64[e]) * SB_M;
  const int row_end = g.offsets[e + 1];
  const int n0 = blockIdx.y * SB_N;
  const int K = g.K;
  const T* A = static_cast<const T*>(g.a);

  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int lr = tid >> 2, lk = (tid & 3) * 4;

  float acc[NB][4][4];
#pragma unroll
  for (int b = 0; b < NB; ++b)
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[b][i][j] = 0.f;

  const int ar = row0 + lr;
  const bool a_ok = ar < row_end;
  const T* a_row = A + static_cast<int64_t>(a_ok ? ar : row0) * K;
  const int bn = n0 + lr;
  const bool b_ok = bn < g.N;
  const T* b1_row = b_row<T>(g.b1, e, b_ok ? bn : 0, K);
  const T* b3_row = kGated ? b_row<T>(g.b3, e, b_ok ? bn : 0, K) : nullptr;

  for (int k0 = 0; k0 < K; k0 += SB_K) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int kk = k0 + lk + q;
      const bool kin = kk < K;
      As[lk + q][lr] = (a_ok && kin) ? to_f(a_row[kk]) : 0.f;
      Bs[0][lk + q][lr] = (b_ok && kin) ? to_f(b1_row[kk]) : 0.f;
      if (kGated) Bs[NB - 1][lk + q][lr] = (b_ok && kin) ? to_f(b3_row[kk]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < SB_K; ++kk) {
      const float4 av = *reinterpret_cast<const float4*>(&As[kk][ty * 4]);
      const float a4[4] = {av.x, av.y, av.z, av.w};
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        const float4 bv = *reinterpret_cast<const float4*>(&Bs[b][kk][tx * 4]);
        const float b4[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[b][i][j] = fmaf(a4[i], b4[j], acc[b][i][j]);
      }
    }
    __syncthreads();
  }

  T* out = static_cast<T*>(g.out);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = row0 + ty * 4 + i;
    if (r >= row_end) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n >= g.N) continue;
      float v;
      if (kGated) {
        v = act_gated(g.ap, acc[0][i][j] + bias_at<T>(g.bias1, e, n, g),
                      acc[NB - 1][i][j] + bias_at<T>(g.bias3, e, n, g));
      } else {
        v = act_single(g.ap.act, acc[0][i][j] + bias_at<T>(g.bias1, e, n, g));
      }
      out[static_cast<int64_t>(r) * g.ldo + n] = from_f<T>(v);
    }
  }
}

template <typename T>
cudaError_t launch_t(const GemmArgs& g, cudaStream_t s) {
  // Upper bound of 64-row tiles over all experts; CTAs past the device-side
  // total return at once, so no host synchronisation is needed.
  const int64_t m_tiles = (g.rows + SB_M - 1) / SB_M + g.E;
  const dim3 grid(static_cast<unsigned>(m_tiles), static_cast<unsigned>((g.N + SB_N - 1) / SB_N));
  if (g.gated)
    simt_gemm_kernel<T, true><<<grid, SB_THREADS, 0, s>>>(g);
  else
    simt_gemm_kernel<T, false><<<grid, SB_THREADS, 0, s>>>(g);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gemm_simt(const GemmArgs& g, cudaStream_t s) {
  if (g.rows == 0 || g.N == 0) return cudaSuccess;
  switch (g.dtype) {
    case kDtF32: return launch_t<float>(g, s);
    case kDtF16: return launch_t<__half>(g, s);
    case kDtBF16: return launch_t<__nv_bfloat16>(g, s);
  }
  return cudaErrorInvalidValue;
}

}  // namespace moe
