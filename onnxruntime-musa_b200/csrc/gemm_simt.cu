// Grouped GEMM on the FFMA pipe (fp32 accumulate) with the MoE epilogues: a cp.async
// pipelined kernel for 16-byte-aligned rows and a scalar kernel for the rest.
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
  pdl_wait();  // launched dependent (launch_dependent): predecessors' data after this
  pdl_launch_dependents();
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

// ---------------------------------------------------------------------------------------
// Pipelined variant for 16-byte-aligned rows: A and B tiles of 64 x PK move by cp.async
// into a PS-stage ring (rows past the expert's end and columns past K are zero-filled), so
// the global loads of the next stages overlap this stage's FMAs.  Shared memory keeps the
// rows K-contiguous; a thread owns rows ty + 16 i and columns tx + 16 j, so the eight
// threads of a 128-bit load phase read eight consecutive rows (a row pitch of an odd number
// of 16-byte units keeps them on distinct banks).  Every output sums its products in
// ascending k, as the scalar kernel does.
constexpr int PK = 32;      // k per stage
constexpr int PS = 3;       // stages
template <typename T> constexpr int pitch() { return PK + 16 / static_cast<int>(sizeof(T)); }
template <typename T, bool kGated> constexpr int pipe_smem() {
  return PS * (kGated ? 3 : 2) * SB_M * pitch<T>() * static_cast<int>(sizeof(T));
}

__device__ __forceinline__ void cp_async16_zfill(void* smem, const void* gmem, bool ok) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem),
               "r"(ok ? 16 : 0)
               : "memory");
}

template <typename T>
__device__ __forceinline__ float4 lds4(const T* p) {
  if constexpr (sizeof(T) == 4) {
    return *reinterpret_cast<const float4*>(p);
  } else {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    const T* e = reinterpret_cast<const T*>(&v);
    return make_float4(to_f(e[0]), to_f(e[1]), to_f(e[2]), to_f(e[3]));
  }
}

template <typename T, bool kGated>
__global__ void __launch_bounds__(SB_THREADS) simt_gemm_pipe_kernel(const GemmArgs g) {
  pdl_wait();  // launched dependent (launch_dependent): predecessors' data after this
  pdl_launch_dependents();
  constexpr int NB = kGated ? 2 : 1;
  constexpr int P = pitch<T>();
  constexpr int VEC = 16 / static_cast<int>(sizeof(T));  // elements per 16-byte piece
  constexpr int PIECES = SB_M * PK / VEC;                 // 16-byte pieces per 64 x PK tile
  extern __shared__ __align__(16) uint8_t pipe_raw[];
  T* sm = reinterpret_cast<T*>(pipe_raw);
  auto tile_ptr = [&](int stage, int m) { return sm + (stage * (NB + 1) + m) * SB_M * P; };

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

  auto load_stage = [&](int stage, int k0) {
    for (int pc = tid; pc < PIECES; pc += SB_THREADS) {
      const int r = pc / (PK / VEC), kc = (pc % (PK / VEC)) * VEC;
      const int k = k0 + kc;
      const bool kin = k < K;
      const int ar = row0 + r;
      const bool aok = kin && ar < row_end;
      cp_async16_zfill(tile_ptr(stage, 0) + r * P + kc, A + static_cast<int64_t>(aok ? ar : row0) * K + (kin ? k : 0), aok);
      const int bn = n0 + r;
      const bool bok = kin && bn < g.N;
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        const T* brow = b_row<T>(b == 0 ? g.b1 : g.b3, e, bok ? bn : 0, K);
        cp_async16_zfill(tile_ptr(stage, 1 + b) + r * P + kc, brow + (kin ? k : 0), bok);
      }
    }
  };

  float acc[NB][4][4];
#pragma unroll
  for (int b = 0; b < NB; ++b)
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[b][i][j] = 0.f;

  const int nk = (K + PK - 1) / PK;
#pragma unroll
  for (int st = 0; st < PS - 1; ++st) {
    if (st < nk) load_stage(st, st * PK);
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  for (int kt = 0; kt < nk; ++kt) {
    asm volatile("cp.async.wait_group %0;" ::"n"(PS - 2) : "memory");
    __syncthreads();
    // The stage read PS - 1 steps ago is free (everyone passed the barrier above).
    if (kt + PS - 1 < nk) load_stage((kt + PS - 1) % PS, (kt + PS - 1) * PK);
    asm volatile("cp.async.commit_group;" ::: "memory");
    const int stage = kt % PS;
    const T* As = tile_ptr(stage, 0);
#pragma unroll
    for (int kk = 0; kk < PK; kk += 4) {
      float4 a4[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a4[i] = lds4(As + (ty + 16 * i) * P + kk);
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        const T* Bs = tile_ptr(stage, 1 + b);
        float4 b4[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) b4[j] = lds4(Bs + (tx + 16 * j) * P + kk);
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float v = acc[b][i][j];
            v = fmaf(a4[i].x, b4[j].x, v);
            v = fmaf(a4[i].y, b4[j].y, v);
            v = fmaf(a4[i].z, b4[j].z, v);
            v = fmaf(a4[i].w, b4[j].w, v);
            acc[b][i][j] = v;
          }
      }
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");

  T* out = static_cast<T*>(g.out);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = row0 + ty + 16 * i;
    if (r >= row_end) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx + 16 * j;
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
  auto aligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  const bool pipe = (static_cast<int64_t>(g.K) * sizeof(T)) % 16 == 0 && aligned(g.a) &&
                    aligned(g.b1.ptr) && (!g.gated || aligned(g.b3.ptr));
  if (pipe) {
    static bool attr_set[2] = {false, false};  // idempotent; a race between first callers is benign
    const int smem = g.gated ? pipe_smem<T, true>() : pipe_smem<T, false>();
    if (!attr_set[g.gated]) {
      cudaError_t st = g.gated ? cudaFuncSetAttribute(simt_gemm_pipe_kernel<T, true>,
                                                      cudaFuncAttributeMaxDynamicSharedMemorySize, smem)
                               : cudaFuncSetAttribute(simt_gemm_pipe_kernel<T, false>,
                                                      cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (st != cudaSuccess) return st;
      attr_set[g.gated] = true;
    }
    return g.gated ? launch_dependent(pdl_layer_enabled(), simt_gemm_pipe_kernel<T, true>, grid, dim3(SB_THREADS), smem, s, g)
                   : launch_dependent(pdl_layer_enabled(), simt_gemm_pipe_kernel<T, false>, grid, dim3(SB_THREADS), smem, s, g);
  }
  return g.gated ? launch_dependent(pdl_layer_enabled(), simt_gemm_kernel<T, true>, grid, dim3(SB_THREADS), 0, s, g)
                 : launch_dependent(pdl_layer_enabled(), simt_gemm_kernel<T, false>, grid, dim3(SB_THREADS), 0, s, g);
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
