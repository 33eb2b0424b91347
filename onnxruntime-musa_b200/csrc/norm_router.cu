// Pre-MoE block in one pass over the hidden states: optional residual add, RMS
// normalisation and the router MatMul that produces the MoE node's router_probs.
//
//   h      = input (+ skip)                          fp32; stored as residual_out (dtype)
//   normed = dtype(h * rsqrt(mean(h^2) + eps) * gamma)   gamma fp32 [H]
//   logits = dtype(normed . router_weight[e])        fp32 accumulation, router_weight [E, H]
//
// Reference analogs: the RMS normalisation the plugin fuses from
// Pow/ReduceMean/Add/Sqrt/Div/Mul (musa/ep/src/fusion/rms_norm_fusion.cc:185) and runs as
// RmsNormKernel (musa/ep/src/kernels/nn/rms_norm_impl.mu:10-45: fp32 gamma,
// rsqrt(mean + eps), value * inv * gamma), followed by the router MatMul on muBLAS
// (musa/ep/src/kernels/math/matmul.cc:239-332).  The logits use the rounded normalised
// values, as the unfused MatMul would.
//
// One warp per row: a first pass sums the squares (16-byte loads), a second writes the
// normalised row (global and a shared-memory copy); the router MatMul then runs on the
// tensor cores over 16-row tiles for fp16/bf16 (norm_router_tc_kernel) or as 16 expert
// dot products at a time per row otherwise.  HBM-bound: x (+ skip) read twice (the second
// read mostly from L2), normed (+ residual) written once.
#include <type_traits>

#include "moe_kernels.h"

namespace moe {

namespace {

constexpr int NR_WARPS = 4;
constexpr int NR_EBLOCK = 16;

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const T* e = reinterpret_cast<const T*>(&u);
  if constexpr (sizeof(T) == 4) {
    // 16 bytes hold 4 floats: two loads for 8 values.
    const uint4 w = *reinterpret_cast<const uint4*>(p + 4);
    const float* a = reinterpret_cast<const float*>(&u);
    const float* b = reinterpret_cast<const float*>(&w);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[j] = a[j];
      v[4 + j] = b[j];
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = to_f(e[j]);
  }
}

template <typename T>
__device__ __forceinline__ void store8(T* p, const float (&v)[8]) {
  if constexpr (sizeof(T) == 4) {
    reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    uint4 u;
    u.x = pack2<T>(v[0], v[1]);
    u.y = pack2<T>(v[2], v[3]);
    u.z = pack2<T>(v[4], v[5]);
    u.w = pack2<T>(v[6], v[7]);
    *reinterpret_cast<uint4*>(p) = u;
  }
}

template <typename T>
__device__ __forceinline__ void load_h(const T* x, const T* skip, int c, float (&h)[8]) {
  load8<T>(x + c, h);
  if (skip != nullptr) {
    float s[8];
    load8<T>(skip + c, s);
#pragma unroll
    for (int j = 0; j < 8; ++j) h[j] += s[j];
  }
}

template <typename T>
__global__ void __launch_bounds__(NR_WARPS * 32)
norm_router_kernel(const T* __restrict__ x, const T* __restrict__ skip,
                   const float* __restrict__ gamma, float eps, const T* __restrict__ wr,
                   int64_t rows, int H, int E, T* __restrict__ residual_out,
                   T* __restrict__ normed, T* __restrict__ logits) {
  extern __shared__ __align__(16) uint8_t nr_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * NR_WARPS + warp;
  if (row >= rows) return;
  T* srow = reinterpret_cast<T*>(nr_smem) + static_cast<int64_t>(warp) * H;
  const T* xr = x + row * H;
  const T* sr = skip != nullptr ? skip + row * H : nullptr;

  float ss = 0.f;
  for (int c = lane * 8; c < H; c += 256) {
    float h[8];
    load_h<T>(xr, sr, c, h);
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = fmaf(h[j], h[j], ss);
    if (residual_out != nullptr) store8<T>(residual_out + row * H + c, h);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = rsqrtf(ss / static_cast<float>(H) + eps);

  for (int c = lane * 8; c < H; c += 256) {
    float h[8];
    load_h<T>(xr, sr, c, h);
    const float4 g0 = __ldg(reinterpret_cast<const float4*>(gamma + c));
    const float4 g1 = __ldg(reinterpret_cast<const float4*>(gamma + c + 4));
    const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
    float n[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) n[j] = h[j] * inv * g[j];
    if (normed != nullptr) store8<T>(normed + row * H + c, n);
    store8<T>(srow + c, n);
  }
  __syncwarp();

  for (int e0 = 0; e0 < E; e0 += NR_EBLOCK) {
    float acc[NR_EBLOCK];
#pragma unroll
    for (int i = 0; i < NR_EBLOCK; ++i) acc[i] = 0.f;
    for (int c = lane * 8; c < H; c += 256) {
      float n[8];
      load8<T>(srow + c, n);  // the rounded normalised values
#pragma unroll
      for (int i = 0; i < NR_EBLOCK; ++i) {
        if (e0 + i >= E) break;
        float w[8];
        load8<T>(wr + static_cast<int64_t>(e0 + i) * H + c, w);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i] = fmaf(n[j], w[j], acc[i]);
      }
    }
#pragma unroll
    for (int i = 0; i < NR_EBLOCK; ++i)
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
    if (lane < NR_EBLOCK && e0 + lane < E) {
      float v = 0.f;
#pragma unroll
      for (int i = 0; i < NR_EBLOCK; ++i)
        if (i == lane) v = acc[i];
      logits[row * E + e0 + lane] = from_f<T>(v);
    }
  }
}

// 16-bit types: a CTA of 8 warps takes 16 rows.  Each warp normalises two rows into a
// shared [16][H + 8] tile (8 elements of padding per row: conflict-free fragment loads,
// zero-filled K tail); then the router MatMul runs on the tensor cores (mma.sync
// m16n8k16, fp32 accumulation), warp w taking expert columns [8j, 8j + 8) for
// j = w, w + 8, ..., so the router weights are read once per 16 rows instead of once per
// row.
constexpr int NR_TC_ROWS = 16;
constexpr int NR_TC_WARPS = 8;

__host__ __device__ constexpr size_t tc_tile_bytes(int64_t H) {
  return static_cast<size_t>(NR_TC_ROWS) * (H + 8) * 2;  // 16-byte multiple (H % 8 == 0)
}

__device__ __forceinline__ void nr_mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                       uint32_t b1, bool bf16) {
  if (bf16)
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  else
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <typename T>
__global__ void __launch_bounds__(NR_TC_WARPS * 32)
norm_router_tc_kernel(const T* __restrict__ x, const T* __restrict__ skip,
                      const float* __restrict__ gamma, float eps, const T* __restrict__ wr,
                      int64_t rows, int H, int E, T* __restrict__ residual_out,
                      T* __restrict__ normed, T* __restrict__ logits) {
  extern __shared__ __align__(16) uint8_t nr_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ld = H + 8;                  // padded row (elements)
  const int Kp = (H + 15) & ~15;         // K rounded up to the MMA depth
  T* tile = reinterpret_cast<T*>(nr_smem);
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * NR_TC_ROWS;

  for (int rr = warp; rr < NR_TC_ROWS; rr += NR_TC_WARPS) {
    const int64_t row = row0 + rr;
    T* srow = tile + rr * ld;
    if (row >= rows) {
      for (int c = lane; c < Kp; c += 32) srow[c] = from_f<T>(0.f);
      continue;
    }
    const T* xr = x + row * H;
    const T* sr = skip != nullptr ? skip + row * H : nullptr;
    float ss = 0.f;
#pragma unroll 4
    for (int c = lane * 8; c < H; c += 256) {
      float h[8];
      load_h<T>(xr, sr, c, h);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(h[j], h[j], ss);
      if (residual_out != nullptr) store8<T>(residual_out + row * H + c, h);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = rsqrtf(ss / static_cast<float>(H) + eps);
#pragma unroll 4
    for (int c = lane * 8; c < H; c += 256) {
      float h[8];
      load_h<T>(xr, sr, c, h);
      const float4 g0 = __ldg(reinterpret_cast<const float4*>(gamma + c));
      const float4 g1 = __ldg(reinterpret_cast<const float4*>(gamma + c + 4));
      const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
      float n[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) n[j] = h[j] * inv * g[j];
      if (normed != nullptr) store8<T>(normed + row * H + c, n);
      store8<T>(srow + c, n);
    }
    for (int c = H + lane; c < Kp; c += 32) srow[c] = from_f<T>(0.f);
  }
  __syncthreads();

  const int g = lane >> 2, t = lane & 3;
  const uint32_t* tw = reinterpret_cast<const uint32_t*>(tile);
  const int ldw = ld / 2;  // padded row in 32-bit words
  // With fewer than 8 expert tiles, `wpt` warps share a tile by splitting K; their
  // partial tiles are summed in shared memory in warp order (deterministic).
  const int ntile = (E + 7) / 8;
  const int wpt = ntile >= 8 ? 1 : (ntile >= 4 ? 2 : (ntile >= 2 ? 4 : 8));
  const int kslice = warp % wpt;
  const int ksteps = Kp / 16;
  const int kper = (ksteps + wpt - 1) / wpt;
  float* red = reinterpret_cast<float*>(nr_smem + tc_tile_bytes(H));  // [8][32][4]
  for (int j = warp / wpt; j < ntile; j += NR_TC_WARPS / wpt) {
    const int e = min(j * 8 + g, E - 1);     // B column of this thread
    const T* wrow = wr + static_cast<int64_t>(e) * H;
    float d[4] = {0.f, 0.f, 0.f, 0.f};
    const int kb = kslice * kper * 16, ke = min(Kp, (kslice + 1) * kper * 16);
    for (int k0 = kb; k0 < ke; k0 += 16) {
      uint32_t a[4];
      a[0] = tw[g * ldw + (k0 >> 1) + t];
      a[1] = tw[(g + 8) * ldw + (k0 >> 1) + t];
      a[2] = tw[g * ldw + (k0 >> 1) + 4 + t];
      a[3] = tw[(g + 8) * ldw + (k0 >> 1) + 4 + t];
      const int ka = k0 + 2 * t, kb = k0 + 8 + 2 * t;
      const uint32_t b0 = ka < H ? __ldg(reinterpret_cast<const uint32_t*>(wrow + ka)) : 0u;
      const uint32_t b1 = kb < H ? __ldg(reinterpret_cast<const uint32_t*>(wrow + kb)) : 0u;
      nr_mma(d, a, b0, b1, sizeof(T) == 2 && !std::is_same<T, __half>::value);
    }
    if (wpt > 1) {
      // One tile per warp group: publish the partial tile, sum in the group's first warp.
#pragma unroll
      for (int q = 0; q < 4; ++q) red[(warp * 32 + lane) * 4 + q] = d[q];
    }
    if (wpt == 1) {
      // d: rows g / g + 8, expert columns j*8 + 2t, + 1
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int64_t row = row0 + g + (q >> 1) * 8;
        const int ec = j * 8 + 2 * t + (q & 1);
        if (row < rows && ec < E) logits[row * E + ec] = from_f<T>(d[q]);
      }
    }
  }
  if (wpt == 1) return;
  __syncthreads();
  const int j = warp / wpt;
  if (kslice != 0 || j >= ntile) return;
  float d[4] = {0.f, 0.f, 0.f, 0.f};
  for (int w2 = warp; w2 < warp + wpt; ++w2)
#pragma unroll
    for (int q = 0; q < 4; ++q) d[q] += red[(w2 * 32 + lane) * 4 + q];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int64_t row = row0 + g + (q >> 1) * 8;
    const int ec = j * 8 + 2 * t + (q & 1);
    if (row < rows && ec < E) logits[row * E + ec] = from_f<T>(d[q]);
  }
}

size_t tc_smem_bytes(int64_t H) {
  return tc_tile_bytes(H) + NR_TC_WARPS * 32 * 4 * sizeof(float);
}

template <typename T>
cudaError_t launch_t(const void* x, const void* skip, const float* gamma, float eps,
                     const void* wr, int64_t rows, int H, int E, void* residual_out,
                     void* normed, void* logits, cudaStream_t s) {
  if constexpr (sizeof(T) == 2) {
    const size_t smem = tc_smem_bytes(H);
    if (smem <= 227 * 1024) {
      if (smem > 48 * 1024) {
        cudaError_t st = cudaFuncSetAttribute(norm_router_tc_kernel<T>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              static_cast<int>(smem));
        if (st != cudaSuccess) return st;
      }
      const int64_t blocks = (rows + NR_TC_ROWS - 1) / NR_TC_ROWS;
      norm_router_tc_kernel<T><<<static_cast<unsigned>(blocks), NR_TC_WARPS * 32, smem, s>>>(
          static_cast<const T*>(x), static_cast<const T*>(skip), gamma, eps,
          static_cast<const T*>(wr), rows, H, E, static_cast<T*>(residual_out),
          static_cast<T*>(normed), static_cast<T*>(logits));
      return cudaGetLastError();
    }
  }
  const size_t smem = static_cast<size_t>(NR_WARPS) * H * sizeof(T);
  if (smem > 48 * 1024) {
    cudaError_t st = cudaFuncSetAttribute(norm_router_kernel<T>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(smem));
    if (st != cudaSuccess) return st;
  }
  const int64_t blocks = (rows + NR_WARPS - 1) / NR_WARPS;
  norm_router_kernel<T><<<static_cast<unsigned>(blocks), NR_WARPS * 32, smem, s>>>(
      static_cast<const T*>(x), static_cast<const T*>(skip), gamma, eps,
      static_cast<const T*>(wr), rows, H, E, static_cast<T*>(residual_out),
      static_cast<T*>(normed), static_cast<T*>(logits));
  return cudaGetLastError();
}

}  // namespace

size_t norm_router_smem_bytes(int dtype, int64_t H) {
  return static_cast<size_t>(NR_WARPS) * H * dtype_bytes(dtype);
}

cudaError_t launch_norm_router(int dtype, const void* x, const void* skip, const float* gamma,
                               float eps, const void* wr, int64_t rows, int H, int E,
                               void* residual_out, void* normed, void* logits, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  switch (dtype) {
    case kDtF32:
      return launch_t<float>(x, skip, gamma, eps, wr, rows, H, E, residual_out, normed, logits, s);
    case kDtF16:
      return launch_t<__half>(x, skip, gamma, eps, wr, rows, H, E, residual_out, normed, logits, s);
    case kDtBF16:
      return launch_t<__nv_bfloat16>(x, skip, gamma, eps, wr, rows, H, E, residual_out, normed,
                                     logits, s);
  }
  return cudaErrorInvalidValue;
}

}  // namespace moe
