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
// fp16/bf16: norm_router_tc_kernel (16-row CTAs, K in chunks, the router MatMul on the
// tensor cores).  fp32: one warp per row: a first pass sums the squares, a second writes
// the normalised row (global and a shared-memory copy), then 16 expert dot products at a
// time.  HBM-bound: x (+ skip) read twice (the second read mostly from L2), normed
// (+ residual) written once.
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

// 16-bit types: a CTA of 8 warps takes NR_TC_LIVE = 8 rows (more CTAs per SM than 16-row
// CTAs; the MMA's rows 8-15 are zero).  A first pass gives each row its 1/rms (a warp per
// row); then K is walked in chunks of NR_KC columns: every thread normalises one 16-byte
// piece of the chunk (writing normed and residual), stages it in shared memory
// ([16][NR_KC + 8]: 8 elements of padding make the fragment loads conflict-free), loads its
// piece of the next chunk into registers, and the warps run the router MatMul on the staged
// chunk with mma.sync m16n8k16 (fp32 accumulation), keeping their expert tiles'
// accumulators in registers across chunks, so the next chunk's global loads overlap this
// chunk's MMAs.  Warp w owns expert columns [8j, 8j + 8) for j = w / wpt, ...; with fewer
// than 8 tiles `wpt` warps share a tile by splitting each chunk's k-steps and sum their
// partials at the end in warp order (deterministic).  ~13 KB of shared memory per CTA.
constexpr int NR_TC_ROWS = 16;             // MMA rows
constexpr int NR_TC_LIVE = 8;              // rows a CTA normalises
constexpr int NR_TC_WARPS = 8;
constexpr int NR_KC = 256;                 // K columns per chunk: one 16-byte piece of one
                                           // live row per thread
constexpr int NR_LD = NR_KC + 8;           // padded tile row (elements)
constexpr int NR_MAX_TPW = 4;              // expert tiles per warp (E <= 256)
static_assert(NR_TC_LIVE * NR_KC / 8 == NR_TC_WARPS * 32, "one piece per thread per chunk");

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
  __shared__ __align__(16) T tile[NR_TC_ROWS * NR_LD];
  __shared__ float s_inv[NR_TC_LIVE];
  __shared__ float red[NR_TC_WARPS * 32 * 4];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * NR_TC_LIVE;
  constexpr bool kBf16 = !std::is_same<T, __half>::value;

  // The MMA's rows NR_TC_LIVE..15 stay zero.
  for (int i = tid; i < (NR_TC_ROWS - NR_TC_LIVE) * NR_LD; i += NR_TC_WARPS * 32)
    tile[NR_TC_LIVE * NR_LD + i] = from_f<T>(0.f);

  // 1/rms of each row.
  for (int rr = warp; rr < NR_TC_LIVE; rr += NR_TC_WARPS) {
    const int64_t row = row0 + rr;
    float ss = 0.f;
    if (row < rows) {
      const T* xr = x + row * H;
      const T* sr = skip != nullptr ? skip + row * H : nullptr;
#pragma unroll 4
      for (int c = lane * 8; c < H; c += 256) {
        float h[8];
        load_h<T>(xr, sr, c, h);
#pragma unroll
        for (int j = 0; j < 8; ++j) ss = fmaf(h[j], h[j], ss);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) s_inv[rr] = row < rows ? rsqrtf(ss / static_cast<float>(H) + eps) : 0.f;
  }

  const int g = lane >> 2, t = lane & 3;
  const int ntile = (E + 7) / 8;
  const int wpt = ntile >= 8 ? 1 : (ntile >= 4 ? 2 : (ntile >= 2 ? 4 : 8));
  const int kslice = warp % wpt;
  const int jstep = NR_TC_WARPS / wpt;
  float d[NR_MAX_TPW][4];
#pragma unroll
  for (int i = 0; i < NR_MAX_TPW; ++i)
#pragma unroll
    for (int q = 0; q < 4; ++q) d[i][q] = 0.f;
  const uint32_t* tw = reinterpret_cast<const uint32_t*>(tile);
  constexpr int LDW = NR_LD / 2;

  // This thread's piece of every chunk: live row rr, columns c0 + cc .. + 7.
  const int rr = tid / (NR_KC / 8), cc = (tid % (NR_KC / 8)) * 8;
  const int64_t prow = row0 + rr;
  const bool row_ok = prow < rows;
  const T* px = x + (row_ok ? prow : 0) * H;
  const T* ps = skip != nullptr ? skip + (row_ok ? prow : 0) * H : nullptr;
  float h[8];
  auto fetch = [&](int c0) {
    if (row_ok && c0 + cc < H) {
      load_h<T>(px, ps, c0 + cc, h);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) h[j] = 0.f;
    }
  };
  fetch(0);
  __syncthreads();  // s_inv and the zero rows

  for (int c0 = 0; c0 < H; c0 += NR_KC) {
    const int cw = min(NR_KC, H - c0);          // multiple of 8
    const int cwp = (cw + 15) & ~15;            // multiple of the MMA depth
    if (cc < cw) {
      float n[8];
      if (row_ok) {
        if (residual_out != nullptr) store8<T>(residual_out + prow * H + c0 + cc, h);
        const float4 g0 = __ldg(reinterpret_cast<const float4*>(gamma + c0 + cc));
        const float4 g1 = __ldg(reinterpret_cast<const float4*>(gamma + c0 + cc + 4));
        const float gm[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
        const float inv = s_inv[rr];
#pragma unroll
        for (int j = 0; j < 8; ++j) n[j] = h[j] * inv * gm[j];
        if (normed != nullptr) store8<T>(normed + prow * H + c0 + cc, n);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) n[j] = 0.f;
      }
      store8<T>(tile + rr * NR_LD + cc, n);
    }
    if (cwp != cw)  // zero the k tail of the last chunk (H % 16 == 8)
      for (int i = tid; i < NR_TC_LIVE * 8; i += NR_TC_WARPS * 32)
        tile[(i >> 3) * NR_LD + cw + (i & 7)] = from_f<T>(0.f);
    __syncthreads();
    if (c0 + NR_KC < H) fetch(c0 + NR_KC);  // in flight during the MMAs below

    const int ks = cwp / 16;
    const int kper = (ks + wpt - 1) / wpt;
    const int kb = kslice * kper, ke = min(ks, kb + kper);
#pragma unroll
    for (int i = 0; i < NR_MAX_TPW; ++i) {
      const int j = warp / wpt + i * jstep;
      if (j >= ntile) break;
      const T* wrow = wr + static_cast<int64_t>(min(j * 8 + g, E - 1)) * H + c0;
      for (int k = kb; k < ke; ++k) {
        uint32_t a[4];
        a[0] = tw[g * LDW + k * 8 + t];
        a[1] = tw[(g + 8) * LDW + k * 8 + t];
        a[2] = tw[g * LDW + k * 8 + 4 + t];
        a[3] = tw[(g + 8) * LDW + k * 8 + 4 + t];
        const int ka = 16 * k + 2 * t, kb2 = ka + 8;
        const uint32_t b0 = ka < cw ? __ldg(reinterpret_cast<const uint32_t*>(wrow + ka)) : 0u;
        const uint32_t b1 = kb2 < cw ? __ldg(reinterpret_cast<const uint32_t*>(wrow + kb2)) : 0u;
        nr_mma(d[i], a, b0, b1, kBf16);
      }
    }
    __syncthreads();  // the next chunk overwrites the tile
  }

  if (wpt > 1) {
#pragma unroll
    for (int q = 0; q < 4; ++q) red[(warp * 32 + lane) * 4 + q] = d[0][q];
    __syncthreads();
    const int j = warp / wpt;
    if (kslice != 0 || j >= ntile) return;
#pragma unroll
    for (int q = 0; q < 4; ++q) d[0][q] = 0.f;
    for (int w2 = warp; w2 < warp + wpt; ++w2)
#pragma unroll
      for (int q = 0; q < 4; ++q) d[0][q] += red[(w2 * 32 + lane) * 4 + q];
  }
  // d: rows g / g + 8 (live rows are g < NR_TC_LIVE), expert columns 8j + 2t, + 1
#pragma unroll
  for (int i = 0; i < NR_MAX_TPW; ++i) {
    const int j = warp / wpt + i * jstep;
    if (j >= ntile || (wpt > 1 && i > 0)) break;
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int64_t row = row0 + g;
      const int ec = j * 8 + 2 * t + q;
      if (g < NR_TC_LIVE && row < rows && ec < E) logits[row * E + ec] = from_f<T>(d[i][q]);
    }
  }
}

template <typename T>
cudaError_t launch_t(const void* x, const void* skip, const float* gamma, float eps,
                     const void* wr, int64_t rows, int H, int E, void* residual_out,
                     void* normed, void* logits, cudaStream_t s) {
  if constexpr (sizeof(T) == 2) {
    const int64_t blocks = (rows + NR_TC_LIVE - 1) / NR_TC_LIVE;
    norm_router_tc_kernel<T><<<static_cast<unsigned>(blocks), NR_TC_WARPS * 32, 0, s>>>(
        static_cast<const T*>(x), static_cast<const T*>(skip), gamma, eps,
        static_cast<const T*>(wr), rows, H, E, static_cast<T*>(residual_out),
        static_cast<T*>(normed), static_cast<T*>(logits));
    return cudaGetLastError();
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
  // fp32 rows go through the per-warp kernel (a shared-memory copy of each row); 16-bit
  // rows through the chunked tensor-core kernel (fixed ~13 KB).
  return dtype == kDtF32 ? static_cast<size_t>(NR_WARPS) * H * 4 : 0;
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
