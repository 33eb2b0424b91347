// Router (softmax + top-k + renormalisation), dispatch plan (per-expert histogram,
// exclusive scan, stable permutation) and the row gather into expert-contiguous
// order.  All integer results are deterministic: no atomic slot claiming.
//
// Reference analogs (MooreThreads/onnxruntime-musa):
//   softmax  musa/ep/src/kernels/math/softmax_impl.mu:49-84 (fp32 accumulation)
//   top-k    musa/ep/src/kernels/math/topk_impl.mu:46-65 (ties -> lower index)
//   scan     musa/ep/src/kernels/math/cumsum_impl.mu:17 (replaced by a two-level scan)
//   gather   musa/ep/src/kernels/tensor/gather_impl.mu:18
#include <algorithm>

#include "moe_kernels.h"

namespace moe {

__device__ __forceinline__ int64_t imin64(int64_t a, int64_t b) { return a < b ? a : b; }

// ------------------------------------------------------------------------ router
// Routes one row with one warp; lane l holds logits l, l+32, ...  Selection compares
// fp32 values, ties to the lower index; NaN logits are read as -inf.  Lanes r < k
// receive the r-th selected expert and its weight.
// Sparse-mixer top-2 (the router of Phi-3.5-MoE, inference form): for each of the two
// picks, m = the largest remaining logit, e* its expert (ties -> lower index); experts with
// (m - s_e) / max(|s_e|, m) > 2 * jitter_eps are dropped and the pick's weight is its
// softmax probability over the experts kept (the second pick also excludes the first).
// The mask tests are IEEE fp32 operations, so the kept sets are reproducible.
template <int kPerLane>
__device__ __forceinline__ void sparse_mixer_row(const float (&v)[kPerLane], int E, int lane,
                                                 int& my_idx, float& my_w) {
  uint32_t taken = 0;
  for (int r = 0; r < 2; ++r) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < kPerLane; ++j) {
      const int e = lane + 32 * j;
      if (e < E && !(taken & (1u << j)) && (v[j] > bv || (v[j] == bv && e < bi))) {
        bv = v[j];
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < kPerLane; ++j) {
      const int e = lane + 32 * j;
      if (e >= E || (taken & (1u << j))) continue;
      const float ratio = (bv - v[j]) / fmaxf(fabsf(v[j]), bv);
      if (!(ratio > 2.0f * kSparseMixerJitterEps)) sum += expf(v[j] - bv);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    if (lane == r) {
      my_idx = bi;
      my_w = 1.0f / sum;
    }
  }
}

// Order-preserving map of fp32 bits to uint32 (larger float -> larger key; NaN is never
// passed) and its inverse.
__device__ __forceinline__ uint32_t float_key(float x) {
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_float(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Lane l's logits of one row (l, l + 32, ...), fp32; NaN and absent experts read -inf.
template <typename T, int kPerLane>
__device__ __forceinline__ void load_row(const T* __restrict__ row, int E, int lane,
                                         float (&v)[kPerLane]) {
#pragma unroll
  for (int j = 0; j < kPerLane; ++j) {
    const int e = lane + 32 * j;
    float x = -INFINITY;
    if (e < E) {
      x = to_f(row[e]);
      if (x != x) x = -INFINITY;
    }
    v[j] = x;
  }
}

// Routing of one row from its logits in registers (see route_row).
template <int kPerLane>
__device__ __forceinline__ void route_vals(const float (&v)[kPerLane], int E, int k,
                                           int normalize, int lane, int& my_idx, float& my_w) {
  if (normalize == kRouteSparseMixer) {
    my_idx = 0;
    my_w = 0.f;
    sparse_mixer_row<kPerLane>(v, E, lane, my_idx, my_w);
    return;
  }
  // Selection runs on order-preserving unsigned keys of the fp32 logits (-0 read as +0,
  // so equal values have equal keys): one warp max-reduction finds the largest remaining
  // value and one min-reduction the lowest expert index holding it (ties -> lower index),
  // the rule of the reference TopK.  The softmax denominator of the full row (only for
  // normalize == 0) keeps a fixed butterfly order: deterministic.
  uint32_t key[kPerLane];
#pragma unroll
  for (int j = 0; j < kPerLane; ++j) key[j] = float_key(v[j] + 0.0f);
  float s = 0.f, m = 0.f;
  if (!normalize) {
    uint32_t km = key[0];
#pragma unroll
    for (int j = 1; j < kPerLane; ++j) km = max(km, key[j]);
    m = key_float(__reduce_max_sync(0xffffffffu, km));
#pragma unroll
    for (int j = 0; j < kPerLane; ++j)
      if (lane + 32 * j < E) s += expf(v[j] - m);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  }

  uint32_t taken = 0;  // bit j: v[j] already selected
  float top_val = 0.f, sel_sum = 0.f, my_val = 0.f;
  my_idx = 0;
  for (int r = 0; r < k; ++r) {
    uint32_t bk = 0;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < kPerLane; ++j) {
      const int e = lane + 32 * j;
      // Strictly greater (or the first valid): among this lane's equal keys the lowest
      // index, which comes first, stays.
      if (e < E && !(taken & (1u << j)) && (bi == 0x7fffffff || key[j] > bk)) {
        bk = key[j];
        bi = e;
      }
    }
    const uint32_t wk = __reduce_max_sync(0xffffffffu, bi == 0x7fffffff ? 0u : bk);
    bi = static_cast<int>(__reduce_min_sync(
        0xffffffffu, (bi != 0x7fffffff && bk == wk) ? static_cast<uint32_t>(bi) : 0x7fffffffu));
    const float bv = key_float(wk);
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    if (r == 0) top_val = bv;
    const float ex = normalize ? expf(bv - top_val) : expf(bv - m);
    sel_sum += ex;
    if (lane == r) { my_val = ex; my_idx = bi; }
  }
  my_w = normalize ? my_val / sel_sum : my_val / s;
}

template <typename T, int kPerLane>
__device__ __forceinline__ void route_row(const T* __restrict__ row, int E, int k, int normalize,
                                          int lane, int& my_idx, float& my_w) {
  float v[kPerLane];
  load_row<T, kPerLane>(row, E, lane, v);
  route_vals<kPerLane>(v, E, k, normalize, lane, my_idx, my_w);
}

// Threads of a routing CTA: 16 warps share a chunk's rows (more rows in flight per SM).
constexpr int kRouteKernelThreads = 512;

// One warp per row, `chunk` rows per CTA; also the CTA's expert histogram.
template <typename T, int kPerLane>
__global__ void __launch_bounds__(kRouteKernelThreads)
route_kernel(const T* __restrict__ logits, int num_rows, int E, int k, int normalize,
             int32_t* __restrict__ expert_idx, float* __restrict__ route_w,
             int32_t* __restrict__ chunk_counts, int chunk, int* __restrict__ clear) {
  extern __shared__ int32_t s_counts[];  // [E]
  if (clear != nullptr && blockIdx.x == 0 && threadIdx.x < kClearWords) clear[threadIdx.x] = 0;
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_counts[e] = 0;
  __syncthreads();

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int row0 = blockIdx.x * chunk;
  const int row_end = min(row0 + chunk, num_rows);
  constexpr int kStride = kRouteKernelThreads / 32;
  // The next row's logits load while this row is routed (hides the load latency).
  float vn[kPerLane];
  if (row0 + warp < row_end)
    load_row<T, kPerLane>(logits + static_cast<int64_t>(row0 + warp) * E, E, lane, vn);
  for (int t = row0 + warp; t < row_end; t += kStride) {
    float v[kPerLane];
#pragma unroll
    for (int j = 0; j < kPerLane; ++j) v[j] = vn[j];
    if (t + kStride < row_end)
      load_row<T, kPerLane>(logits + static_cast<int64_t>(t + kStride) * E, E, lane, vn);
    int my_idx;
    float w;
    route_vals<kPerLane>(v, E, k, normalize, lane, my_idx, w);
    if (lane < k) {
      expert_idx[static_cast<int64_t>(t) * k + lane] = my_idx;
      route_w[static_cast<int64_t>(t) * k + lane] = w;
      atomicAdd(&s_counts[my_idx], 1);
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x)
    chunk_counts[static_cast<int64_t>(blockIdx.x) * E + e] = s_counts[e];
}

// ------------------------------------------------------------- small dispatch
// Routing and the whole dispatch plan of a small call (T*k <= kSmallDispatchRows) in
// one CTA: warp-per-row routing, expert counts, exclusive scan, and the stable rank of
// each routed row within its expert by counting earlier rows of the same expert.
template <typename T, int kPerLane>
__global__ void __launch_bounds__(1024)
small_dispatch_kernel(const T* __restrict__ logits, int num_rows, int E, int k, int normalize,
                      int32_t* __restrict__ expert_idx, float* __restrict__ route_w,
                      int32_t* __restrict__ expert_offsets, int32_t* __restrict__ permuted_pos,
                      int32_t* __restrict__ permuted_src, int* __restrict__ clear) {
  // The decode chain's next kernel (the activation prep) reads only the layer input, so it
  // may start now (it waits for this kernel before it exits).
  pdl_launch_dependents();
  __shared__ int32_t s_idx[kSmallDispatchRows];
  if (clear != nullptr && threadIdx.x < kClearWords) clear[threadIdx.x] = 0;
  __shared__ int32_t s_cnt[kMaxExperts + 1];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  for (int e = threadIdx.x; e <= E; e += blockDim.x) s_cnt[e] = 0;
  __syncthreads();
  for (int t = warp; t < num_rows; t += 32) {
    int my_idx;
    float w;
    route_row<T, kPerLane>(logits + static_cast<int64_t>(t) * E, E, k, normalize, lane, my_idx, w);
    if (lane < k) {
      expert_idx[t * k + lane] = my_idx;
      route_w[t * k + lane] = w;
      s_idx[t * k + lane] = my_idx;
      atomicAdd(&s_cnt[my_idx], 1);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int32_t o = 0;
    for (int e = 0; e < E; ++e) {
      const int32_t c = s_cnt[e];
      s_cnt[e] = o;
      o += c;
    }
    s_cnt[E] = o;
  }
  __syncthreads();
  for (int e = threadIdx.x; e <= E; e += blockDim.x) expert_offsets[e] = s_cnt[e];
  const int R = num_rows * k;
  for (int i = threadIdx.x; i < R; i += blockDim.x) {
    const int e = s_idx[i];
    int rank = 0;
    for (int j = 0; j < i; ++j) rank += s_idx[j] == e;
    const int p = s_cnt[e] + rank;
    permuted_pos[i] = p;
    permuted_src[p] = i;
  }
}

// ---------------------------------------------------------- histogram (external)
// Per-chunk histogram of an existing expert_idx (used when routing is supplied).
__global__ void __launch_bounds__(kRouteThreads)
histogram_kernel(const int32_t* __restrict__ expert_idx, int num_rows, int k, int E,
                 int32_t* __restrict__ chunk_counts, int* __restrict__ err, int chunk) {
  extern __shared__ int32_t s_counts[];
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_counts[e] = 0;
  __syncthreads();
  const int64_t base = static_cast<int64_t>(blockIdx.x) * chunk * k;
  const int64_t end = imin64(base + static_cast<int64_t>(chunk) * k,
                                   static_cast<int64_t>(num_rows) * k);
  for (int64_t i = base + threadIdx.x; i < end; i += blockDim.x) {
    const int e = expert_idx[i];
    if (e < 0 || e >= E) { atomicExch(err, kErrBadExpert); continue; }
    atomicAdd(&s_counts[e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x)
    chunk_counts[static_cast<int64_t>(blockIdx.x) * E + e] = s_counts[e];
}

// ---------------------------------------------------------------------- scan
constexpr int kScanParts = 16;  // most threads per expert in the column scan
// Single CTA.  Column scan over chunks per expert (chunk_base), then an exclusive
// scan over experts (expert_offsets) and the prefix of 128-row and 64-row tile
// counts used by the grouped-GEMM schedulers.
__global__ void __launch_bounds__(1024)
scan_kernel(const int32_t* __restrict__ chunk_counts, int num_chunks, int E,
            int32_t* __restrict__ chunk_base, int32_t* __restrict__ expert_offsets,
            int32_t* __restrict__ tiles128, int32_t* __restrict__ tiles64,
            int32_t* __restrict__ tiles256) {
  pdl_wait();  // launched dependent (launch_dependent): predecessors' data after this
  pdl_launch_dependents();
  extern __shared__ int32_t s_cnt[];  // [E], then [kScanParts][E] part sums
  // P threads per expert (P = blockDim / E rounded down to a power of two, <= 16) each
  // sum a contiguous range of chunks (independent loads), then write that range's running
  // bases from the exclusive prefix of the earlier parts.
  int P = 1;
  while (P * 2 * E <= static_cast<int>(blockDim.x) && P < kScanParts) P *= 2;
  int32_t* s_part = s_cnt + E;
  const int e = threadIdx.x / P, part = threadIdx.x % P;
  const int per = (num_chunks + P - 1) / P;
  const int c0 = min(num_chunks, part * per), c1 = min(num_chunks, c0 + per);
  int32_t sum = 0;
  if (e < E) {
#pragma unroll 8
    for (int c = c0; c < c1; ++c) sum += chunk_counts[static_cast<int64_t>(c) * E + e];
    s_part[part * E + e] = sum;
  }
  __syncthreads();
  if (e < E) {
    int32_t run = 0;
    for (int q = 0; q < part; ++q) run += s_part[q * E + e];
    for (int c = c0; c < c1; ++c) {
      const int64_t i = static_cast<int64_t>(c) * E + e;
      chunk_base[i] = run;
      run += chunk_counts[i];
    }
    if (part == P - 1) s_cnt[e] = run;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int32_t o = 0, t128 = 0, t64 = 0, t256 = 0;
    for (int e = 0; e < E; ++e) {
      expert_offsets[e] = o;
      tiles128[e] = t128;
      tiles64[e] = t64;
      tiles256[e] = t256;
      const int32_t c = s_cnt[e];
      o += c;
      t128 += (c + 127) / 128;
      t64 += (c + 63) / 64;
      t256 += (c + 255) / 256;
    }
    expert_offsets[E] = o;
    tiles128[E] = t128;
    tiles64[E] = t64;
    tiles256[E] = t256;
  }
}

// ------------------------------------------------------------------ permutation
// One CTA per routing chunk.  Entries are ranked within their expert in
// (token, slot) order: __match_any_sync gives the rank inside a warp, a per-warp
// count table the rank across warps, and a running per-expert counter the rank
// across the groups of the chunk.
__global__ void __launch_bounds__(kRouteThreads)
permute_kernel(const int32_t* __restrict__ expert_idx, int num_rows, int k, int E,
               const int32_t* __restrict__ expert_offsets,
               const int32_t* __restrict__ chunk_base, int32_t* __restrict__ permuted_pos,
               int32_t* __restrict__ permuted_src, int chunk) {
  pdl_wait();  // launched dependent (launch_dependent): predecessors' data after this
  pdl_launch_dependents();
  extern __shared__ int32_t smem[];
  constexpr int kWarps = kRouteThreads / 32;
  int32_t* s_warp = smem;               // [kWarps][E]
  int32_t* s_run = smem + kWarps * E;   // [E]
  int32_t* s_base = s_run + E;          // [E]
  for (int i = threadIdx.x; i < kWarps * E; i += blockDim.x) s_warp[i] = 0;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    s_run[e] = 0;
    s_base[e] = expert_offsets[e] + chunk_base[static_cast<int64_t>(blockIdx.x) * E + e];
  }
  __syncthreads();

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t base = static_cast<int64_t>(blockIdx.x) * chunk * k;
  const int64_t end = imin64(base + static_cast<int64_t>(chunk) * k,
                                   static_cast<int64_t>(num_rows) * k);
  const uint32_t lt_mask = (1u << lane) - 1u;
  for (int64_t g = base; g < end; g += kRouteThreads) {
    const int64_t i = g + threadIdx.x;
    const bool valid = i < end;
    int e = valid ? expert_idx[i] : -1;
    if (e >= E || e < -1) e = -1;  // out-of-range ids were flagged by the router/histogram
    const uint32_t peers = __match_any_sync(0xffffffffu, e);
    const int lane_rank = __popc(peers & lt_mask);
    const bool leader = (peers & lt_mask) == 0;
    if (e >= 0 && leader) s_warp[warp * E + e] = __popc(peers);
    __syncthreads();
    if (e >= 0) {
      int r = s_run[e] + lane_rank;
      for (int w = 0; w < warp; ++w) r += s_warp[w * E + e];
      const int32_t p = s_base[e] + r;
      permuted_pos[i] = p;
      permuted_src[p] = static_cast<int32_t>(i);
    }
    __syncthreads();
    for (int ee = threadIdx.x; ee < E; ee += blockDim.x) {
      int add = 0;
      for (int w = 0; w < kWarps; ++w) { add += s_warp[w * E + ee]; s_warp[w * E + ee] = 0; }
      s_run[ee] += add;
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------------ gather
// Xp[p, :] = x[permuted_src[p] / k, :].  One warp per permuted row, 16-byte
// vectors when the row is 16-byte aligned.
__global__ void __launch_bounds__(256)
gather_rows_kernel(const uint8_t* __restrict__ x, int64_t row_bytes, int k,
                   const int32_t* __restrict__ permuted_src, int64_t num_perm_rows,
                   uint8_t* __restrict__ xp) {
  pdl_wait();  // launched dependent (launch_dependent): predecessors' data after this
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t p = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (p >= num_perm_rows) return;
  const int64_t t = permuted_src[p] / k;
  const uint8_t* src = x + t * row_bytes;
  uint8_t* dst = xp + p * row_bytes;
  if ((row_bytes & 15) == 0) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    uint4* d4 = reinterpret_cast<uint4*>(dst);
    for (int64_t i = lane; i < row_bytes / 16; i += 32) d4[i] = __ldg(s4 + i);
  } else {
    for (int64_t i = lane; i < row_bytes; i += 32) dst[i] = src[i];
  }
}

// ------------------------------------------------------------------------ combine
// out[t, :] = sum_j w[t, j] * Y[pos[t, j], :], fp32 accumulation in slot order.
template <typename T>
__global__ void __launch_bounds__(256)
combine_kernel(const T* __restrict__ y, const int32_t* __restrict__ permuted_pos,
               const float* __restrict__ route_w, int num_rows, int k, int H,
               T* __restrict__ out) {
  pdl_wait();  // launched dependent (launch_dependent): predecessors' data after this
  pdl_launch_dependents();
  const int t = blockIdx.x;
  if (t >= num_rows) return;
  const int32_t* pos = permuted_pos + static_cast<int64_t>(t) * k;
  const float* w = route_w + static_cast<int64_t>(t) * k;
  if constexpr (sizeof(T) == 2) {
    if ((H & 7) == 0) {
      for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int j = 0; j < k; ++j) {
          const uint4 v = *reinterpret_cast<const uint4*>(y + static_cast<int64_t>(pos[j]) * H + c);
          const T* e = reinterpret_cast<const T*>(&v);
          const float wj = w[j];
#pragma unroll
          for (int q = 0; q < 8; ++q) acc[q] += wj * to_f(e[q]);
        }
        uint4 o;
        uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
        for (int q = 0; q < 4; ++q) ow[q] = pack2<T>(acc[2 * q], acc[2 * q + 1]);
        *reinterpret_cast<uint4*>(out + static_cast<int64_t>(t) * H + c) = o;
      }
      return;
    }
  }
  for (int c = threadIdx.x; c < H; c += blockDim.x) {
    float acc = 0.f;
    for (int j = 0; j < k; ++j) acc += w[j] * to_f(y[static_cast<int64_t>(pos[j]) * H + c]);
    out[static_cast<int64_t>(t) * H + c] = from_f<T>(acc);
  }
}

__global__ void fill_f32_kernel(float* __restrict__ dst, float v, int64_t n,
                                int* __restrict__ clear) {
  if (clear != nullptr && blockIdx.x == 0 && threadIdx.x < kClearWords) clear[threadIdx.x] = 0;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    dst[i] = v;
}

// One warp per row: fp32 sum of an fp16 row, lanes over 16-byte pieces, fixed butterfly.
__global__ void __launch_bounds__(256)
row_sums_kernel(const __half* __restrict__ a, int64_t rows, int K, float* __restrict__ out) {
  pdl_wait();  // launched dependent (launch_dependent): predecessors' data after this
  pdl_launch_dependents();
  const int64_t r = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const __half* row = a + r * K;
  float acc = 0.f;
  for (int c = lane * 8; c < K; c += 256) {
    const uint4 u = *reinterpret_cast<const uint4*>(row + c);
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __half22float2(h[j]);
      acc += f.x + f.y;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) out[r] = acc;
}

// ------------------------------------------------------------------ launchers
cudaError_t launch_row_sums(const void* a, int64_t rows, int K, float* out, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  return launch_dependent(pdl_layer_enabled(), row_sums_kernel, dim3(static_cast<unsigned>((rows + 7) / 8)), dim3(256), 0, s,
      static_cast<const __half*>(a), rows, K, out);
}

cudaError_t launch_fill_f32(float* dst, float value, int64_t n, cudaStream_t s, int* clear) {
  if (n == 0) return cudaSuccess;
  const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 1184));
  fill_f32_kernel<<<blocks, 256, 0, s>>>(dst, value, n, clear);
  return cudaGetLastError();
}

template <typename T>
static cudaError_t launch_route_t(const void* logits, int T_, int E, int k, int normalize,
                                  int32_t* idx, float* w, int32_t* chunk_counts,
                                  cudaStream_t s, int chunk, int* clear) {
  const int chunks = num_route_chunks(T_, chunk);
  const size_t sm = static_cast<size_t>(E) * sizeof(int32_t);
  const T* l = static_cast<const T*>(logits);
  const int per_lane = (E + 31) / 32;
  if (per_lane <= 1)
    route_kernel<T, 1><<<chunks, kRouteKernelThreads, sm, s>>>(l, T_, E, k, normalize, idx, w, chunk_counts, chunk, clear);
  else if (per_lane <= 2)
    route_kernel<T, 2><<<chunks, kRouteKernelThreads, sm, s>>>(l, T_, E, k, normalize, idx, w, chunk_counts, chunk, clear);
  else if (per_lane <= 4)
    route_kernel<T, 4><<<chunks, kRouteKernelThreads, sm, s>>>(l, T_, E, k, normalize, idx, w, chunk_counts, chunk, clear);
  else
    route_kernel<T, 8><<<chunks, kRouteKernelThreads, sm, s>>>(l, T_, E, k, normalize, idx, w, chunk_counts, chunk, clear);
  return cudaGetLastError();
}

cudaError_t launch_route(int dtype, const void* logits, int T_, int E, int k, int normalize,
                         int32_t* idx, float* w, int32_t* chunk_counts, cudaStream_t s,
                         int chunk, int* clear) {
  if (T_ == 0) return cudaSuccess;
  switch (dtype) {
    case kDtF32: return launch_route_t<float>(logits, T_, E, k, normalize, idx, w, chunk_counts, s, chunk, clear);
    case kDtF16: return launch_route_t<__half>(logits, T_, E, k, normalize, idx, w, chunk_counts, s, chunk, clear);
    case kDtBF16: return launch_route_t<__nv_bfloat16>(logits, T_, E, k, normalize, idx, w, chunk_counts, s, chunk, clear);
  }
  return cudaErrorInvalidValue;
}

template <typename T>
static cudaError_t launch_small_dispatch_t(const void* logits, int T_, int E, int k, int normalize,
                                           int32_t* idx, float* w, int32_t* offsets, int32_t* pos,
                                           int32_t* src, cudaStream_t s, int* clear) {
  const T* l = static_cast<const T*>(logits);
  const int per_lane = (E + 31) / 32;
  if (per_lane <= 1)
    small_dispatch_kernel<T, 1><<<1, 1024, 0, s>>>(l, T_, E, k, normalize, idx, w, offsets, pos, src, clear);
  else if (per_lane <= 2)
    small_dispatch_kernel<T, 2><<<1, 1024, 0, s>>>(l, T_, E, k, normalize, idx, w, offsets, pos, src, clear);
  else if (per_lane <= 4)
    small_dispatch_kernel<T, 4><<<1, 1024, 0, s>>>(l, T_, E, k, normalize, idx, w, offsets, pos, src, clear);
  else
    small_dispatch_kernel<T, 8><<<1, 1024, 0, s>>>(l, T_, E, k, normalize, idx, w, offsets, pos, src, clear);
  return cudaGetLastError();
}

cudaError_t launch_small_dispatch(int dtype, const void* logits, int T_, int E, int k,
                                  int normalize, int32_t* idx, float* w, int32_t* offsets,
                                  int32_t* pos, int32_t* src, cudaStream_t s, int* clear) {
  if (T_ == 0) return cudaSuccess;
  switch (dtype) {
    case kDtF32: return launch_small_dispatch_t<float>(logits, T_, E, k, normalize, idx, w, offsets, pos, src, s, clear);
    case kDtF16: return launch_small_dispatch_t<__half>(logits, T_, E, k, normalize, idx, w, offsets, pos, src, s, clear);
    case kDtBF16: return launch_small_dispatch_t<__nv_bfloat16>(logits, T_, E, k, normalize, idx, w, offsets, pos, src, s, clear);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_histogram(const int32_t* idx, int T_, int k, int E, int32_t* chunk_counts,
                             int* err, cudaStream_t s, int chunk) {
  if (T_ == 0) return cudaSuccess;
  histogram_kernel<<<num_route_chunks(T_, chunk), kRouteThreads, E * sizeof(int32_t), s>>>(
      idx, T_, k, E, chunk_counts, err, chunk);
  return cudaGetLastError();
}

cudaError_t launch_plan(const int32_t* idx, int T_, int k, int E, const int32_t* chunk_counts,
                        int32_t* chunk_base, int32_t* offsets, int32_t* tiles128,
                        int32_t* tiles64, int32_t* tiles256, int32_t* pos, int32_t* src,
                        cudaStream_t s, int chunk) {
  const int chunks = num_route_chunks(T_, chunk);
  cudaError_t st = launch_dependent(pdl_layer_enabled(), scan_kernel, dim3(1), dim3(1024),
                                    (1 + kScanParts) * E * sizeof(int32_t), s,
                                    chunk_counts, chunks, E, chunk_base, offsets, tiles128,
                                    tiles64, tiles256);
  if (st != cudaSuccess || T_ == 0) return st;
  const size_t sm = (static_cast<size_t>(kRouteThreads / 32) + 2) * E * sizeof(int32_t);
  return launch_dependent(pdl_layer_enabled(), permute_kernel, dim3(chunks), dim3(kRouteThreads), sm, s, idx, T_, k, E,
                          offsets, chunk_base, pos, src, chunk);
}

cudaError_t launch_gather(const void* x, int64_t row_bytes, int k, const int32_t* src,
                          int64_t rows, void* xp, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  const int64_t blocks = (rows + 7) / 8;
  return launch_dependent(pdl_layer_enabled(), gather_rows_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, s,
                          static_cast<const uint8_t*>(x), row_bytes, k, src, rows,
                          static_cast<uint8_t*>(xp));
}

cudaError_t launch_combine(int dtype, const void* y, const int32_t* pos, const float* w,
                           int T_, int k, int H, void* out, cudaStream_t s) {
  if (T_ == 0) return cudaSuccess;
  switch (dtype) {
    case kDtF32:
      return launch_dependent(pdl_layer_enabled(), combine_kernel<float>, dim3(T_), dim3(256), 0, s,
                              static_cast<const float*>(y), pos, w, T_, k, H,
                              static_cast<float*>(out));
    case kDtF16:
      return launch_dependent(pdl_layer_enabled(), combine_kernel<__half>, dim3(T_), dim3(256), 0, s,
                              static_cast<const __half*>(y), pos, w, T_, k, H,
                              static_cast<__half*>(out));
    case kDtBF16:
      return launch_dependent(pdl_layer_enabled(), combine_kernel<__nv_bfloat16>, dim3(T_), dim3(256), 0, s,
                              static_cast<const __nv_bfloat16*>(y), pos, w, T_, k, H,
                              static_cast<__nv_bfloat16*>(out));
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace moe
