// Grouped expert GEMM on the 5th-generation tensor cores (tcgen05) for sm_100a.
//
// One persistent CTA per SM walks a device-side tile list (expert, n-tile, m-tile)
// built from the per-expert row offsets, so no host round trip is needed between
// routing and the GEMM.  Per CTA, warp-specialised:
//   warp 0      TMA producer: A tile 128x64 (permuted activations) and B tile
//               256x64 (one expert's weight rows) per stage, 128-byte swizzle.
//   warp 1      MMA issuer: tcgen05.mma kind::f16, M=128 N=256 K=16, fp32
//               accumulator in TMEM; two accumulators (2 x 256 columns) so the
//               epilogue of tile i overlaps the mainloop of tile i+1.
//   warps 2..9  epilogue (two warps per 32-lane TMEM quarter, each taking half the
//               columns): tcgen05.ld of its lane quarter, bias + activation
//               (gated: act(g) * u, where columns 0..127 hold the gate tile and
//               128..255 the linear tile of the same 128 output columns), and a
//               store of the 16-bit result rows.  Rows of the tile that belong to
//               the next expert are computed but never stored.
// Reference analog: muDNN MatMul / muBLAS GemmStridedBatched plus GemmPostKernel
// (musa/ep/src/kernels/math/matmul.cc:239-332, shared_inc/blas_utils.h:237-262,
//  math/gemm_post_kernels.mu:27-53), which this single kernel replaces.
#include <algorithm>
#include <mutex>
#include <type_traits>

#include "moe_kernels.h"

namespace moe {

namespace {

constexpr int BM = 128;
constexpr int BN = 256;  // MMA N (gated: 128 gate + 128 linear)
constexpr int BK = 64;   // one 128-byte swizzle atom of 16-bit elements
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_BYTES = BN * BK * 2;
constexpr int B_HALF = B_BYTES / 2;
constexpr int THREADS = 320;      // warp 0 TMA, warp 1 MMA, warps 2..9 epilogue
constexpr int EPI_WARPS = 8;      // two warps per TMEM lane quarter, splitting the columns
constexpr int TMEM_COLS = 512;
constexpr int SMEM_BYTES =
    1024 /*align slack*/ + STAGES * (A_BYTES + B_BYTES) + 64 * 8 /*barriers*/ +
    2 * (kMaxExperts + 1) * 4;

struct TcParams {
  const int32_t* offsets;
  const int32_t* tiles;   // prefix of per-expert m-tile counts (128 or 256 rows per tile)
  int E;
  int K;
  int N;            // output columns
  int n_tiles;      // per expert
  int gated;
  int b1_g, b3_g;   // interleave coordinates
  int b1_noff, b3_noff;
  const void* bias1;
  const void* bias3;
  int bias_stride;
  int64_t bias_e_stride;
  ActParams ap;
  void* out;
  int64_t ldo;
  int* err;
  // Packed (QMoE) B operands: codes with zero point 2^(bits-1) and fp16 scales, one per
  // stored row (block_size 0) or per block of block_size along K.
  const __half* scales1;
  const __half* scales3;
  int qblock;
  int b1_G, b3_G;
  int b1_rows, b3_rows;  // stored rows of one expert
  // Test hook: the producers issue no loads, so the consumers' bounded waits expire and
  // the kernel unwinds with an error code (exercises failure handling without a fault).
  int test_stall;
};

__device__ __forceinline__ void decode_tile(int L, const int32_t* s_tiles, int E, int n_tiles,
                                            int& e, int& m, int& n) {
  // Largest e with s_tiles[e] * n_tiles <= L.
  int lo = 0, hi = E - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (s_tiles[mid] * n_tiles <= L) lo = mid; else hi = mid - 1;
  }
  e = lo;
  const int local = L - s_tiles[e] * n_tiles;
  const int mt = s_tiles[e + 1] - s_tiles[e];
  n = local / mt;  // m fastest: the m-tiles of one weight tile run back to back (L2 reuse)
  m = local - n * mt;
}

template <typename T>
__device__ __forceinline__ float bias_val(const void* bias, int e, int n, const TcParams& p) {
  if (bias == nullptr) return 0.f;
  return to_f(static_cast<const T*>(bias)[e * p.bias_e_stride +
                                          static_cast<int64_t>(n) * p.bias_stride]);
}

template <typename T>
__device__ __forceinline__ void store16(T* dst, const float (&v)[16], int valid_cols) {
  if (valid_cols >= 16) {
    uint4 o0, o1;
    uint32_t* w0 = reinterpret_cast<uint32_t*>(&o0);
    uint32_t* w1 = reinterpret_cast<uint32_t*>(&o1);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      w0[q] = pack2<T>(v[2 * q], v[2 * q + 1]);
      w1[q] = pack2<T>(v[8 + 2 * q], v[8 + 2 * q + 1]);
    }
    reinterpret_cast<uint4*>(dst)[0] = o0;
    reinterpret_cast<uint4*>(dst)[1] = o1;
  } else {
#pragma unroll
    for (int q = 0; q < 16; ++q)
      if (q < valid_cols) dst[q] = from_f<T>(v[q]);
  }
}

// Fast-math activations for the 16-bit epilogue (inputs and outputs are fp16/bf16,
// so the few-ulp error of the approximate exp and reciprocal is far below the
// output rounding).
__device__ __forceinline__ float fast_sigmoid(float x) { return __frcp_rn(1.0f + __expf(-x)); }

__device__ __forceinline__ float fast_act_single(int act, float x) {
  switch (act) {
    case kRelu: return fmaxf(x, 0.0f);
    case kGelu: return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
    case kSilu: return x * fast_sigmoid(x);
    default: return x;
  }
}

__device__ __forceinline__ float fast_act_gated(const ActParams& p, float g, float u) {
  if (p.act == kSwiglu) {
    g = fminf(g, p.limit);
    u = fminf(fmaxf(u, -p.limit), p.limit);
    return g * fast_sigmoid(p.alpha * g) * (u + p.beta);
  }
  return fast_act_single(p.act, g) * u;
}

// Epilogue of one accumulator tile for the calling warp's 32 TMEM lanes (one output
// row per thread), accumulator columns [c0, c1).  Gated: columns [0,128) hold the gate
// and [128,256) the linear half of output columns n0..n0+127 (c ranges over the gate
// columns); plain: columns [0,256) are outputs n0..n0+255.
template <typename T>
__device__ __forceinline__ void epilogue_rows(const TcParams& p, uint32_t taddr, int row,
                                              bool valid, int e, int n0, int c0, int c1) {
  T* orow = static_cast<T*>(p.out) + static_cast<int64_t>(row) * p.ldo;
  const bool has_b1 = p.bias1 != nullptr, has_b3 = p.bias3 != nullptr;
  if (p.gated) {
#pragma unroll 1
    for (int c = c0; c < c1; c += 16) {
      float g[16], u[16];
      tmem_ld16(taddr + c, g);
      tmem_ld16(taddr + BN / 2 + c, u);
      tmem_ld_wait();
      const int col = n0 + c;
      if (valid && col < p.N) {
        float v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int cj = min(col + j, p.N - 1);
          const float gb = has_b1 ? g[j] + bias_val<T>(p.bias1, e, cj, p) : g[j];
          const float ub = has_b3 ? u[j] + bias_val<T>(p.bias3, e, cj, p) : u[j];
          v[j] = fast_act_gated(p.ap, gb, ub);
        }
        store16<T>(orow + col, v, p.N - col);
      }
    }
  } else {
#pragma unroll 1
    for (int c = c0; c < c1; c += 16) {
      float a[16];
      tmem_ld16(taddr + c, a);
      tmem_ld_wait();
      const int col = n0 + c;
      if (valid && col < p.N) {
        float v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int cj = min(col + j, p.N - 1);
          const float ab = has_b1 ? a[j] + bias_val<T>(p.bias1, e, cj, p) : a[j];
          v[j] = fast_act_single(p.ap.act, ab);
        }
        store16<T>(orow + col, v, p.N - col);
      }
    }
  }
}

// Column range of epilogue warp `w` (2..9): warps 2..5 take the first half of the
// tile's columns, warps 6..9 the second half.
__device__ __forceinline__ void epi_cols(const TcParams& p, int warp, int& c0, int& c1) {
  const int width = p.gated ? BN / 2 : BN;
  const int half = width / 2;
  c0 = warp < 6 ? 0 : half;
  c1 = c0 + half;
}

template <typename T>
__global__ void __launch_bounds__(THREADS, 1)
tc_grouped_gemm_kernel(const __grid_constant__ CUtensorMap map_a,
                       const __grid_constant__ CUtensorMap map_b1,
                       const __grid_constant__ CUtensorMap map_b3, const TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = bars + 2 * STAGES + 2;
  uint64_t* done = bars + 2 * STAGES + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int32_t* s_tiles = reinterpret_cast<int32_t*>(bars + 64);
  int32_t* s_offs = s_tiles + (kMaxExperts + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int E = p.E;

  for (int i = threadIdx.x; i <= E; i += blockDim.x) {
    s_tiles[i] = p.tiles[i];
    s_offs[i] = p.offsets[i];
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], EPI_WARPS);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b1);
    if (p.gated) tma_prefetch_desc(&map_b3);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int total = s_tiles[E] * p.n_tiles;
  const int nk = (p.K + BK - 1) / BK;

  if (warp == 0) {
    // ------------------------------------------------------------- TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int L = blockIdx.x; L < total && !*abort_flag && !p.test_stall; L += gridDim.x) {
        int e, m, n;
        decode_tile(L, s_tiles, E, p.n_tiles, e, m, n);
        const int row0 = s_offs[e] + m * BM;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1)) {
            atomicExch(p.err, kErrTimeoutProducer);
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], A_BYTES + B_BYTES);
          uint8_t* a_dst = sA + stage * A_BYTES;
          uint8_t* b_dst = sB + stage * B_BYTES;
          const int kc = kb * BK;
          tma_load_2d(a_dst, &map_a, &full[stage], kc, row0);
          if (p.gated) {
            const int n0 = n * (BN / 2);
            tma_load_4d(b_dst, &map_b1, &full[stage], kc, p.b1_g, n0 + p.b1_noff, e);
            tma_load_4d(b_dst + B_HALF, &map_b3, &full[stage], kc, p.b3_g, n0 + p.b3_noff, e);
          } else {
            const int n0 = n * BN;
            tma_load_4d(b_dst, &map_b1, &full[stage], kc, p.b1_g, n0 + p.b1_noff, e);
            tma_load_4d(b_dst + B_HALF, &map_b1, &full[stage], kc, p.b1_g,
                        n0 + BN / 2 + p.b1_noff, e);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // --------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t kFmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
      const uint32_t idesc = idesc_f16(kFmt, BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int i = 0;
      for (int L = blockIdx.x; L < total && !*abort_flag; L += gridDim.x, ++i) {
        const int acc = i & 1;
        const uint32_t acc_phase = (i >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1)) {
          atomicExch(p.err, kErrTimeoutMma);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&full[stage], phase)) {
            atomicExch(p.err, kErrTimeoutMma);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = smem_desc_k_sw128(a_addr + kk * 32);
            const uint64_t bd = smem_desc_k_sw128(b_addr + kk * 32);
            tc_mma_f16(d_tmem, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          tc_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        tc_commit(&tfull[acc]);
      }
      // All MMAs of this CTA have retired once `done` completes.
      tc_commit(done);
      mbar_wait(done, 0);
    }
  } else {
    // ----------------------------------------------------------------- epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int r_in_tile = q * 32 + lane;
    int ec0, ec1;
    epi_cols(p, warp, ec0, ec1);
    int i = 0;
    for (int L = blockIdx.x; L < total && !*abort_flag; L += gridDim.x, ++i) {
      const int acc = i & 1;
      const uint32_t acc_phase = (i >> 1) & 1;
      if (!mbar_wait(&tfull[acc], acc_phase)) {
        atomicExch(p.err, kErrTimeoutEpilogue);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      int e, m, n;
      decode_tile(L, s_tiles, E, p.n_tiles, e, m, n);
      const int row = s_offs[e] + m * BM + r_in_tile;
      const bool valid = row < s_offs[e + 1];
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
      epilogue_rows<T>(p, taddr, row, valid, e, p.gated ? n * (BN / 2) : n * BN, ec0, ec1);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}


// ---------------------------------------------------------------------------
// CTA-pair variant (tcgen05 cta_group::2): a cluster of 2 CTAs on 2 SMs computes a
// 256x256 tile with M=256 MMAs issued by the leader CTA.  Each CTA stages its own
// 128 rows of A and its own 128 rows of B (gate rows in CTA 0 and linear rows in CTA 1
// when gated), so per SM the operand traffic per MMA is half that of the single-CTA
// kernel.  Both CTAs' TMA loads complete on the leader's `full` barrier (which expects
// the bytes of both); MMA completion is committed to the barriers of both CTAs.  No
// TMA load is multicast.  Accumulators: 128 lanes x 256 columns per CTA, double
// buffered; each CTA's epilogue drains its own rows and then arrives on the leader's
// `tempty` barrier (16 arrivals: 8 warps x 2 CTAs).
constexpr int P_BM = 256;         // rows per pair tile
constexpr int P_STAGES = 6;
constexpr int P_STAGE_BYTES = A_BYTES + B_HALF;  // per CTA: 128x64 of A + 128x64 of B
constexpr int P_SMEM_BYTES =
    1024 + P_STAGES * P_STAGE_BYTES + 64 * 8 + 2 * (kMaxExperts + 1) * 4;

template <typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
tc_pair_grouped_gemm_kernel(const __grid_constant__ CUtensorMap map_a,
                            const __grid_constant__ CUtensorMap map_b1,
                            const __grid_constant__ CUtensorMap map_b3, const TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + P_STAGES * A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + P_STAGES * B_HALF);
  uint64_t* full = bars;
  uint64_t* empty = bars + P_STAGES;
  uint64_t* tfull = bars + 2 * P_STAGES;
  uint64_t* tempty = bars + 2 * P_STAGES + 2;
  uint64_t* done = bars + 2 * P_STAGES + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * P_STAGES + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int32_t* s_tiles = reinterpret_cast<int32_t*>(bars + 64);
  int32_t* s_offs = s_tiles + (kMaxExperts + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int E = p.E;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  for (int i = threadIdx.x; i <= E; i += blockDim.x) {
    s_tiles[i] = p.tiles[i];
    s_offs[i] = p.offsets[i];
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * EPI_WARPS);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b1);
    if (p.gated) tma_prefetch_desc(&map_b3);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers are initialised before any remote signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int total = s_tiles[E] * p.n_tiles;
  const int nk = (p.K + BK - 1) / BK;
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;

  if (warp == 0) {
    // ------------------------------------------------------------- TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int L = pair; L < total && !*abort_flag && !p.test_stall; L += npairs) {
        int e, m, n;
        decode_tile(L, s_tiles, E, p.n_tiles, e, m, n);
        const int row0 = s_offs[e] + m * P_BM + static_cast<int>(rank) * BM;
        const CUtensorMap* bmap = (p.gated && rank == 1) ? &map_b3 : &map_b1;
        int bg, brow;
        if (p.gated) {
          bg = rank == 1 ? p.b3_g : p.b1_g;
          brow = n * (BN / 2) + (rank == 1 ? p.b3_noff : p.b1_noff);
        } else {
          bg = p.b1_g;
          brow = n * BN + static_cast<int>(rank) * (BN / 2) + p.b1_noff;
        }
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1)) {
            atomicExch(p.err, kErrTimeoutProducer);
            *abort_flag = 1;
            break;
          }
          const uint32_t full_leader = mapa_shared(smem_u32(&full[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * P_STAGE_BYTES);
          const int kc = kb * BK;
          tma_load_2d_pair(sA + stage * A_BYTES, &map_a, full_leader, kc, row0);
          tma_load_4d_pair(sB + stage * B_HALF, bmap, full_leader, kc, bg, brow, e);
          if (++stage == P_STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------- MMA issuer (leader CTA only)
    if (lane == 0 && leader) {
      constexpr uint32_t kFmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
      const uint32_t idesc = idesc_f16(kFmt, P_BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int i = 0;
      for (int L = pair; L < total && !*abort_flag; L += npairs, ++i) {
        const int acc = i & 1;
        const uint32_t acc_phase = (i >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1)) {
          atomicExch(p.err, kErrTimeoutMma);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&full[stage], phase)) {
            atomicExch(p.err, kErrTimeoutMma);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * B_HALF);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            tc_mma_f16_pair(d_tmem, smem_desc_k_sw128(a_addr + kk * 32),
                            smem_desc_k_sw128(b_addr + kk * 32), idesc,
                            (kb | kk) != 0 ? 1u : 0u);
          }
          tc_commit_pair(&empty[stage], 0x3);
          if (++stage == P_STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        tc_commit_pair(&tfull[acc], 0x3);
      }
      tc_commit_pair(done, 0x1);
      mbar_wait(done, 0);
    }
  } else {
    // ----------------------------------------------------- epilogue (both CTAs)
    const int q = warp & 3;
    const int r_in_tile = static_cast<int>(rank) * BM + q * 32 + lane;
    int ec0, ec1;
    epi_cols(p, warp, ec0, ec1);
    int i = 0;
    for (int L = pair; L < total && !*abort_flag; L += npairs, ++i) {
      const int acc = i & 1;
      const uint32_t acc_phase = (i >> 1) & 1;
      if (!mbar_wait(&tfull[acc], acc_phase)) {
        atomicExch(p.err, kErrTimeoutEpilogue);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      int e, m, n;
      decode_tile(L, s_tiles, E, p.n_tiles, e, m, n);
      const int row = s_offs[e] + m * P_BM + r_in_tile;
      const bool valid = row < s_offs[e + 1];
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
      epilogue_rows<T>(p, taddr, row, valid, e, p.gated ? n * (BN / 2) : n * BN, ec0, ec1);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), 0));
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its peer may still signal it or read its smem
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}


// ---------------------------------------------------------------------------
// QMoE prefill: the CTA-pair kernel with int4/int8 B operands converted in shared
// memory; the unpacked weights never exist in HBM.  Three rings per CTA:
//   A ring (QA stages)   fp16 activations, TMA, completion on the leader's `fullA`;
//   P ring (QP stages)   packed codes of this CTA's 128 B rows (uint8 tile, 32/64-byte
//                        swizzled), TMA by a second producer warp, released by the
//                        converters: it runs further ahead than the A ring, so HBM
//                        latency is off the conversion's critical path;
//   B ring (QB stages)   fp16 B tiles in the 128-byte-swizzled K-major layout of the MMA
//                        descriptor, written by eight converter warps (two groups on
//                        alternate k-blocks, one B row per thread: (q - zp) * scale), made visible to the tensor
//                        core with fence.proxy.async, announced on the leader's `cdone`.
// The leader's MMA waits for `fullA` and `cdone` of both CTAs and releases the A and B
// slots of both CTAs with multicast commits.
constexpr int QA = 4;
constexpr int QB = 6;
constexpr int QP = 6;
constexpr int Q_THREADS = 608;   // warps 0 A TMA, 1 MMA, 2..9 epilogue, 10..17 converters, 18 P TMA
constexpr int CONV_WARPS = 8;
constexpr int kConvGroups = 4;   // converter groups working on different k-blocks
constexpr int Q_PWARP = 18;
template <int BITS> constexpr int q_packed_bytes() { return BM * BK * BITS / 8; }
template <int BITS> constexpr int q_smem_bytes() {
  return 1024 + QA * A_BYTES + QB * B_HALF + QP * q_packed_bytes<BITS>() + 64 * 8 +
         2 * (kMaxExperts + 1) * 4;
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// 8 codes (one 16-byte output chunk, natural order) -> fp16 (q - zp) * s.
template <int BITS>
__device__ __forceinline__ uint4 convert8(const uint8_t* codes, __half2 s2) {
  uint4 o;
  uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
  if (BITS == 8) {
    const uint2 w = *reinterpret_cast<const uint2*>(codes);
    const __half2 zp = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
    ow[0] = h2u(__hmul2(__hsub2(u2h(__byte_perm(w.x, 0x64646464u, 0x4140u)), zp), s2));
    ow[1] = h2u(__hmul2(__hsub2(u2h(__byte_perm(w.x, 0x64646464u, 0x4342u)), zp), s2));
    ow[2] = h2u(__hmul2(__hsub2(u2h(__byte_perm(w.y, 0x64646464u, 0x4140u)), zp), s2));
    ow[3] = h2u(__hmul2(__hsub2(u2h(__byte_perm(w.y, 0x64646464u, 0x4342u)), zp), s2));
  } else {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(codes);
    const __half2 zp = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t b = (w >> (8 * i)) & 0xFFu;
      const uint32_t u = (b & 0xFu) | ((b & 0xF0u) << 12) | 0x64006400u;
      ow[i] = h2u(__hmul2(__hsub2(u2h(u), zp), s2));
    }
  }
  return o;
}

template <int BITS>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Q_THREADS, 1)
tc_pair_qgemm_kernel(const __grid_constant__ CUtensorMap map_a,
                     const __grid_constant__ CUtensorMap map_q1,
                     const __grid_constant__ CUtensorMap map_q3, const TcParams p) {
  constexpr int PB = q_packed_bytes<BITS>();
  constexpr int ROW_BYTES = BK * BITS / 8;  // packed bytes of one B row per k-block
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + QA * A_BYTES;
  uint8_t* sP = sB + QB * B_HALF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + QP * PB);
  uint64_t* fullA = bars;                  // [QA]
  uint64_t* emptyA = fullA + QA;           // [QA]
  uint64_t* fullP = emptyA + QA;           // [QP]
  uint64_t* emptyP = fullP + QP;           // [QP]
  uint64_t* cdone = emptyP + QP;           // [QB]  (leader: both CTAs' converters)
  uint64_t* emptyB = cdone + QB;           // [QB]
  uint64_t* tfull = emptyB + QB;           // [2]
  uint64_t* tempty = tfull + 2;            // [2]
  uint64_t* done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int32_t* s_tiles = reinterpret_cast<int32_t*>(bars + 64);
  int32_t* s_offs = s_tiles + (kMaxExperts + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int E = p.E;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  for (int i = threadIdx.x; i <= E; i += blockDim.x) {
    s_tiles[i] = p.tiles[i];
    s_offs[i] = p.offsets[i];
  }
  if (threadIdx.x == 0) {
    for (int st = 0; st < QA; ++st) {
      mbar_init(&fullA[st], 1);
      mbar_init(&emptyA[st], 1);
    }
    for (int st = 0; st < QP; ++st) {
      mbar_init(&fullP[st], 1);
      mbar_init(&emptyP[st], CONV_WARPS / kConvGroups);
    }
    for (int st = 0; st < QB; ++st) {
      mbar_init(&cdone[st], 2 * CONV_WARPS / kConvGroups);  // one group's warps x 2 CTAs
      mbar_init(&emptyB[st], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * EPI_WARPS);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_q1);
    if (p.gated) tma_prefetch_desc(&map_q3);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int total = s_tiles[E] * p.n_tiles;
  const int nk = (p.K + BK - 1) / BK;
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;
  // This CTA's B rows come from operand 3 (linear half) in CTA 1 of a gated pass.
  const bool use3 = p.gated && rank == 1;

  if (warp == 0) {
    // ---------------------------------------------------------- A producer (TMA)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int L = pair; L < total && !*abort_flag && !p.test_stall; L += npairs) {
        int e, m, n;
        decode_tile(L, s_tiles, E, p.n_tiles, e, m, n);
        const int row0 = s_offs[e] + m * P_BM + static_cast<int>(rank) * BM;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&emptyA[stage], phase ^ 1)) {
            atomicExch(p.err, kErrTimeoutProducer);
            *abort_flag = 1;
            break;
          }
          const uint32_t full_leader = mapa_shared(smem_u32(&fullA[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&fullA[stage], 2 * A_BYTES);
          tma_load_2d_pair(sA + stage * A_BYTES, &map_a, full_leader, kb * BK, row0);
          if (++stage == QA) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == Q_PWARP) {
    // ----------------------------------------------------- packed-code producer (TMA)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int L = pair; L < total && !*abort_flag && !p.test_stall; L += npairs) {
        int e, m, n;
        decode_tile(L, s_tiles, E, p.n_tiles, e, m, n);
        const CUtensorMap* qmap = use3 ? &map_q3 : &map_q1;
        const int bg = use3 ? p.b3_g : p.b1_g;
        const int brow = p.gated ? n * (BN / 2) + (use3 ? p.b3_noff : p.b1_noff)
                                 : n * BN + static_cast<int>(rank) * (BN / 2) + p.b1_noff;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&emptyP[stage], phase ^ 1)) {
            atomicExch(p.err, kErrTimeoutProducer);
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&fullP[stage], PB);
          tma_load_4d(sP + stage * PB, qmap, &fullP[stage], kb * ROW_BYTES, bg, brow, e);
          if (++stage == QP) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------- MMA issuer (leader CTA only)
    if (lane == 0 && leader) {
      const uint32_t idesc = idesc_f16(0u, P_BM, BN);
      int sa = 0, sb = 0;
      uint32_t pa = 0, pb = 0;
      int i = 0;
      for (int L = pair; L < total && !*abort_flag; L += npairs, ++i) {
        const int acc = i & 1;
        const uint32_t acc_phase = (i >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1)) {
          atomicExch(p.err, kErrTimeoutMma);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&fullA[sa], pa) || !mbar_wait(&cdone[sb], pb)) {
            atomicExch(p.err, kErrTimeoutMma);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + sa * A_BYTES);
          const uint32_t b_addr = smem_u32(sB + sb * B_HALF);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            tc_mma_f16_pair(d_tmem, smem_desc_k_sw128(a_addr + kk * 32),
                            smem_desc_k_sw128(b_addr + kk * 32), idesc,
                            (kb | kk) != 0 ? 1u : 0u);
          }
          tc_commit_pair(&emptyA[sa], 0x3);
          tc_commit_pair(&emptyB[sb], 0x3);
          if (++sa == QA) { sa = 0; pa ^= 1; }
          if (++sb == QB) { sb = 0; pb ^= 1; }
        }
        if (!ok) break;
        tc_commit_pair(&tfull[acc], 0x3);
      }
      tc_commit_pair(done, 0x1);
      mbar_wait(done, 0);
    }
  } else if (warp >= 2 + EPI_WARPS) {
    // ------------------------------------------------------- converters (both CTAs)
    // kConvGroups groups of warps take k-blocks round robin (group h: kb = h, h+G, ...),
    // so that many conversions are in flight; each thread converts kRowsPerThread B rows.
    const int ct = threadIdx.x - (2 + EPI_WARPS) * 32;  // 0 .. 255
    constexpr int kThreadsPerGroup = CONV_WARPS * 32 / kConvGroups;
    constexpr int kRowsPerThread = BM / kThreadsPerGroup;
    const int grp = ct / kThreadsPerGroup;
    const int r0 = ct % kThreadsPerGroup;                // rows r0 + j * kThreadsPerGroup
    const __half* scales = use3 ? p.scales3 : p.scales1;
    const int G = use3 ? p.b3_G : p.b1_G;
    const int g = use3 ? p.b3_g : p.b1_g;
    const int noff = use3 ? p.b3_noff : p.b1_noff;
    const int rows_e = use3 ? p.b3_rows : p.b1_rows;
    const int nb = p.qblock ? (p.K + p.qblock - 1) / p.qblock : 1;
    const uint32_t cdone_leader0 = mapa_shared(smem_u32(&cdone[0]), 0);
    // Global k-block counter of this CTA (continues across tiles); ring slot and phase
    // of k-block gi: gi % Q, (gi / Q) & 1.
    int it = 0;
    for (int L = pair; L < total && !*abort_flag; L += npairs) {
      int e, m, n;
      decode_tile(L, s_tiles, E, p.n_tiles, e, m, n);
      const __half* srs[kRowsPerThread];
      __half2 row_scale[kRowsPerThread];
#pragma unroll
      for (int j = 0; j < kRowsPerThread; ++j) {
        const int r = r0 + j * kThreadsPerGroup;
        const int nrow = p.gated ? n * (BN / 2) + r : n * BN + static_cast<int>(rank) * (BN / 2) + r;
        const int64_t srow = static_cast<int64_t>(e) * rows_e +
                             static_cast<int64_t>(min(nrow, p.N - 1) + noff) * G + g;
        srs[j] = scales + srow * nb;
        row_scale[j] = __half2half2(srs[j][0]);
      }
      bool ok = true;
      const int kb0 = ((grp - it) % kConvGroups + kConvGroups) % kConvGroups;
      for (int kb = kb0; kb < nk; kb += kConvGroups) {
        const int gi = it + kb;  // global k-block index
        const int sp = gi % QP, sb = gi % QB;
        const uint32_t pp = (gi / QP) & 1, pb = (gi / QB) & 1;
        if (!mbar_wait(&fullP[sp], pp) || !mbar_wait(&emptyB[sb], pb ^ 1)) {
          atomicExch(p.err, kErrTimeoutProducer);
          *abort_flag = 1;
          ok = false;
          break;
        }
#pragma unroll
        for (int j = 0; j < kRowsPerThread; ++j) {
          const int r = r0 + j * kThreadsPerGroup;
          const uint8_t* prow = sP + sp * PB + r * ROW_BYTES;
          uint8_t* brow_s = sB + sb * B_HALF + r * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) {  // chunks of 8 codes
            const int byte_off = c * BITS;     // byte offset of code 8c in the packed row
            const int chunk = byte_off >> 4;
            const int phys = BITS == 8 ? (chunk ^ ((r >> 1) & 3)) : (chunk ^ ((r >> 2) & 1));
            const uint8_t* codes = prow + phys * 16 + (byte_off & 15);
            const __half2 s2 =
                p.qblock ? __half2half2(srs[j][min(kb * BK + 8 * c, p.K - 1) / p.qblock])
                         : row_scale[j];
            const uint4 o = convert8<BITS>(codes, s2);
            *reinterpret_cast<uint4*>(brow_s + ((c ^ (r & 7)) * 16)) = o;
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive_cluster(cdone_leader0 + sb * 8);
          mbar_arrive(&emptyP[sp]);
        }
      }
      if (!ok) break;
      it += nk;
    }
  } else {
    // ----------------------------------------------------- epilogue (both CTAs)
    const int q = warp & 3;
    const int r_in_tile = static_cast<int>(rank) * BM + q * 32 + lane;
    int ec0, ec1;
    epi_cols(p, warp, ec0, ec1);
    int i = 0;
    for (int L = pair; L < total && !*abort_flag; L += npairs, ++i) {
      const int acc = i & 1;
      const uint32_t acc_phase = (i >> 1) & 1;
      if (!mbar_wait(&tfull[acc], acc_phase)) {
        atomicExch(p.err, kErrTimeoutEpilogue);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      int e, m, n;
      decode_tile(L, s_tiles, E, p.n_tiles, e, m, n);
      const int row = s_offs[e] + m * P_BM + r_in_tile;
      const bool valid = row < s_offs[e + 1];
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
      epilogue_rows<__half>(p, taddr, row, valid, e, p.gated ? n * (BN / 2) : n * BN, ec0, ec1);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), 0));
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// ----------------------------------------------------------------- host side
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

CUtensorMapDataType tma_dtype(int dt) {
  return dt == kDtBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

// A: [rows, K] row-major, box 128 rows x 64 columns.
bool make_map_a(CUtensorMap* m, int dt, const void* ptr, int64_t rows, int K) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
  cuuint32_t box[2] = {BK, BM};
  cuuint32_t es[2] = {1, 1};
  return enc(m, tma_dtype(dt), 2, const_cast<void*>(ptr), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

// B: weights of all experts viewed as [E][Nrows/G][G][K], box 1 x 128 x 1 x 64.
bool make_map_b(CUtensorMap* m, int dt, const GemmOperandB& b, int K, int E) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  const cuuint64_t rows_g = static_cast<cuuint64_t>(b.n_rows / b.G);
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(b.G), rows_g,
                        static_cast<cuuint64_t>(E)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(K) * 2,
                           static_cast<cuuint64_t>(K) * 2 * b.G,
                           static_cast<cuuint64_t>(K) * 2 * b.n_rows};
  cuuint32_t box[4] = {BK, 1, BN / 2, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  return enc(m, tma_dtype(dt), 4, const_cast<void*>(b.ptr), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

template <typename T>
cudaError_t launch_t(const GemmArgs& g, int num_sms, bool pair, cudaStream_t s) {
  CUtensorMap ma, mb1, mb3;
  if (!make_map_a(&ma, g.dtype, g.a, g.rows, g.K)) return cudaErrorInvalidValue;
  if (!make_map_b(&mb1, g.dtype, g.b1, g.K, g.E)) return cudaErrorInvalidValue;
  if (g.gated) {
    if (!make_map_b(&mb3, g.dtype, g.b3, g.K, g.E)) return cudaErrorInvalidValue;
  } else {
    mb3 = mb1;
  }
  TcParams p;
  p.offsets = g.offsets;
  p.tiles = pair ? g.tiles256 : g.tiles128;
  p.E = g.E;
  p.K = g.K;
  p.N = g.N;
  p.gated = g.gated ? 1 : 0;
  p.n_tiles = g.gated ? (g.N + BN / 2 - 1) / (BN / 2) : (g.N + BN - 1) / BN;
  p.b1_g = g.b1.g;
  p.b3_g = g.b3.g;
  p.b1_noff = g.b1.n_off;
  p.b3_noff = g.b3.n_off;
  p.bias1 = g.bias1;
  p.bias3 = g.bias3;
  p.bias_stride = g.bias_stride;
  p.bias_e_stride = g.bias_e_stride;
  p.ap = g.ap;
  p.out = g.out;
  p.ldo = g.ldo;
  p.err = g.err;
  p.test_stall = g.test_stall;
  // The attribute call is idempotent; a race between first callers is benign.
  static bool attr_set[2] = {false, false};
  if (!attr_set[pair]) {
    cudaError_t st = pair ? cudaFuncSetAttribute(tc_pair_grouped_gemm_kernel<T>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 P_SMEM_BYTES)
                          : cudaFuncSetAttribute(tc_grouped_gemm_kernel<T>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 SMEM_BYTES);
    if (st != cudaSuccess) return st;
    attr_set[pair] = true;
  }
  // The real tile count lives on the device; an upper bound sizes the grid.
  const int rows_per_tile = pair ? P_BM : BM;
  const int64_t ub = ((g.rows + rows_per_tile - 1) / rows_per_tile + g.E) * p.n_tiles;
  if (pair) {
    const int64_t pairs = std::min<int64_t>(ub, num_sms / 2);
    tc_pair_grouped_gemm_kernel<T><<<static_cast<int>(2 * pairs), THREADS, P_SMEM_BYTES, s>>>(
        ma, mb1, mb3, p);
  } else {
    const int grid = static_cast<int>(std::min<int64_t>(ub, num_sms));
    tc_grouped_gemm_kernel<T><<<grid, THREADS, SMEM_BYTES, s>>>(ma, mb1, mb3, p);
  }
  return cudaGetLastError();
}


// Packed B: uint8 codes of all experts viewed as [E][Nrows/G][G][K*bits/8], box
// 1 x 128 x 1 x (64*bits/8) bytes, swizzled so the converters read it without bank
// conflicts (64-byte swizzle for int8 rows of 64 B, 32-byte for int4 rows of 32 B).
bool make_map_q(CUtensorMap* m, const GemmOperandB& b, int K, int bits, int E) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  const cuuint64_t kb = static_cast<cuuint64_t>(K) * bits / 8;
  const cuuint64_t rows_g = static_cast<cuuint64_t>(b.n_rows / b.G);
  cuuint64_t dims[4] = {kb, static_cast<cuuint64_t>(b.G), rows_g, static_cast<cuuint64_t>(E)};
  cuuint64_t strides[3] = {kb, kb * b.G, kb * b.n_rows};
  cuuint32_t box[4] = {static_cast<cuuint32_t>(BK * bits / 8), 1, BN / 2, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(b.ptr), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE,
             bits == 8 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

template <int BITS>
cudaError_t launch_q(const GemmArgs& g, int num_sms, cudaStream_t s) {
  CUtensorMap ma, mq1, mq3;
  if (!make_map_a(&ma, g.dtype, g.a, g.rows, g.K)) return cudaErrorInvalidValue;
  if (!make_map_q(&mq1, g.b1, g.K, BITS, g.E)) return cudaErrorInvalidValue;
  if (g.gated) {
    if (!make_map_q(&mq3, g.b3, g.K, BITS, g.E)) return cudaErrorInvalidValue;
  } else {
    mq3 = mq1;
  }
  TcParams p{};
  p.offsets = g.offsets;
  p.tiles = g.tiles256;
  p.E = g.E;
  p.K = g.K;
  p.N = g.N;
  p.gated = g.gated ? 1 : 0;
  p.n_tiles = g.gated ? (g.N + BN / 2 - 1) / (BN / 2) : (g.N + BN - 1) / BN;
  p.b1_g = g.b1.g;
  p.b3_g = g.b3.g;
  p.b1_noff = g.b1.n_off;
  p.b3_noff = g.b3.n_off;
  p.bias1 = g.bias1;
  p.bias3 = g.bias3;
  p.bias_stride = g.bias_stride;
  p.bias_e_stride = g.bias_e_stride;
  p.ap = g.ap;
  p.out = g.out;
  p.ldo = g.ldo;
  p.err = g.err;
  p.test_stall = g.test_stall;
  p.scales1 = static_cast<const __half*>(g.b1.scales);
  p.scales3 = static_cast<const __half*>(g.gated ? g.b3.scales : g.b1.scales);
  p.qblock = g.qblock;
  p.b1_G = g.b1.G;
  p.b3_G = g.gated ? g.b3.G : 1;
  p.b1_rows = g.b1.n_rows;
  p.b3_rows = g.gated ? g.b3.n_rows : g.b1.n_rows;
  static bool attr_set = false;  // idempotent; a race between first callers is benign
  if (!attr_set) {
    cudaError_t st = cudaFuncSetAttribute(tc_pair_qgemm_kernel<BITS>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          q_smem_bytes<BITS>());
    if (st != cudaSuccess) return st;
    attr_set = true;
  }
  const int64_t ub = ((g.rows + P_BM - 1) / P_BM + g.E) * p.n_tiles;
  const int64_t pairs = std::min<int64_t>(ub, num_sms / 2);
  tc_pair_qgemm_kernel<BITS><<<static_cast<int>(2 * pairs), Q_THREADS, q_smem_bytes<BITS>(), s>>>(
      ma, mq1, mq3, p);
  return cudaGetLastError();
}

}  // namespace

bool tc_q_supported(const GemmArgs& g) {
  if (g.dtype != kDtF16 || (g.qbits != 4 && g.qbits != 8)) return false;
  if ((static_cast<int64_t>(g.K) * g.qbits / 8) % 16 != 0 || g.K % BK != 0) return false;
  if (g.qblock != 0 && (g.qblock % 8 != 0)) return false;
  if (g.ldo % 8 != 0 || g.E > kMaxExperts) return false;
  if (g.b1.scales == nullptr || (g.gated && g.b3.scales == nullptr)) return false;
  auto aligned = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  if (!aligned(g.a) || !aligned(g.b1.ptr) || !aligned(g.out)) return false;
  if (g.gated && !aligned(g.b3.ptr)) return false;
  return get_encode_fn() != nullptr;
}

cudaError_t launch_gemm_tc_q(const GemmArgs& g, int num_sms, cudaStream_t s) {
  if (g.rows == 0 || g.N == 0) return cudaSuccess;
  return g.qbits == 4 ? launch_q<4>(g, num_sms, s) : launch_q<8>(g, num_sms, s);
}

namespace {
}  // namespace

bool tc_supported(const GemmArgs& g) {
  if (g.dtype != kDtF16 && g.dtype != kDtBF16) return false;
  if (g.K % 8 != 0 || g.K <= 0) return false;
  if (g.ldo % 8 != 0) return false;
  if (g.E > kMaxExperts) return false;
  auto aligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!aligned(g.a) || !aligned(g.b1.ptr) || !aligned(g.out)) return false;
  if (g.gated && !aligned(g.b3.ptr)) return false;
  return get_encode_fn() != nullptr;
}

cudaError_t launch_gemm_tc(const GemmArgs& g, int num_sms, int mode, cudaStream_t s) {
  if (g.rows == 0 || g.N == 0) return cudaSuccess;
  // mode 0: choose (CTA pairs when experts average >= 256 rows), 1: single CTA, 2: pairs.
  const bool pair = mode == 2 || (mode == 0 && g.rows >= 256 * static_cast<int64_t>(g.E));
  if (g.dtype == kDtF16) return launch_t<__half>(g, num_sms, pair, s);
  if (g.dtype == kDtBF16) return launch_t<__nv_bfloat16>(g, num_sms, pair, s);
  return cudaErrorInvalidValue;
}

}  // namespace moe
