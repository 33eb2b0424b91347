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
#include <cstdio>
#include <type_traits>
#include <vector>

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
    1024 /*align slack*/ + STAGES * (A_BYTES + B_BYTES) + EPI_WARPS * 2048 /*epilogue staging*/ +
    64 * 8 /*barriers*/ + 2 * (kMaxExperts + 1) * 4;

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
  // CTA-pair kernel: last tiles of an expert with <= swap_max rows run swapped (0 = never).
  int swap_max;
  // CTA-pair kernel: zeroed counter from which pairs claim tiles in order (dynamic
  // schedule); nullptr = static round-robin.
  int* tile_counter;
  // Output row remap (expert-parallel return over peer memory): row p of segment q
  // (seg_start[q] <= p < seg_start[q+1]) goes to row seg_dst[q] + p - seg_start[q] of
  // out_peers[q % remap_world]; seg_start == nullptr: row p of `out`.
  const int32_t* seg_start;
  const int32_t* seg_dst;
  int nseg;
  int remap_world;
  void* out_peers[kMaxEpRanks];
  int trace;   // diagnostics: CTA 0 records per-tile phase timestamps (MOE_B200_GEMM_TRACE)
  // Packed operands with one scale per row (block_size 0): 0 = the converters apply
  // (q - zp) * s; 1 = they write exact q - zp and the epilogue multiplies column n by its
  // scale; 2 = they write the biased codes 1024 + q and the epilogue applies
  // s_n * (acc - qbias * rowsum[row]) with qbias = 1024 + zp.
  int qepi;
  float qbias;
  const float* rowsum;
  // CTA-pair kernel: A row p is row a_src[p] / a_k of the map's tensor (TMA gather4,
  // four rows per lane of the producer warp); nullptr = A rows p of the map's tensor.
  const int32_t* a_src;
  int a_k;
  // Fused routing-weighted combine (GemmArgs.comb_*; comb_cnt == nullptr: off).
  unsigned* comb_cnt;
  const int32_t* comb_src;
  const int32_t* comb_pos;
  const float* comb_w;
  void* comb_out;
  int comb_k;
};

// Per-tile phase trace of CTA 0 (diagnostics only).  Entry i: [2i] = %globaltimer ns,
// [2i+1] = event << 32 | tile.
constexpr unsigned kTraceCap = 16384;
__device__ unsigned long long g_tile_trace[2 * kTraceCap];
__device__ unsigned int g_trace_n;
enum TraceEvent : unsigned {
  kTrClaim = 1, kTrProdDone = 2, kTrMmaStart = 3, kTrMmaFirst = 4, kTrMmaDone = 5,
  kTrEpiStart = 6, kTrEpiDone = 7,
};
__device__ __forceinline__ void trace(const TcParams& p, unsigned ev, int tile) {
  if (!p.trace || blockIdx.x != 0) return;
  const unsigned i = atomicAdd(&g_trace_n, 1u);
  if (i < kTraceCap) {
    g_tile_trace[2 * i] = globaltimer_ns();
    g_tile_trace[2 * i + 1] = (static_cast<unsigned long long>(ev) << 32) |
                              static_cast<unsigned>(tile);
  }
}

template <typename T>
__device__ __forceinline__ T* out_row(const TcParams& p, int row) {
  if (p.seg_start == nullptr) return static_cast<T*>(p.out) + static_cast<int64_t>(row) * p.ldo;
  int lo = 0, hi = p.nseg - 1;  // the last segment starting at or before `row`
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(&p.seg_start[mid]) <= row) lo = mid; else hi = mid - 1;
  }
  const int dst = __ldg(&p.seg_dst[lo]) + row - __ldg(&p.seg_start[lo]);
  return static_cast<T*>(p.out_peers[lo % p.remap_world]) + static_cast<int64_t>(dst) * p.ldo;
}

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

// Fast-math activations for the 16-bit epilogue (inputs and outputs are fp16/bf16,
// so the few-ulp error of the approximate exp and reciprocal is far below the output
// rounding).  The activation is dispatched once per chunk of n values, each variant a
// straight loop: a per-element switch, unrolled over the chunk with erf, exp and an IEEE
// reciprocal inlined in every copy, ran the epilogue out of the instruction cache
// (2.8 us per 32 values, ~10x the whole rest of the epilogue).
__device__ __forceinline__ float fast_sigmoid(float x) {
  return __fdividef(1.0f, 1.0f + __expf(-x));
}

template <int n>
__device__ __forceinline__ void act_chunk(int act, float (&v)[n]) {
  switch (act) {
    case kRelu:
#pragma unroll
      for (int j = 0; j < n; ++j) v[j] = fmaxf(v[j], 0.0f);
      break;
    case kGelu:
#pragma unroll
      for (int j = 0; j < n; ++j) v[j] = 0.5f * v[j] * (1.0f + erff(v[j] * 0.70710678118654752f));
      break;
    case kSilu:
#pragma unroll
      for (int j = 0; j < n; ++j) v[j] = v[j] * fast_sigmoid(v[j]);
      break;
    default:
      break;
  }
}

// v[j] = act(g[j]) * u[j] (swiglu: the clamped, alpha-scaled form with u + beta).
template <int n>
__device__ __forceinline__ void act_gated_chunk(const ActParams& ap, float (&g)[n],
                                                const float (&u)[n]) {
  if (ap.act == kSwiglu) {
    const float lim = ap.limit, al = ap.alpha, be = ap.beta;
#pragma unroll
    for (int j = 0; j < n; ++j) {
      const float gc = fminf(g[j], lim);
      const float uc = fminf(fmaxf(u[j], -lim), lim);
      g[j] = gc * fast_sigmoid(al * gc) * (uc + be);
    }
    return;
  }
  act_chunk<n>(ap.act, g);
#pragma unroll
  for (int j = 0; j < n; ++j) g[j] *= u[j];
}

// Adds bias[e, col0 + j] (clamped to column N - 1) to v[0..n).
template <typename T, int n>
__device__ __forceinline__ void add_bias(float (&v)[n], const void* bias, int e, int col0,
                                         const TcParams& p) {
  if (bias == nullptr) return;
#pragma unroll
  for (int j = 0; j < n; ++j) v[j] += bias_val<T>(bias, e, min(col0 + j, p.N - 1), p);
}

// Epilogue of one accumulator tile for the calling warp's 32 TMEM lanes (one output
// row per lane), accumulator columns [c0, c1) in chunks of 32 output columns.  Gated:
// columns [0,128) hold the gate and [128,256) the linear half of output columns
// n0..n0+127 (c ranges over the gate columns); plain: columns [0,256) are outputs
// n0..n0+255.  Each chunk goes through the warp's 2 KB staging area (32 rows x 64 B,
// 16-byte granules XOR-swizzled by row so both the row-wise writes and the column-wise
// reads are conflict-free) and leaves as 16-byte stores that cover 8 rows x 64 B per
// instruction, instead of one 16-byte piece of 32 different rows.
constexpr int EPI_CHUNK = 32;                 // output columns per staged chunk
constexpr int EPI_STAGE_BYTES = 32 * EPI_CHUNK * 2;  // per epilogue warp

// Per-row-scaled packed operands (qepi 1 / 2): v[j] = s(col0 + j) * (v[j] - off), s the
// scale of output column col0 + j of expert e in the operand's stored-row addressing.
template <int n>
__device__ __forceinline__ void q_scale_cols(float (&v)[n], const __half* scales, int rows_e,
                                             int G, int g, int noff, int e, int col0, int N,
                                             float off) {
#pragma unroll
  for (int j = 0; j < n; ++j) {
    const int64_t srow = static_cast<int64_t>(e) * rows_e +
                         static_cast<int64_t>(min(col0 + j, N - 1) + noff) * G + g;
    v[j] = __half2float(__ldg(scales + srow)) * (v[j] - off);
  }
}

// Fused combine of the (token, 32-column segment) items a warp completed: item (s, l) for
// each bit l of masks[s], token = lane l's `tok`, columns col_base + s * 32 + [0, 32).
// Four lanes take an item (8 columns each, one 16-byte load per slot row), eight items per
// pass; each sums the token's k fc2 rows, read from L2 (other CTAs wrote them), in slot
// order in fp32, exactly as the separate combine kernel sums them.
template <typename T, int S>
__device__ __forceinline__ void combine_items(const TcParams& p, const unsigned (&masks)[S],
                                              int tok, int col_base, int lane) {
  int total = 0;
#pragma unroll
  for (int s = 0; s < S; ++s) total += __popc(masks[s]);
  const int k = p.comb_k;
  const T* y = static_cast<const T*>(p.out);
#pragma unroll 1
  for (int it0 = 0; it0 < total; it0 += 8) {
    const int it = it0 + (lane >> 2);
    int s_sel = -1, l_sel = 0, rem = it;
#pragma unroll
    for (int s = 0; s < S; ++s) {
      const int c = __popc(masks[s]);
      if (s_sel < 0 && it < total) {
        if (rem < c) {
          s_sel = s;
          l_sel = static_cast<int>(__fns(masks[s], 0, rem + 1));
        } else {
          rem -= c;
        }
      }
    }
    const int t = __shfl_sync(0xffffffffu, tok, l_sel);
    const int col = col_base + s_sel * 32 + (lane & 3) * 8;
    if (s_sel < 0 || col >= p.N) continue;
    const int32_t* pos = p.comb_pos + static_cast<int64_t>(t) * k;
    const float* w = p.comb_w + static_cast<int64_t>(t) * k;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
    for (int j = 0; j < k; ++j) {
      const uint4 v = __ldcg(reinterpret_cast<const uint4*>(
          y + static_cast<int64_t>(__ldg(pos + j)) * p.ldo + col));
      const T* e = reinterpret_cast<const T*>(&v);
      const float wj = __ldg(w + j);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] += wj * to_f(e[q]);
    }
    uint4 o;
    o.x = pack2<T>(acc[0], acc[1]);
    o.y = pack2<T>(acc[2], acc[3]);
    o.z = pack2<T>(acc[4], acc[5]);
    o.w = pack2<T>(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(static_cast<T*>(p.comb_out) + static_cast<int64_t>(t) * p.N + col) = o;
  }
}

// One arrival of permuted row `row` at 32-column segment `seg` (after the caller's
// stores of that segment and a device-scope fence): true when it completes the token's
// k rows, the caller then owns the segment's combine.
__device__ __forceinline__ bool combine_arrive(const TcParams& p, int row, int seg, int& tok) {
  tok = __ldg(p.comb_src + row) / p.comb_k;
  unsigned* c = p.comb_cnt + static_cast<int64_t>(tok) * ((p.N + 31) / 32) + seg;
  return atomicAdd(c, 1u) == static_cast<unsigned>(p.comb_k - 1);
}

// Scale of output column `col` of expert e (stored-row addressing), for the swapped tiles.
__device__ __forceinline__ float q_scale_at(const __half* scales, int rows_e, int G, int g,
                                            int noff, int e, int col) {
  return __half2float(__ldg(scales + static_cast<int64_t>(e) * rows_e +
                            static_cast<int64_t>(col + noff) * G + g));
}

template <typename T>
__device__ __forceinline__ void epilogue_rows(const TcParams& p, uint32_t taddr, int row,
                                              bool valid, int e, int n0, int c0, int c1,
                                              uint8_t* stage, int lane) {
  const unsigned long long my_row =
      valid ? reinterpret_cast<unsigned long long>(out_row<T>(p, row)) : 0ull;
  const float qoff = (p.qepi == 2 && valid) ? p.qbias * __ldg(p.rowsum + row) : 0.f;
  uint4* st_row = reinterpret_cast<uint4*>(stage + lane * (EPI_CHUNK * 2));
  const int wsw = (lane >> 1) & 3;
#pragma unroll 1
  for (int c = c0; c < c1; c += EPI_CHUNK) {
    const int col = n0 + c;
    // Two halves of 16 columns (fewer live registers), each packed into two granules.
#pragma unroll
    for (int hs = 0; hs < 2; ++hs) {
      const int ch = c + 16 * hs, colh = col + 16 * hs;
      float v[16];
      if (p.gated) {
        float u[16];
        tmem_ld16(taddr + ch, v);
        tmem_ld16(taddr + BN / 2 + ch, u);
        tmem_ld_wait();
        if (p.qepi) {
          q_scale_cols<16>(v, p.scales1, p.b1_rows, p.b1_G, p.b1_g, p.b1_noff, e, colh, p.N, qoff);
          q_scale_cols<16>(u, p.scales3, p.b3_rows, p.b3_G, p.b3_g, p.b3_noff, e, colh, p.N, qoff);
        }
        add_bias<T, 16>(v, p.bias1, e, colh, p);
        add_bias<T, 16>(u, p.bias3, e, colh, p);
        act_gated_chunk<16>(p.ap, v, u);
      } else {
        tmem_ld16(taddr + ch, v);
        tmem_ld_wait();
        if (p.qepi)
          q_scale_cols<16>(v, p.scales1, p.b1_rows, p.b1_G, p.b1_g, p.b1_noff, e, colh, p.N, qoff);
        add_bias<T, 16>(v, p.bias1, e, colh, p);
        act_chunk<16>(p.ap.act, v);
      }
#pragma unroll
      for (int qq = 0; qq < 2; ++qq) {
        const int q = 2 * hs + qq;
        uint4 w;
        w.x = pack2<T>(v[8 * qq + 0], v[8 * qq + 1]);
        w.y = pack2<T>(v[8 * qq + 2], v[8 * qq + 3]);
        w.z = pack2<T>(v[8 * qq + 4], v[8 * qq + 5]);
        w.w = pack2<T>(v[8 * qq + 6], v[8 * qq + 7]);
        st_row[q ^ wsw] = w;
      }
    }
    __syncwarp();
#pragma unroll
    for (int pass = 0; pass < 4; ++pass) {
      const int r = pass * 8 + (lane >> 2), q = lane & 3;
      T* rp = reinterpret_cast<T*>(__shfl_sync(0xffffffffu, my_row, r));
      const uint4 w = reinterpret_cast<const uint4*>(stage + r * (EPI_CHUNK * 2))[q ^ ((r >> 1) & 3)];
      if (rp != nullptr && col + 8 * q + 8 <= p.N) *reinterpret_cast<uint4*>(rp + col + 8 * q) = w;
    }
    __syncwarp();
  }
}

// Fused combine after a row tile's stores (called once the tile's TMEM accumulator is
// released, so the MMA of the next tile overlaps it): publish the warp's stores of rows
// [32] x columns [n0 + c0, n0 + c1), count each row's arrival at every 32-column segment
// (one lane's atomics are independent and overlap), and combine the segments this warp
// completed.
template <typename T>
__device__ __forceinline__ void combine_rows(const TcParams& p, int row, bool valid, int n0,
                                             int c0, int c1, int lane) {
  __threadfence();
  __syncwarp();
  constexpr int kSeg = BN / 2 / 32;  // a warp's columns: half of an (ungated) tile
  unsigned masks[kSeg];
  int tok = 0;
#pragma unroll
  for (int i = 0; i < kSeg; ++i) {
    const int c = c0 + i * 32;
    const bool last = valid && c < c1 && n0 + c < p.N && combine_arrive(p, row, (n0 + c) / 32, tok);
    masks[i] = __ballot_sync(0xffffffffu, last);
  }
  __threadfence();
  combine_items<T, kSeg>(p, masks, tok, n0 + c0, lane);
  __syncwarp();
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
  pdl_wait();  // launched dependent (launch_dependent): predecessors' data after this
  pdl_launch_dependents();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* epi_stage = sB + STAGES * B_BYTES;  // [EPI_WARPS][32 rows x 64 B]
  uint64_t* bars = reinterpret_cast<uint64_t*>(epi_stage + EPI_WARPS * EPI_STAGE_BYTES);
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
      epilogue_rows<T>(p, taddr, row, valid, e, p.gated ? n * (BN / 2) : n * BN, ec0, ec1,
                       epi_stage + (warp - 2) * EPI_STAGE_BYTES, lane);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      if (p.comb_cnt != nullptr) combine_rows<T>(p, row, valid, n * BN, ec0, ec1, lane);
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
constexpr int P_SMEM_BYTES = 1024 + P_STAGES * P_STAGE_BYTES + 16 * 32 * 4 * 4 /*exchange*/ +
                             EPI_WARPS * 2048 /*epilogue staging*/ + 64 * 8 +
                             2 * (kMaxExperts + 1) * 4;

constexpr int SW_TOK_ROWS = 64;   // token rows per TMA box of a swapped tile (1-2 per CTA)
constexpr int kPairSwapLimit = 240;  // largest swapped tail (rows); 256 is a full tile
constexpr int SW_HALF = 64;       // gated swapped tile: gate rows, then linear rows, per CTA
constexpr int XCH_SLOTS = 4;      // gate/linear exchange slots (lane quarter pair x column half)
constexpr int XCH_BYTES = XCH_SLOTS * 16 * 32 * 4;

// One tile of the pair kernel.  A tile whose rows (the expert's last, ragged m-tile) are at
// most swap_max is computed swapped: D[w, t] = sum_k W[w, k] X[t, k] with the 256 weight rows
// of the tile as M (128 per CTA, in TMEM lanes) and its rows as N = nt (rows rounded up to
// 16; nt / 2 per CTA), so its MMA work scales with the rows instead of a full 256.
struct PairTile {
  int e, m, n;
  int r0;     // first permuted row
  int rows;   // valid rows (<= 256)
  int nt;     // swapped: MMA N; 0 for a normal tile
};

__device__ __forceinline__ PairTile pair_tile(int L, const int32_t* s_tiles,
                                              const int32_t* s_offs, const TcParams& p) {
  PairTile t;
  decode_tile(L, s_tiles, p.E, p.n_tiles, t.e, t.m, t.n);
  t.r0 = s_offs[t.e] + t.m * P_BM;
  t.rows = min(P_BM, s_offs[t.e + 1] - t.r0);
  t.nt = t.rows <= p.swap_max ? (t.rows + 15) & ~15 : 0;
  return t;
}

// Gate/linear hand-over of the gated swapped epilogue: one slot of 16 columns x 32 lanes
// of fp32, filled by a linear-quarter warp and drained by its gate-quarter partner.
struct Exchange {
  float* buf;        // [XCH_SLOTS][16][32]
  uint64_t* full;    // [XCH_SLOTS], 32 arrivals (the linear warp's lanes)
  uint64_t* empty;   // [XCH_SLOTS], 32 arrivals (the gate warp's lanes)
};

// Epilogue of a swapped tile for the calling warp (TMEM lane quarter q, column chunks of
// 16 starting at c_first, stride 32).  Returns false when a bounded wait expired.
//  plain: lane l of CTA `rank` holds output column f = n*256 + rank*128 + q*32 + l for the
//         tile's rows (TMEM columns);
//  gated: lanes 0..63 of CTA `rank` hold the gate rows and lanes 64..127 the linear rows of
//         output columns f = n*128 + rank*64 + [0, 64); a linear-quarter warp (q = 2, 3)
//         passes its chunk (+ bias) through shared memory to the gate-quarter warp q - 2,
//         which applies the activation and stores.
template <typename T>
__device__ __forceinline__ bool epilogue_swapped(const TcParams& p, const PairTile& t,
                                                 uint32_t taddr, int rank, int q, int lane,
                                                 int half, const Exchange& x, uint32_t& xuse) {
  const int c_first = 16 * half;
  if (p.gated) {
    const bool lin = q >= 2;
    const int f = t.n * (BN / 2) + rank * SW_HALF + (q & 1) * 32 + lane;
    const bool fok = f < p.N;
    const int fc = min(f, p.N - 1);
    const int slot = (q & 1) * 2 + half;
    float* buf = x.buf + slot * 16 * 32;
    const float own_bias = lin ? bias_val<T>(p.bias3, t.e, fc, p) : bias_val<T>(p.bias1, t.e, fc, p);
    // qepi 1 (exact codes, one scale per output column): scale, then bias.
    const float own_scale =
        !p.qepi ? 1.f
        : lin   ? q_scale_at(p.scales3, p.b3_rows, p.b3_G, p.b3_g, p.b3_noff, t.e, fc)
                : q_scale_at(p.scales1, p.b1_rows, p.b1_G, p.b1_g, p.b1_noff, t.e, fc);
#pragma unroll 1
    for (int c = c_first; c < t.nt; c += 32, ++xuse) {
      const uint32_t par = xuse & 1;
      float v[16];
      tmem_ld16(taddr + c, v);
      tmem_ld_wait();
      if (lin) {
        if (!mbar_wait(&x.empty[slot], par ^ 1)) return false;
#pragma unroll
        for (int j = 0; j < 16; ++j) buf[j * 32 + lane] = v[j] * own_scale + own_bias;
        mbar_arrive(&x.full[slot]);
      } else {
        if (!mbar_wait(&x.full[slot], par)) return false;
        float u[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) u[j] = buf[j * 32 + lane];
        mbar_arrive(&x.empty[slot]);
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = v[j] * own_scale + own_bias;
        act_gated_chunk<16>(p.ap, v, u);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int tok = c + j;
          if (fok && tok < t.rows) out_row<T>(p, t.r0 + tok)[f] = from_f<T>(v[j]);
        }
      }
    }
  } else {
    const int f = t.n * BN + rank * (BN / 2) + q * 32 + lane;
    const bool fok = f < p.N;
    const float b = bias_val<T>(p.bias1, t.e, min(f, p.N - 1), p);
    const float sc = p.qepi ? q_scale_at(p.scales1, p.b1_rows, p.b1_G, p.b1_g, p.b1_noff, t.e,
                                         min(f, p.N - 1))
                            : 1.f;
#pragma unroll 1
    for (int c = c_first; c < t.nt; c += 32) {
      float v[16];
      tmem_ld16(taddr + c, v);
      tmem_ld_wait();
      // Lane j < 16 resolves the output row of row c + j once for the warp.
      const int my_tok = c + (lane & 15);
      const unsigned long long my_row =
          my_tok < t.rows ? reinterpret_cast<unsigned long long>(out_row<T>(p, t.r0 + my_tok)) : 0ull;
      if (p.qepi == 2) {  // biased codes: s_n * (acc - (1024 + zp) * rowsum[row])
#pragma unroll
        for (int j = 0; j < 16; ++j)
          v[j] = sc * (v[j] - p.qbias * __ldg(p.rowsum + t.r0 + min(c + j, t.rows - 1))) + b;
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = v[j] * sc + b;
      }
      act_chunk<16>(p.ap.act, v);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        T* row = reinterpret_cast<T*>(__shfl_sync(0xffffffffu, my_row, j));
        if (fok && c + j < t.rows) row[f] = from_f<T>(v[j]);
      }
      if (p.comb_cnt != nullptr) {
        // Rows c .. c+15 of this warp's 32 columns are stored: lane j < 16 counts row c + j's
        // arrival at the segment and, if it completes it, combines it.
        __threadfence();
        __syncwarp();
        const int seg_col = t.n * BN + rank * (BN / 2) + q * 32;
        int tok = 0;
        const bool done = lane < 16 && c + lane < t.rows && seg_col < p.N &&
                          combine_arrive(p, t.r0 + c + lane, seg_col / 32, tok);
        const unsigned masks[1] = {__ballot_sync(0xffffffffu, done)};
        __threadfence();
        combine_items<T, 1>(p, masks, tok, seg_col, lane);
        __syncwarp();
      }
    }
  }
  return true;
}

// Tile queue of the pair kernel.  The leader's producer claims tile numbers in order
// (atomic counter) and publishes each in a TQ-deep queue in both CTAs' shared memory; the
// consumers (leader MMA and epilogue warps, peer producer and epilogue warps) read it and
// release the slot on the leader's tq_empty.  -1 ends the schedule.  Claiming in order
// keeps the m-tiles that share a weight tile running at the same time (L2 reuse) while
// pairs that drew cheap (swapped) tiles take more of them.
constexpr int TQ = 4;
constexpr int TQ_CONSUMERS = 2 + 2 * EPI_WARPS;

__device__ __forceinline__ bool tq_take(int it, const volatile int* s_tq, uint64_t* tq_full,
                                        uint64_t* tq_empty, bool leader, int& L) {
  const int slot = it % TQ;
  if (!mbar_wait_cluster(&tq_full[slot], (it / TQ) & 1)) return false;
  L = s_tq[slot];
  if (leader) mbar_arrive(&tq_empty[slot]);
  else mbar_arrive_cluster(mapa_shared(smem_u32(&tq_empty[slot]), 0));
  return true;
}

template <typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
tc_pair_grouped_gemm_kernel(const __grid_constant__ CUtensorMap map_a,
                            const __grid_constant__ CUtensorMap map_b1,
                            const __grid_constant__ CUtensorMap map_b3,
                            const __grid_constant__ CUtensorMap map_a_sw,
                            const __grid_constant__ CUtensorMap map_b1_sw,
                            const __grid_constant__ CUtensorMap map_b3_sw, const TcParams p) {
  pdl_wait();  // launched dependent (launch_dependent): predecessors' data after this
  pdl_launch_dependents();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + P_STAGES * A_BYTES;
  float* xbuf = reinterpret_cast<float*>(sB + P_STAGES * B_HALF);
  uint8_t* epi_stage = sB + P_STAGES * B_HALF + XCH_BYTES;  // [EPI_WARPS][32 rows x 64 B]
  uint64_t* bars = reinterpret_cast<uint64_t*>(epi_stage + EPI_WARPS * EPI_STAGE_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + P_STAGES;
  uint64_t* tfull = bars + 2 * P_STAGES;
  uint64_t* tempty = bars + 2 * P_STAGES + 2;
  uint64_t* done = bars + 2 * P_STAGES + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * P_STAGES + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const Exchange xch{xbuf, bars + 32, bars + 32 + XCH_SLOTS};
  uint64_t* tq_full = bars + 40;
  uint64_t* tq_empty = bars + 44;
  volatile int* s_tq = reinterpret_cast<volatile int*>(bars + 48);
  int32_t* s_tiles = reinterpret_cast<int32_t*>(bars + 64);
  int32_t* s_offs = s_tiles + (kMaxExperts + 1);
  static_assert(2 * P_STAGES + 6 <= 32, "pair kernel barrier slots overlap the exchange");
  static_assert(32 + 2 * XCH_SLOTS <= 40 && TQ == 4, "pair kernel barrier slots overlap");

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
    for (int i = 0; i < XCH_SLOTS; ++i) {
      mbar_init(&xch.full[i], 32);
      mbar_init(&xch.empty[i], 32);
    }
    for (int i = 0; i < TQ; ++i) {
      mbar_init(&tq_full[i], 1);
      mbar_init(&tq_empty[i], TQ_CONSUMERS);
    }
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
    // Lane 0 claims tiles, waits for free slots and loads B (and A when it is not
    // gathered).  With a gathered A (p.a_src) every lane loads four A rows per k-block
    // with one gather4: lane l rows 4l..4l+3 of this CTA's share of the tile.
    const bool gather = p.a_src != nullptr;
    int stage = 0;
    uint32_t phase = 0;
    for (int it = 0;; ++it) {
      int L = -1;
      if (lane == 0) {
        if (leader) {
          const int slot = it % TQ;
          if (!mbar_wait_cluster(&tq_empty[slot], ((it / TQ) & 1) ^ 1)) {
            atomicExch(p.err, kErrTimeoutProducer);
            *abort_flag = 1;
          }
          L = *abort_flag ? -1
                          : (p.tile_counter != nullptr ? atomicAdd(p.tile_counter, 1)
                                                       : pair + it * npairs);
          if (L >= total) L = -1;
          s_tq[slot] = L;
          st_cluster_s32(mapa_shared(smem_u32(const_cast<int*>(&s_tq[slot])), 1), L);
          mbar_arrive(&tq_full[slot]);
          mbar_arrive_cluster(mapa_shared(smem_u32(&tq_full[slot]), 1));
        } else if (*abort_flag || !tq_take(it, s_tq, tq_full, tq_empty, false, L)) {
          atomicExch(p.err, kErrTimeoutProducer);
          *abort_flag = 1;
          L = -1;
        }
      }
      L = __shfl_sync(0xffffffffu, L, 0);
      if (L < 0) break;
      if (lane == 0) trace(p, kTrClaim, L);
      if (p.test_stall) continue;
      const PairTile t = pair_tile(L, s_tiles, s_offs, p);
      const int e = t.e, n = t.n;
      const int row0 = t.nt ? t.r0 + static_cast<int>(rank) * (t.nt / 2)
                            : t.r0 + static_cast<int>(rank) * BM;
      const CUtensorMap* bmap = (p.gated && rank == 1) ? &map_b3 : &map_b1;
      int bg, brow;
      if (p.gated) {
        bg = rank == 1 ? p.b3_g : p.b1_g;
        brow = n * (BN / 2) + (rank == 1 ? p.b3_noff : p.b1_noff);
      } else {
        bg = p.b1_g;
        brow = n * BN + static_cast<int>(rank) * (BN / 2) + p.b1_noff;
      }
      // Swapped gated tile: this CTA's weight rows are the 64 gate rows, then the 64
      // linear rows, of output columns n*128 + rank*64 + [0,64).
      const int sw_col = n * (BN / 2) + static_cast<int>(rank) * SW_HALF;
      const int tok_boxes = (t.nt / 2 + SW_TOK_ROWS - 1) / SW_TOK_ROWS;  // 1 or 2
      // A rows of this CTA: 128 (normal tile) or nt / 2 (swapped; a multiple of 8).
      const int a_rows = t.nt ? t.nt / 2 : BM;
      const uint32_t a_bytes =
          gather ? a_rows * BK * 2 : (t.nt ? tok_boxes * SW_TOK_ROWS * BK * 2 : A_BYTES);
      const uint32_t tx = 2 * (B_HALF + a_bytes);
      // Gathered rows of this lane: source rows of the tile's rows past the expert's end
      // are replaced by a valid row (their outputs are never stored).
      int g0 = 0, g1 = 0, g2 = 0, g3 = 0;
      const bool g_issue = gather && 4 * lane < a_rows;
      if (g_issue) {
        const int end = t.r0 + t.rows;
        const int rb = row0 + 4 * lane;
        g0 = rb + 0 < end ? __ldg(p.a_src + rb + 0) / p.a_k : 0;
        g1 = rb + 1 < end ? __ldg(p.a_src + rb + 1) / p.a_k : 0;
        g2 = rb + 2 < end ? __ldg(p.a_src + rb + 2) / p.a_k : 0;
        g3 = rb + 3 < end ? __ldg(p.a_src + rb + 3) / p.a_k : 0;
      }
      bool ok = true;
      for (int kb = 0; kb < nk; ++kb) {
        if (lane == 0 && !mbar_wait(&empty[stage], phase ^ 1)) {
          atomicExch(p.err, kErrTimeoutProducer);
          *abort_flag = 1;
          ok = false;
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
        const uint32_t full_leader = mapa_shared(smem_u32(&full[stage]), 0);
        const int kc = kb * BK;
        uint8_t* a_dst = sA + stage * A_BYTES;
        uint8_t* b_dst = sB + stage * B_HALF;
        if (lane == 0) {
          if (leader) mbar_arrive_expect_tx(&full[stage], tx);
          if (!t.nt) {
            if (!gather) tma_load_2d_pair(a_dst, &map_a, full_leader, kc, row0);
            tma_load_4d_pair(b_dst, bmap, full_leader, kc, bg, brow, e);
          } else {
            if (!gather)
              for (int j = 0; j < tok_boxes; ++j)
                tma_load_2d_pair(a_dst + j * SW_TOK_ROWS * BK * 2, &map_a_sw, full_leader, kc,
                                 row0 + j * SW_TOK_ROWS);
            if (p.gated) {
              tma_load_4d_pair(b_dst, &map_b1_sw, full_leader, kc, p.b1_g, sw_col + p.b1_noff, e);
              tma_load_4d_pair(b_dst + SW_HALF * BK * 2, &map_b3_sw, full_leader, kc, p.b3_g,
                               sw_col + p.b3_noff, e);
            } else {
              tma_load_4d_pair(b_dst, bmap, full_leader, kc, bg, brow, e);
            }
          }
        }
        if (g_issue)
          tma_gather4_pair(a_dst + lane * 4 * BK * 2, &map_a, full_leader, kc, g0, g1, g2, g3);
        if (++stage == P_STAGES) { stage = 0; phase ^= 1; }
      }
      // After a timeout the next claim publishes -1 (abort_flag), so the consumers stop.
      if (lane == 0 && ok) trace(p, kTrProdDone, L);
    }
  } else if (warp == 1) {
    // ------------------------------------------------- MMA issuer (leader CTA only)
    if (lane == 0 && leader) {
      constexpr uint32_t kFmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
      const uint32_t idesc = idesc_f16(kFmt, P_BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      for (int i = 0;; ++i) {
        int L;
        if (*abort_flag || !tq_take(i, s_tq, tq_full, tq_empty, true, L)) {
          atomicExch(p.err, kErrTimeoutMma);
          *abort_flag = 1;
          break;
        }
        if (L < 0) break;
        const int acc = i & 1;
        const uint32_t acc_phase = (i >> 1) & 1;
        const PairTile t = pair_tile(L, s_tiles, s_offs, p);
        const uint32_t id = t.nt ? idesc_f16(kFmt, P_BM, t.nt) : idesc;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1)) {
          atomicExch(p.err, kErrTimeoutMma);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        trace(p, kTrMmaStart, L);
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
          if (kb == 0) trace(p, kTrMmaFirst, L);
          const uint32_t x_addr = smem_u32(sA + stage * A_BYTES);
          const uint32_t w_addr = smem_u32(sB + stage * B_HALF);
          const uint32_t a_addr = t.nt ? w_addr : x_addr;
          const uint32_t b_addr = t.nt ? x_addr : w_addr;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            tc_mma_f16_pair(d_tmem, smem_desc_k_sw128(a_addr + kk * 32),
                            smem_desc_k_sw128(b_addr + kk * 32), id,
                            (kb | kk) != 0 ? 1u : 0u);
          }
          tc_commit_pair(&empty[stage], 0x3);
          if (++stage == P_STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        tc_commit_pair(&tfull[acc], 0x3);
        trace(p, kTrMmaDone, L);
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
    uint32_t xuse = 0;
    for (int i = 0;; ++i) {
      int L = -1, ok = 1;
      if (lane == 0) {
        ok = !*abort_flag && tq_take(i, s_tq, tq_full, tq_empty, leader, L);
        if (!ok) {
          atomicExch(p.err, kErrTimeoutEpilogue);
          *abort_flag = 1;
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      L = __shfl_sync(0xffffffffu, L, 0);
      if (!ok || L < 0) break;
      const int acc = i & 1;
      const uint32_t acc_phase = (i >> 1) & 1;
      if (!mbar_wait(&tfull[acc], acc_phase)) {
        atomicExch(p.err, kErrTimeoutEpilogue);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      if (warp == 2 && lane == 0) trace(p, kTrEpiStart, L);
      const PairTile t = pair_tile(L, s_tiles, s_offs, p);
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
      if (t.nt) {
        if (!epilogue_swapped<T>(p, t, taddr, static_cast<int>(rank), q, lane, warp < 6 ? 0 : 1,
                                 xch, xuse)) {
          atomicExch(p.err, kErrTimeoutEpilogue);
          *abort_flag = 1;
          break;
        }
      } else {
        const int row = t.r0 + r_in_tile;
        const bool valid = row < t.r0 + t.rows;
        epilogue_rows<T>(p, taddr, row, valid, t.e, p.gated ? t.n * (BN / 2) : t.n * BN, ec0,
                         ec1, epi_stage + (warp - 2) * EPI_STAGE_BYTES, lane);
      }
      tc_fence_before();
      __syncwarp();
      if (warp == 2 && lane == 0) trace(p, kTrEpiDone, L);
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), 0));
      if (p.comb_cnt != nullptr && !t.nt)
        combine_rows<T>(p, t.r0 + r_in_tile, t.r0 + r_in_tile < t.r0 + t.rows, t.n * BN, ec0,
                        ec1, lane);
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
// Packed ring depth: 6, or 5 for int8 so the epilogue staging still fits in 227 KB.
template <int BITS> constexpr int qp_stages() { return BITS == 8 ? 5 : 6; }
constexpr int Q_THREADS = 608;   // warps 0 A TMA, 1 MMA, 2..9 epilogue, 10..17 converters, 18 P TMA
constexpr int CONV_WARPS = 8;
constexpr int kConvGroups = 4;   // converter groups working on different k-blocks
constexpr int Q_PWARP = 18;
template <int BITS> constexpr int q_packed_bytes() { return BM * BK * BITS / 8; }
template <int BITS> constexpr int q_smem_bytes() {
  return 1024 + QA * A_BYTES + QB * B_HALF + qp_stages<BITS>() * q_packed_bytes<BITS>() +
         EPI_WARPS * 2048 /*epilogue staging*/ + 64 * 8 + 2 * (kMaxExperts + 1) * 4;
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// 8 codes (one 16-byte output chunk, natural order) -> fp16: (q - zp) * s (QEPI 0),
// q - zp (QEPI 1, scale applied in the epilogue) or the biased code 1024 + q (QEPI 2).
// w: the 8 codes (int8: both words; int4: w.x only).
template <int BITS, int QEPI>
__device__ __forceinline__ uint4 convert8(uint2 w, __half2 s2) {
  uint4 o;
  uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
  auto fin = [&](uint32_t biased, __half2 zp) -> uint32_t {
    if (QEPI == 2) return biased;
    const __half2 d = __hsub2(u2h(biased), zp);
    return h2u(QEPI == 1 ? d : __hmul2(d, s2));
  };
  if (BITS == 8) {
    const __half2 zp = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
    ow[0] = fin(__byte_perm(w.x, 0x64646464u, 0x4140u), zp);
    ow[1] = fin(__byte_perm(w.x, 0x64646464u, 0x4342u), zp);
    ow[2] = fin(__byte_perm(w.y, 0x64646464u, 0x4140u), zp);
    ow[3] = fin(__byte_perm(w.y, 0x64646464u, 0x4342u), zp);
  } else {
    const __half2 zp = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t b = (w.x >> (8 * i)) & 0xFFu;
      ow[i] = fin((b & 0xFu) | ((b & 0xF0u) << 12) | 0x64006400u, zp);
    }
  }
  return o;
}

template <int BITS, int QEPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Q_THREADS, 1)
tc_pair_qgemm_kernel(const __grid_constant__ CUtensorMap map_a,
                     const __grid_constant__ CUtensorMap map_q1,
                     const __grid_constant__ CUtensorMap map_q3,
                     const __grid_constant__ CUtensorMap map_a_sw, const TcParams p) {
  pdl_wait();  // launched dependent (launch_dependent): predecessors' data after this
  pdl_launch_dependents();
  constexpr int PB = q_packed_bytes<BITS>();
  constexpr int ROW_BYTES = BK * BITS / 8;  // packed bytes of one B row per k-block
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + QA * A_BYTES;
  uint8_t* sP = sB + QB * B_HALF;
  constexpr int QP = qp_stages<BITS>();
  uint8_t* epi_stage = sP + QP * PB;  // [EPI_WARPS][32 rows x 64 B]
  uint64_t* bars = reinterpret_cast<uint64_t*>(epi_stage + EPI_WARPS * EPI_STAGE_BYTES);
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
        // A swapped tail tile (ungated pass, <= swap_max rows) loads only its rows: nt / 2
        // per CTA in boxes of SW_TOK_ROWS (the weights then act as the MMA's M side).
        const PairTile t = pair_tile(L, s_tiles, s_offs, p);
        const int row0 = t.nt ? t.r0 + static_cast<int>(rank) * (t.nt / 2)
                              : t.r0 + static_cast<int>(rank) * BM;
        const int tok_boxes = (t.nt / 2 + SW_TOK_ROWS - 1) / SW_TOK_ROWS;
        const uint32_t a_tx = t.nt ? 2u * tok_boxes * SW_TOK_ROWS * BK * 2 : 2u * A_BYTES;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&emptyA[stage], phase ^ 1)) {
            atomicExch(p.err, kErrTimeoutProducer);
            *abort_flag = 1;
            break;
          }
          const uint32_t full_leader = mapa_shared(smem_u32(&fullA[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&fullA[stage], a_tx);
          if (t.nt) {
            for (int j = 0; j < tok_boxes; ++j)
              tma_load_2d_pair(sA + stage * A_BYTES + j * SW_TOK_ROWS * BK * 2, &map_a_sw,
                               full_leader, kb * BK, row0 + j * SW_TOK_ROWS);
          } else {
            tma_load_2d_pair(sA + stage * A_BYTES, &map_a, full_leader, kb * BK, row0);
          }
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
        const PairTile t = pair_tile(L, s_tiles, s_offs, p);
        const uint32_t id = t.nt ? idesc_f16(0u, P_BM, t.nt) : idesc;
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&fullA[sa], pa) || !mbar_wait(&cdone[sb], pb)) {
            atomicExch(p.err, kErrTimeoutMma);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t x_addr = smem_u32(sA + sa * A_BYTES);
          const uint32_t w_addr = smem_u32(sB + sb * B_HALF);
          const uint32_t a_addr = t.nt ? w_addr : x_addr;
          const uint32_t b_addr = t.nt ? x_addr : w_addr;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            tc_mma_f16_pair(d_tmem, smem_desc_k_sw128(a_addr + kk * 32),
                            smem_desc_k_sw128(b_addr + kk * 32), id,
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
          // One 16-byte load per swizzled chunk of the packed row (16 int8 or 32 int4
          // codes; the eight rows of a load phase hit eight distinct 16-byte bank groups),
          // then 8 codes per 16-byte store of the B tile.
          constexpr int kPerLoad = 16 / BITS;  // chunks of 8 codes per 16-byte load
#pragma unroll
          for (int m = 0; m < 8 / kPerLoad; ++m) {
            const int phys = BITS == 8 ? (m ^ ((r >> 1) & 3)) : (m ^ ((r >> 2) & 1));
            const uint4 w16 = *reinterpret_cast<const uint4*>(prow + phys * 16);
            const uint32_t ww[4] = {w16.x, w16.y, w16.z, w16.w};
#pragma unroll
            for (int u = 0; u < kPerLoad; ++u) {
              const int c = m * kPerLoad + u;  // chunk of 8 codes
              const uint2 w = BITS == 8 ? make_uint2(ww[2 * u], ww[2 * u + 1])
                                        : make_uint2(ww[u], 0u);
              const __half2 s2 =
                  p.qblock ? __half2half2(srs[j][min(kb * BK + 8 * c, p.K - 1) / p.qblock])
                           : row_scale[j];
              const uint4 o = convert8<BITS, QEPI>(w, s2);
              *reinterpret_cast<uint4*>(brow_s + ((c ^ (r & 7)) * 16)) = o;
            }
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
    const Exchange no_xch{nullptr, nullptr, nullptr};
    uint32_t xuse = 0;
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
      const PairTile t = pair_tile(L, s_tiles, s_offs, p);
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
      if (t.nt) {  // ungated passes only: the gate/linear exchange is never used
        if (!epilogue_swapped<__half>(p, t, taddr, static_cast<int>(rank), q, lane,
                                      warp < 6 ? 0 : 1, no_xch, xuse)) {
          atomicExch(p.err, kErrTimeoutEpilogue);
          *abort_flag = 1;
          break;
        }
      } else {
        const int row = t.r0 + r_in_tile;
        const bool valid = row < t.r0 + t.rows;
        epilogue_rows<__half>(p, taddr, row, valid, t.e, p.gated ? t.n * (BN / 2) : t.n * BN,
                              ec0, ec1, epi_stage + (warp - 2) * EPI_STAGE_BYTES, lane);
      }
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

// A: [rows, K] row-major, box box_rows x 64 columns.
bool make_map_a(CUtensorMap* m, int dt, const void* ptr, int64_t rows, int K,
                int box_rows = BM) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
  cuuint32_t box[2] = {BK, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t es[2] = {1, 1};
  return enc(m, tma_dtype(dt), 2, const_cast<void*>(ptr), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

// B: weights of all experts viewed as [E][Nrows/G][G][K], box 1 x box_rows x 1 x 64.
bool make_map_b(CUtensorMap* m, int dt, const GemmOperandB& b, int K, int E,
                int box_rows = BN / 2) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  const cuuint64_t rows_g = static_cast<cuuint64_t>(b.n_rows / b.G);
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(b.G), rows_g,
                        static_cast<cuuint64_t>(E)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(K) * 2,
                           static_cast<cuuint64_t>(K) * 2 * b.G,
                           static_cast<cuuint64_t>(K) * 2 * b.n_rows};
  cuuint32_t box[4] = {BK, 1, static_cast<cuuint32_t>(box_rows), 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  return enc(m, tma_dtype(dt), 4, const_cast<void*>(b.ptr), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

// Appends CTA 0's trace of the launch just enqueued to `path` (diagnostics only:
// synchronises the stream).  Lines: launch, K, event, tile, ns since the first entry.
void dump_trace(const char* path, int K, cudaStream_t s) {
  unsigned n = 0;
  if (cudaStreamSynchronize(s) != cudaSuccess ||
      cudaMemcpyFromSymbol(&n, g_trace_n, sizeof(n)) != cudaSuccess)
    return;
  n = std::min(n, kTraceCap);
  std::vector<unsigned long long> buf(2 * static_cast<size_t>(n));
  if (n == 0 || cudaMemcpyFromSymbol(buf.data(), g_tile_trace, buf.size() * 8) != cudaSuccess)
    return;
  unsigned long long t0 = ~0ull;
  for (unsigned i = 0; i < n; ++i) t0 = std::min(t0, buf[2 * i]);
  FILE* f = std::fopen(path, "a");
  if (f == nullptr) return;
  static int launch = 0;
  for (unsigned i = 0; i < n; ++i)
    std::fprintf(f, "%d,%d,%u,%u,%llu\n", launch, K, static_cast<unsigned>(buf[2 * i + 1] >> 32),
                 static_cast<unsigned>(buf[2 * i + 1] & 0xffffffffu), buf[2 * i] - t0);
  std::fclose(f);
  ++launch;
}

template <typename T>
cudaError_t launch_t(const GemmArgs& g, int num_sms, bool pair, cudaStream_t s) {
  CUtensorMap ma, mb1, mb3;
  // Gathered A (pair kernel only): the map covers the un-permuted rows with a one-row box.
  const bool gather = pair && g.gather_src != nullptr;
  if (gather) {
    if (!make_map_a(&ma, g.dtype, g.gather_x, g.gather_x_rows, g.K, 1)) return cudaErrorInvalidValue;
  } else if (!make_map_a(&ma, g.dtype, g.a, g.rows, g.K)) {
    return cudaErrorInvalidValue;
  }
  if (!make_map_b(&mb1, g.dtype, g.b1, g.K, g.E)) return cudaErrorInvalidValue;
  if (g.gated) {
    if (!make_map_b(&mb3, g.dtype, g.b3, g.K, g.E)) return cudaErrorInvalidValue;
  } else {
    mb3 = mb1;
  }
  TcParams p{};
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
  p.swap_max = pair ? std::max(0, std::min(g.swap_max, kPairSwapLimit)) / 16 * 16 : 0;
  p.tile_counter = pair ? g.tile_counter : nullptr;
  p.seg_start = g.seg_start;
  p.seg_dst = g.seg_dst;
  p.nseg = g.nseg;
  p.remap_world = g.remap_world;
  for (int i = 0; i < kMaxEpRanks; ++i) p.out_peers[i] = g.out_peers[i];
  // Weights holding exact integer codes with one fp16 scale per output row (qepi 1): the
  // epilogues scale the fp32 sums.  Biased codes (qepi 2) exist only in the packed kernel.
  if (g.qepi == 2 || (g.qepi == 1 && (g.dtype != kDtF16 || g.b1.scales == nullptr ||
                                      (g.gated && g.b3.scales == nullptr))))
    return cudaErrorInvalidValue;
  p.qepi = g.qepi;
  if (g.qepi) {
    p.scales1 = static_cast<const __half*>(g.b1.scales);
    p.scales3 = static_cast<const __half*>(g.gated ? g.b3.scales : g.b1.scales);
    p.b1_G = g.b1.G;
    p.b3_G = g.gated ? g.b3.G : 1;
    p.b1_rows = g.b1.n_rows;
    p.b3_rows = g.gated ? g.b3.n_rows : g.b1.n_rows;
  }
  if (g.comb_cnt != nullptr && (g.gated || g.seg_start != nullptr || g.N % 8 != 0))
    return cudaErrorInvalidValue;
  p.comb_cnt = g.comb_cnt;
  p.comb_src = g.comb_src;
  p.comb_pos = g.comb_pos;
  p.comb_w = g.comb_w;
  p.comb_out = g.comb_out;
  p.comb_k = g.comb_k;
  p.a_src = gather ? g.gather_src : nullptr;
  p.a_k = gather ? g.gather_k : 1;
  const char* trace_path = pair ? std::getenv("MOE_B200_GEMM_TRACE") : nullptr;
  p.trace = trace_path != nullptr ? 1 : 0;



  if (p.trace) {
    const unsigned zero = 0;
    cudaMemcpyToSymbolAsync(g_trace_n, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, s);
  }
  CUtensorMap ma_sw = ma, mb1_sw = mb1, mb3_sw = mb3;
  if (p.swap_max > 0) {
    if (!gather && !make_map_a(&ma_sw, g.dtype, g.a, g.rows, g.K, SW_TOK_ROWS))
      return cudaErrorInvalidValue;
    if (g.gated) {
      if (!make_map_b(&mb1_sw, g.dtype, g.b1, g.K, g.E, SW_HALF) ||
          !make_map_b(&mb3_sw, g.dtype, g.b3, g.K, g.E, SW_HALF))
        return cudaErrorInvalidValue;
    }
  }
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
    cudaError_t st = launch_dependent(pdl_layer_enabled(), tc_pair_grouped_gemm_kernel<T>,
                                      dim3(static_cast<unsigned>(2 * pairs)), dim3(THREADS),
                                      P_SMEM_BYTES, s, ma, mb1, mb3, ma_sw, mb1_sw, mb3_sw, p);
    if (st != cudaSuccess) return st;
    if (p.trace) dump_trace(trace_path, g.K, s);
  } else {
    const int grid = static_cast<int>(std::min<int64_t>(ub, num_sms));
    cudaError_t st = launch_dependent(pdl_layer_enabled(), tc_grouped_gemm_kernel<T>, dim3(grid), dim3(THREADS),
                                      SMEM_BYTES, s, ma, mb1, mb3, p);
    if (st != cudaSuccess) return st;
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

template <int BITS, int QEPI>
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
  p.qepi = QEPI;
  p.qbias = 1024.0f + static_cast<float>(1 << (BITS - 1));
  p.rowsum = g.rowsum;
  // Swapped tail tiles in the ungated pass (fc2): the last m-tile of an expert with at most
  // swap_max rows runs with the converted weights as M and its rows as N.
  p.swap_max = g.gated ? 0 : std::max(0, std::min(g.swap_max, kPairSwapLimit)) / 16 * 16;
  CUtensorMap ma_sw = ma;
  if (p.swap_max > 0 && !make_map_a(&ma_sw, g.dtype, g.a, g.rows, g.K, SW_TOK_ROWS))
    return cudaErrorInvalidValue;
  p.seg_start = g.seg_start;
  p.seg_dst = g.seg_dst;
  p.nseg = g.nseg;
  p.remap_world = g.remap_world;
  for (int i = 0; i < kMaxEpRanks; ++i) p.out_peers[i] = g.out_peers[i];
  static bool attr_set = false;  // idempotent; a race between first callers is benign
  if (!attr_set) {
    cudaError_t st = cudaFuncSetAttribute(tc_pair_qgemm_kernel<BITS, QEPI>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          q_smem_bytes<BITS>());
    if (st != cudaSuccess) return st;
    attr_set = true;
  }
  const int64_t ub = ((g.rows + P_BM - 1) / P_BM + g.E) * p.n_tiles;
  const int64_t pairs = std::min<int64_t>(ub, num_sms / 2);
  return launch_dependent(pdl_layer_enabled(), tc_pair_qgemm_kernel<BITS, QEPI>, dim3(static_cast<unsigned>(2 * pairs)),
                          dim3(Q_THREADS), q_smem_bytes<BITS>(), s, ma, mq1, mq3, ma_sw, p);
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
  // Epilogue-side scaling needs one scale per stored row (block_size 0); the biased codes
  // also need the A row sums.
  const int mode = g.qblock != 0 ? 0 : (g.qepi == 2 && g.rowsum == nullptr ? 1 : g.qepi);
  if (g.qbits == 4) {
    if (mode == 2) return launch_q<4, 2>(g, num_sms, s);
    if (mode == 1) return launch_q<4, 1>(g, num_sms, s);
    return launch_q<4, 0>(g, num_sms, s);
  }
  if (mode == 2) return launch_q<8, 2>(g, num_sms, s);
  if (mode == 1) return launch_q<8, 1>(g, num_sms, s);
  return launch_q<8, 0>(g, num_sms, s);
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

namespace {
// mode 0: choose (CTA pairs when experts average >= 256 rows), 1: single CTA, 2: pairs.
bool use_pair(const GemmArgs& g, int mode) {
  return mode == 2 || (mode == 0 && g.rows >= 256 * static_cast<int64_t>(g.E));
}
}  // namespace

bool tc_pair_gathers(const GemmArgs& g, int mode) {
  if (g.gather_src == nullptr || g.gather_x == nullptr || g.gather_x_rows < 1 || g.gather_k < 1)
    return false;
  if ((reinterpret_cast<uintptr_t>(g.gather_x) & 15) != 0) return false;
  return tc_supported(g) && use_pair(g, mode);
}

cudaError_t launch_gemm_tc(const GemmArgs& g, int num_sms, int mode, cudaStream_t s) {
  if (g.rows == 0 || g.N == 0) return cudaSuccess;
  // A gathered A needs the pair kernel (callers gather into g.a otherwise).
  if (g.gather_src != nullptr && !tc_pair_gathers(g, mode)) return cudaErrorInvalidValue;
  const bool pair = use_pair(g, mode);
  if (g.dtype == kDtF16) return launch_t<__half>(g, num_sms, pair, s);
  if (g.dtype == kDtBF16) return launch_t<__nv_bfloat16>(g, num_sms, pair, s);
  return cudaErrorInvalidValue;
}

}  // namespace moe
