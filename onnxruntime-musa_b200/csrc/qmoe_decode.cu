// QMoE decode path: weight-streaming grouped GEMM for small routed-row counts.
//
// At decode sizes (T*k routed rows in the tens) a QMoE layer is bound by reading
// the packed weights of the touched experts from HBM.  This kernel streams them once:
// each warp owns 16 output rows of one expert (16 gate + 16 linear rows when gated),
// loads their packed int4/int8 codes for a 128-wide K chunk with 16-byte coalesced
// loads (the next chunk is prefetched into a second register set), dequantises in
// registers ((q - zero_point) * scale in half2 arithmetic, exact before the scale) and
// feeds the codes straight into mma.sync m16n8k16 as the A operand, with the expert's
// routed token rows as the B operand (swap-AB: D[weight row, token]).  Experts with no
// routed rows launch CTAs that exit immediately, so untouched experts cost no traffic.
//
// K permutation: within a 128-wide chunk, thread t (of the 4 sharing a row) holds the
// 32 consecutive codes [32t, 32t+32).  MMA step j (0..7) uses, for that thread, codes
// 32t+4j .. 32t+4j+3 in the fragment slots {2t, 2t+1, 2t+8, 2t+9}; the B fragment is
// gathered with the same mapping (one 8-byte load of 4 consecutive activations), so the
// products are summed over exactly the same k pairs as an in-order dot product.
//
// fc2 (a long K = inter_size) is split over K across CTAs; each split writes fp32
// partial sums [split][row][col] and the combine kernel adds splits in fixed order,
// so the result is deterministic.
#include "qmoe_decode.h"

namespace moe {

namespace {

constexpr int QD_WARPS = 4;
constexpr int QD_CHUNK = 128;

__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                              uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// Two int4 codes of one byte -> half2 (q_lo - 8, q_hi - 8) * s.  1024 + q is built by
// placing q in the mantissa of 1024.0h (0x6400); the subtraction is exact.
__device__ __forceinline__ uint32_t deq4(uint32_t byte, __half2 s2) {
  const uint32_t u = (byte & 0xFu) | ((byte & 0xF0u) << 12) | 0x64006400u;
  const __half2 v = __hsub2(bits_h2(u), __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408)));
  return h2_bits(__hmul2(v, s2));
}
// Bytes (b0, b1) of a word selected by `sel` -> half2 (b0 - 128, b1 - 128) * s.
__device__ __forceinline__ uint32_t deq8(uint32_t word, uint32_t sel, __half2 s2) {
  const uint32_t u = __byte_perm(word, 0x64646464u, sel);
  const __half2 v = __hsub2(bits_h2(u), __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480)));
  return h2_bits(__hmul2(v, s2));
}

// Packed codes of one weight row for one chunk: 64 bytes (int4) or 128 bytes (int8),
// of which this thread holds 16 or 32.
template <int BITS> struct Codes { uint4 v[BITS / 4]; };

template <int BITS>
__device__ __forceinline__ void load_codes(Codes<BITS>& c, const uint8_t* row, int chunk, int t) {
  const uint4* p = reinterpret_cast<const uint4*>(row + static_cast<int64_t>(chunk) * (QD_CHUNK * BITS / 8) +
                                                  t * (32 * BITS / 8));
#pragma unroll
  for (int i = 0; i < BITS / 4; ++i) c.v[i] = __ldg(p + i);
}

// A-fragment registers (slots 2t..: codes 32t+4j .. 32t+4j+3) of step j.
template <int BITS>
__device__ __forceinline__ void frag(const Codes<BITS>& c, int j, __half2 s2, uint32_t& lo,
                                     uint32_t& hi) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(c.v);
  if (BITS == 4) {
    const uint32_t word = w[j >> 1];                 // bytes 2j, 2j+1 live in word j/2
    const uint32_t sh = (j & 1) * 16;
    lo = deq4((word >> sh) & 0xFFu, s2);
    hi = deq4((word >> (sh + 8)) & 0xFFu, s2);
  } else {
    const uint32_t word = w[j];                      // bytes 4j .. 4j+3
    lo = deq8(word, 0x4140u, s2);
    hi = deq8(word, 0x4342u, s2);
  }
}

struct RowPtrs {
  const uint8_t* r0;   // row n0+g
  const uint8_t* r8;   // row n0+g+8
  const __half* s0;    // scales of those rows
  const __half* s8;
};

__device__ __forceinline__ RowPtrs row_ptrs(const QOperand& b, int e, int n, int N, int K, int bits,
                                            int nb) {
  const int na = min(n, N - 1), nb8 = min(n + 8, N - 1);
  const int64_t row_bytes = static_cast<int64_t>(K) * bits / 8;
  const int64_t sr0 = static_cast<int64_t>(e) * b.n_rows + static_cast<int64_t>(na + b.n_off) * b.G + b.g;
  const int64_t sr8 = static_cast<int64_t>(e) * b.n_rows + static_cast<int64_t>(nb8 + b.n_off) * b.G + b.g;
  RowPtrs r;
  r.r0 = b.q + sr0 * row_bytes;
  r.r8 = b.q + sr8 * row_bytes;
  r.s0 = b.scales + sr0 * nb;
  r.s8 = b.scales + sr8 * nb;
  return r;
}

template <int BITS, int NG, bool GATED>
__device__ __forceinline__ void run_pass(const QDecodeArgs& a, int e, int row_begin, int cnt,
                                         int tok0, int n0, int c_begin, int c_end, int split) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int nb = a.block_size ? (a.K + a.block_size - 1) / a.block_size : 1;
  constexpr int NT = GATED ? 2 : 1;
  RowPtrs rp[NT];
  rp[0] = row_ptrs(a.b1, e, n0 + g, a.N, a.K, BITS, nb);
  if (GATED) rp[NT - 1] = row_ptrs(a.b3, e, n0 + g, a.N, a.K, BITS, nb);

  float acc[NT][NG][4];
#pragma unroll
  for (int x = 0; x < NT; ++x)
#pragma unroll
    for (int y = 0; y < NG; ++y)
#pragma unroll
      for (int z = 0; z < 4; ++z) acc[x][y][z] = 0.f;

  // Activation row pointers of this thread's B columns (token g of each group).
  const __half* xrow[NG];
  bool tok_ok[NG];
#pragma unroll
  for (int gi = 0; gi < NG; ++gi) {
    const int tok = tok0 + gi * 8 + g;
    tok_ok[gi] = tok < cnt;
    xrow[gi] = a.x + static_cast<int64_t>(row_begin + (tok_ok[gi] ? tok : 0)) * a.K + 32 * t;
  }

  Codes<BITS> cur[NT][2], nxt[NT][2];
#pragma unroll
  for (int x = 0; x < NT; ++x) {
    load_codes<BITS>(cur[x][0], rp[x].r0, c_begin, t);
    load_codes<BITS>(cur[x][1], rp[x].r8, c_begin, t);
  }
  for (int c = c_begin; c < c_end; ++c) {
    if (c + 1 < c_end) {
#pragma unroll
      for (int x = 0; x < NT; ++x) {
        load_codes<BITS>(nxt[x][0], rp[x].r0, c + 1, t);
        load_codes<BITS>(nxt[x][1], rp[x].r8, c + 1, t);
      }
    }
    const int sidx = a.block_size ? (c * QD_CHUNK + 32 * t) / a.block_size : 0;
    __half2 s0[NT], s8[NT];
#pragma unroll
    for (int x = 0; x < NT; ++x) {
      s0[x] = __half2half2(rp[x].s0[sidx]);
      s8[x] = __half2half2(rp[x].s8[sidx]);
    }
#pragma unroll
    for (int j = 0; j < QD_CHUNK / 16; ++j) {
      uint32_t af[NT][4];
#pragma unroll
      for (int x = 0; x < NT; ++x) {
        frag<BITS>(cur[x][0], j, s0[x], af[x][0], af[x][2]);
        frag<BITS>(cur[x][1], j, s8[x], af[x][1], af[x][3]);
      }
#pragma unroll
      for (int gi = 0; gi < NG; ++gi) {
        uint2 bv = make_uint2(0u, 0u);
        if (tok_ok[gi]) bv = __ldg(reinterpret_cast<const uint2*>(xrow[gi] + c * QD_CHUNK + 4 * j));
#pragma unroll
        for (int x = 0; x < NT; ++x) mma_f16_16816(acc[x][gi], af[x], bv.x, bv.y);
      }
    }
    if (c + 1 < c_end) {
#pragma unroll
      for (int x = 0; x < NT; ++x) {
        cur[x][0] = nxt[x][0];
        cur[x][1] = nxt[x][1];
      }
    }
  }

  // Epilogue: acc[x][gi] = {D(n0+g, 2t), D(n0+g, 2t+1), D(n0+g+8, 2t), D(n0+g+8, 2t+1)}
#pragma unroll
  for (int gi = 0; gi < NG; ++gi) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int n = n0 + g + ((q >> 1) ? 8 : 0);
      const int tok = tok0 + gi * 8 + 2 * t + (q & 1);
      if (n >= a.N || tok >= cnt) continue;
      const int64_t row = row_begin + tok;
      float v = acc[0][gi][q];
      if (a.out_partial != nullptr) {
        if (split == 0 && a.bias1 != nullptr)
          v += __half2float(static_cast<const __half*>(a.bias1)[e * a.bias_e_stride +
                                                                static_cast<int64_t>(n) * a.bias_stride]);
        a.out_partial[(static_cast<int64_t>(split) * a.rows + row) * a.ldo + n] = v;
      } else {
        if (a.bias1 != nullptr)
          v += __half2float(static_cast<const __half*>(a.bias1)[e * a.bias_e_stride +
                                                                static_cast<int64_t>(n) * a.bias_stride]);
        if (GATED) {
          float u = acc[NT - 1][gi][q];
          if (a.bias3 != nullptr)
            u += __half2float(static_cast<const __half*>(a.bias3)[e * a.bias_e_stride +
                                                                  static_cast<int64_t>(n) * a.bias_stride]);
          v = act_gated(a.ap, v, u);
        } else {
          v = act_single(a.ap.act, v);
        }
        a.out[row * a.ldo + n] = __float2half_rn(v);
      }
    }
  }
}

template <int BITS, bool GATED>
__global__ void __launch_bounds__(QD_WARPS * 32) qmoe_decode_kernel(const QDecodeArgs a) {
  const int e = blockIdx.y;
  const int row_begin = a.offsets[e];
  const int cnt = a.offsets[e + 1] - row_begin;
  if (cnt == 0) return;
  const int warp = threadIdx.x >> 5;
  const int n0 = (blockIdx.x * QD_WARPS + warp) * 16;
  if (n0 >= a.N) return;
  const int nchunks = a.K / QD_CHUNK;
  const int split = blockIdx.z;
  const int per = (nchunks + a.splits - 1) / a.splits;
  const int c_begin = split * per;
  const int c_end = min(nchunks, c_begin + per);
  if (c_begin >= c_end) {
    // An empty split still owns its partial-sum slice: write zeros (bias lives in split 0).
    if (a.out_partial != nullptr) {
      const int lane = threadIdx.x & 31;
      for (int i = lane; i < 16 * cnt; i += 32) {
        const int n = n0 + (i & 15), tok = i >> 4;
        if (n < a.N)
          a.out_partial[(static_cast<int64_t>(split) * a.rows + row_begin + tok) * a.ldo + n] = 0.f;
      }
    }
    return;
  }
  // Up to 32 routed rows per pass over the weights (4 groups of 8 MMA columns).
  for (int tok0 = 0; tok0 < cnt; tok0 += 32) {
    const int groups = min(4, (cnt - tok0 + 7) / 8);
    if (groups <= 1) run_pass<BITS, 1, GATED>(a, e, row_begin, cnt, tok0, n0, c_begin, c_end, split);
    else if (groups <= 2) run_pass<BITS, 2, GATED>(a, e, row_begin, cnt, tok0, n0, c_begin, c_end, split);
    else run_pass<BITS, 4, GATED>(a, e, row_begin, cnt, tok0, n0, c_begin, c_end, split);
  }
}

// out[t] = sum_j w[t,j] * sum_s partial[s][pos[t,j]] (fixed order), fp32 -> fp16.
__global__ void __launch_bounds__(256)
combine_partials_kernel(const float* __restrict__ part, int splits, int64_t rows,
                        const int32_t* __restrict__ pos, const float* __restrict__ w, int k,
                        int H, __half* __restrict__ out) {
  const int t = blockIdx.x;
  for (int c = threadIdx.x; c < H; c += blockDim.x) {
    float acc = 0.f;
    for (int j = 0; j < k; ++j) {
      const int64_t r = pos[static_cast<int64_t>(t) * k + j];
      float y = 0.f;
      for (int s = 0; s < splits; ++s) y += part[(static_cast<int64_t>(s) * rows + r) * H + c];
      acc += w[static_cast<int64_t>(t) * k + j] * y;
    }
    out[static_cast<int64_t>(t) * H + c] = __float2half_rn(acc);
  }
}

}  // namespace

bool qmoe_decode_supported(int dtype, int bits, int block_size, int64_t H, int64_t I) {
  if (dtype != kDtF16) return false;
  if (bits != 4 && bits != 8) return false;
  if (block_size != 0 && block_size < 32) return false;
  return H % QD_CHUNK == 0 && I % QD_CHUNK == 0;
}

cudaError_t launch_qmoe_decode(const QDecodeArgs& a, int max_experts_touched, cudaStream_t s) {
  const dim3 block(QD_WARPS * 32);
  const dim3 grid((a.N + QD_WARPS * 16 - 1) / (QD_WARPS * 16), a.E, a.splits);
  (void)max_experts_touched;
  if (a.bits == 4) {
    if (a.gated) qmoe_decode_kernel<4, true><<<grid, block, 0, s>>>(a);
    else qmoe_decode_kernel<4, false><<<grid, block, 0, s>>>(a);
  } else {
    if (a.gated) qmoe_decode_kernel<8, true><<<grid, block, 0, s>>>(a);
    else qmoe_decode_kernel<8, false><<<grid, block, 0, s>>>(a);
  }
  return cudaGetLastError();
}

cudaError_t launch_combine_partials(const float* part, int splits, int64_t rows, const int32_t* pos,
                                    const float* w, int T, int k, int H, void* out, cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  combine_partials_kernel<<<T, 256, 0, s>>>(part, splits, rows, pos, w, k, H,
                                            static_cast<__half*>(out));
  return cudaGetLastError();
}

}  // namespace moe
