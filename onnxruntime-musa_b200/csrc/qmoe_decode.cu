// QMoE decode path: weight-streaming grouped GEMM for small routed-row counts.
//
// At decode sizes (T*k routed rows in the tens) a QMoE layer is bound by reading the
// packed weights of the touched experts from HBM.  This kernel streams them once: each
// warp owns 16 output rows of one expert (16 gate + 16 linear rows when gated) and
// walks K in 128-wide chunks.  The codes reach shared memory through a warp-private
// cp.async ring (4 KB to 14 KB per warp in flight, enough bytes per SM to cover HBM
// latency), are converted to fp16 in registers and fed to mma.sync m16n8k16 as the A
// operand, with the expert's routed token rows as the B operand (swap-AB:
// D[weight row, token]).  Token rows are read in place from the layer input through the
// inverse permutation, so no gather pass runs.  Experts with no routed rows launch CTAs
// that exit at once: untouched experts cost no traffic.
//
// Scale modes (kScale):
//   kScaleRow    one scale per output row: the MMA runs on the integer codes (exact in
//                fp16) and the fp32 sum is scaled once at the end;
//   kScaleChunk  block scales covering whole 128-wide chunks (block_size >= 128): codes
//                exact, each chunk's fp32 partial sum is scaled and accumulated;
//   kScaleElem   smaller blocks: codes are scaled during the fp16 conversion.
//
// K permutation.  A dot product may take its k terms in any order as long as A and B
// agree.  Thread t (of the 4 sharing a row) handles the 32 consecutive codes
// [32t, 32t+32) of a chunk and places 4 of them per MMA step in the fragment slots
// {2t, 2t+1, 2t+8, 2t+9}; the B fragment is gathered with the same mapping:
//   * int8, and int4 with per-code conversion: step j takes codes 32t+4j .. 32t+4j+3 in
//     order (int4: (q - 8) exact, times the block scale in kScaleElem);
//   * int4 biased codes (the default for the exact modes): word m (codes 8m..8m+7) is split by one mask per half2 into
//     pairs (c_i, c_{i+4}) (steps 2m / 2m+1 take pairs (0,1) / (2,3), after one shift for
//     the second); the activations come pre-arranged in that order (launch_qdec_prep).
//     The masked words are used as they are: low nibbles read as 1024 + q and high
//     nibbles, masked in place, as 1024 + 16 q, whose activations are pre-scaled by 1/16;
//     the constant part, 1032 * (sum of even-slot x) + 1152 * (sum of odd-slot x/16) per
//     chunk and token (zero point 8 included), is subtracted from the chunk's sum.  This
//     removes all per-code arithmetic but one logic op per half2; the products are exact
//     in fp32 and the subtraction costs ~1e-3 absolute per chunk on sums of order 1e4.
//
// fc2 (long K = inter_size) is split over K across CTAs; each split writes fp32 partial
// sums [split][row][col] and the combine kernel adds splits in a fixed order, so the
// result is deterministic.
#include <algorithm>
#include <cstdlib>
#include "qmoe_decode.h"

namespace moe {

namespace {

constexpr int QD_WARPS = 4;
constexpr int QD_CHUNK = 128;
// Stages of the per-warp ring: 6 for int4 and 3 for int8 (the same bytes in flight), sized
// so four CTAs fit on one SM.
// Stages of the per-warp ring: 6 for int4 and 3 for int8 (the same bytes in flight), sized
// so four CTAs fit on one SM.  (Shallower rings at 5-6 CTAs per SM for the one-group
// passes measured slower: C3 T=1 0.0955 -> 0.1015 ms, C5 T=1 0.067 -> 0.074 ms.)
template <int BITS, int NGMAX> constexpr int qd_stages() { return BITS == 4 ? 6 : 3; }

enum ScaleMode { kScaleRow = 0, kScaleChunk = 1, kScaleElem = 2 };

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

// 1024 + q for a code q placed in the mantissa of 1024.0h (0x6400); subtracting
// 1024 + zero_point is exact.
__device__ __forceinline__ __half2 h2c(uint16_t bits) {
  return __halves2half2(__ushort_as_half(bits), __ushort_as_half(bits));
}
// Codes (lo nibble, hi nibble) of one byte -> (q_lo - 8, q_hi - 8) * s.
__device__ __forceinline__ uint32_t deq4_scaled(uint32_t byte, __half2 s2) {
  const uint32_t u = (byte & 0xFu) | ((byte & 0xF0u) << 12) | 0x64006400u;
  return h2_bits(__hmul2(__hsub2(bits_h2(u), h2c(0x6408)), s2));
}
// Codes (lo nibble, hi nibble) of one byte -> (q_lo - 8, q_hi - 8), exact in fp16.
__device__ __forceinline__ uint32_t deq4_exact(uint32_t byte) {
  const uint32_t u = (byte & 0xFu) | ((byte & 0xF0u) << 12) | 0x64006400u;
  return h2_bits(__hsub2(bits_h2(u), h2c(0x6408)));
}
// Biased codes of the low nibbles i, i+4 (1024 + q) and, masked in place, of the high
// nibbles i+1, i+5 (1024 + 16 q) of a word shifted right by 4i.
// One three-input logic op each, (shifted & mask) | bias, with the bias 0x64006400 held in
// a register (`bias`, see opaque_bias): with both constants as immediates the compiler
// emitted two logic ops per conversion (the instruction takes one immediate), which
// doubled the kernel's logic-op count.
__device__ __forceinline__ uint32_t raw4_lo(uint32_t shifted, uint32_t bias) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(shifted), "n"(0x000F000F), "r"(bias));
  return d;
}
__device__ __forceinline__ uint32_t raw4_hi(uint32_t shifted, uint32_t bias) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(shifted), "n"(0x00F000F0), "r"(bias));
  return d;
}
// 0x64006400 in a register the compiler cannot fold back into an immediate.
__device__ __forceinline__ uint32_t opaque_bias() {
  uint32_t b;
  asm volatile("mov.b32 %0, 0x64006400;" : "=r"(b));
  return b;
}
// Bytes of a word selected by `sel` -> (b - 128) exact, optionally scaled.
__device__ __forceinline__ uint32_t deq8(uint32_t word, uint32_t sel) {
  return h2_bits(__hsub2(bits_h2(__byte_perm(word, 0x64646464u, sel)), h2c(0x6480)));
}
__device__ __forceinline__ uint32_t deq8_scaled(uint32_t word, uint32_t sel, __half2 s2) {
  return h2_bits(__hmul2(bits_h2(deq8(word, sel)), s2));
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Stored row of output row n (clamped into range) of expert e.
__device__ __forceinline__ int64_t stored_row(const QOperand& b, int e, int n, int N) {
  return static_cast<int64_t>(e) * b.n_rows + static_cast<int64_t>(min(n, N - 1) + b.n_off) * b.G +
         b.g;
}

template <int BITS, int NG, bool GATED, int kScale, bool RAW4, int STAGES, bool PF>
__device__ __forceinline__ void run_pass(const QDecodeArgs& a, int e, int row_begin, int cnt,
                                         int tok0, int n0, int c_begin, int c_end, int split,
                                         uint8_t* ring) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int nb = a.block_size ? (a.K + a.block_size - 1) / a.block_size : 1;
  constexpr int NT = GATED ? 2 : 1;
  constexpr int ROW_CHUNK = QD_CHUNK * BITS / 8;  // bytes of one row per chunk
  constexpr int PPR = ROW_CHUNK / 16;              // 16-byte pieces per row chunk
  constexpr int STAGE = NT * 16 * ROW_CHUNK;       // bytes per stage of this warp
  constexpr int PER_LANE = NT * 16 * PPR / 32;     // pieces each lane copies per chunk
  const int64_t row_bytes = static_cast<int64_t>(a.K) * BITS / 8;

  // Sources of the cp.async pieces of this lane (fixed across chunks).
  const uint8_t* src[PER_LANE];
#pragma unroll
  for (int i = 0; i < PER_LANE; ++i) {
    const int p = lane + 32 * i;
    const int x = p / (16 * PPR);
    const int r = (p / PPR) % 16;
    const QOperand& b = (GATED && x == 1) ? a.b3 : a.b1;
    src[i] = b.q + stored_row(b, e, n0 + r, a.N) * row_bytes + (p % PPR) * 16;
  }
  auto issue = [&](int c, int stage) {
    uint8_t* dst = ring + stage * STAGE;
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i)
      cp_async16(dst + (lane + 32 * i) * 16, src[i] + static_cast<int64_t>(c) * ROW_CHUNK);
  };

  // Scale rows of this thread (rows n0+g and n0+g+8 of each tile).
  const __half* sc0[NT];
  const __half* sc8[NT];
#pragma unroll
  for (int x = 0; x < NT; ++x) {
    const QOperand& b = (GATED && x == 1) ? a.b3 : a.b1;
    sc0[x] = b.scales + stored_row(b, e, n0 + g, a.N) * nb;
    sc8[x] = b.scales + stored_row(b, e, n0 + g + 8, a.N) * nb;
  }

  float acc[NT][NG][4];
#pragma unroll
  for (int x = 0; x < NT; ++x)
#pragma unroll
    for (int y = 0; y < NG; ++y)
#pragma unroll
      for (int z = 0; z < 4; ++z) acc[x][y][z] = 0.f;

  // Activation rows of this thread's B columns (token g of each group).
  const __half* xrow[NG];
  bool tok_ok[NG];
#pragma unroll
  for (int gi = 0; gi < NG; ++gi) {
    const int tok = tok0 + gi * 8 + g;
    tok_ok[gi] = tok < cnt;
    const int64_t prow = row_begin + (tok_ok[gi] ? tok : 0);
    const int64_t xr = a.src_rows ? a.src_rows[prow] / a.k : prow;
    xrow[gi] = a.x + xr * a.K + 32 * t;
  }
  // Biased-code int4: offset terms of this thread's D columns (tokens 2t, 2t+1 of a group).
  static_assert(!RAW4 || (BITS == 4 && kScale != kScaleElem), "biased codes: int4, exact modes");
  constexpr bool kRaw4 = RAW4;
  [[maybe_unused]] const int nch = a.K / QD_CHUNK;
  const float* crow[NG][2];
  if constexpr (kRaw4) {
#pragma unroll
    for (int gi = 0; gi < NG; ++gi)
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int tok = min(tok0 + gi * 8 + 2 * t + u, cnt - 1);
        const int64_t prow = row_begin + tok;
        const int64_t xr = a.src_rows ? a.src_rows[prow] / a.k : prow;
        crow[gi][u] = a.xcorr + xr * nch;
      }
  }

  __syncwarp();
#pragma unroll
  for (int st = 0; st < STAGES - 1; ++st) {
    if (c_begin + st < c_end) issue(c_begin + st, st);
    cp_async_commit();
  }
  // Ring slots of the chunk consumed and of the chunk issued, and the block-scale index of
  // the chunk (kScaleChunk: a block spans cpb whole chunks), advanced without divisions.
  int stage = 0, stage_next = STAGES - 1;
  const int cpb = kScale == kScaleChunk ? a.block_size / QD_CHUNK : 1;
  int sblk = kScale == kScaleChunk ? c_begin / cpb : 0;
  int ssub = kScale == kScaleChunk ? c_begin - sblk * cpb : 0;
  // The next chunk's activations (and offset terms, and chunk scales) load while this chunk
  // computes: they come from L2, and a load issued just before its use would stall the warp
  // for a full L2 round trip every chunk.
  [[maybe_unused]] const uint32_t bias6400 = opaque_bias();
  // One-group passes of one-group kernels only (PF): wider passes, and the kernels that
  // also hold them, have no registers for a second buffer.
  constexpr bool kPf = PF && NG == 1;
  constexpr int M = QD_CHUNK / 32;
  // Two register buffers of prefetched values, used in turn by consecutive chunks (no
  // copies between them).
  uint4 xbuf[2][M][NG];
  float obuf[2][NG][2];
  float fbuf0[2][NT], fbuf8[2][NT];
  auto load_x = [&](int cc, uint4 (&xd)[M][NG], float (&od)[NG][2]) {
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int gi = 0; gi < NG; ++gi)
        xd[m][gi] = tok_ok[gi]
                        ? __ldg(reinterpret_cast<const uint4*>(xrow[gi] + cc * QD_CHUNK + 8 * m))
                        : make_uint4(0u, 0u, 0u, 0u);
    if constexpr (kRaw4) {
#pragma unroll
      for (int gi = 0; gi < NG; ++gi) {
        od[gi][0] = __ldg(crow[gi][0] + cc);
        od[gi][1] = __ldg(crow[gi][1] + cc);
      }
    }
  };
  auto load_scales = [&](int si, float (&f0d)[NT], float (&f8d)[NT]) {
    if constexpr (kScale == kScaleChunk) {
#pragma unroll
      for (int x = 0; x < NT; ++x) {
        f0d[x] = __half2float(sc0[x][si]);
        f8d[x] = __half2float(sc8[x][si]);
      }
    }
  };
  if (kPf && c_begin < c_end) {
    load_x(c_begin, xbuf[0], obuf[0]);
    load_scales(sblk, fbuf0[0], fbuf8[0]);
  }
  // One chunk: reads the buffer `cur` (prefetched, or loaded now in wider passes) and
  // prefetches the next chunk into `nxt`.
  auto chunk = [&](int c, uint4 (&xcur)[M][NG], float (&ocur)[NG][2], float (&fcur0)[NT],
                   float (&fcur8)[NT], uint4 (&xnxt)[M][NG], float (&onxt)[NG][2],
                   float (&fnxt0)[NT], float (&fnxt8)[NT]) {
    if (!kPf) {
      if constexpr (kRaw4) {
#pragma unroll
        for (int gi = 0; gi < NG; ++gi) {
          ocur[gi][0] = __ldg(crow[gi][0] + c);
          ocur[gi][1] = __ldg(crow[gi][1] + c);
        }
      }
      load_scales(sblk, fcur0, fcur8);
    }
    if (kScale == kScaleChunk && ++ssub == cpb) {
      ssub = 0;
      ++sblk;
    }
    if (kPf && c + 1 < c_end) {
      load_x(c + 1, xnxt, onxt);
      load_scales(sblk, fnxt0, fnxt8);
    }
    cp_async_wait<STAGES - 2>();
    __syncwarp();
    const uint8_t* sb = ring + stage * STAGE;
    uint4 code[NT][2][BITS / 4];  // [tile][row g / g+8][16-byte words]
#pragma unroll
    for (int x = 0; x < NT; ++x) {
      const uint4* r0 = reinterpret_cast<const uint4*>(sb + (x * 16 + g) * ROW_CHUNK + t * (ROW_CHUNK / 4));
      const uint4* r8 = reinterpret_cast<const uint4*>(sb + (x * 16 + g + 8) * ROW_CHUNK + t * (ROW_CHUNK / 4));
#pragma unroll
      for (int i = 0; i < BITS / 4; ++i) {
        code[x][0][i] = r0[i];
        code[x][1][i] = r8[i];
      }
    }
    __syncwarp();
    if (c + STAGES - 1 < c_end) issue(c + STAGES - 1, stage_next);
    cp_async_commit();
    stage_next = stage_next + 1 == STAGES ? 0 : stage_next + 1;
    stage = stage + 1 == STAGES ? 0 : stage + 1;

    __half2 s0[NT], s8[NT];
    if (kScale == kScaleElem) {
      const int sidx = (c * QD_CHUNK + 32 * t) / a.block_size;
#pragma unroll
      for (int x = 0; x < NT; ++x) {
        s0[x] = __half2half2(sc0[x][sidx]);
        s8[x] = __half2half2(sc8[x][sidx]);
      }
    }
    constexpr int PX = kScale == kScaleChunk ? NT : 1;
    constexpr int PG = kScale == kScaleChunk ? NG : 1;
    float part[PX][PG][4];
    if (kScale == kScaleChunk) {
#pragma unroll
      for (int x = 0; x < PX; ++x)
#pragma unroll
        for (int y = 0; y < PG; ++y)
#pragma unroll
          for (int z = 0; z < 4; ++z) part[x][y][z] = 0.f;
    }

    // Steps are taken in pairs (j = 2m, 2m+1) that share one 16-byte activation load
    // per token group: activations 32t+8m .. 32t+8m+7.
#pragma unroll
    for (int m = 0; m < QD_CHUNK / 32; ++m) {
      uint4 xv[NG];
#pragma unroll
      for (int gi = 0; gi < NG; ++gi)
        xv[gi] = kPf ? xcur[m][gi]
             : (tok_ok[gi] ? __ldg(reinterpret_cast<const uint4*>(xrow[gi] + c * QD_CHUNK + 8 * m))
                           : make_uint4(0u, 0u, 0u, 0u));
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int j = 2 * m + h;
        uint32_t af[NT][4];
#pragma unroll
        for (int x = 0; x < NT; ++x) {
#pragma unroll
          for (int r = 0; r < 2; ++r) {  // r=0: row g -> a0/a2, r=1: row g+8 -> a1/a3
            const uint32_t* w = reinterpret_cast<const uint32_t*>(code[x][r]);
            uint32_t lo, hi;
            if (kRaw4) {
              const uint32_t word = w[m] >> (h * 8);  // pairs (0,4),(1,5) or (2,6),(3,7)
              lo = raw4_lo(word, bias6400);
              hi = raw4_hi(word, bias6400);
            } else if (BITS == 4 && kScale == kScaleElem) {
              const uint32_t word = w[m] >> (h * 16);
              const __half2 s2 = r ? s8[x] : s0[x];
              lo = deq4_scaled(word & 0xFFu, s2);
              hi = deq4_scaled((word >> 8) & 0xFFu, s2);
            } else if (BITS == 4) {  // exact codes, scale applied to the fp32 sums
              const uint32_t word = w[m] >> (h * 16);
              lo = deq4_exact(word & 0xFFu);
              hi = deq4_exact((word >> 8) & 0xFFu);
            } else if (kScale == kScaleElem) {
              const __half2 s2 = r ? s8[x] : s0[x];
              lo = deq8_scaled(w[j], 0x4140u, s2);
              hi = deq8_scaled(w[j], 0x4342u, s2);
            } else {
              lo = deq8(w[j], 0x4140u);
              hi = deq8(w[j], 0x4342u);
            }
            af[x][r] = lo;
            af[x][r + 2] = hi;
          }
        }
#pragma unroll
        for (int gi = 0; gi < NG; ++gi) {
          uint32_t b0, b1;
          if (kRaw4) {
            // Pre-arranged: (x_i, x_{i+4}) then (x_{i+1}/16, x_{i+5}/16).
            b0 = h ? xv[gi].z : xv[gi].x;
            b1 = h ? xv[gi].w : xv[gi].y;
          } else {
            b0 = h ? xv[gi].z : xv[gi].x;  // activations 4j, 4j+1
            b1 = h ? xv[gi].w : xv[gi].y;  // activations 4j+2, 4j+3
          }
#pragma unroll
          for (int x = 0; x < NT; ++x) {
            if (kScale == kScaleChunk) mma_f16_16816(part[x < PX ? x : 0][gi < PG ? gi : 0], af[x], b0, b1);
            else mma_f16_16816(acc[x][gi], af[x], b0, b1);
          }
        }
      }
    }
    if constexpr (kRaw4) {
#pragma unroll
      for (int gi = 0; gi < NG; ++gi) {
        const float o0 = ocur[gi][0], o1 = ocur[gi][1];
#pragma unroll
        for (int x = 0; x < NT; ++x) {
          float* d = kScale == kScaleChunk ? part[x < PX ? x : 0][gi < PG ? gi : 0] : acc[x][gi];
          d[0] -= o0;
          d[1] -= o1;
          d[2] -= o0;
          d[3] -= o1;
        }
      }
    }
    if (kScale == kScaleChunk) {
#pragma unroll
      for (int x = 0; x < NT; ++x) {
        const float f0 = fcur0[x], f8 = fcur8[x];
#pragma unroll
        for (int gi = 0; gi < NG; ++gi) {
          const float* pp = part[x < PX ? x : 0][gi < PG ? gi : 0];
          acc[x][gi][0] = fmaf(f0, pp[0], acc[x][gi][0]);
          acc[x][gi][1] = fmaf(f0, pp[1], acc[x][gi][1]);
          acc[x][gi][2] = fmaf(f8, pp[2], acc[x][gi][2]);
          acc[x][gi][3] = fmaf(f8, pp[3], acc[x][gi][3]);
        }
      }
    }
    };
  if constexpr (kPf) {
    for (int c = c_begin; c < c_end; c += 2) {
      chunk(c, xbuf[0], obuf[0], fbuf0[0], fbuf8[0], xbuf[1], obuf[1], fbuf0[1], fbuf8[1]);
      if (c + 1 < c_end)
        chunk(c + 1, xbuf[1], obuf[1], fbuf0[1], fbuf8[1], xbuf[0], obuf[0], fbuf0[0], fbuf8[0]);
    }
  } else {
    for (int c = c_begin; c < c_end; ++c)
      chunk(c, xbuf[0], obuf[0], fbuf0[0], fbuf8[0], xbuf[0], obuf[0], fbuf0[0], fbuf8[0]);
  }
  cp_async_wait<0>();
  __syncwarp();
  if (kScale == kScaleRow) {
#pragma unroll
    for (int x = 0; x < NT; ++x) {
      const float f0 = __half2float(sc0[x][0]), f8 = __half2float(sc8[x][0]);
#pragma unroll
      for (int gi = 0; gi < NG; ++gi) {
        acc[x][gi][0] *= f0;
        acc[x][gi][1] *= f0;
        acc[x][gi][2] *= f8;
        acc[x][gi][3] *= f8;
      }
    }
  }

  // Epilogue: acc[x][gi] = {D(n0+g, 2t), D(n0+g, 2t+1), D(n0+g+8, 2t), D(n0+g+8, 2t+1)}
  const __half* b1p = static_cast<const __half*>(a.bias1);
  const __half* b3p = static_cast<const __half*>(a.bias3);
#pragma unroll
  for (int gi = 0; gi < NG; ++gi) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int n = n0 + g + ((q >> 1) ? 8 : 0);
      const int tok = tok0 + gi * 8 + 2 * t + (q & 1);
      if (n >= a.N || tok >= cnt) continue;
      const int64_t row = row_begin + tok;
      float v = acc[0][gi][q];
      const int64_t bi = e * a.bias_e_stride + static_cast<int64_t>(n) * a.bias_stride;
      if (a.out_partial != nullptr) {
        // Split-K partial sums; biases and the activation are applied by the reader.
        float* prow = a.out_partial + (static_cast<int64_t>(split) * a.rows + row) * a.ldo;
        prow[n] = v;
        if (GATED) prow[a.N + n] = acc[NT - 1][gi][q];
      } else {
        if (b1p != nullptr) v += __half2float(b1p[bi]);
        if (GATED) {
          float u = acc[NT - 1][gi][q];
          if (b3p != nullptr) u += __half2float(b3p[bi]);
          v = act_gated(a.ap, v, u);
        } else {
          v = act_single(a.ap.act, v);
        }
        a.out[row * a.ldo + n] = __float2half_rn(v);
      }
    }
  }
}

// One thread per group of 8 activations; the 16 threads of a 128-wide chunk sum the
// chunk's offset term with a fixed butterfly (deterministic).
__global__ void __launch_bounds__(256)
qdec_prep_kernel(const __half* __restrict__ x, int64_t rows, int K, __half* __restrict__ xp,
                 float* __restrict__ corr, int x_from_previous) {
  const int64_t groups = rows * (K / 8);
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  // Launched dependent.  x_from_previous: x is the previous kernel's output, so wait first;
  // else x predates the layer call (its routing kernel started after every earlier kernel
  // finished) and only the exit has to wait.
  if (x_from_previous) {
    pdl_wait();
    pdl_launch_dependents();
  }
  float part = 0.f;
  if (gid < groups) {
    const uint4 v = reinterpret_cast<const uint4*>(x)[gid];
    const __half2 q01 = bits_h2(v.x), q23 = bits_h2(v.y), q45 = bits_h2(v.z), q67 = bits_h2(v.w);
    const __half2 sixteenth = __float2half2_rn(0.0625f);
    const __half2 e04 = __lows2half2(q01, q45), e26 = __lows2half2(q23, q67);
    const __half2 o15 = __hmul2(__highs2half2(q01, q45), sixteenth);
    const __half2 o37 = __hmul2(__highs2half2(q23, q67), sixteenth);
    reinterpret_cast<uint4*>(xp)[gid] = make_uint4(h2_bits(e04), h2_bits(o15), h2_bits(e26),
                                                   h2_bits(o37));
    const float2 fe04 = __half22float2(e04), fe26 = __half22float2(e26);
    const float2 fo15 = __half22float2(o15), fo37 = __half22float2(o37);
    part = 1032.0f * ((fe04.x + fe04.y) + (fe26.x + fe26.y)) +
           1152.0f * ((fo15.x + fo15.y) + (fo37.x + fo37.y));
  }
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  if (gid < groups && (gid & 15) == 0) corr[gid >> 4] = part;
  if (!x_from_previous) {
    pdl_wait();
    pdl_launch_dependents();
  }
}

template <int BITS, bool GATED, int NGMAX>
constexpr int ring_bytes() { return qd_stages<BITS, NGMAX>() * (GATED ? 2 : 1) * 16 * QD_CHUNK * BITS / 8; }

// NGMAX: most groups of 8 routed rows one pass takes (1, 2 or 4; the host bounds it by the
// routed rows, so small calls compile only the narrow passes and keep their registers).
// The int4 gated 4-group pass runs 3 CTAs per SM with up to 168 registers instead of 4 CTAs
// with 128 and ~400 bytes of spills: 4% faster at C3 T=64 on B200; every other variant
// measured the same or faster at 4 CTAs per SM.
template <int BITS, bool GATED, int NGMAX>
constexpr int qd_min_blocks() {
  return (BITS == 4 && GATED && NGMAX == 4) ? 3 : 4;
}

template <int BITS, bool GATED, int kScale, bool RAW4, int NGMAX>
__global__ void __launch_bounds__(QD_WARPS * 32, (qd_min_blocks<BITS, GATED, NGMAX>()))
qmoe_decode_kernel(const QDecodeArgs a) {
  extern __shared__ __align__(128) uint8_t s_ring[];  // one ring per warp
  uint8_t* ring = s_ring + (threadIdx.x >> 5) * ring_bytes<BITS, GATED, NGMAX>();
  // Launched dependent: every input (offsets, activations) comes from earlier kernels.
  pdl_wait();
  pdl_launch_dependents();
  // Grid rows cover the experts that can hold rows (min(E, routed rows)): row j takes the
  // j-th expert with rows, found from the offsets.
  int e = blockIdx.y;
  if (gridDim.y < static_cast<unsigned>(a.E)) {
    __shared__ int s_cnt[QD_WARPS];
    __shared__ int s_e;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (threadIdx.x == 0) s_e = -1;
    int before = 0;  // experts with rows ahead of this 128-wide chunk
    for (int c0 = 0; c0 < a.E; c0 += QD_WARPS * 32) {
      const int ex = c0 + static_cast<int>(threadIdx.x);
      const bool has = ex < a.E && a.offsets[ex + 1] > a.offsets[ex];
      const unsigned m = __ballot_sync(0xffffffffu, has);
      if (lane == 0) s_cnt[w] = __popc(m);
      __syncthreads();
      int rank = before + __popc(m & ((1u << lane) - 1u));
      int total = 0;
#pragma unroll
      for (int i = 0; i < QD_WARPS; ++i) {
        if (i < w) rank += s_cnt[i];
        total += s_cnt[i];
      }
      if (has && rank == static_cast<int>(blockIdx.y)) s_e = ex;
      before += total;
      __syncthreads();
    }
    e = s_e;
    if (e < 0) return;
  }
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
    // An empty split still owns its partial-sum slice: write zeros.
    if (a.out_partial != nullptr) {
      const int lane = threadIdx.x & 31;
      for (int i = lane; i < 16 * cnt; i += 32) {
        const int n = n0 + (i & 15), tok = i >> 4;
        if (n >= a.N) continue;
        float* prow = a.out_partial + (static_cast<int64_t>(split) * a.rows + row_begin + tok) * a.ldo;
        prow[n] = 0.f;
        if (GATED) prow[a.N + n] = 0.f;
      }
    }
    return;
  }
  // Up to NGMAX groups of 8 routed rows per pass over the weights.
  static_assert(NGMAX == 1 || NGMAX == 2 || NGMAX == 4, "NGMAX is 1, 2 or 4");
  for (int tok0 = 0; tok0 < cnt; tok0 += 8 * NGMAX) {
    const int groups = min(NGMAX, (cnt - tok0 + 7) / 8);
    if (NGMAX == 1 || groups <= 1)
      run_pass<BITS, 1, GATED, kScale, RAW4, qd_stages<BITS, NGMAX>(), NGMAX == 1>(a, e, row_begin, cnt, tok0, n0, c_begin, c_end, split, ring);
    else if (NGMAX == 2 || groups <= 2)
      run_pass<BITS, 2, GATED, kScale, RAW4, qd_stages<BITS, NGMAX>(), NGMAX == 1>(a, e, row_begin, cnt, tok0, n0, c_begin, c_end, split, ring);
    else
      run_pass<BITS, 4, GATED, kScale, RAW4, qd_stages<BITS, NGMAX>(), NGMAX == 1>(a, e, row_begin, cnt, tok0, n0, c_begin, c_end, split, ring);
  }
}

// Expert of permuted row r (binary search over the offsets).
__device__ __forceinline__ int expert_of(const int32_t* offsets, int E, int64_t r) {
  int lo = 0, hi = E - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (offsets[mid] <= r) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// fc1 finalisation of split-K partial sums: act[r, n] = act(sum_s P[s][r][n] + b1,
// sum_s P[s][r][N + n] + b3) in fixed split order, fp32 -> fp16.
__global__ void __launch_bounds__(256)
finalize_fc1_kernel(const QDecodeArgs a, __half* __restrict__ act) {
  const int64_t r = blockIdx.y;
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  pdl_wait();  // launched dependent: the partial sums come from the previous kernel
  pdl_launch_dependents();
  if (n >= a.N) return;
  const int e = expert_of(a.offsets, a.E, r);
  const int64_t bi = e * a.bias_e_stride + static_cast<int64_t>(n) * a.bias_stride;
  // All splits' loads in flight at once; the sums keep the split order.
  float pg[kQmoeMaxSplits], pu[kQmoeMaxSplits];
#pragma unroll
  for (int s = 0; s < kQmoeMaxSplits; ++s) {
    const float* prow = a.out_partial + (static_cast<int64_t>(s) * a.rows + r) * a.ldo;
    pg[s] = s < a.splits ? prow[n] : 0.f;
    pu[s] = s < a.splits && a.gated ? prow[a.N + n] : 0.f;
  }
  float g = 0.f, u = 0.f;
#pragma unroll
  for (int s = 0; s < kQmoeMaxSplits; ++s) {
    if (s < a.splits) {
      g += pg[s];
      u += pu[s];
    }
  }
  const __half* b1p = static_cast<const __half*>(a.bias1);
  const __half* b3p = static_cast<const __half*>(a.bias3);
  if (b1p != nullptr) g += __half2float(b1p[bi]);
  float v;
  if (a.gated) {
    if (b3p != nullptr) u += __half2float(b3p[bi]);
    v = act_gated(a.ap, g, u);
  } else {
    v = act_single(a.ap.act, g);
  }
  act[r * a.N + n] = __float2half_rn(v);
}

// out[t] = sum_j w[t,j] * (sum_s partial[s][pos[t,j]] + bias) (fixed order), fp32 -> fp16.
__global__ void __launch_bounds__(256)
combine_partials_kernel(const float* __restrict__ part, int splits, int64_t rows,
                        const int32_t* __restrict__ pos, const float* __restrict__ w, int k,
                        int H, const int32_t* __restrict__ offsets, int E,
                        const __half* __restrict__ bias, __half* __restrict__ out) {
  const int t = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  pdl_wait();  // launched dependent: the partial sums come from the previous kernel
  pdl_launch_dependents();
  if (c >= H) return;
  float acc = 0.f;
  for (int j = 0; j < k; ++j) {
    const int64_t r = pos[static_cast<int64_t>(t) * k + j];
    // All splits' loads (and the bias) in flight at once; the sums keep the split order.
    float pv[kQmoeMaxSplits];
#pragma unroll
    for (int s = 0; s < kQmoeMaxSplits; ++s)
      pv[s] = s < splits ? part[(static_cast<int64_t>(s) * rows + r) * H + c] : 0.f;
    const float b =
        bias != nullptr ? __half2float(bias[static_cast<int64_t>(expert_of(offsets, E, r)) * H + c])
                        : 0.f;
    float y = 0.f;
#pragma unroll
    for (int s = 0; s < kQmoeMaxSplits; ++s)
      if (s < splits) y += pv[s];
    if (bias != nullptr) y += b;
    acc += w[static_cast<int64_t>(t) * k + j] * y;
  }
  out[static_cast<int64_t>(t) * H + c] = __float2half_rn(acc);
}

template <int BITS, bool GATED, int kScale, bool RAW4, int NGMAX>
cudaError_t launch_decode_n(const QDecodeArgs& a, cudaStream_t s) {
  constexpr int kSmem = QD_WARPS * ring_bytes<BITS, GATED, NGMAX>();
  static bool attr_set = false;  // idempotent; a race between first callers is benign
  if (!attr_set) {
    cudaError_t st = cudaFuncSetAttribute(qmoe_decode_kernel<BITS, GATED, kScale, RAW4, NGMAX>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (st != cudaSuccess) return st;
    attr_set = true;
  }
  // At most min(E, routed rows) experts hold rows: CTAs for the others would exit at once.
  const int ey = static_cast<int>(std::min<int64_t>(a.E, std::max<int64_t>(a.rows, 1)));
  const dim3 grid((a.N + QD_WARPS * 16 - 1) / (QD_WARPS * 16), ey, a.splits);
  return launch_dependent(pdl_enabled(), qmoe_decode_kernel<BITS, GATED, kScale, RAW4, NGMAX>, grid,
                          dim3(QD_WARPS * 32), kSmem, s, a);
}

// An expert holds at most all routed rows: groups of 8 per pass up to min(4, ceil(rows / 8)).
template <int BITS, bool GATED, int kScale, bool RAW4>
cudaError_t launch_decode_t(const QDecodeArgs& a, cudaStream_t s) {
  // MOE_B200_QDEC_MAXNG=1/2 caps the groups of one pass (measurement runs).
  static const int max_ng = [] {
    const char* v = std::getenv("MOE_B200_QDEC_MAXNG");
    return v != nullptr ? std::atoi(v) : 4;
  }();
  if (a.rows <= 8 || max_ng <= 1) return launch_decode_n<BITS, GATED, kScale, RAW4, 1>(a, s);
  if (a.rows <= 16 || max_ng <= 2) return launch_decode_n<BITS, GATED, kScale, RAW4, 2>(a, s);
  return launch_decode_n<BITS, GATED, kScale, RAW4, 4>(a, s);
}

// The biased-code int4 kernels run exactly when the caller supplied the arranged
// activations and offset terms (xcorr); every other combination runs per-code conversion.
template <int BITS, bool GATED>
cudaError_t launch_decode_b(const QDecodeArgs& a, cudaStream_t s) {
  const bool raw = a.xcorr != nullptr;
  if (BITS == 4 && raw && a.block_size % QD_CHUNK != 0 && a.block_size != 0)
    return cudaErrorInvalidValue;
  if (a.block_size == 0)
    return raw ? launch_decode_t<BITS, GATED, kScaleRow, BITS == 4>(a, s)
               : launch_decode_t<BITS, GATED, kScaleRow, false>(a, s);
  if (a.block_size % QD_CHUNK == 0)
    return raw ? launch_decode_t<BITS, GATED, kScaleChunk, BITS == 4>(a, s)
               : launch_decode_t<BITS, GATED, kScaleChunk, false>(a, s);
  return launch_decode_t<BITS, GATED, kScaleElem, false>(a, s);
}

}  // namespace

bool qmoe_decode_supported(int dtype, int bits, int block_size, int64_t H, int64_t I) {
  if (dtype != kDtF16) return false;
  if (bits != 4 && bits != 8) return false;
  if (block_size != 0 && block_size < 32) return false;
  return H % QD_CHUNK == 0 && I % QD_CHUNK == 0;
}

cudaError_t launch_qmoe_decode(const QDecodeArgs& a, int max_experts_touched, cudaStream_t s) {
  (void)max_experts_touched;
  if (a.bits == 4) return a.gated ? launch_decode_b<4, true>(a, s) : launch_decode_b<4, false>(a, s);
  return a.gated ? launch_decode_b<8, true>(a, s) : launch_decode_b<8, false>(a, s);
}

cudaError_t launch_qdec_prep(const __half* x, int64_t rows, int K, __half* xp, float* corr,
                             bool x_from_previous, cudaStream_t s) {
  const int64_t groups = rows * (K / 8);
  if (groups == 0) return cudaSuccess;
  return launch_dependent(pdl_enabled(), qdec_prep_kernel, dim3(static_cast<unsigned>((groups + 255) / 256)),
                          dim3(256), 0, s, x, rows, K, xp, corr, x_from_previous ? 1 : 0);
}

cudaError_t launch_finalize_fc1(const QDecodeArgs& a, __half* act, cudaStream_t s) {
  if (a.rows == 0) return cudaSuccess;
  const dim3 grid((a.N + 255) / 256, static_cast<unsigned>(a.rows));
  return launch_dependent(pdl_enabled(), finalize_fc1_kernel, grid, dim3(256), 0, s, a, act);
}

cudaError_t launch_combine_partials(const float* part, int splits, int64_t rows, const int32_t* pos,
                                    const float* w, int T, int k, int H, const int32_t* offsets,
                                    int E, const void* bias, void* out, cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  const dim3 grid((H + 255) / 256, T);
  return launch_dependent(pdl_enabled(), combine_partials_kernel, grid, dim3(256), 0, s, part, splits, rows, pos,
                          w, k, H, offsets, E, static_cast<const __half*>(bias),
                          static_cast<__half*>(out));
}

}  // namespace moe
