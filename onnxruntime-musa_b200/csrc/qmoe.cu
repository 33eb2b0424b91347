// QMoE dequantisation kernels.  HBM-bound byte work: each thread turns 8 codes
// (4 bytes of int4 or 8 bytes of int8) into one 16-byte vector of fp16/bf16.
#include <algorithm>
#include <cstdlib>

#include "qmoe.h"
#include "qmoe_decode.h"

namespace moe {

namespace {

size_t align256(size_t v) { return (v + 255) / 256 * 256; }

template <typename T, int kBits>
__global__ void __launch_bounds__(256)
dequant_vec8_kernel(const uint8_t* __restrict__ q, const T* __restrict__ scales, int64_t rows,
                    int K, int block_size, int num_blocks, T* __restrict__ out) {
  const int64_t groups_per_row = K / 8;
  const int64_t total = rows * groups_per_row;
  for (int64_t gi = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; gi < total;
       gi += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = gi / groups_per_row;
    const int k0 = static_cast<int>(gi - r * groups_per_row) * 8;
    const float s = scales == nullptr ? 1.f
                    : block_size == 0  ? to_f(scales[r])
                                       : to_f(scales[r * num_blocks + k0 / block_size]);
    float v[8];
    if (kBits == 4) {
      const uint32_t word =
          *reinterpret_cast<const uint32_t*>(q + r * (K / 2) + k0 / 2);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        v[j] = static_cast<float>(static_cast<int>((word >> (4 * j)) & 0xF) - 8) * s;
    } else {
      const uint2 words = *reinterpret_cast<const uint2*>(q + r * K + k0);
      const uint32_t w2[2] = {words.x, words.y};
#pragma unroll
      for (int j = 0; j < 8; ++j)
        v[j] = static_cast<float>(static_cast<int>((w2[j >> 2] >> (8 * (j & 3))) & 0xFF) - 128) * s;
    }
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) ow[j] = pack2<T>(v[2 * j], v[2 * j + 1]);
    *reinterpret_cast<uint4*>(out + r * K + k0) = o;
  }
}

template <typename T>
__global__ void __launch_bounds__(256)
dequant_scalar_kernel(const uint8_t* __restrict__ q, const T* __restrict__ scales, int64_t rows,
                      int K, int bits, int block_size, int num_blocks, T* __restrict__ out) {
  const int64_t total = rows * K;
  const int64_t row_bytes = bits == 4 ? (K + 1) / 2 : K;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / K;
    const int c = static_cast<int>(i - r * K);
    int code;
    if (bits == 4) {
      const uint8_t b = q[r * row_bytes + c / 2];
      code = ((c & 1) ? (b >> 4) : (b & 0xF)) - 8;
    } else {
      code = static_cast<int>(q[r * row_bytes + c]) - 128;
    }
    const float s = scales == nullptr ? 1.f
                    : block_size == 0  ? to_f(scales[r])
                                       : to_f(scales[r * num_blocks + c / block_size]);
    out[i] = from_f<T>(static_cast<float>(code) * s);
  }
}

template <typename T>
cudaError_t dequant_t(const void* q, const void* scales, int64_t rows, int K, int bits,
                      int block_size, void* out, cudaStream_t s) {
  const int nb = block_size ? (K + block_size - 1) / block_size : 0;
  const T* sc = static_cast<const T*>(scales);
  const uint8_t* qb = static_cast<const uint8_t*>(q);
  T* o = static_cast<T*>(out);
  const bool vec = (K % 8) == 0 && (block_size == 0 || block_size % 8 == 0);
  const int64_t work = vec ? rows * (K / 8) : rows * K;
  const int blocks = static_cast<int>(std::min<int64_t>((work + 255) / 256, 148 * 16));
  if (vec) {
    if (bits == 4)
      dequant_vec8_kernel<T, 4><<<blocks, 256, 0, s>>>(qb, sc, rows, K, block_size, nb, o);
    else
      dequant_vec8_kernel<T, 8><<<blocks, 256, 0, s>>>(qb, sc, rows, K, block_size, nb, o);
  } else {
    dequant_scalar_kernel<T><<<blocks, 256, 0, s>>>(qb, sc, rows, K, bits, block_size, nb, o);
  }
  return cudaGetLastError();
}

// Sets *diff when out[r, c] differs (bitwise) from the dequantisation the kernels above
// would write for codes q and scales (scales == nullptr: exact codes).
template <typename T>
__global__ void __launch_bounds__(256)
dequant_compare_kernel(const uint8_t* __restrict__ q, const T* __restrict__ scales, int64_t rows,
                       int K, int bits, int block_size, int num_blocks, const T* __restrict__ out,
                       int* __restrict__ diff) {
  const int64_t total = rows * K;
  const int64_t row_bytes = bits == 4 ? (K + 1) / 2 : K;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / K;
    const int c = static_cast<int>(i - r * K);
    int code;
    if (bits == 4) {
      const uint8_t b = q[r * row_bytes + c / 2];
      code = ((c & 1) ? (b >> 4) : (b & 0xF)) - 8;
    } else {
      code = static_cast<int>(q[r * row_bytes + c]) - 128;
    }
    const float s = scales == nullptr ? 1.f
                    : block_size == 0  ? to_f(scales[r])
                                       : to_f(scales[r * num_blocks + c / block_size]);
    const T v = from_f<T>(static_cast<float>(code) * s);
    if (*reinterpret_cast<const uint16_t*>(&v) != reinterpret_cast<const uint16_t*>(out)[i])
      *diff = 1;
  }
}

template <typename T>
cudaError_t dequant_compare_t(const void* q, const void* scales, int64_t rows, int K, int bits,
                              int block_size, const void* out, int* diff, cudaStream_t s) {
  const int nb = block_size ? (K + block_size - 1) / block_size : 0;
  const int blocks = static_cast<int>(std::min<int64_t>((rows * K + 255) / 256, 148 * 16));
  dequant_compare_kernel<T><<<blocks, 256, 0, s>>>(
      static_cast<const uint8_t*>(q), static_cast<const T*>(scales), rows, K, bits, block_size,
      nb, static_cast<const T*>(out), diff);
  return cudaGetLastError();
}

cudaError_t dequant_compare(int dtype, const void* q, const void* scales, int64_t rows, int K,
                            int bits, int block_size, const void* out, int* diff,
                            cudaStream_t s) {
  if (rows == 0 || K == 0) return cudaSuccess;
  if (dtype == kDtF16)
    return dequant_compare_t<__half>(q, scales, rows, K, bits, block_size, out, diff, s);
  if (dtype == kDtBF16)
    return dequant_compare_t<__nv_bfloat16>(q, scales, rows, K, bits, block_size, out, diff, s);
  return cudaErrorInvalidValue;
}

cudaError_t dequant(int dtype, const void* q, const void* scales, int64_t rows, int K, int bits,
                    int block_size, void* out, cudaStream_t s) {
  if (rows == 0 || K == 0) return cudaSuccess;
  if (dtype == kDtF16) return dequant_t<__half>(q, scales, rows, K, bits, block_size, out, s);
  if (dtype == kDtBF16)
    return dequant_t<__nv_bfloat16>(q, scales, rows, K, bits, block_size, out, s);
  return cudaErrorInvalidValue;
}

}  // namespace

int64_t fc1_rows(const moe_b200_problem& p) {
  const bool fused = p.attrs.activation_type == MOE_B200_ACT_SWIGLU && p.attrs.swiglu_fusion != 0;
  return fused ? 2 * p.inter_size : p.inter_size;
}

bool qmoe_use_decode(const moe_b200_problem& p) {
  if (p.attrs.expert_weight_bits == 0) return false;
  if (std::getenv("MOE_B200_QMOE_NO_DECODE") != nullptr) return false;
  // MOE_B200_QMOE_DECODE_MAX_ROWS moves the switch-over point (for measurement).
  int64_t max_rows = kQmoeDecodeMaxRows;
  if (const char* v = std::getenv("MOE_B200_QMOE_DECODE_MAX_ROWS")) max_rows = std::atoll(v);
  max_rows = std::min<int64_t>(max_rows, kSmallDispatchRows);
  return p.num_rows * p.attrs.k <= max_rows &&
         qmoe_decode_supported(p.dtype, p.attrs.expert_weight_bits, p.attrs.block_size,
                               p.hidden_size, p.inter_size);
}

namespace {

// K splits of a decode pass over N output rows of K columns: enough warp tiles
// (16 rows each) to fill the GPU several times over when few experts are touched.
int decode_splits(const moe_b200_problem& p, int64_t N, int64_t K) {
  const int64_t touched = std::min<int64_t>(p.num_experts, p.num_rows * p.attrs.k);
  const int64_t tiles = (N + 15) / 16 * std::max<int64_t>(touched, 1);
  const int64_t target = 148 * 4 * 8;  // 8 waves of 4 warps per SM
  const int s = static_cast<int>((target + tiles - 1) / tiles);
  const int chunks = static_cast<int>(K / 128);
  // MOE_B200_QDEC_SPLITS fixes the split count (measurement runs).
  if (const char* v = std::getenv("MOE_B200_QDEC_SPLITS"))
    return std::max(1, std::min({std::atoi(v), kQmoeMaxSplits, chunks}));
  return std::max(1, std::min({s, kQmoeMaxSplits, chunks}));
}
int fc1_splits(const moe_b200_problem& p) { return decode_splits(p, p.inter_size, p.hidden_size); }
int fc2_splits(const moe_b200_problem& p) { return decode_splits(p, p.hidden_size, p.inter_size); }

// int4 with exact codes runs the biased-code kernel on pre-arranged activations
// (launch_qdec_prep); MOE_B200_QDEC_RAW4=0 keeps the per-code conversion (comparison runs).
bool raw4(const moe_b200_problem& p) {
  const int bs = p.attrs.block_size;
  if (p.attrs.expert_weight_bits != 4 || (bs != 0 && bs % 128 != 0)) return false;
  const char* v = std::getenv("MOE_B200_QDEC_RAW4");
  return v == nullptr || v[0] != '0';
}

// Workspace of the decode path: fc1 partials [S1][R][2I], fc2 partials [S2][R][H], and for
// the biased-code int4 path the arranged activations and offset terms of fc1 ([T][H],
// [T][H/128]) and fc2 ([R][I], [R][I/128]).
size_t fc1_partial_bytes(const moe_b200_problem& p) {
  const int s1 = fc1_splits(p);
  if (s1 == 1) return 0;
  return align256(static_cast<size_t>(s1) * p.num_rows * p.attrs.k * 2 * p.inter_size * sizeof(float));
}

size_t fc2_partial_bytes(const moe_b200_problem& p) {
  return align256(static_cast<size_t>(fc2_splits(p)) * p.num_rows * p.attrs.k * p.hidden_size *
                  sizeof(float));
}
struct Raw4Ws {
  size_t xp1, c1, xp2, c2, total;
};
Raw4Ws raw4_ws(const moe_b200_problem& p) {
  Raw4Ws w{};
  if (!raw4(p)) return w;
  const size_t T = p.num_rows, R = p.num_rows * p.attrs.k, H = p.hidden_size, I = p.inter_size;
  size_t o = fc1_partial_bytes(p) + fc2_partial_bytes(p);
  w.xp1 = o;
  o += align256(T * H * 2);
  w.c1 = o;
  o += align256(T * (H / 128) * 4);
  w.xp2 = o;
  o += align256(R * I * 2);
  w.c2 = o;
  o += align256(R * (I / 128) * 4);
  w.total = o - fc1_partial_bytes(p) - fc2_partial_bytes(p);
  return w;
}

}  // namespace

int qmoe_decode_fc1(const moe_b200_problem& p, const moe_b200_tensors& t, const int32_t* src,
                    void* act, const int32_t* offsets, uint8_t* ws, cudaStream_t s) {
  if (t.fc1_scales == nullptr || t.fc2_scales == nullptr || (p.has_fc3 && t.fc3_scales == nullptr))
    return set_error(MOE_B200_INVALID_ARGUMENT, "QMoE scales are required");
  const int64_t E = p.num_experts, H = p.hidden_size, I = p.inter_size;
  const int64_t R = p.num_rows * p.attrs.k;
  const bool fused = p.attrs.activation_type == MOE_B200_ACT_SWIGLU && p.attrs.swiglu_fusion != 0;
  const int N1 = static_cast<int>(fc1_rows(p));
  const auto* s1 = static_cast<const __half*>(t.fc1_scales);
  QDecodeArgs a{};
  a.x = static_cast<const __half*>(t.input);  // routed row p reads input row src[p] / k
  a.src_rows = src;
  a.k = p.attrs.k;
  a.rows = R;
  a.K = static_cast<int>(H);
  a.N = static_cast<int>(I);
  a.E = static_cast<int>(E);
  a.offsets = offsets;
  a.bits = p.attrs.expert_weight_bits;
  a.block_size = p.attrs.block_size;
  a.ap = ActParams{p.attrs.activation_type, p.attrs.activation_alpha, p.attrs.activation_beta,
                   p.attrs.swiglu_limit};
  a.bias_stride = 1;
  a.bias_e_stride = I;
  const uint8_t* q1 = static_cast<const uint8_t*>(t.fc1_weights);
  if (p.has_fc3) {
    a.gated = true;
    a.b1 = QOperand{q1, s1, 0, 1, 0, static_cast<int>(I)};
    a.b3 = QOperand{static_cast<const uint8_t*>(t.fc3_weights),
                    static_cast<const __half*>(t.fc3_scales), 0, 1, 0, static_cast<int>(I)};
    a.bias1 = t.fc1_bias;
    a.bias3 = t.fc3_bias;
  } else if (fused) {
    a.gated = true;
    a.bias_e_stride = 2 * I;
    if (p.attrs.swiglu_fusion == 1) {
      a.b1 = QOperand{q1, s1, 0, 2, 0, N1};
      a.b3 = QOperand{q1, s1, 1, 2, 0, N1};
      a.bias1 = t.fc1_bias;
      a.bias3 = t.fc1_bias ? static_cast<const __half*>(t.fc1_bias) + 1 : nullptr;
      a.bias_stride = 2;
    } else {
      a.b1 = QOperand{q1, s1, 0, 1, 0, N1};
      a.b3 = QOperand{q1, s1, 0, 1, static_cast<int>(I), N1};
      a.bias1 = t.fc1_bias;
      a.bias3 = t.fc1_bias ? static_cast<const __half*>(t.fc1_bias) + I : nullptr;
    }
  } else {
    a.gated = false;
    a.b1 = QOperand{q1, s1, 0, 1, 0, static_cast<int>(I)};
    a.bias1 = t.fc1_bias;
  }
  a.splits = fc1_splits(p);
  if (raw4(p)) {
    const Raw4Ws w = raw4_ws(p);
    auto* xp = reinterpret_cast<__half*>(ws + w.xp1);
    auto* corr = reinterpret_cast<float*>(ws + w.c1);
    cudaError_t st = launch_qdec_prep(a.x, p.num_rows, a.K, xp, corr, false, s);
    if (st != cudaSuccess)
      return set_error(MOE_B200_EP_FAIL, "QMoE fc1 activation prep: %s", cudaGetErrorString(st));
    a.x = xp;
    a.xcorr = corr;
  }
  if (a.splits == 1) {
    a.out = static_cast<__half*>(act);
    a.ldo = I;
  } else {
    a.out_partial = reinterpret_cast<float*>(ws);
    a.ldo = a.gated ? 2 * I : I;
  }
  cudaError_t st = launch_qmoe_decode(a, static_cast<int>(E), s);
  if (st == cudaSuccess && a.splits > 1) st = launch_finalize_fc1(a, static_cast<__half*>(act), s);
  if (st != cudaSuccess) return set_error(MOE_B200_EP_FAIL, "QMoE fc1 decode: %s", cudaGetErrorString(st));
  return MOE_B200_OK;
}

int qmoe_decode_fc2(const moe_b200_problem& p, const moe_b200_tensors& t, const void* act,
                    const int32_t* offsets, uint8_t* ws, cudaStream_t s) {
  const int64_t E = p.num_experts, H = p.hidden_size, I = p.inter_size;
  const int64_t R = p.num_rows * p.attrs.k;
  QDecodeArgs b{};
  b.x = static_cast<const __half*>(act);
  b.src_rows = nullptr;
  b.k = p.attrs.k;
  b.rows = R;
  b.K = static_cast<int>(I);
  b.N = static_cast<int>(H);
  b.E = static_cast<int>(E);
  b.offsets = offsets;
  b.bits = p.attrs.expert_weight_bits;
  b.block_size = p.attrs.block_size;
  b.gated = false;
  b.b1 = QOperand{static_cast<const uint8_t*>(t.fc2_weights),
                  static_cast<const __half*>(t.fc2_scales), 0, 1, 0, static_cast<int>(H)};
  b.ap = ActParams{kIdentity, 1.f, 0.f, INFINITY};
  b.bias_stride = 1;
  b.bias_e_stride = H;
  b.out_partial = reinterpret_cast<float*>(ws + fc1_partial_bytes(p));
  b.ldo = H;
  b.splits = fc2_splits(p);
  if (raw4(p)) {
    const Raw4Ws w = raw4_ws(p);
    auto* xp = reinterpret_cast<__half*>(ws + w.xp2);
    auto* corr = reinterpret_cast<float*>(ws + w.c2);
    cudaError_t st = launch_qdec_prep(b.x, R, b.K, xp, corr, true, s);
    if (st != cudaSuccess)
      return set_error(MOE_B200_EP_FAIL, "QMoE fc2 activation prep: %s", cudaGetErrorString(st));
    b.x = xp;
    b.xcorr = corr;
  }
  cudaError_t st = launch_qmoe_decode(b, static_cast<int>(E), s);
  if (st != cudaSuccess) return set_error(MOE_B200_EP_FAIL, "QMoE fc2 decode: %s", cudaGetErrorString(st));
  return MOE_B200_OK;
}

int qmoe_decode_combine(const moe_b200_problem& p, const moe_b200_tensors& t, const uint8_t* ws,
                        const int32_t* offsets, const int32_t* pos, const float* w,
                        cudaStream_t s) {
  const int64_t R = p.num_rows * p.attrs.k;
  cudaError_t st = launch_combine_partials(
      reinterpret_cast<const float*>(ws + fc1_partial_bytes(p)), fc2_splits(p), R, pos, w,
      static_cast<int>(p.num_rows), p.attrs.k, static_cast<int>(p.hidden_size), offsets,
      static_cast<int>(p.num_experts), t.fc2_bias, t.output, s);
  if (st != cudaSuccess) return set_error(MOE_B200_EP_FAIL, "QMoE combine: %s", cudaGetErrorString(st));
  return MOE_B200_OK;
}

bool qmoe_use_fused(const moe_b200_problem& p) {
  const int bits = p.attrs.expert_weight_bits;
  if (bits == 0 || qmoe_use_decode(p) || p.dtype != kDtF16) return false;
  if (std::getenv("MOE_B200_QMOE_DEQUANT") != nullptr) return false;
  // Beyond ~16K routed rows the fp16 GEMM on dequantised copies is faster: the one-off
  // dequantisation is amortised, and the fp16 kernel reaches a higher tensor rate.
  if (p.num_rows * p.attrs.k > kQmoeFusedMaxRows) return false;
  const int bs = p.attrs.block_size;
  auto k_ok = [&](int64_t K) { return K % 64 == 0 && (K * bits / 8) % 16 == 0; };
  return k_ok(p.hidden_size) && k_ok(p.inter_size) && (bs == 0 || bs % 8 == 0);
}

size_t qmoe_workspace_bytes(const moe_b200_problem& p) {
  if (p.attrs.expert_weight_bits == 0 || qmoe_use_fused(p)) return 0;
  if (qmoe_use_decode(p)) return fc1_partial_bytes(p) + fc2_partial_bytes(p) + raw4_ws(p).total;
  return qmoe_dequantized_bytes(p);
}

bool qmoe_dequantized_exact(const moe_b200_problem& p) {
  return p.attrs.expert_weight_bits != 0 && p.attrs.block_size == 0 && p.dtype == kDtF16;
}

size_t qmoe_dequantized_bytes(const moe_b200_problem& p) {
  const size_t es = dtype_bytes(p.dtype);
  const int64_t E = p.num_experts, H = p.hidden_size, I = p.inter_size;
  size_t b = align256(E * fc1_rows(p) * H * es) + align256(E * H * I * es);
  if (p.has_fc3) b += align256(E * I * H * es);
  return b;
}

int qmoe_dequantize_into(const moe_b200_problem& p, const moe_b200_tensors& t, uint8_t* dst,
                         QmoeDequantOut* out, cudaStream_t s) {
  if (t.fc1_scales == nullptr || t.fc2_scales == nullptr || (p.has_fc3 && t.fc3_scales == nullptr))
    return MOE_B200_INVALID_ARGUMENT;
  const size_t es = dtype_bytes(p.dtype);
  const int64_t E = p.num_experts, H = p.hidden_size, I = p.inter_size;
  const int bits = p.attrs.expert_weight_bits, bs = p.attrs.block_size;
  uint8_t* w1 = dst;
  uint8_t* w2 = w1 + align256(E * fc1_rows(p) * H * es);
  uint8_t* w3 = w2 + align256(E * H * I * es);
  // Per-row scales: the copies hold the exact codes (q - zero point) and the GEMM
  // epilogues apply the scale to the fp32 sums, so the weights carry no fp16 rounding.
  const bool exact = qmoe_dequantized_exact(p);
  auto sc = [&](const void* scales) { return exact ? nullptr : scales; };
  cudaError_t st = dequant(p.dtype, t.fc1_weights, sc(t.fc1_scales), E * fc1_rows(p),
                           static_cast<int>(H), bits, bs, w1, s);
  if (st == cudaSuccess)
    st = dequant(p.dtype, t.fc2_weights, sc(t.fc2_scales), E * H, static_cast<int>(I), bits, bs,
                 w2, s);
  if (st == cudaSuccess && p.has_fc3)
    st = dequant(p.dtype, t.fc3_weights, sc(t.fc3_scales), E * I, static_cast<int>(H), bits, bs,
                 w3, s);
  if (st != cudaSuccess) return MOE_B200_EP_FAIL;
  out->w1 = w1;
  out->w2 = w2;
  out->w3 = p.has_fc3 ? w3 : nullptr;
  return MOE_B200_OK;
}

int qmoe_dequantized_differs(const moe_b200_problem& p, const moe_b200_tensors& t,
                             const QmoeDequantOut& have, int* diff_dev, cudaStream_t s,
                             bool* differs) {
  const int64_t E = p.num_experts, H = p.hidden_size, I = p.inter_size;
  const int bits = p.attrs.expert_weight_bits, bs = p.attrs.block_size;
  const bool exact = qmoe_dequantized_exact(p);
  auto sc = [&](const void* scales) { return exact ? nullptr : scales; };
  cudaError_t st = cudaMemsetAsync(diff_dev, 0, sizeof(int), s);
  if (st == cudaSuccess)
    st = dequant_compare(p.dtype, t.fc1_weights, sc(t.fc1_scales), E * fc1_rows(p),
                         static_cast<int>(H), bits, bs, have.w1, diff_dev, s);
  if (st == cudaSuccess)
    st = dequant_compare(p.dtype, t.fc2_weights, sc(t.fc2_scales), E * H, static_cast<int>(I),
                         bits, bs, have.w2, diff_dev, s);
  if (st == cudaSuccess && p.has_fc3)
    st = dequant_compare(p.dtype, t.fc3_weights, sc(t.fc3_scales), E * I, static_cast<int>(H),
                         bits, bs, have.w3, diff_dev, s);
  int h = 0;
  if (st == cudaSuccess) st = cudaMemcpyAsync(&h, diff_dev, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (st == cudaSuccess) st = cudaStreamSynchronize(s);
  if (st != cudaSuccess) return set_error(MOE_B200_EP_FAIL, "prepack compare: %s", cudaGetErrorString(st));
  *differs = h != 0;
  return MOE_B200_OK;
}

int qmoe_dequantize(const moe_b200_problem& p, const moe_b200_tensors& t, uint8_t* ws,
                    const int32_t* expert_offsets, QmoeDequantOut* out, cudaStream_t s) {
  (void)expert_offsets;
  return qmoe_dequantize_into(p, t, ws, out, s);
}

}  // namespace moe
