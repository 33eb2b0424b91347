// QMoE dequantisation kernels.  HBM-bound byte work: each thread turns 8 codes
// (4 bytes of int4 or 8 bytes of int8) into one 16-byte vector of fp16/bf16.
#include "qmoe.h"

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
    const float s = block_size == 0
                        ? to_f(scales[r])
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
    const float s = block_size == 0 ? to_f(scales[r]) : to_f(scales[r * num_blocks + c / block_size]);
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

cudaError_t dequant(int dtype, const void* q, const void* scales, int64_t rows, int K, int bits,
                    int block_size, void* out, cudaStream_t s) {
  if (rows == 0 || K == 0) return cudaSuccess;
  if (dtype == kDtF16) return dequant_t<__half>(q, scales, rows, K, bits, block_size, out, s);
  if (dtype == kDtBF16)
    return dequant_t<__nv_bfloat16>(q, scales, rows, K, bits, block_size, out, s);
  return cudaErrorInvalidValue;
}

int64_t fc1_rows(const moe_b200_problem& p) {
  const bool fused = p.attrs.activation_type == MOE_B200_ACT_SWIGLU && p.attrs.swiglu_fusion != 0;
  return fused ? 2 * p.inter_size : p.inter_size;
}

}  // namespace

size_t qmoe_workspace_bytes(const moe_b200_problem& p) {
  if (p.attrs.expert_weight_bits == 0) return 0;
  const size_t es = dtype_bytes(p.dtype);
  const int64_t E = p.num_experts, H = p.hidden_size, I = p.inter_size;
  size_t b = align256(E * fc1_rows(p) * H * es) + align256(E * H * I * es);
  if (p.has_fc3) b += align256(E * I * H * es);
  return b;
}

int qmoe_dequantize(const moe_b200_problem& p, const moe_b200_tensors& t, uint8_t* ws,
                    const int32_t* expert_offsets, QmoeDequantOut* out, cudaStream_t s) {
  (void)expert_offsets;
  if (t.fc1_scales == nullptr || t.fc2_scales == nullptr || (p.has_fc3 && t.fc3_scales == nullptr))
    return MOE_B200_INVALID_ARGUMENT;
  const size_t es = dtype_bytes(p.dtype);
  const int64_t E = p.num_experts, H = p.hidden_size, I = p.inter_size;
  const int bits = p.attrs.expert_weight_bits, bs = p.attrs.block_size;
  uint8_t* w1 = ws;
  uint8_t* w2 = w1 + align256(E * fc1_rows(p) * H * es);
  uint8_t* w3 = w2 + align256(E * H * I * es);
  cudaError_t st = dequant(p.dtype, t.fc1_weights, t.fc1_scales, E * fc1_rows(p),
                           static_cast<int>(H), bits, bs, w1, s);
  if (st == cudaSuccess)
    st = dequant(p.dtype, t.fc2_weights, t.fc2_scales, E * H, static_cast<int>(I), bits, bs, w2, s);
  if (st == cudaSuccess && p.has_fc3)
    st = dequant(p.dtype, t.fc3_weights, t.fc3_scales, E * I, static_cast<int>(H), bits, bs, w3, s);
  if (st != cudaSuccess) return MOE_B200_EP_FAIL;
  out->w1 = w1;
  out->w2 = w2;
  out->w3 = p.has_fc3 ? w3 : nullptr;
  return MOE_B200_OK;
}

}  // namespace moe
