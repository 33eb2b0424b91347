// QMoE weight prepack and its sharing registry.
//
// The reference parses the session option "ep.musa.enable_prepack_weight_sharing"
// into EpConfig::enable_prepack_weight_sharing (musa/ep/src/ep_factory.cc:472-478,
// ep.h:35) and has no kernel that uses it.  Here a QMoE node's constant weights are
// dequantised once, when the session is initialised (the role of OpKernel::PrePack),
// into one device allocation; prefill-sized calls then run the fp16/bf16 tensor-core
// GEMMs on it with no per-call dequantisation.  With sharing on, nodes whose codes and
// scales have identical content (the same model loaded by several sessions) hold one
// copy: a registry keyed by the shape and a 64-bit content hash, reference counted.
//
// The content hash is the wrapping sum, over the 8-byte words w_i of each tensor, of
// mix(w_i ^ mix(i + salt)), where mix is the splitmix64 finaliser (S. Vigna,
// "splitmix64", public domain; the two xor-shift-multiply rounds with the constants
// of the published generator).  A sum is independent of the order in which threads
// add their words, so the hash is deterministic for any launch shape.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "prepack.h"
#include "qmoe.h"

namespace moe {

namespace {

__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

__global__ void __launch_bounds__(256)
content_hash_kernel(const uint8_t* __restrict__ p, int64_t n, uint64_t salt,
                    unsigned long long* __restrict__ out) {
  const int64_t nw = n / 8;
  const bool aligned = (reinterpret_cast<uintptr_t>(p) & 7) == 0;
  uint64_t acc = 0;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < nw;
       i += stride) {
    uint64_t w = 0;
    if (aligned) {
      w = __ldg(reinterpret_cast<const unsigned long long*>(p) + i);
    } else {
      for (int b = 0; b < 8; ++b) w |= static_cast<uint64_t>(p[8 * i + b]) << (8 * b);
    }
    acc += mix64(w ^ mix64(static_cast<uint64_t>(i) + salt));
  }
  if (blockIdx.x == 0 && threadIdx.x == 0 && (n & 7) != 0) {
    uint64_t w = 0;
    for (int64_t b = nw * 8; b < n; ++b) w |= static_cast<uint64_t>(p[b]) << (8 * (b - nw * 8));
    acc += mix64(w ^ mix64(static_cast<uint64_t>(nw) + salt));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) atomicAdd(out, static_cast<unsigned long long>(acc));
}

struct HashPart {
  const void* ptr;
  int64_t bytes;
};

// Content hash of the parts, in order: each part is hashed with its index as salt and
// the per-part sums are chained on the host together with the part sizes.
int content_hash(const HashPart* parts, int n, cudaStream_t s, uint64_t* key) {
  unsigned long long* d = nullptr;
  cudaError_t ce = cudaMallocAsync(&d, sizeof(unsigned long long) * n, s);
  if (ce == cudaSuccess) ce = cudaMemsetAsync(d, 0, sizeof(unsigned long long) * n, s);
  for (int i = 0; i < n && ce == cudaSuccess; ++i) {
    if (parts[i].bytes == 0) continue;
    const int64_t words = (parts[i].bytes + 7) / 8;
    const int blocks = static_cast<int>(std::min<int64_t>((words + 255) / 256, 148 * 16));
    content_hash_kernel<<<blocks, 256, 0, s>>>(static_cast<const uint8_t*>(parts[i].ptr),
                                               parts[i].bytes, 0x9e3779b97f4a7c15ull * (i + 1),
                                               d + i);
    ce = cudaGetLastError();
  }
  std::vector<unsigned long long> h(n, 0);
  if (ce == cudaSuccess)
    ce = cudaMemcpyAsync(h.data(), d, sizeof(unsigned long long) * n, cudaMemcpyDeviceToHost, s);
  if (d != nullptr) cudaFreeAsync(d, s);
  if (ce == cudaSuccess) ce = cudaStreamSynchronize(s);
  if (ce != cudaSuccess)
    return set_error(MOE_B200_EP_FAIL, "prepack content hash: %s", cudaGetErrorString(ce));
  uint64_t k = 0x243f6a8885a308d3ull;
  for (int i = 0; i < n; ++i)
    k = mix64(k ^ mix64(h[i] + static_cast<uint64_t>(parts[i].bytes)));
  *key = k;
  return MOE_B200_OK;
}

std::mutex g_registry_mu;
std::vector<moe_b200_prepacked*> g_registry;  // shared prepacks, guarded by g_registry_mu

bool same_shape(const moe_b200_prepacked& a, const moe_b200_prepacked& b) {
  return a.device == b.device && a.dtype == b.dtype && a.E == b.E && a.H == b.H && a.I == b.I &&
         a.n1 == b.n1 && a.has_fc3 == b.has_fc3 && a.bits == b.bits && a.block == b.block;
}

// A registered prepack whose key and shape match is shared only if its dequantised copies
// are, bit for bit, those of the new weights: the 64-bit key is a sum of mixed words, so
// different weights can collide (deliberately, too); equal dequantised copies are exactly
// the condition under which sharing gives the same outputs.
int same_content(const moe_b200_prepacked& e, const moe_b200_problem& p,
                 const moe_b200_tensors& t, cudaStream_t s, bool* differs) {
  int* diff = nullptr;
  cudaError_t ce = cudaMalloc(&diff, sizeof(int));
  if (ce != cudaSuccess)
    return set_error(MOE_B200_EP_FAIL, "prepack compare: %s", cudaGetErrorString(ce));
  const QmoeDequantOut have{e.w1, e.w2, e.w3};
  const int st = qmoe_dequantized_differs(p, t, have, diff, s, differs);
  cudaFree(diff);
  return st;
}

void free_prepack(moe_b200_prepacked* pk) {
  if (pk->base != nullptr) cudaFree(pk->base);  // waits for work in flight on the device
  delete pk;
}

}  // namespace

bool prepack_matches(const moe_b200_prepacked& pk, const moe_b200_problem& p) {
  return pk.dtype == p.dtype && pk.E == p.num_experts && pk.H == p.hidden_size &&
         pk.I == p.inter_size && pk.n1 == fc1_rows(p) && pk.has_fc3 == (p.has_fc3 ? 1 : 0) &&
         pk.bits == p.attrs.expert_weight_bits && pk.block == p.attrs.block_size;
}

bool prepack_applies(const moe_b200_prepacked* pk, const moe_b200_problem& p) {
  if (pk == nullptr || p.attrs.expert_weight_bits == 0 || !prepack_matches(*pk, p)) return false;
  if (qmoe_use_decode(p)) return false;
  int64_t min_rows = kPrepackMinRows;
  if (const char* v = std::getenv("MOE_B200_PREPACK_MIN_ROWS")) min_rows = std::atoll(v);
  return p.num_rows * p.attrs.k >= min_rows;
}

}  // namespace moe

extern "C" {

int moe_b200_prepack_create(const moe_b200_problem* problem, const moe_b200_tensors* weights,
                            int32_t share, void* stream, moe_b200_prepacked** out) {
  moe::clear_stale_cuda_error();
  using moe::set_error;
  if (problem == nullptr || weights == nullptr || out == nullptr)
    return set_error(MOE_B200_INVALID_ARGUMENT, "problem, weights and out must be non-NULL");
  *out = nullptr;
  const moe_b200_problem& p = *problem;
  const int bits = p.attrs.expert_weight_bits;
  if (bits != 4 && bits != 8)
    return set_error(MOE_B200_INVALID_ARGUMENT,
                     "prepack is for QMoE weights: expert_weight_bits=%d must be 4 or 8", bits);
  size_t ws_unused = 0;  // the same shape and attribute checks as a layer call
  int vst = moe_b200_workspace_size(problem, &ws_unused);
  if (vst != MOE_B200_OK) return vst;
  const int bs = p.attrs.block_size;
  const moe_b200_tensors& t = *weights;
  if (t.fc1_weights == nullptr || t.fc2_weights == nullptr || t.fc1_scales == nullptr ||
      t.fc2_scales == nullptr || (p.has_fc3 && (t.fc3_weights == nullptr || t.fc3_scales == nullptr)))
    return set_error(MOE_B200_INVALID_ARGUMENT, "prepack: weights and scales must be non-NULL");

  auto* pk = new moe_b200_prepacked();
  cudaGetDevice(&pk->device);
  pk->dtype = p.dtype;
  pk->E = p.num_experts;
  pk->H = p.hidden_size;
  pk->I = p.inter_size;
  pk->n1 = moe::fc1_rows(p);
  pk->has_fc3 = p.has_fc3 ? 1 : 0;
  pk->bits = bits;
  pk->block = bs;
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  if (share) {
    const int64_t E = pk->E, H = pk->H, I = pk->I, n1 = pk->n1;
    auto nb = [&](int64_t K) { return bs ? (K + bs - 1) / bs : 1; };
    const int64_t es = moe::dtype_bytes(p.dtype);
    const moe::HashPart parts[6] = {
        {t.fc1_weights, E * n1 * H * bits / 8}, {t.fc1_scales, E * n1 * nb(H) * es},
        {t.fc2_weights, E * H * I * bits / 8},  {t.fc2_scales, E * H * nb(I) * es},
        {p.has_fc3 ? t.fc3_weights : nullptr, p.has_fc3 ? E * I * H * bits / 8 : 0},
        {p.has_fc3 ? t.fc3_scales : nullptr, p.has_fc3 ? E * I * nb(H) * es : 0}};
    int st = moe::content_hash(parts, 6, s, &pk->key);
    if (st != MOE_B200_OK) {
      delete pk;
      return st;
    }
    std::lock_guard<std::mutex> lock(moe::g_registry_mu);
    for (moe_b200_prepacked* e : moe::g_registry) {
      if (e->key == pk->key && moe::same_shape(*e, *pk)) {
        bool differs = true;
        st = moe::same_content(*e, p, t, s, &differs);
        if (st != MOE_B200_OK) {
          delete pk;
          return st;
        }
        if (differs) continue;  // a hash collision: these weights get their own copy
        e->refs.fetch_add(1);
        delete pk;
        *out = e;
        return MOE_B200_OK;
      }
    }
  }

  pk->bytes = moe::qmoe_dequantized_bytes(p);
  cudaError_t ce = cudaMalloc(&pk->base, pk->bytes);
  if (ce != cudaSuccess) {
    delete pk;
    return set_error(MOE_B200_EP_FAIL, "prepack allocation of %zu bytes: %s",
                     static_cast<size_t>(moe::qmoe_dequantized_bytes(p)), cudaGetErrorString(ce));
  }
  moe::QmoeDequantOut dq{};
  int st = moe::qmoe_dequantize_into(p, t, static_cast<uint8_t*>(pk->base), &dq, s);
  if (st == MOE_B200_OK) {
    ce = cudaStreamSynchronize(s);  // usable from any stream once this returns
    if (ce != cudaSuccess) st = set_error(MOE_B200_EP_FAIL, "prepack: %s", cudaGetErrorString(ce));
  } else {
    st = set_error(st, "prepack: dequantisation failed");
  }
  if (st != MOE_B200_OK) {
    moe::free_prepack(pk);
    return st;
  }
  pk->w1 = dq.w1;
  pk->w2 = dq.w2;
  pk->w3 = dq.w3;
  if (share) {
    std::lock_guard<std::mutex> lock(moe::g_registry_mu);
    // Another thread may have registered the same content meanwhile: keep one copy.
    for (moe_b200_prepacked* e : moe::g_registry) {
      bool differs = true;
      if (e->key == pk->key && moe::same_shape(*e, *pk) &&
          moe::same_content(*e, p, t, s, &differs) == MOE_B200_OK && !differs) {
        e->refs.fetch_add(1);
        moe::free_prepack(pk);
        *out = e;
        return MOE_B200_OK;
      }
    }
    pk->shared = true;
    moe::g_registry.push_back(pk);
  }
  *out = pk;
  return MOE_B200_OK;
}

int moe_b200_prepack_info(const moe_b200_prepacked* pk, size_t* bytes, int32_t* refs) {
  if (pk == nullptr) return moe::set_error(MOE_B200_INVALID_ARGUMENT, "prepack is NULL");
  if (bytes != nullptr) *bytes = pk->bytes;
  if (refs != nullptr) *refs = pk->refs.load();
  return MOE_B200_OK;
}

int moe_b200_prepack_release(moe_b200_prepacked* pk) {
  if (pk == nullptr) return MOE_B200_OK;
  if (pk->shared) {
    std::lock_guard<std::mutex> lock(moe::g_registry_mu);
    if (pk->refs.fetch_sub(1) != 1) return MOE_B200_OK;
    auto& r = moe::g_registry;
    for (size_t i = 0; i < r.size(); ++i)
      if (r[i] == pk) {
        r.erase(r.begin() + static_cast<std::ptrdiff_t>(i));
        break;
      }
  } else if (pk->refs.fetch_sub(1) != 1) {
    return MOE_B200_OK;
  }
  moe::free_prepack(pk);
  return MOE_B200_OK;
}

}  // extern "C"
