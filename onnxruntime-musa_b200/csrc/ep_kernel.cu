// The per-node MoE / QMoE kernel object and the CUDA runtime layer of the C ABI.
//
// moe_b200_kernel mirrors what the reference's kernel framework gives every op:
// attributes read once at creation (AttrOrDefault, kernels/shared_inc/
// kernel_attributes.h:21-37), a const, re-entrant Compute that validates input
// shapes and types and returns a status (kernel_base.h:45-84), and a Release.
// Scratch memory is a per-stream cached workspace grown with stream-ordered
// allocation, the role of DeferredDeviceFreeQueue / AllocateDeviceMemoryOnStream
// (kernels/shared_inc/kernel_memory.h:67-252).
#include <cerrno>
#include <cstdint>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>

#include "../../include/moe_b200.h"
#include "moe_kernels.h"
#include "prepack.h"

namespace {

using moe::set_error;
#define efail moe::set_error

bool parse_int(const char* s, int64_t* out) {
  if (s == nullptr || *s == '\0') return false;
  char* end = nullptr;
  errno = 0;
  const long long v = std::strtoll(s, &end, 10);
  if (errno != 0 || end == s || *end != '\0') return false;
  *out = v;
  return true;
}

bool parse_float(const char* s, float* out) {
  if (s == nullptr || *s == '\0') return false;
  char* end = nullptr;
  errno = 0;
  const float v = std::strtof(s, &end);
  if (errno != 0 || end == s || *end != '\0') return false;
  *out = v;
  return true;
}

int activation_from_name(const char* s) {
  if (!std::strcmp(s, "relu")) return MOE_B200_ACT_RELU;
  if (!std::strcmp(s, "gelu")) return MOE_B200_ACT_GELU;
  if (!std::strcmp(s, "silu")) return MOE_B200_ACT_SILU;
  if (!std::strcmp(s, "identity")) return MOE_B200_ACT_IDENTITY;
  if (!std::strcmp(s, "swiglu")) return MOE_B200_ACT_SWIGLU;
  return -1;
}

}  // namespace

struct moe_b200_kernel {
  bool quantized = false;
  moe_b200_attrs attrs{};
  std::mutex mu;
  struct Ws {
    void* ptr = nullptr;
    size_t bytes = 0;
  };
  std::unordered_map<cudaStream_t, Ws> ws;  // guarded by mu
  // Pre-pack (QMoE): the prepack and the device pointers of the weight and scale
  // inputs it was made from (fc1 w/s, fc2 w/s, fc3 w/s); computes whose inputs are
  // these pointers use it.
  moe_b200_prepacked* pk = nullptr;
  const void* pk_src[6] = {};
};

namespace {

int64_t numel_prefix(const moe_b200_tensor_ref& t, int upto) {
  int64_t n = 1;
  for (int i = 0; i < upto; ++i) n *= t.dims[i];
  return n;
}

std::string shape_str(const moe_b200_tensor_ref& t) {
  std::string s = "[";
  for (int i = 0; i < t.rank; ++i) {
    if (i) s += ",";
    s += std::to_string(t.dims[i]);
  }
  return s + "]";
}

}  // namespace

extern "C" {

static const char* op_name(const moe_b200_kernel* kern) {
  return kern == nullptr ? "?" : (kern->quantized ? "QMoE" : "MoE");
}

int moe_b200_kernel_create(const char* op_type, int32_t num_attrs, const char* const* names,
                           const char* const* values, moe_b200_kernel** kernel) {
  if (kernel == nullptr || op_type == nullptr)
    return (efail(MOE_B200_INVALID_ARGUMENT, "op_type and kernel must be non-NULL"));
  const bool q = std::strcmp(op_type, "QMoE") == 0;
  if (!q && std::strcmp(op_type, "MoE") != 0)
    return (efail(MOE_B200_NOT_IMPLEMENTED, "unsupported op_type '%s'", op_type));
  moe_b200_attrs a{};
  a.activation_type = MOE_B200_ACT_RELU;
  a.k = 1;
  a.normalize_routing_weights = 0;
  a.use_sparse_mixer = 0;
  a.swiglu_fusion = 0;
  a.swiglu_limit = INFINITY;
  a.activation_alpha = 1.0f;
  a.activation_beta = 0.0f;
  a.expert_weight_bits = q ? 4 : 0;
  a.block_size = 0;
  for (int i = 0; i < num_attrs; ++i) {
    const char* n = names[i];
    const char* v = values[i];
    int64_t iv = 0;
    float fv = 0.f;
    if (!std::strcmp(n, "activation_type")) {
      a.activation_type = activation_from_name(v);
      if (a.activation_type < 0)
        return (efail(MOE_B200_INVALID_ARGUMENT, "unsupported activation_type '%s'", v));
    } else if (!std::strcmp(n, "k") || !std::strcmp(n, "normalize_routing_weights") ||
               !std::strcmp(n, "use_sparse_mixer") || !std::strcmp(n, "swiglu_fusion") ||
               !std::strcmp(n, "expert_weight_bits") || !std::strcmp(n, "block_size")) {
      if (!parse_int(v, &iv))
        return (efail(MOE_B200_INVALID_ARGUMENT, "attribute %s: '%s' is not an integer", n, v));
      if (!std::strcmp(n, "k")) a.k = static_cast<int32_t>(iv);
      else if (!std::strcmp(n, "normalize_routing_weights")) a.normalize_routing_weights = static_cast<int32_t>(iv);
      else if (!std::strcmp(n, "use_sparse_mixer")) a.use_sparse_mixer = static_cast<int32_t>(iv);
      else if (!std::strcmp(n, "swiglu_fusion")) a.swiglu_fusion = static_cast<int32_t>(iv);
      else if (!std::strcmp(n, "expert_weight_bits")) {
        if (!q) return (efail(MOE_B200_INVALID_ARGUMENT, "expert_weight_bits is a QMoE attribute"));
        a.expert_weight_bits = static_cast<int32_t>(iv);
      } else {
        if (!q) return (efail(MOE_B200_INVALID_ARGUMENT, "block_size is a QMoE attribute"));
        a.block_size = static_cast<int32_t>(iv);
      }
    } else if (!std::strcmp(n, "swiglu_limit") || !std::strcmp(n, "activation_alpha") ||
               !std::strcmp(n, "activation_beta")) {
      if (!parse_float(v, &fv))
        return (efail(MOE_B200_INVALID_ARGUMENT, "attribute %s: '%s' is not a float", n, v));
      if (!std::strcmp(n, "swiglu_limit")) a.swiglu_limit = fv;
      else if (!std::strcmp(n, "activation_alpha")) a.activation_alpha = fv;
      else a.activation_beta = fv;
    } else {
      return (efail(MOE_B200_INVALID_ARGUMENT, "unknown attribute '%s' for %s", n, op_type));
    }
  }
  if (a.k < 1) return (efail(MOE_B200_INVALID_ARGUMENT, "k=%d must be >= 1", a.k));
  if (q && a.expert_weight_bits != 4 && a.expert_weight_bits != 8)
    return (efail(MOE_B200_INVALID_ARGUMENT, "expert_weight_bits=%d must be 4 or 8",
                        a.expert_weight_bits));
  auto* kern = new moe_b200_kernel();
  kern->quantized = q;
  kern->attrs = a;
  *kernel = kern;
  if (std::getenv("MOE_B200_TRACE_KERNELS") != nullptr) {
    std::fprintf(stderr, "MOE_B200_KERNEL_CREATE %s impl=%p k=%d bits=%d block=%d\n",
                 op_name(kern), static_cast<void*>(kern), a.k, a.expert_weight_bits,
                 a.block_size);
    std::fflush(stderr);
  }
  return MOE_B200_OK;
}

static int kernel_compute_impl(moe_b200_kernel* kern, int32_t num_inputs,
                               const moe_b200_tensor_ref* in, moe_b200_tensor_ref* output,
                               void* stream);

// Kernel trace of the reference EP (OpKernelBase::ComputeImpl,
// musa/ep/src/kernels/shared_inc/kernel_base.h:45-84): with MOE_B200_TRACE_KERNELS set,
// one BEGIN and one END line per compute on stderr, flushed; with MOE_B200_TRACE_SYNC as
// well, a successful compute synchronises its stream so an asynchronous fault is reported
// (EP_FAIL) at the kernel that caused it.
int moe_b200_kernel_compute(moe_b200_kernel* kern, int32_t num_inputs,
                            const moe_b200_tensor_ref* in, moe_b200_tensor_ref* output,
                            void* stream) {
  const bool trace = std::getenv("MOE_B200_TRACE_KERNELS") != nullptr;
  if (trace) {
    std::fprintf(stderr, "MOE_B200_KERNEL_BEGIN %s impl=%p\n", op_name(kern),
                 static_cast<void*>(kern));
    std::fflush(stderr);
  }
  int rc = kernel_compute_impl(kern, num_inputs, in, output, stream);
  if (trace) {
    if (rc == MOE_B200_OK && std::getenv("MOE_B200_TRACE_SYNC") != nullptr) {
      const cudaError_t st = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
      if (st != cudaSuccess)
        rc = efail(MOE_B200_EP_FAIL, "stream synchronize: %s", cudaGetErrorString(st));
    }
    std::fprintf(stderr, "MOE_B200_KERNEL_END %s impl=%p status=%d\n", op_name(kern),
                 static_cast<void*>(kern), rc);
    std::fflush(stderr);
  }
  return rc;
}

static int kernel_compute_impl(moe_b200_kernel* kern, int32_t num_inputs,
                               const moe_b200_tensor_ref* in, moe_b200_tensor_ref* output,
                               void* stream) {
  moe::clear_stale_cuda_error();
  if (kern == nullptr || in == nullptr || output == nullptr)
    return (efail(MOE_B200_INVALID_ARGUMENT, "kernel, inputs and output must be non-NULL"));
  const bool q = kern->quantized;
  // Schema input slots.
  const int kInput = 0, kRouter = 1;
  const int kFc1W = 2, kFc1S = q ? 3 : -1, kFc1B = q ? 4 : 3;
  const int kFc2W = q ? 5 : 4, kFc2S = q ? 6 : -1, kFc2B = q ? 7 : 5;
  const int kFc3W = q ? 8 : 6, kFc3S = q ? 9 : -1, kFc3B = q ? 10 : 7;
  const int max_inputs = q ? 14 : 8;
  if (num_inputs < (q ? 7 : 5) || num_inputs > max_inputs)
    return (efail(MOE_B200_INVALID_ARGUMENT, "%s takes %d..%d inputs, got %d",
                        q ? "QMoE" : "MoE", q ? 7 : 5, max_inputs, num_inputs));
  // An input is present when it has data or is a zero-size tensor (whose data
  // pointer may legitimately be NULL); absent optional inputs have rank 0, no data.
  auto present = [&](const moe_b200_tensor_ref& t) {
    if (t.data != nullptr) return true;
    if (t.rank <= 0 || t.rank > 4) return false;
    for (int d = 0; d < t.rank; ++d)
      if (t.dims[d] == 0) return true;
    return false;
  };
  auto get = [&](int i) -> const moe_b200_tensor_ref* {
    if (i < 0 || i >= num_inputs || !present(in[i])) return nullptr;
    return &in[i];
  };
  if (q) {
    for (int i = 11; i < num_inputs; ++i)
      if (in[i].data != nullptr)
        return (efail(MOE_B200_NOT_IMPLEMENTED,
                            "QMoE zero-point inputs (asymmetric weights) are not supported"));
  }
  const moe_b200_tensor_ref* x = get(kInput);
  const moe_b200_tensor_ref* r = get(kRouter);
  const moe_b200_tensor_ref* w1 = get(kFc1W);
  const moe_b200_tensor_ref* w2 = get(kFc2W);
  const moe_b200_tensor_ref* w3 = get(kFc3W);
  if (!x || !r || !w1 || !w2)
    return (efail(MOE_B200_INVALID_ARGUMENT, "input, router_probs, fc1 and fc2 weights are required"));
  const int dt = x->elem_type;
  if (dt != MOE_B200_FLOAT && dt != MOE_B200_FLOAT16 && dt != MOE_B200_BFLOAT16)
    return (efail(MOE_B200_NOT_IMPLEMENTED, "input element type %d is not supported", dt));
  if (x->rank != 2 && x->rank != 3)
    return (efail(MOE_B200_INVALID_ARGUMENT, "input must be 2-D or 3-D, got %s",
                        shape_str(*x).c_str()));
  const int64_t H = x->dims[x->rank - 1];
  const int64_t T = numel_prefix(*x, x->rank - 1);
  if (r->rank != 2 || r->dims[0] != T || r->elem_type != dt)
    return (efail(MOE_B200_INVALID_ARGUMENT, "router_probs must be [%lld, E] of the input type, got %s",
                        (long long)T, shape_str(*r).c_str()));
  const int64_t E = r->dims[1];
  const int bits = q ? kern->attrs.expert_weight_bits : 16;
  const int wdt = q ? MOE_B200_UINT8 : dt;
  auto packed = [&](int64_t K) { return q ? K * bits / 8 : K; };
  if (w1->rank != 3 || w1->dims[0] != E || w1->dims[2] != packed(H) || w1->elem_type != wdt)
    return (efail(MOE_B200_INVALID_ARGUMENT, "fc1_experts_weights must be [%lld, N, %lld], got %s",
                        (long long)E, (long long)packed(H), shape_str(*w1).c_str()));
  if (w2->rank != 3 || w2->dims[0] != E || w2->dims[1] != H || w2->elem_type != wdt)
    return (efail(MOE_B200_INVALID_ARGUMENT, "fc2_experts_weights must be [%lld, %lld, I], got %s",
                        (long long)E, (long long)H, shape_str(*w2).c_str()));
  const int64_t I = q ? w2->dims[2] * 8 / bits : w2->dims[2];
  const bool fused = kern->attrs.activation_type == MOE_B200_ACT_SWIGLU && kern->attrs.swiglu_fusion != 0;
  const int64_t N1 = fused ? 2 * I : I;
  if (w1->dims[1] != N1)
    return (efail(MOE_B200_INVALID_ARGUMENT, "fc1_experts_weights has %lld rows, expected %lld",
                        (long long)w1->dims[1], (long long)N1));
  if (w3 && (w3->rank != 3 || w3->dims[0] != E || w3->dims[1] != I || w3->dims[2] != packed(H) ||
             w3->elem_type != wdt))
    return (efail(MOE_B200_INVALID_ARGUMENT, "fc3_experts_weights must be [%lld, %lld, %lld], got %s",
                        (long long)E, (long long)I, (long long)packed(H), shape_str(*w3).c_str()));
  auto check_bias = [&](int slot, int64_t n, const char* name) -> int {
    const moe_b200_tensor_ref* b = get(slot);
    if (!b) return MOE_B200_OK;
    if (b->rank != 2 || b->dims[0] != E || b->dims[1] != n || b->elem_type != dt)
      return efail(MOE_B200_INVALID_ARGUMENT, "%s must be [%lld, %lld], got %s", name,
                   (long long)E, (long long)n, shape_str(*b).c_str());
    return MOE_B200_OK;
  };
  int st = check_bias(kFc1B, N1, "fc1_experts_bias");
  if (st == MOE_B200_OK) st = check_bias(kFc2B, H, "fc2_experts_bias");
  if (st == MOE_B200_OK) st = check_bias(kFc3B, I, "fc3_experts_bias");
  if (st != MOE_B200_OK) return (st);
  if (get(kFc3B) && !w3)
    return (efail(MOE_B200_INVALID_ARGUMENT, "fc3_experts_bias given without fc3 weights"));
  if (q) {
    const int bs = kern->attrs.block_size;
    auto check_scales = [&](int slot, int64_t n, int64_t K, const char* name) -> int {
      const moe_b200_tensor_ref* s = get(slot);
      if (!s) return efail(MOE_B200_INVALID_ARGUMENT, "%s is required", name);
      const int64_t nb = bs ? (K + bs - 1) / bs : 0;
      const bool ok = s->elem_type == dt && s->dims[0] == E && s->dims[1] == n &&
                      (bs ? (s->rank == 3 && s->dims[2] == nb) : s->rank == 2);
      if (!ok) return efail(MOE_B200_INVALID_ARGUMENT, "%s has shape %s", name, shape_str(*s).c_str());
      return MOE_B200_OK;
    };
    st = check_scales(kFc1S, N1, H, "fc1_scales");
    if (st == MOE_B200_OK) st = check_scales(kFc2S, H, I, "fc2_scales");
    if (st == MOE_B200_OK && w3) st = check_scales(kFc3S, I, H, "fc3_scales");
    if (st != MOE_B200_OK) return (st);
  }
  if (!present(*output) || output->elem_type != dt || output->rank != x->rank)
    return (efail(MOE_B200_INVALID_ARGUMENT, "output must match the input's type and rank"));
  for (int i = 0; i < x->rank; ++i)
    if (output->dims[i] != x->dims[i])
      return (efail(MOE_B200_INVALID_ARGUMENT, "output shape %s differs from input %s",
                          shape_str(*output).c_str(), shape_str(*x).c_str()));

  moe_b200_problem p{};
  p.num_rows = T;
  p.hidden_size = H;
  p.inter_size = I;
  p.num_experts = E;
  p.dtype = dt;
  p.has_fc3 = w3 != nullptr;
  p.attrs = kern->attrs;
  if (!q) p.attrs.expert_weight_bits = 0;
  const moe_b200_prepacked* pk = nullptr;
  if (q && kern->pk != nullptr) {
    const void* src[6] = {w1->data, in[kFc1S].data, w2->data, in[kFc2S].data,
                          w3 ? w3->data : nullptr, w3 ? in[kFc3S].data : nullptr};
    if (std::memcmp(src, kern->pk_src, sizeof(src)) == 0) pk = kern->pk;
  }
  size_t need = 0;
  st = moe_b200_workspace_size_prepacked(&p, pk, &need);
  if (st != MOE_B200_OK) return st;

  moe_b200_tensors t{};
  t.input = x->data;
  t.router_probs = r->data;
  t.fc1_weights = w1->data;
  t.fc1_bias = get(kFc1B) ? in[kFc1B].data : nullptr;
  t.fc2_weights = w2->data;
  t.fc2_bias = get(kFc2B) ? in[kFc2B].data : nullptr;
  t.fc3_weights = w3 ? w3->data : nullptr;
  t.fc3_bias = get(kFc3B) ? in[kFc3B].data : nullptr;
  if (q) {
    t.fc1_scales = in[kFc1S].data;
    t.fc2_scales = in[kFc2S].data;
    t.fc3_scales = w3 ? in[kFc3S].data : nullptr;
  }
  t.output = const_cast<void*>(output->data);

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  void* wsp = nullptr;
  {
    std::lock_guard<std::mutex> lock(kern->mu);
    auto& w = kern->ws[s];
    if (w.bytes < need) {
      if (w.ptr) cudaFreeAsync(w.ptr, s);
      w.ptr = nullptr;
      w.bytes = 0;
      cudaError_t ce = cudaMallocAsync(&w.ptr, need, s);
      if (ce != cudaSuccess)
        return (efail(MOE_B200_EP_FAIL, "workspace allocation of %zu bytes: %s", need,
                            cudaGetErrorString(ce)));
      w.bytes = need;
    }
    wsp = w.ptr;
    // The call below only enqueues work on `s`; a concurrent caller on another
    // stream has its own workspace, and callers sharing a stream are ordered by it.
  }
  return moe_b200_forward_prepacked(&p, &t, pk, wsp, need, stream, nullptr, 0);
}

int moe_b200_kernel_prepack(moe_b200_kernel* kern, int32_t num_inputs,
                            const moe_b200_tensor_ref* in, int32_t share, void* stream,
                            int32_t* is_packed) {
  moe::clear_stale_cuda_error();
  if (kern == nullptr || in == nullptr)
    return (efail(MOE_B200_INVALID_ARGUMENT, "kernel and inputs must be non-NULL"));
  if (is_packed != nullptr) *is_packed = 0;
  if (!kern->quantized)
    return MOE_B200_OK;  // MoE weights are used as given: nothing to pack
  // QMoE schema slots: fc1 w/s/b 2..4, fc2 w/s/b 5..7, fc3 w/s/b 8..10.
  if (num_inputs < 7)
    return (efail(MOE_B200_INVALID_ARGUMENT, "QMoE pre-pack needs inputs up to fc2_experts_bias"));
  const moe_b200_tensor_ref& w1 = in[2];
  const moe_b200_tensor_ref& s1 = in[3];
  const moe_b200_tensor_ref& w2 = in[5];
  const moe_b200_tensor_ref& s2 = in[6];
  const bool has3 = num_inputs > 8 && in[8].data != nullptr;
  if (w1.data == nullptr || w2.data == nullptr || s1.data == nullptr || s2.data == nullptr ||
      w1.rank != 3 || w2.rank != 3 || s1.rank < 2)
    return (efail(MOE_B200_INVALID_ARGUMENT, "QMoE pre-pack: fc1/fc2 weights and scales are required"));
  if (has3 && (num_inputs < 10 || in[9].data == nullptr))
    return (efail(MOE_B200_INVALID_ARGUMENT, "QMoE pre-pack: fc3_scales is required with fc3 weights"));
  const int bits = kern->attrs.expert_weight_bits;
  moe_b200_problem p{};
  p.num_rows = 0;
  p.num_experts = w1.dims[0];
  p.hidden_size = w2.dims[1];
  p.inter_size = w2.dims[2] * 8 / bits;
  p.dtype = s1.elem_type;
  p.has_fc3 = has3 ? 1 : 0;
  p.attrs = kern->attrs;
  if (w1.dims[2] * 8 / bits != p.hidden_size || w1.elem_type != MOE_B200_UINT8 ||
      w2.elem_type != MOE_B200_UINT8)
    return (efail(MOE_B200_INVALID_ARGUMENT, "QMoE pre-pack: fc1 %s and fc2 %s weights disagree",
                  shape_str(w1).c_str(), shape_str(w2).c_str()));
  const int64_t n1 = (p.attrs.activation_type == MOE_B200_ACT_SWIGLU && p.attrs.swiglu_fusion != 0)
                         ? 2 * p.inter_size : p.inter_size;
  if (w1.dims[1] != n1)
    return (efail(MOE_B200_INVALID_ARGUMENT, "QMoE pre-pack: fc1 has %lld rows, expected %lld",
                  (long long)w1.dims[1], (long long)n1));
  moe_b200_tensors t{};
  t.fc1_weights = w1.data;
  t.fc1_scales = s1.data;
  t.fc2_weights = w2.data;
  t.fc2_scales = s2.data;
  t.fc3_weights = has3 ? in[8].data : nullptr;
  t.fc3_scales = has3 ? in[9].data : nullptr;
  moe_b200_prepacked* pk = nullptr;
  int st = moe_b200_prepack_create(&p, &t, share, stream, &pk);
  if (st != MOE_B200_OK) return st;
  std::lock_guard<std::mutex> lock(kern->mu);
  if (kern->pk != nullptr) moe_b200_prepack_release(kern->pk);
  kern->pk = pk;
  const void* src[6] = {t.fc1_weights, t.fc1_scales, t.fc2_weights, t.fc2_scales,
                        t.fc3_weights, t.fc3_scales};
  std::memcpy(kern->pk_src, src, sizeof(src));
  return MOE_B200_OK;
}

int moe_b200_kernel_release(moe_b200_kernel* kern) {
  if (kern == nullptr) return MOE_B200_OK;
  if (std::getenv("MOE_B200_TRACE_KERNELS") != nullptr) {
    std::fprintf(stderr, "MOE_B200_KERNEL_RELEASE %s impl=%p\n", op_name(kern),
                 static_cast<void*>(kern));
    std::fflush(stderr);
  }
  {
    std::lock_guard<std::mutex> lock(kern->mu);
    for (auto& kv : kern->ws)
      if (kv.second.ptr) {
        cudaStreamSynchronize(kv.first);
        cudaFree(kv.second.ptr);
      }
    kern->ws.clear();
    if (kern->pk != nullptr) moe_b200_prepack_release(kern->pk);
    kern->pk = nullptr;
  }
  delete kern;
  return MOE_B200_OK;
}

// ------------------------------------------------------------- provider options
namespace {

bool parse_whole_int(const char* v, int32_t* out) {
  if (v == nullptr || *v == '\0') return false;
  char* end = nullptr;
  errno = 0;
  const long x = std::strtol(v, &end, 10);
  if (errno != 0 || end == v || *end != '\0' || x < INT32_MIN || x > INT32_MAX) return false;
  *out = static_cast<int32_t>(x);
  return true;
}

}  // namespace

int moe_b200_provider_options_parse(int32_t num_options, const char* const* keys,
                                    const char* const* values,
                                    moe_b200_provider_options* o) {
  if (o == nullptr || num_options < 0 || (num_options > 0 && (keys == nullptr || values == nullptr)))
    return (efail(MOE_B200_INVALID_ARGUMENT, "options, keys and values must be non-NULL"));
  moe_b200_provider_options r{};
  r.do_copy_in_default_stream = 1;
  r.ep_world_size = 1;
  struct IntKey { const char* name; int32_t* dst; };
  const IntKey ints[] = {{"device_id", &r.device_id},
                         {"has_user_compute_stream", &r.has_user_compute_stream},
                         {"use_ep_level_unified_stream", &r.use_ep_level_unified_stream},
                         {"do_copy_in_default_stream", &r.do_copy_in_default_stream},
                         {"ep_world_size", &r.ep_world_size},
                         {"ep_rank", &r.ep_rank}};
  for (int i = 0; i < num_options; ++i) {
    const char* k = keys[i];
    const char* v = values[i] != nullptr ? values[i] : "";
    if (k == nullptr) return (efail(MOE_B200_INVALID_ARGUMENT, "option key %d is NULL", i));
    bool known = false;
    for (const IntKey& ik : ints) {
      if (std::strcmp(k, ik.name) != 0) continue;
      known = true;
      if (!parse_whole_int(v, ik.dst))
        return (efail(MOE_B200_INVALID_ARGUMENT,
                      "Invalid provider option '%s': expected integer, got '%s'.", k, v));
    }
    if (known) continue;
    if (!std::strcmp(k, "user_compute_stream")) {
      if (*v == '\0' || !std::strcmp(v, "0") || !std::strcmp(v, "nullptr")) {
        r.user_compute_stream = nullptr;
        continue;
      }
      char* end = nullptr;
      errno = 0;
      const unsigned long long x = std::strtoull(v, &end, 0);
      if (errno != 0 || end == v || *end != '\0')
        return (efail(MOE_B200_INVALID_ARGUMENT,
                      "Invalid provider option 'user_compute_stream': expected uintptr_t "
                      "string, got '%s'.", v));
      r.user_compute_stream = reinterpret_cast<void*>(static_cast<uintptr_t>(x));
    } else if (!std::strcmp(k, "ep.musa.enable_prepack_weight_sharing")) {
      r.enable_prepack_weight_sharing = std::strcmp(v, "1") == 0 ? 1 : 0;  // "1" enables
    }
  }
  if (r.user_compute_stream != nullptr) r.has_user_compute_stream = 1;
  if (r.device_id < 0)
    return (efail(MOE_B200_INVALID_ARGUMENT,
                  "Provider option 'device_id' must be a non-negative integer."));
  const IntKey flags[] = {{"has_user_compute_stream", &r.has_user_compute_stream},
                          {"use_ep_level_unified_stream", &r.use_ep_level_unified_stream},
                          {"do_copy_in_default_stream", &r.do_copy_in_default_stream}};
  for (const IntKey& f : flags)
    if (*f.dst != 0 && *f.dst != 1)
      return (efail(MOE_B200_INVALID_ARGUMENT,
                    "Invalid provider option '%s': expected 0 or 1, got %d.", f.name, *f.dst));
  if (r.has_user_compute_stream && r.user_compute_stream == nullptr)
    return (efail(MOE_B200_INVALID_ARGUMENT,
                  "Provider option 'has_user_compute_stream' is set but "
                  "'user_compute_stream' is null."));
  if (r.has_user_compute_stream) r.use_ep_level_unified_stream = 1;
  if (r.ep_world_size < 1 || r.ep_rank < 0 || r.ep_rank >= r.ep_world_size)
    return (efail(MOE_B200_INVALID_ARGUMENT,
                  "ep_world_size >= 1 and 0 <= ep_rank < ep_world_size required (got %d / %d)",
                  r.ep_world_size, r.ep_rank));
  *o = r;
  return MOE_B200_OK;
}

// ------------------------------------------------------------------ runtime layer
#define RT_CHECK(expr, what)                                                            \
  do {                                                                                  \
    cudaError_t _st = (expr);                                                           \
    if (_st != cudaSuccess) {                                                           \
      (void)cudaGetLastError(); /* the failure is returned here, not left behind */      \
      return (efail(MOE_B200_EP_FAIL, "%s: %s", what, cudaGetErrorString(_st)));         \
    }                                                                                   \
  } while (0)

int moe_b200_device_count(int32_t* count) {
  if (!count) return (efail(MOE_B200_INVALID_ARGUMENT, "count is NULL"));
  int n = 0;
  cudaError_t st = cudaGetDeviceCount(&n);
  *count = st == cudaSuccess ? n : 0;  // no driver / no device: zero devices, not an error
  return MOE_B200_OK;
}

int moe_b200_device_props_get(int32_t device_id, moe_b200_device_props* props) {
  if (!props) return (efail(MOE_B200_INVALID_ARGUMENT, "props is NULL"));
  cudaDeviceProp dp;
  RT_CHECK(cudaGetDeviceProperties(&dp, device_id), "cudaGetDeviceProperties");
  std::memset(props, 0, sizeof(*props));
  std::snprintf(props->name, sizeof(props->name), "%s", dp.name);
  props->vendor_id = 0x10DE;
  props->device_id = device_id;
  props->sm_count = dp.multiProcessorCount;
  props->cc_major = dp.major;
  props->cc_minor = dp.minor;
  props->total_memory = dp.totalGlobalMem;
  props->pci_bus_id = dp.pciBusID;
  return MOE_B200_OK;
}

int moe_b200_set_device(int32_t device_id) {
  RT_CHECK(cudaSetDevice(device_id), "cudaSetDevice");
  return MOE_B200_OK;
}

int moe_b200_alloc(size_t bytes, void** ptr) {
  if (!ptr) return (efail(MOE_B200_INVALID_ARGUMENT, "ptr is NULL"));
  *ptr = nullptr;
  if (bytes == 0) return MOE_B200_OK;
  RT_CHECK(cudaMalloc(ptr, bytes), "cudaMalloc");
  return MOE_B200_OK;
}

int moe_b200_free(void* ptr) {
  if (ptr) RT_CHECK(cudaFree(ptr), "cudaFree");
  return MOE_B200_OK;
}

int moe_b200_alloc_pinned(size_t bytes, void** ptr) {
  if (!ptr) return (efail(MOE_B200_INVALID_ARGUMENT, "ptr is NULL"));
  *ptr = nullptr;
  if (bytes == 0) return MOE_B200_OK;
  RT_CHECK(cudaHostAlloc(ptr, bytes, cudaHostAllocDefault), "cudaHostAlloc");
  return MOE_B200_OK;
}

int moe_b200_free_pinned(void* ptr) {
  if (ptr) RT_CHECK(cudaFreeHost(ptr), "cudaFreeHost");
  return MOE_B200_OK;
}

int moe_b200_stream_create(void** stream) {
  if (!stream) return (efail(MOE_B200_INVALID_ARGUMENT, "stream is NULL"));
  cudaStream_t s = nullptr;
  RT_CHECK(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate");
  *stream = s;
  return MOE_B200_OK;
}

int moe_b200_stream_destroy(void* stream) {
  if (stream) {
    RT_CHECK(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "cudaStreamSynchronize");
    RT_CHECK(cudaStreamDestroy(static_cast<cudaStream_t>(stream)), "cudaStreamDestroy");
  }
  return MOE_B200_OK;
}

int moe_b200_stream_synchronize(void* stream) {
  RT_CHECK(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "cudaStreamSynchronize");
  return MOE_B200_OK;
}

int moe_b200_notification_create(void** event) {
  if (!event) return (efail(MOE_B200_INVALID_ARGUMENT, "event is NULL"));
  cudaEvent_t e = nullptr;
  RT_CHECK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
  *event = e;
  return MOE_B200_OK;
}

int moe_b200_notification_activate(void* event, void* stream) {
  RT_CHECK(cudaEventRecord(static_cast<cudaEvent_t>(event), static_cast<cudaStream_t>(stream)),
           "cudaEventRecord");
  return MOE_B200_OK;
}

int moe_b200_notification_wait(void* event, void* stream) {
  RT_CHECK(cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), static_cast<cudaEvent_t>(event), 0),
           "cudaStreamWaitEvent");
  return MOE_B200_OK;
}

int moe_b200_notification_synchronize(void* event) {
  RT_CHECK(cudaEventSynchronize(static_cast<cudaEvent_t>(event)), "cudaEventSynchronize");
  return MOE_B200_OK;
}

int moe_b200_notification_destroy(void* event) {
  if (event) RT_CHECK(cudaEventDestroy(static_cast<cudaEvent_t>(event)), "cudaEventDestroy");
  return MOE_B200_OK;
}

// Ordering follows MusaDataTransfer::CopyImpl (musa/ep/src/ep_data_transfer.cc:108-161):
// device-bound copies are stream-ordered and return at once; a device-to-host copy with a
// stream waits for that stream only (other workers' streams keep running), and without
// one waits for the whole device first, since a synchronous copy on the legacy stream does
// not order work on non-blocking streams; host-to-host copies wait for the given stream
// (the producer of the source) and then copy on the host.
int moe_b200_copy(void* dst, const void* src, size_t bytes, int32_t kind, void* stream) {
  if (bytes == 0 || dst == src) return MOE_B200_OK;
  if (!dst || !src) return (efail(MOE_B200_INVALID_ARGUMENT, "copy with NULL pointer"));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (kind) {
    case 0:
      if (s) RT_CHECK(cudaStreamSynchronize(s), "cudaStreamSynchronize");
      std::memcpy(dst, src, bytes);
      return MOE_B200_OK;
    case 1:
      RT_CHECK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, s), "cudaMemcpyAsync");
      return MOE_B200_OK;
    case 2:
      if (!s) RT_CHECK(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
      RT_CHECK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, s), "cudaMemcpyAsync");
      RT_CHECK(cudaStreamSynchronize(s), "cudaStreamSynchronize");
      return MOE_B200_OK;
    case 3:
      RT_CHECK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, s), "cudaMemcpyAsync");
      return MOE_B200_OK;
    default:
      return (efail(MOE_B200_INVALID_ARGUMENT, "copy kind %d", kind));
  }
}

}  // extern "C"
