// Host side of libmoe_b200: problem validation, workspace planning, the launch
// sequence of one MoE / QMoE layer call, the per-node kernel object and the thin
// CUDA runtime layer that stands in for the reference's MUSA runtime plumbing.
//
// Call sequence of one layer (all on the caller's stream, no host sync):
//   route       softmax/top-k per row + per-chunk expert histogram
//   plan        per-expert offsets (exclusive scan), GEMM tile prefixes, stable
//               permutation (expert, token, slot)
//   gather      x rows -> expert-contiguous activations Xp
//   fc1(+fc3)   grouped GEMM, activation fused in the epilogue  -> act [R, I]
//   fc2         grouped GEMM, bias fused                          -> Y [R, H] (aliases Xp)
//   combine     out[t] = sum_j w[t, j] * Y[pos[t, j]]
#include <nvtx3/nvToolsExt.h>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/moe_b200.h"
#include "ep_p2p.h"
#include "moe_kernels.h"
#include "prepack.h"
#include "qmoe.h"

using namespace moe;

// ------------------------------------------------------------------ errors
namespace {

thread_local std::string g_last_error;

}  // namespace

bool moe::pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("MOE_B200_PDL");
    return v == nullptr || std::strcmp(v, "0") != 0;
  }();
  return on;
}

bool moe::pdl_layer_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("MOE_B200_PDL_LAYER");
    return v != nullptr && std::strcmp(v, "0") != 0 && v[0] != '\0';
  }();
  return on;
}

int moe::set_error(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

namespace {

template <typename... A>
int fail(int code, const char* fmt, A... args) {
  return moe::set_error(code, fmt, args...);
}
int fail(int code, const char* msg) { return moe::set_error(code, "%s", msg); }

int cuda_fail(cudaError_t st, const char* what) {
  return fail(MOE_B200_EP_FAIL, "%s: %s", what, cudaGetErrorString(st));
}

#define MOE_CUDA_CHECK(expr, what)                   \
  do {                                               \
    cudaError_t _st = (expr);                        \
    if (_st != cudaSuccess) return cuda_fail(_st, what); \
  } while (0)

bool env_flag(const char* name) {
  const char* v = std::getenv(name);
  return v != nullptr && v[0] != '\0' && std::strcmp(v, "0") != 0;
}

int device_sm_count() {
  static int counts[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (counts[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    counts[dev] = n > 0 ? n : 148;
  }
  return counts[dev];
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

bool is_float_type(int dt) {
  return dt == MOE_B200_FLOAT || dt == MOE_B200_FLOAT16 || dt == MOE_B200_BFLOAT16;
}

// ------------------------------------------------------------ workspace plan
struct WsLayout {
  size_t idx, w, chunk_counts, chunk_base, offsets, tiles128, tiles64, tiles256, pos, src, err;
  size_t rowsum, comb, xp, act, qmoe, total;
};

// Smallest inter_size (fc2's K) at which the combine runs inside the fc2 epilogue.
constexpr int64_t kFusedCombineMinInter = 4096;

bool swiglu_fused(const moe_b200_problem& p) {
  return p.attrs.activation_type == MOE_B200_ACT_SWIGLU && p.attrs.swiglu_fusion != 0;
}

// `prepacked`: the call runs on prepacked weights (no dequantised copies in the workspace).
WsLayout plan_workspace(const moe_b200_problem& p, bool prepacked = false) {
  WsLayout L{};
  const int64_t T = p.num_rows, E = p.num_experts, k = p.attrs.k;
  const int64_t R = T * k;
  const int64_t chunks = num_route_chunks(T, layer_route_chunk(T));
  const size_t es = static_cast<size_t>(dtype_bytes(p.dtype));
  size_t o = 0;
  auto take = [&](size_t bytes) { size_t at = o; o = align_up(o + bytes, 256); return at; };
  L.idx = take(R * 4);
  L.w = take(R * 4);
  L.chunk_counts = take(std::max<int64_t>(chunks, 1) * E * 4);
  L.chunk_base = take(std::max<int64_t>(chunks, 1) * E * 4);
  L.offsets = take((E + 1) * 4);
  L.tiles128 = take((E + 1) * 4);
  L.tiles64 = take((E + 1) * 4);
  L.tiles256 = take((E + 1) * 4);
  L.pos = take(R * 4);
  L.src = take(R * 4);
  L.err = take(16);
  L.rowsum = take(R * 4);                // A row sums of the packed (QMoE) GEMMs
  L.comb = take(T * ((p.hidden_size + 31) / 32) * 4);  // fused-combine arrival counters
  L.xp = take(R * p.hidden_size * es);   // gathered input, later fc2 output
  L.act = take(R * p.inter_size * es);
  L.qmoe = take(prepacked ? 0 : qmoe_workspace_bytes(p));
  L.total = o;
  return L;
}

// Routing mode of a layer call (launch_route's `normalize` argument).
int route_mode(const moe_b200_problem& p) {
  return p.attrs.use_sparse_mixer ? kRouteSparseMixer : (p.attrs.normalize_routing_weights ? 1 : 0);
}

int validate_problem(const moe_b200_problem* p) {
  if (p == nullptr) return fail(MOE_B200_INVALID_ARGUMENT, "problem is NULL");
  if (!is_float_type(p->dtype))
    return fail(MOE_B200_NOT_IMPLEMENTED, "unsupported element type %d", p->dtype);
  if (p->num_rows < 0 || p->hidden_size <= 0 || p->inter_size <= 0 || p->num_experts <= 0)
    return fail(MOE_B200_INVALID_ARGUMENT,
                "invalid shape: num_rows=%lld hidden=%lld inter=%lld experts=%lld",
                (long long)p->num_rows, (long long)p->hidden_size, (long long)p->inter_size,
                (long long)p->num_experts);
  if (p->num_experts > kMaxExperts)
    return fail(MOE_B200_NOT_IMPLEMENTED, "num_experts=%lld exceeds %d",
                (long long)p->num_experts, kMaxExperts);
  const auto& a = p->attrs;
  if (a.k < 1 || a.k > p->num_experts || a.k > kMaxK)
    return fail(MOE_B200_INVALID_ARGUMENT, "k=%d must be in [1, min(num_experts, %d)]", a.k,
                kMaxK);
  if (a.activation_type < MOE_B200_ACT_RELU || a.activation_type > MOE_B200_ACT_SWIGLU)
    return fail(MOE_B200_INVALID_ARGUMENT, "invalid activation_type %d", a.activation_type);
  if (a.use_sparse_mixer != 0 && a.use_sparse_mixer != 1)
    return fail(MOE_B200_INVALID_ARGUMENT, "use_sparse_mixer=%d must be 0 or 1", a.use_sparse_mixer);
  if (a.use_sparse_mixer != 0 && a.k != 2)
    return fail(MOE_B200_INVALID_ARGUMENT, "use_sparse_mixer=1 routes top-2: k=%d must be 2", a.k);
  if (a.swiglu_fusion < 0 || a.swiglu_fusion > 2)
    return fail(MOE_B200_INVALID_ARGUMENT, "swiglu_fusion=%d must be 0, 1 or 2", a.swiglu_fusion);
  if (a.activation_type == MOE_B200_ACT_SWIGLU && a.swiglu_fusion == 0 && !p->has_fc3)
    return fail(MOE_B200_INVALID_ARGUMENT,
                "activation_type=swiglu with swiglu_fusion=0 needs fc3 weights");
  if (a.swiglu_fusion != 0 && p->has_fc3)
    return fail(MOE_B200_INVALID_ARGUMENT, "fused swiglu (swiglu_fusion=%d) excludes fc3",
                a.swiglu_fusion);
  if (a.expert_weight_bits != 0 && a.expert_weight_bits != 4 && a.expert_weight_bits != 8)
    return fail(MOE_B200_INVALID_ARGUMENT, "expert_weight_bits=%d must be 4 or 8",
                a.expert_weight_bits);
  if (a.expert_weight_bits != 0) {
    if (p->dtype == MOE_B200_FLOAT)
      return fail(MOE_B200_NOT_IMPLEMENTED, "QMoE with float32 activations is not supported");
    if (a.block_size != 0 && (a.block_size < 16 || (a.block_size & (a.block_size - 1)) != 0))
      return fail(MOE_B200_INVALID_ARGUMENT,
                  "block_size=%d must be 0 or a power of two >= 16", a.block_size);
    if (a.expert_weight_bits == 4 && ((p->hidden_size | p->inter_size) & 1))
      return fail(MOE_B200_INVALID_ARGUMENT, "4-bit weights need even hidden and inter sizes");
  }
  const int64_t R = p->num_rows * a.k;
  if (R > (int64_t)1 << 30)
    return fail(MOE_B200_INVALID_ARGUMENT, "num_rows * k = %lld is too large", (long long)R);
  return MOE_B200_OK;
}

ActParams act_params(const moe_b200_attrs& a) {
  ActParams ap;
  ap.act = a.activation_type;
  ap.alpha = a.activation_alpha;
  ap.beta = a.activation_beta;
  ap.limit = a.swiglu_limit;
  return ap;
}

// fc1 (+fc3) pass description for MoE weights of element type p.dtype (or the
// dequantised copies of QMoE weights).
GemmArgs fc1_args(const moe_b200_problem& p, const void* w1, const void* b1, const void* w3,
                  const void* b3) {
  const int I = static_cast<int>(p.inter_size);
  const int H = static_cast<int>(p.hidden_size);
  GemmArgs g{};
  g.dtype = p.dtype;
  g.K = H;
  g.N = I;
  g.E = static_cast<int>(p.num_experts);
  g.ap = act_params(p.attrs);
  g.bias_stride = 1;
  if (p.has_fc3) {
    g.gated = true;
    g.b1 = {w1, 0, 1, 0, I};
    g.b3 = {w3, 0, 1, 0, I};
    g.bias1 = b1;
    g.bias3 = b3;
    g.bias_e_stride = I;
  } else if (swiglu_fused(p)) {
    const size_t es = dtype_bytes(p.dtype);
    g.gated = true;
    g.bias_e_stride = 2 * I;
    if (p.attrs.swiglu_fusion == 1) {
      g.b1 = {w1, 0, 2, 0, 2 * I};
      g.b3 = {w1, 1, 2, 0, 2 * I};
      g.bias1 = b1;
      g.bias3 = b1 ? static_cast<const uint8_t*>(b1) + es : nullptr;
      g.bias_stride = 2;
    } else {
      g.b1 = {w1, 0, 1, 0, 2 * I};
      g.b3 = {w1, 0, 1, I, 2 * I};
      g.bias1 = b1;
      g.bias3 = b1 ? static_cast<const uint8_t*>(b1) + es * I : nullptr;
    }
  } else {
    g.gated = false;
    g.b1 = {w1, 0, 1, 0, I};
    g.bias1 = b1;
    g.bias_e_stride = I;
  }
  return g;
}

GemmArgs fc2_args(const moe_b200_problem& p, const void* w2, const void* b2) {
  const int I = static_cast<int>(p.inter_size);
  const int H = static_cast<int>(p.hidden_size);
  GemmArgs g{};
  g.dtype = p.dtype;
  g.K = I;
  g.N = H;
  g.E = static_cast<int>(p.num_experts);
  g.gated = false;
  g.b1 = {w2, 0, 1, 0, H};
  g.bias1 = b2;
  g.bias_stride = 1;
  g.bias_e_stride = H;
  g.ap = ActParams{kIdentity, 1.f, 0.f, INFINITY};
  return g;
}

// MOE_B200_FORCE_SIMT=1 selects the FFMA GEMMs; MOE_B200_TC_MODE=1|2 forces the
// single-CTA or CTA-pair tensor-core kernel (used by tests to cover both);
// MOE_B200_PAIR_SWAP_MAX overrides the swapped-tail-tile limit.
cudaError_t run_gemm(GemmArgs& g, cudaStream_t s) {
  const bool tc = !env_flag("MOE_B200_FORCE_SIMT") && tc_supported(g);
  const char* m = std::getenv("MOE_B200_TC_MODE");
  const int mode = m ? std::atoi(m) : 0;
  // A gathered A (set only with MOE_B200_GATHER_FUSION=1): the CTA-pair kernel loads the
  // rows itself with TMA gather4 (four 128-byte rows per instruction); other kernels get
  // a gather pass into g.a first.  The fused loads are exact but slower on B200 (C2 fc1
  // 4.39 ms against 1.62 ms with the separate gather): at about 90 cycles per gather4, the
  // 32 instructions a 128-row A tile needs per k-block take ~4x the k-block's MMA time.
  if (g.gather_src != nullptr) {
    const bool fuse = tc && tc_pair_gathers(g, mode);
    if (!fuse) {
      cudaError_t st = launch_gather(g.gather_x, static_cast<int64_t>(g.K) * dtype_bytes(g.dtype),
                                     g.gather_k, g.gather_src, g.rows, const_cast<void*>(g.a), s);
      if (st != cudaSuccess) return st;
      g.gather_src = nullptr;
      g.gather_x = nullptr;
    }
  }
  if (tc) {
    // MOE_B200_PAIR_SWAP_MAX: row limit of the pair kernel's swapped tail tiles (0 = off).
    if (const char* sw = std::getenv("MOE_B200_PAIR_SWAP_MAX")) g.swap_max = std::atoi(sw);
    // MOE_B200_PAIR_STATIC=1: static round-robin tile schedule (comparison runs).
    if (env_flag("MOE_B200_PAIR_STATIC")) g.tile_counter = nullptr;
    return launch_gemm_tc(g, device_sm_count(), mode, s);
  }
  // The FFMA kernels apply no per-row scales: exact-code weights need the tensor cores.
  if (g.qepi != 0) return cudaErrorInvalidValue;
  return launch_gemm_simt(g, s);
}

// Marks a GEMM pass's B operands as packed QMoE codes with their scales.  For a fused
// swiglu fc1 both operands share fc1's scales (same stored-row addressing as the codes).
void set_quantized(const moe_b200_problem& p, GemmArgs& g, const void* scales_a,
                   const void* scales_b) {
  g.qbits = p.attrs.expert_weight_bits;
  g.qblock = p.attrs.block_size;
  g.b1.scales = scales_a;
  if (g.gated) g.b3.scales = scales_b != nullptr ? scales_b : scales_a;
}

// Stage boundaries recorded when `ev` is non-NULL (kNumStages + 1 events).
enum Stage { kStRoute = 0, kStPlan, kStGather, kStDequant, kStFc1, kStFc2, kStCombine, kNumStages };

// NVTX ranges, one per stage of a layer call ("moe_b200/route", ...), as the host
// enqueues it: a profiler filters on them (ncu --nvtx --nvtx-include "moe_b200/fc1/").
// Without a tool attached an NVTX call is a null-pointer check.
constexpr const char* kStageNames[kNumStages] = {
    "moe_b200/route", "moe_b200/plan", "moe_b200/gather", "moe_b200/dequant",
    "moe_b200/fc1", "moe_b200/fc2", "moe_b200/combine"};

struct StageRanges {
  bool open = false;
  void enter(int i) {
    if (open) nvtxRangePop();
    open = i >= 0 && i < kNumStages;
    if (open) nvtxRangePushA(kStageNames[i]);
  }
  ~StageRanges() { if (open) nvtxRangePop(); }
};

// One layer call.  With `given_idx` (k == 1) the routing is supplied by the caller: rows
// of `input` are already assigned to experts (expert parallelism: the rows a rank
// received), every routing weight is 1, and the output row i is expert(row i)'s FFN
// output; router_probs is not read.
int forward_impl(const moe_b200_problem& p, const moe_b200_tensors& t, uint8_t* ws,
                 size_t ws_bytes, cudaStream_t s, cudaEvent_t* ev = nullptr,
                 const int32_t* given_idx = nullptr, const moe_b200_prepacked* pk = nullptr) {
  StageRanges ranges;
  auto mark = [&](int i) {
    if (ev && ev[i]) cudaEventRecord(ev[i], s);
    ranges.enter(i);
  };
  const bool use_pk = prepack_applies(pk, p);
  const WsLayout L = plan_workspace(p, use_pk);
  if (ws_bytes < L.total)
    return fail(MOE_B200_INVALID_ARGUMENT, "workspace of %zu bytes is smaller than %zu",
                ws_bytes, L.total);
  if ((reinterpret_cast<uintptr_t>(ws) & 255) != 0)
    return fail(MOE_B200_INVALID_ARGUMENT, "workspace must be 256-byte aligned");
  if (t.fc1_weights == nullptr || t.fc2_weights == nullptr)
    return fail(MOE_B200_INVALID_ARGUMENT, "fc1/fc2 weights must be non-NULL");
  if (p.num_rows > 0 && (t.input == nullptr || t.output == nullptr ||
                         (t.router_probs == nullptr && given_idx == nullptr)))
    return fail(MOE_B200_INVALID_ARGUMENT, "input, router_probs and output must be non-NULL");
  if (given_idx != nullptr && p.attrs.k != 1)
    return fail(MOE_B200_INVALID_ARGUMENT, "rows with given experts need k == 1");
  if (p.has_fc3 && t.fc3_weights == nullptr)
    return fail(MOE_B200_INVALID_ARGUMENT, "has_fc3 is set but fc3_weights is NULL");
  const int T = static_cast<int>(p.num_rows);
  const int E = static_cast<int>(p.num_experts);
  const int k = p.attrs.k;
  const int H = static_cast<int>(p.hidden_size);
  const int I = static_cast<int>(p.inter_size);
  const int64_t R = static_cast<int64_t>(T) * k;
  if (T == 0) return MOE_B200_OK;

  auto* idx = reinterpret_cast<int32_t*>(ws + L.idx);
  auto* w = reinterpret_cast<float*>(ws + L.w);
  auto* cc = reinterpret_cast<int32_t*>(ws + L.chunk_counts);
  auto* cb = reinterpret_cast<int32_t*>(ws + L.chunk_base);
  auto* offs = reinterpret_cast<int32_t*>(ws + L.offsets);
  auto* t128 = reinterpret_cast<int32_t*>(ws + L.tiles128);
  auto* t64 = reinterpret_cast<int32_t*>(ws + L.tiles64);
  auto* t256 = reinterpret_cast<int32_t*>(ws + L.tiles256);
  auto* pos = reinterpret_cast<int32_t*>(ws + L.pos);
  auto* src = reinterpret_cast<int32_t*>(ws + L.src);
  auto* err = reinterpret_cast<int*>(ws + L.err);
  void* xp = ws + L.xp;
  void* act = ws + L.act;

  // err[0]: device error word; err[1], err[2]: tile counters of the fc1 / fc2 GEMMs.
  // Zeroed by the call's first kernel (route, small dispatch or unit-weight fill): a
  // memset here would put a copy-engine operation between the previous call's kernels
  // and this one's.
  const size_t es = dtype_bytes(p.dtype);
  const int chunk = layer_route_chunk(T);
  if (given_idx != nullptr) {
    // Supplied routing: unit weights, histogram and plan of the given expert ids.
    mark(kStRoute);
    MOE_CUDA_CHECK(launch_fill_f32(w, 1.0f, R, s, err), "unit weights");
    MOE_CUDA_CHECK(launch_histogram(given_idx, T, 1, E, cc, err, s, chunk), "histogram");
    mark(kStPlan);
    MOE_CUDA_CHECK(launch_plan(given_idx, T, 1, E, cc, cb, offs, t128, t64, t256, pos, src, s,
                               chunk),
                   "plan");
    if (qmoe_use_decode(p)) {
      mark(kStGather);
      mark(kStDequant);
      mark(kStFc1);
      int st = qmoe_decode_fc1(p, t, src, act, offs, ws + L.qmoe, s);
      if (st != MOE_B200_OK) return st;
      mark(kStFc2);
      st = qmoe_decode_fc2(p, t, act, offs, ws + L.qmoe, s);
      if (st != MOE_B200_OK) return st;
      mark(kStCombine);
      st = qmoe_decode_combine(p, t, ws + L.qmoe, offs, pos, w, s);
      if (st != MOE_B200_OK) return st;
      mark(kNumStages);
      return MOE_B200_OK;
    }
  } else if (qmoe_use_decode(p)) {
    // Decode-sized QMoE: one CTA routes and plans, then the packed weights of the
    // touched experts are streamed once (token rows are read in place: no gather).
    mark(kStRoute);
    MOE_CUDA_CHECK(launch_small_dispatch(p.dtype, t.router_probs, T, E, k,
                                         route_mode(p), idx, w, offs, pos,
                                         src, s, err),
                   "route");
    mark(kStPlan);
    mark(kStGather);
    mark(kStDequant);
    mark(kStFc1);
    int st = qmoe_decode_fc1(p, t, src, act, offs, ws + L.qmoe, s);
    if (st != MOE_B200_OK) return st;
    mark(kStFc2);
    st = qmoe_decode_fc2(p, t, act, offs, ws + L.qmoe, s);
    if (st != MOE_B200_OK) return st;
    mark(kStCombine);
    st = qmoe_decode_combine(p, t, ws + L.qmoe, offs, pos, w, s);
    if (st != MOE_B200_OK) return st;
    mark(kNumStages);
    return MOE_B200_OK;
  }
  if (given_idx == nullptr) {
    mark(kStRoute);
    MOE_CUDA_CHECK(launch_route(p.dtype, t.router_probs, T, E, k,
                                route_mode(p), idx, w, cc, s, chunk, err),
                   "route");
    mark(kStPlan);
    MOE_CUDA_CHECK(launch_plan(idx, T, k, E, cc, cb, offs, t128, t64, t256, pos, src, s, chunk),
                   "plan");
  }
  // Routed rows gathered into xp (expert order).  With MOE_B200_GATHER_FUSION=1 the fc1
  // GEMM gets the un-permuted input instead (run_gemm: TMA gather4 in the CTA-pair kernel,
  // else a gather pass just before the GEMM).
  const bool fused_q = !use_pk && qmoe_use_fused(p);
  const bool gather_in_gemm = !fused_q && env_flag("MOE_B200_GATHER_FUSION");
  mark(kStGather);
  if (!gather_in_gemm)
    MOE_CUDA_CHECK(launch_gather(t.input, static_cast<int64_t>(H) * es, k, src, R, xp, s),
                   "gather");

  const void* w1 = t.fc1_weights;
  const void* w2 = t.fc2_weights;
  const void* w3 = t.fc3_weights;
  mark(kStDequant);
  if (use_pk) {
    // Weights dequantised once at session initialisation (moe_b200_prepack_create).
    w1 = pk->w1;
    w2 = pk->w2;
    w3 = pk->w3;
  } else if (p.attrs.expert_weight_bits != 0 && !fused_q) {
    // QMoE prefill: dequantise the weights of every expert into the workspace, then run
    // the same grouped GEMMs.
    QmoeDequantOut dq;
    int st = qmoe_dequantize(p, t, ws + L.qmoe, offs, &dq, s);
    if (st != MOE_B200_OK) return st;
    w1 = dq.w1;
    w2 = dq.w2;
    w3 = dq.w3;
  }

  GemmArgs g1 = fc1_args(p, w1, t.fc1_bias, w3, t.fc3_bias);
  g1.a = xp;
  g1.rows = R;
  if (gather_in_gemm) {
    g1.gather_x = t.input;
    g1.gather_src = src;
    g1.gather_k = k;
    g1.gather_x_rows = T;
  }
  g1.offsets = offs;
  g1.tiles128 = t128;
  g1.tiles64 = t64;
  g1.tiles256 = t256;
  g1.out = act;
  g1.ldo = I;
  g1.err = err;
  g1.tile_counter = err + 1;
  // MOE_B200_TEST_STALL=1 (tests only): the GEMM producers issue no loads, the kernel's
  // bounded waits expire and the call reports the device error instead of hanging.
  g1.test_stall = env_flag("MOE_B200_TEST_STALL") ? 1 : 0;
  // Dequantised copies holding exact codes: the epilogue applies the per-row scales.
  const bool row_scaled = !fused_q && p.attrs.expert_weight_bits != 0 &&
                          qmoe_dequantized_exact(p);
  if (fused_q || row_scaled) set_quantized(p, g1, t.fc1_scales, t.fc3_scales);
  if (row_scaled) g1.qepi = 1;
  // Per-row scales (block_size 0): the scale moves to the epilogue.  int8 codes go to the
  // tensor cores biased (1024 + q) and the epilogue subtracts (1024 + 128) * rowsum: the
  // constant part is ~15x the signal (|q - 128| ~ 74), within what the fp32 accumulation
  // carries.  int4 codes stay exact (q - 8): their constant part would be ~220x the signal
  // (|q - 8| ~ 4.6), and over a full-K accumulation that pushed a few outputs past the
  // fp16 tolerance.  MOE_B200_QGEMM_EPI=0/1/2 forces a mode (comparison runs).
  auto* rowsum = reinterpret_cast<float*>(ws + L.rowsum);
  int qepi = 0;
  if (fused_q && p.attrs.block_size == 0) {
    const char* v = std::getenv("MOE_B200_QGEMM_EPI");
    qepi = v != nullptr ? std::atoi(v) : (p.attrs.expert_weight_bits == 8 ? 2 : 1);
  }
  if (fused_q) g1.qepi = qepi;
  g1.rowsum = qepi == 2 ? rowsum : nullptr;
  mark(kStFc1);
  if (fused_q) {
    if (!tc_q_supported(g1))
      return fail(MOE_B200_NOT_IMPLEMENTED, "QMoE fc1: operands not 16-byte aligned");
    if (qepi == 2) MOE_CUDA_CHECK(launch_row_sums(xp, R, H, rowsum, s), "fc1 row sums");
    MOE_CUDA_CHECK(launch_gemm_tc_q(g1, device_sm_count(), s), "fc1 grouped GEMM (packed)");
  } else {
    MOE_CUDA_CHECK(run_gemm(g1, s), "fc1 grouped GEMM");
  }

  GemmArgs g2 = fc2_args(p, w2, t.fc2_bias);
  g2.a = act;
  g2.rows = R;
  g2.offsets = offs;
  g2.tiles128 = t128;
  g2.tiles64 = t64;
  g2.tiles256 = t256;
  g2.out = xp;  // Y aliases the gathered input, dead after fc1
  g2.ldo = H;
  g2.err = err;
  g2.tile_counter = err + 2;
  g2.test_stall = g1.test_stall;
  if (fused_q || row_scaled) set_quantized(p, g2, t.fc2_scales, nullptr);
  g2.qepi = row_scaled ? 1 : qepi;
  g2.rowsum = qepi == 2 ? rowsum : nullptr;
  // Combine fused into the fc2 epilogue: the epilogue counts the arrivals of each token's
  // k rows per 32-column segment and the completing one sums them into the output, so no
  // separate combine pass runs.  It pays where fc2's tiles are long enough (K = inter_size)
  // for the MMA to hide the epilogue's extra reads: C2 (I = 14336) 2.51 -> 2.46 ms per
  // layer; at C4 (I = 768, k = 8) the epilogue was already as long as the MMA and fc2 grew
  // by more than the 0.12 ms combine pass.  MOE_B200_FUSED_COMBINE=0/1 forces it.
  const char* fc_env = std::getenv("MOE_B200_FUSED_COMBINE");
  const bool fuse_wanted = fc_env != nullptr ? (fc_env[0] != '\0' && std::strcmp(fc_env, "0") != 0)
                                             : p.inter_size >= kFusedCombineMinInter;
  const bool fuse_combine = !fused_q && p.num_rows > 0 && fuse_wanted &&
                            !env_flag("MOE_B200_FORCE_SIMT") && tc_supported(g2) &&
                            H % 8 == 0;
  if (fuse_combine) {
    g2.comb_cnt = reinterpret_cast<unsigned*>(ws + L.comb);
    g2.comb_src = src;
    g2.comb_pos = pos;
    g2.comb_w = w;
    g2.comb_out = t.output;
    g2.comb_k = k;
    MOE_CUDA_CHECK(cudaMemsetAsync(ws + L.comb, 0,
                                   static_cast<size_t>(T) * ((H + 31) / 32) * 4, s),
                   "combine counters");
  }
  mark(kStFc2);
  if (fused_q) {
    if (!tc_q_supported(g2))
      return fail(MOE_B200_NOT_IMPLEMENTED, "QMoE fc2: operands not 16-byte aligned");
    if (qepi == 2) MOE_CUDA_CHECK(launch_row_sums(act, R, I, rowsum, s), "fc2 row sums");
    MOE_CUDA_CHECK(launch_gemm_tc_q(g2, device_sm_count(), s), "fc2 grouped GEMM (packed)");
  } else {
    MOE_CUDA_CHECK(run_gemm(g2, s), "fc2 grouped GEMM");
  }

  mark(kStCombine);
  if (!fuse_combine)
    MOE_CUDA_CHECK(launch_combine(p.dtype, xp, pos, w, T, k, H, t.output, s), "combine");
  mark(kNumStages);

  if (env_flag("MOE_B200_TRACE_SYNC")) {
    MOE_CUDA_CHECK(cudaStreamSynchronize(s), "stream synchronize");
    int herr = 0;
    MOE_CUDA_CHECK(cudaMemcpy(&herr, err, sizeof(int), cudaMemcpyDeviceToHost), "read error word");
    if (herr != 0) return fail(MOE_B200_EP_FAIL, "device error code %d", herr);
  }
  return MOE_B200_OK;
}

// ------------------------------------------------ device-side expert parallelism
struct EpWsLayout {
  size_t idx, w, cc, cb, myoff, t128, t64, t256, pos, src, err;
  size_t send_base, eoff, rt128, rt64, rt256, seg_start, seg_dst, act, total;
};

EpWsLayout plan_ep_workspace(const moe_b200_ep_comm* c, const moe_b200_problem& p) {
  EpWsLayout L{};
  const int64_t T = p.num_rows, E = c->num_experts, k = p.attrs.k, W = c->world, El = E / W;
  const int64_t R = T * k;
  const int64_t chunks = std::max<int64_t>(num_route_chunks(T, layer_route_chunk(T)), 1);
  size_t o = 0;
  auto take = [&](size_t bytes) { size_t at = o; o = align_up(o + bytes, 256); return at; };
  L.idx = take(R * 4);
  L.w = take(R * 4);
  L.cc = take(chunks * E * 4);
  L.cb = take(chunks * E * 4);
  L.myoff = take((E + 1) * 4);
  L.t128 = take((E + 1) * 4);
  L.t64 = take((E + 1) * 4);
  L.t256 = take((E + 1) * 4);
  L.pos = take(R * 4);
  L.src = take(R * 4);
  L.err = take(16);
  L.send_base = take(E * 4);
  L.eoff = take((El + 1) * 4);
  L.rt128 = take((El + 1) * 4);
  L.rt64 = take((El + 1) * 4);
  L.rt256 = take((El + 1) * 4);
  L.seg_start = take((El * W + 1) * 4);
  L.seg_dst = take(El * W * 4);
  L.act = take(static_cast<size_t>(c->cap_rows) * p.inter_size * dtype_bytes(p.dtype));
  L.total = o;
  return L;
}

}  // namespace

namespace moe {

size_t ep_workspace_bytes(const moe_b200_ep_comm* c, const moe_b200_problem& p) {
  return plan_ep_workspace(c, p).total;
}

// One layer call of the device-side expert-parallel path: route and plan over all E
// experts, exchange counts (device), send rows into the owners' receive buffers, expert
// FFN on the received rows with the fc2 epilogue storing into the senders' return
// buffers, combine.  Local weights: [E / W, ...].  No host synchronisation.
int ep_forward_impl(moe_b200_ep_comm* c, const moe_b200_problem& p, const moe_b200_tensors& t,
                    uint8_t* ws, size_t ws_bytes, cudaStream_t s, cudaEvent_t* ev) {
  // Phase boundaries (kEpNumPhases + 1 events when `ev` is non-NULL): route+plan, counts,
  // send rows, wait rows, fc1, fc2 (with the return stores), wait return, combine.
  auto mark = [&](int i) { if (ev && ev[i]) cudaEventRecord(ev[i], s); };
  const int W = c->world, E = c->num_experts, El = E / W, r = c->rank;
  moe_b200_problem global = p;  // routing is over all E experts (k <= E, not E / W)
  global.num_experts = E;
  int st = validate_problem(&global);
  if (st != MOE_B200_OK) return st;
  if (p.num_experts != El)
    return fail(MOE_B200_INVALID_ARGUMENT, "problem.num_experts=%lld must be the local %d",
                (long long)p.num_experts, El);
  if (p.dtype != c->dtype || p.hidden_size != c->hidden || p.num_rows > c->max_rows ||
      p.attrs.k > c->k_max)
    return fail(MOE_B200_INVALID_ARGUMENT,
                "problem (dtype %d, hidden %lld, rows %lld, k %d) outside the communicator's "
                "(dtype %d, hidden %lld, rows <= %lld, k <= %d)",
                p.dtype, (long long)p.hidden_size, (long long)p.num_rows, p.attrs.k, c->dtype,
                (long long)c->hidden, (long long)c->max_rows, c->k_max);
  const bool quant = p.attrs.expert_weight_bits != 0;
  if (quant && (t.fc1_scales == nullptr || t.fc2_scales == nullptr ||
                (p.has_fc3 && t.fc3_scales == nullptr)))
    return fail(MOE_B200_INVALID_ARGUMENT, "QMoE: fc1/fc2(/fc3) scales must be non-NULL");
  if (p.attrs.k > E) return fail(MOE_B200_INVALID_ARGUMENT, "k=%d > %d experts", p.attrs.k, E);
  if (t.fc1_weights == nullptr || t.fc2_weights == nullptr || (p.has_fc3 && !t.fc3_weights))
    return fail(MOE_B200_INVALID_ARGUMENT, "local fc1/fc2(/fc3) weights must be non-NULL");
  const int T = static_cast<int>(p.num_rows), k = p.attrs.k;
  const int H = static_cast<int>(p.hidden_size), I = static_cast<int>(p.inter_size);
  if (T > 0 && (t.input == nullptr || t.router_probs == nullptr || t.output == nullptr))
    return fail(MOE_B200_INVALID_ARGUMENT, "input, router_probs and output must be non-NULL");
  const EpWsLayout L = plan_ep_workspace(c, p);
  if (ws_bytes < L.total || (reinterpret_cast<uintptr_t>(ws) & 255) != 0)
    return fail(MOE_B200_INVALID_ARGUMENT, "workspace must be 256-byte aligned and >= %zu bytes",
                L.total);
  auto i32 = [&](size_t off) { return reinterpret_cast<int32_t*>(ws + off); };
  int* err = reinterpret_cast<int*>(ws + L.err);
  const uint32_t epoch = ++c->epoch;
  const int64_t R = static_cast<int64_t>(T) * k;
  const int chunk = layer_route_chunk(T);
  const size_t es = dtype_bytes(p.dtype);

  mark(0);
  // Route and plan over all E experts (expert-ordered rows of this rank's tokens).
  MOE_CUDA_CHECK(launch_route(p.dtype, t.router_probs, T, E, k,
                              route_mode(p), i32(L.idx),
                              reinterpret_cast<float*>(ws + L.w), i32(L.cc), s, chunk),
                 "route");
  if (T > 0)
    MOE_CUDA_CHECK(launch_plan(i32(L.idx), T, k, E, i32(L.cc), i32(L.cb), i32(L.myoff),
                               i32(L.t128), i32(L.t64), i32(L.t256), i32(L.pos), i32(L.src), s,
                               chunk),
                   "plan");
  const EpTables tab{i32(L.send_base), i32(L.eoff), i32(L.rt128), i32(L.rt64), i32(L.rt256),
                     i32(L.seg_start), i32(L.seg_dst)};
  mark(1);
  MOE_CUDA_CHECK(launch_ep_exchange_counts(c->peers, c->lay, r, W, E, epoch,
                                           T > 0 ? i32(L.myoff) : nullptr, tab, err, s),
                 "count exchange");
  mark(2);
  // Deduplicated dispatch when a token's k experts often share a rank (k >= 4): each
  // token crosses NVLink once per destination and the receiver gathers its rows locally.
  // MOE_B200_EP_DEDUP=0/1 forces it (1 needs a region created with k_max >= 4).
  const char* dd = std::getenv("MOE_B200_EP_DEDUP");
  const bool dedup = c->lay.tok != 0 && (dd != nullptr ? dd[0] != '0' : k >= kEpDedupMinK);
  MOE_CUDA_CHECK(launch_ep_send_rows(c->peers, c->lay, r, W, E, t.input,
                                     static_cast<int64_t>(H) * es, k, i32(L.idx), i32(L.src), R,
                                     tab.send_base, c->max_rows, dedup, err, s),
                 "send rows");
  // MOE_B200_TEST_STALL=1 (tests only): the rows and return flags are never raised, so the
  // bounded waits expire and the call reports device error kErrTimeoutPeer.
  const bool stall = env_flag("MOE_B200_TEST_STALL");
  if (!stall)
    MOE_CUDA_CHECK(launch_ep_signal(c->peers, c->lay, r, W, kEpRows, epoch, s), "signal rows");
  mark(3);
  MOE_CUDA_CHECK(launch_ep_wait(c->sym, c->lay, W, kEpRows, epoch, err, s), "wait rows");
  if (dedup)
    MOE_CUDA_CHECK(launch_ep_gather_tokens(c->sym, c->lay, static_cast<int64_t>(H) * es,
                                           tab.eoff + El, c->cap_rows, err, s),
                   "gather received tokens");

  mark(4);
  // Expert FFN on the received rows (row count known on the device only: the GEMMs are
  // sized for the communicator's capacity and schedule from the device offsets).
  void* act = ws + L.act;
  moe_b200_problem pl = p;
  GemmArgs g1 = fc1_args(pl, t.fc1_weights, t.fc1_bias, t.fc3_weights, t.fc3_bias);
  g1.a = c->sym + c->lay.recv;
  g1.rows = c->cap_rows;
  g1.offsets = tab.eoff;
  g1.tiles128 = tab.t128;
  g1.tiles64 = tab.t64;
  g1.tiles256 = tab.t256;
  g1.out = act;
  g1.ldo = I;
  g1.err = err;
  g1.tile_counter = err + 1;
  // QMoE: the code-converting pair GEMM on the received rows.  With one scale per row the
  // codes stay exact and the scale moves to the epilogue (no row sums: the receive buffer
  // is sized for the capacity, not the rows that arrived).
  if (quant) {
    set_quantized(pl, g1, t.fc1_scales, t.fc3_scales);
    g1.qepi = p.attrs.block_size == 0 ? 1 : 0;
    if (!tc_q_supported(g1))
      return fail(MOE_B200_NOT_IMPLEMENTED, "expert-parallel QMoE fc1: operands unsupported");
    MOE_CUDA_CHECK(launch_gemm_tc_q(g1, device_sm_count(), s), "fc1 grouped GEMM (packed)");
  } else {
    if (!tc_supported(g1))
      return fail(MOE_B200_NOT_IMPLEMENTED, "expert-parallel fc1: tensor-core path unsupported");
    MOE_CUDA_CHECK(launch_gemm_tc(g1, device_sm_count(), 2, s), "fc1 grouped GEMM");
  }
  mark(5);
  GemmArgs g2 = fc2_args(pl, t.fc2_weights, t.fc2_bias);
  g2.a = act;
  g2.rows = c->cap_rows;
  g2.offsets = tab.eoff;
  g2.tiles128 = tab.t128;
  g2.tiles64 = tab.t64;
  g2.tiles256 = tab.t256;
  g2.out = c->sym + c->lay.ret;  // alignment check only: rows go to the senders' buffers
  g2.ldo = H;
  g2.err = err;
  g2.tile_counter = err + 2;
  g2.seg_start = tab.seg_start;
  g2.seg_dst = tab.seg_dst;
  g2.nseg = El * W;
  g2.remap_world = W;
  for (int d = 0; d < W; ++d) g2.out_peers[d] = c->peers.base[d] + c->lay.ret;
  if (quant) {
    set_quantized(pl, g2, t.fc2_scales, nullptr);
    g2.qepi = g1.qepi;
    if (!tc_q_supported(g2))
      return fail(MOE_B200_NOT_IMPLEMENTED, "expert-parallel QMoE fc2: operands unsupported");
    MOE_CUDA_CHECK(launch_gemm_tc_q(g2, device_sm_count(), s), "fc2 grouped GEMM (packed)");
  } else {
    if (!tc_supported(g2))
      return fail(MOE_B200_NOT_IMPLEMENTED, "expert-parallel fc2: tensor-core path unsupported");
    MOE_CUDA_CHECK(launch_gemm_tc(g2, device_sm_count(), 2, s), "fc2 grouped GEMM");
  }
  if (!stall)
    MOE_CUDA_CHECK(launch_ep_signal(c->peers, c->lay, r, W, kEpReturn, epoch, s),
                   "signal return");
  mark(6);
  MOE_CUDA_CHECK(launch_ep_wait(c->sym, c->lay, W, kEpReturn, epoch, err, s), "wait return");
  mark(7);
  MOE_CUDA_CHECK(launch_combine(p.dtype, c->sym + c->lay.ret, i32(L.pos),
                                reinterpret_cast<float*>(ws + L.w), T, k, H, t.output, s),
                 "combine");
  mark(8);
  if (env_flag("MOE_B200_TRACE_SYNC")) {
    MOE_CUDA_CHECK(cudaStreamSynchronize(s), "stream synchronize");
    int herr = 0;
    MOE_CUDA_CHECK(cudaMemcpy(&herr, err, sizeof(int), cudaMemcpyDeviceToHost), "read error word");
    if (herr != 0) return fail(MOE_B200_EP_FAIL, "device error code %d", herr);
  }
  return MOE_B200_OK;
}

}  // namespace moe

// ==================================================================== C ABI
extern "C" {

int moe_b200_abi_version(void) { return MOE_B200_ABI_VERSION; }

const char* moe_b200_last_error(void) { return g_last_error.c_str(); }

int moe_b200_workspace_size(const moe_b200_problem* problem, size_t* bytes) {
  int st = validate_problem(problem);
  if (st != MOE_B200_OK) return st;
  if (bytes == nullptr) return fail(MOE_B200_INVALID_ARGUMENT, "bytes is NULL");
  *bytes = plan_workspace(*problem).total;
  return MOE_B200_OK;
}

int moe_b200_forward(const moe_b200_problem* problem, const moe_b200_tensors* t,
                     void* workspace, size_t workspace_bytes, void* stream) {
  moe::clear_stale_cuda_error();
  int st = validate_problem(problem);
  if (st != MOE_B200_OK) return st;
  if (t == nullptr) return fail(MOE_B200_INVALID_ARGUMENT, "tensors is NULL");
  return forward_impl(*problem, *t, static_cast<uint8_t*>(workspace), workspace_bytes,
                      static_cast<cudaStream_t>(stream));
}

int moe_b200_forward_timed(const moe_b200_problem* problem, const moe_b200_tensors* t,
                           void* workspace, size_t workspace_bytes, void* stream,
                           float* stage_ms, int32_t num_stages) {
  moe::clear_stale_cuda_error();
  int st = validate_problem(problem);
  if (st != MOE_B200_OK) return st;
  if (t == nullptr || stage_ms == nullptr || num_stages < kNumStages)
    return fail(MOE_B200_INVALID_ARGUMENT, "tensors/stage_ms NULL or num_stages < %d", kNumStages);
  cudaEvent_t ev[kNumStages + 1];
  for (int i = 0; i <= kNumStages; ++i) MOE_CUDA_CHECK(cudaEventCreate(&ev[i]), "cudaEventCreate");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  st = forward_impl(*problem, *t, static_cast<uint8_t*>(workspace), workspace_bytes, s, ev);
  if (st == MOE_B200_OK && problem->num_rows > 0) {
    cudaError_t ce = cudaEventSynchronize(ev[kNumStages]);
    for (int i = 0; i < kNumStages && ce == cudaSuccess; ++i)
      ce = cudaEventElapsedTime(&stage_ms[i], ev[i], ev[i + 1]);
    if (ce != cudaSuccess) st = cuda_fail(ce, "stage timing");
  } else if (st == MOE_B200_OK) {
    for (int i = 0; i < kNumStages; ++i) stage_ms[i] = 0.f;
  }
  for (int i = 0; i <= kNumStages; ++i) cudaEventDestroy(ev[i]);
  return st;
}

int moe_b200_forward_staged(const moe_b200_problem* problem, const moe_b200_tensors* t,
                            void* workspace, size_t workspace_bytes, void* stream,
                            void* const* events, int32_t num_events) {
  moe::clear_stale_cuda_error();
  int st = validate_problem(problem);
  if (st != MOE_B200_OK) return st;
  if (t == nullptr || events == nullptr || num_events < kNumStages + 1)
    return fail(MOE_B200_INVALID_ARGUMENT, "tensors/events NULL or num_events < %d",
                kNumStages + 1);
  cudaEvent_t ev[kNumStages + 1];
  for (int i = 0; i <= kNumStages; ++i) ev[i] = static_cast<cudaEvent_t>(events[i]);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  st = forward_impl(*problem, *t, static_cast<uint8_t*>(workspace), workspace_bytes, s, ev);
  if (st == MOE_B200_OK && problem->num_rows == 0)
    for (int i = 0; i <= kNumStages; ++i)
      if (ev[i]) MOE_CUDA_CHECK(cudaEventRecord(ev[i], s), "event");
  return st;
}

int moe_b200_workspace_size_prepacked(const moe_b200_problem* problem,
                                      const moe_b200_prepacked* prepacked, size_t* bytes) {
  int st = validate_problem(problem);
  if (st != MOE_B200_OK) return st;
  if (bytes == nullptr) return fail(MOE_B200_INVALID_ARGUMENT, "bytes is NULL");
  *bytes = plan_workspace(*problem, prepack_applies(prepacked, *problem)).total;
  return MOE_B200_OK;
}

int moe_b200_forward_prepacked(const moe_b200_problem* problem, const moe_b200_tensors* t,
                               const moe_b200_prepacked* prepacked, void* workspace,
                               size_t workspace_bytes, void* stream, void* const* events,
                               int32_t num_events) {
  moe::clear_stale_cuda_error();
  int st = validate_problem(problem);
  if (st != MOE_B200_OK) return st;
  if (t == nullptr) return fail(MOE_B200_INVALID_ARGUMENT, "tensors is NULL");
  if (events != nullptr && num_events < kNumStages + 1)
    return fail(MOE_B200_INVALID_ARGUMENT, "num_events=%d < %d", num_events, kNumStages + 1);
  if (prepacked != nullptr && problem->attrs.expert_weight_bits != 0 &&
      !prepack_matches(*prepacked, *problem))
    return fail(MOE_B200_INVALID_ARGUMENT, "the prepack was made for other weight shapes");
  cudaEvent_t ev[kNumStages + 1];
  for (int i = 0; i <= kNumStages; ++i)
    ev[i] = events != nullptr ? static_cast<cudaEvent_t>(events[i]) : nullptr;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  st = forward_impl(*problem, *t, static_cast<uint8_t*>(workspace), workspace_bytes, s,
                    events != nullptr ? ev : nullptr, nullptr, prepacked);
  if (st == MOE_B200_OK && events != nullptr && problem->num_rows == 0)
    for (int i = 0; i <= kNumStages; ++i)
      if (ev[i]) MOE_CUDA_CHECK(cudaEventRecord(ev[i], s), "event");
  return st;
}

int moe_b200_ep_dispatch(const moe_b200_problem* problem, const void* router_probs,
                         const void* input, void* send_rows, int32_t* expert_offsets,
                         int32_t* permuted_pos, float* route_weight, void* workspace,
                         size_t workspace_bytes, void* stream) {
  moe::clear_stale_cuda_error();
  int st = validate_problem(problem);
  if (st != MOE_B200_OK) return st;
  const moe_b200_problem& p = *problem;
  const WsLayout L = plan_workspace(p);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (workspace_bytes < L.total || (reinterpret_cast<uintptr_t>(ws) & 255) != 0)
    return fail(MOE_B200_INVALID_ARGUMENT, "workspace must be 256-byte aligned and >= %zu bytes",
                L.total);
  if (expert_offsets == nullptr || (p.num_rows > 0 && (router_probs == nullptr || input == nullptr ||
                                                       send_rows == nullptr ||
                                                       permuted_pos == nullptr ||
                                                       route_weight == nullptr)))
    return fail(MOE_B200_INVALID_ARGUMENT, "ep_dispatch: NULL buffer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int T = static_cast<int>(p.num_rows), E = static_cast<int>(p.num_experts), k = p.attrs.k;
  if (T == 0) {
    MOE_CUDA_CHECK(cudaMemsetAsync(expert_offsets, 0, (E + 1) * sizeof(int32_t), s), "offsets");
    return MOE_B200_OK;
  }
  auto* idx = reinterpret_cast<int32_t*>(ws + L.idx);
  auto* cc = reinterpret_cast<int32_t*>(ws + L.chunk_counts);
  auto* cb = reinterpret_cast<int32_t*>(ws + L.chunk_base);
  auto* t128 = reinterpret_cast<int32_t*>(ws + L.tiles128);
  auto* t64 = reinterpret_cast<int32_t*>(ws + L.tiles64);
  auto* t256 = reinterpret_cast<int32_t*>(ws + L.tiles256);
  auto* src = reinterpret_cast<int32_t*>(ws + L.src);
  const int chunk = layer_route_chunk(T);
  MOE_CUDA_CHECK(launch_route(p.dtype, router_probs, T, E, k, route_mode(p),
                              idx, route_weight, cc, s, chunk),
                 "route");
  MOE_CUDA_CHECK(launch_plan(idx, T, k, E, cc, cb, expert_offsets, t128, t64, t256, permuted_pos,
                             src, s, chunk),
                 "plan");
  MOE_CUDA_CHECK(launch_gather(input, static_cast<int64_t>(p.hidden_size) * dtype_bytes(p.dtype),
                               k, src, static_cast<int64_t>(T) * k, send_rows, s),
                 "gather");
  return MOE_B200_OK;
}

int moe_b200_expert_ffn(const moe_b200_problem* problem, const moe_b200_tensors* t,
                        const int32_t* row_expert, void* workspace, size_t workspace_bytes,
                        void* stream) {
  moe::clear_stale_cuda_error();
  int st = validate_problem(problem);
  if (st != MOE_B200_OK) return st;
  if (t == nullptr || (problem->num_rows > 0 && row_expert == nullptr))
    return fail(MOE_B200_INVALID_ARGUMENT, "expert_ffn: NULL tensors or row_expert");
  return forward_impl(*problem, *t, static_cast<uint8_t*>(workspace), workspace_bytes,
                      static_cast<cudaStream_t>(stream), nullptr, row_expert);
}

int moe_b200_ep_combine(int32_t dtype, int64_t num_rows, int64_t hidden_size, int32_t k,
                        const void* expert_rows, const int32_t* permuted_pos,
                        const float* route_weight, void* output, void* stream) {
  moe::clear_stale_cuda_error();
  if (!is_float_type(dtype)) return fail(MOE_B200_NOT_IMPLEMENTED, "unsupported dtype %d", dtype);
  if (num_rows < 0 || hidden_size <= 0 || k < 1)
    return fail(MOE_B200_INVALID_ARGUMENT, "ep_combine: invalid shape");
  if (num_rows == 0) return MOE_B200_OK;
  MOE_CUDA_CHECK(launch_combine(dtype, expert_rows, permuted_pos, route_weight,
                                static_cast<int>(num_rows), k, static_cast<int>(hidden_size),
                                output, static_cast<cudaStream_t>(stream)),
                 "combine");
  return MOE_B200_OK;
}

int moe_b200_route(const void* router_probs, int32_t dtype, int64_t num_rows,
                   int64_t num_experts, int32_t k, int32_t normalize_routing_weights,
                   int32_t* expert_idx, float* route_weight, void* stream) {
  moe::clear_stale_cuda_error();
  if (!is_float_type(dtype)) return fail(MOE_B200_NOT_IMPLEMENTED, "unsupported dtype %d", dtype);
  if (num_experts < 1 || num_experts > kMaxExperts || k < 1 || k > num_experts || k > kMaxK ||
      num_rows < 0)
    return fail(MOE_B200_INVALID_ARGUMENT, "invalid routing shape");
  if (normalize_routing_weights < 0 || normalize_routing_weights > kRouteSparseMixer ||
      (normalize_routing_weights == kRouteSparseMixer && k != 2))
    return fail(MOE_B200_INVALID_ARGUMENT,
                "routing mode %d: 0, 1, or 2 (sparse mixer, k = 2)", normalize_routing_weights);
  if (num_rows == 0) return MOE_B200_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t* cc = nullptr;
  // The histogram of this standalone call is not needed; give it a scratch buffer.
  const size_t bytes = static_cast<size_t>(num_route_chunks(num_rows)) * num_experts * 4;
  MOE_CUDA_CHECK(cudaMallocAsync(reinterpret_cast<void**>(&cc), bytes, s), "alloc");
  cudaError_t e = launch_route(dtype, router_probs, static_cast<int>(num_rows),
                               static_cast<int>(num_experts), k, normalize_routing_weights,
                               expert_idx, route_weight, cc, s);
  cudaFreeAsync(cc, s);
  if (e != cudaSuccess) return cuda_fail(e, "route");
  return MOE_B200_OK;
}

int moe_b200_norm_router(int32_t dtype, int64_t num_rows, int64_t hidden_size,
                         int64_t num_experts, const void* input, const void* skip,
                         const float* gamma, float epsilon, const void* router_weight,
                         void* residual_out, void* normed, void* router_logits, void* stream) {
  moe::clear_stale_cuda_error();
  if (!is_float_type(dtype)) return fail(MOE_B200_NOT_IMPLEMENTED, "unsupported dtype %d", dtype);
  if (num_rows < 0 || hidden_size < 8 || hidden_size % 8 != 0 || num_experts < 1)
    return fail(MOE_B200_INVALID_ARGUMENT,
                "norm_router: rows >= 0, hidden_size a multiple of 8 and num_experts >= 1");
  if (norm_router_smem_bytes(dtype, hidden_size) > 227 * 1024)
    return fail(MOE_B200_NOT_IMPLEMENTED, "norm_router: hidden_size=%lld too large",
                (long long)hidden_size);
  if (num_rows == 0) return MOE_B200_OK;
  if (input == nullptr || gamma == nullptr || router_weight == nullptr || router_logits == nullptr)
    return fail(MOE_B200_INVALID_ARGUMENT, "norm_router: input, gamma, router_weight and "
                                           "router_logits must be non-NULL");
  auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  if (!a16(input) || !a16(skip) || !a16(gamma) || !a16(router_weight) || !a16(residual_out) ||
      !a16(normed))
    return fail(MOE_B200_INVALID_ARGUMENT, "norm_router: buffers must be 16-byte aligned");
  MOE_CUDA_CHECK(launch_norm_router(dtype, input, skip, gamma, epsilon, router_weight, num_rows,
                                    static_cast<int>(hidden_size), static_cast<int>(num_experts),
                                    skip != nullptr ? residual_out : nullptr, normed,
                                    router_logits, static_cast<cudaStream_t>(stream)),
                 "norm_router");
  return MOE_B200_OK;
}

size_t moe_b200_permute_workspace_size(int64_t num_rows, int32_t k, int64_t num_experts) {
  (void)k;
  const size_t chunks = std::max<int64_t>(num_route_chunks(num_rows), 1);
  return align_up(chunks * num_experts * 4, 256) * 2 + align_up((num_experts + 1) * 4, 256) * 3 +
         256;
}

int moe_b200_permute(const int32_t* expert_idx, int64_t num_rows, int32_t k,
                     int64_t num_experts, int32_t* expert_offsets, int32_t* permuted_pos,
                     int32_t* permuted_src, void* workspace, size_t workspace_bytes,
                     void* stream) {
  moe::clear_stale_cuda_error();
  if (num_experts < 1 || num_experts > kMaxExperts || k < 1 || num_rows < 0)
    return fail(MOE_B200_INVALID_ARGUMENT, "invalid permutation shape");
  if (workspace_bytes < moe_b200_permute_workspace_size(num_rows, k, num_experts))
    return fail(MOE_B200_INVALID_ARGUMENT, "permute workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t chunks = std::max<int64_t>(num_route_chunks(num_rows), 1);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const size_t cbytes = align_up(chunks * num_experts * 4, 256);
  const size_t tbytes = align_up((num_experts + 1) * 4, 256);
  auto* cc = reinterpret_cast<int32_t*>(ws);
  auto* cb = reinterpret_cast<int32_t*>(ws + cbytes);
  auto* t128 = reinterpret_cast<int32_t*>(ws + 2 * cbytes);
  auto* t64 = reinterpret_cast<int32_t*>(ws + 2 * cbytes + tbytes);
  auto* t256 = reinterpret_cast<int32_t*>(ws + 2 * cbytes + 2 * tbytes);
  auto* err = reinterpret_cast<int*>(ws + 2 * cbytes + 3 * tbytes);
  const int T = static_cast<int>(num_rows), E = static_cast<int>(num_experts);
  MOE_CUDA_CHECK(cudaMemsetAsync(err, 0, sizeof(int), s), "clear error word");
  if (T == 0) MOE_CUDA_CHECK(cudaMemsetAsync(cc, 0, cbytes, s), "clear counts");
  MOE_CUDA_CHECK(launch_histogram(expert_idx, T, k, E, cc, err, s), "histogram");
  MOE_CUDA_CHECK(launch_plan(expert_idx, T, k, E, cc, cb, expert_offsets, t128, t64, t256,
                             permuted_pos, permuted_src, s),
                 "plan");
  int herr = 0;
  MOE_CUDA_CHECK(cudaMemcpyAsync(&herr, err, sizeof(int), cudaMemcpyDeviceToHost, s),
                 "read error word");
  MOE_CUDA_CHECK(cudaStreamSynchronize(s), "stream synchronize");
  if (herr == kErrBadExpert) return fail(MOE_B200_INVALID_ARGUMENT, "expert index out of range");
  return MOE_B200_OK;
}

}  // extern "C"
