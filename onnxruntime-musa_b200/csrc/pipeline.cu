// Host-buffer execution of one MoE / QMoE layer: a stream of calls whose inputs and
// outputs live in (pinned) host memory, with the host<->device copies of neighbouring
// calls overlapping the layer's compute.
//
// Reference analog: a session run whose inputs are CPU tensors: the plugin's data
// transfer copies them to the device (MusaDataTransfer::CopyImpl,
// musa/ep/src/ep_data_transfer.cc:108-161), the kernel runs on the compute stream, and
// with do_copy_in_default_stream = 0 the copies use their own streams ordered by
// notifications (MusaSyncStream / MusaNotification, musa/ep/src/ep_stream.cc:30-185).
//
// Three streams and `depth` device staging slots (input, router logits, output):
//   copy-in    H2D of call i into slot i % depth, after the compute of call i - depth
//              has finished reading that slot;
//   compute    the layer (moe_b200_forward) of call i, after its H2D and after the D2H
//              of call i - depth has drained the slot's output;
//   copy-out   D2H of call i, after its compute.
// Every dependency is a CUDA event waited on by a stream: submit never blocks the host.
#include <cuda_runtime.h>

#include <algorithm>
#include <vector>

#include "../../include/moe_b200.h"
#include "moe_kernels.h"
#include "prepack.h"

struct moe_b200_pipeline {
  moe_b200_problem problem{};   // num_rows = the largest call
  moe_b200_tensors weights{};
  int device = 0;
  int depth = 0;
  int64_t calls = 0;
  size_t in_bytes = 0, lg_bytes = 0, out_bytes = 0;  // per row
  cudaStream_t s_in = nullptr, s_comp = nullptr, s_out = nullptr;
  void* workspace = nullptr;
  size_t ws_bytes = 0;
  moe_b200_prepacked* prepacked = nullptr;  // one reference held
  struct Slot {
    void* x = nullptr;
    void* lg = nullptr;
    void* out = nullptr;
    cudaEvent_t in_done = nullptr, comp_done = nullptr, out_done = nullptr;
  };
  std::vector<Slot> slots;
};

namespace {

int cuda_fail(cudaError_t st, const char* what) {
  return moe::set_error(MOE_B200_EP_FAIL, "%s: %s", what, cudaGetErrorString(st));
}

#define PL_CHECK(expr, what)                                  \
  do {                                                        \
    cudaError_t _st = (expr);                                 \
    if (_st != cudaSuccess) return cuda_fail(_st, what);      \
  } while (0)

void destroy(moe_b200_pipeline* pl) {
  if (pl == nullptr) return;
  cudaSetDevice(pl->device);
  for (auto& s : pl->slots) {
    cudaFree(s.x);
    cudaFree(s.lg);
    cudaFree(s.out);
    if (s.in_done) cudaEventDestroy(s.in_done);
    if (s.comp_done) cudaEventDestroy(s.comp_done);
    if (s.out_done) cudaEventDestroy(s.out_done);
  }
  cudaFree(pl->workspace);
  if (pl->prepacked != nullptr) moe_b200_prepack_release(pl->prepacked);
  if (pl->s_in) cudaStreamDestroy(pl->s_in);
  if (pl->s_comp) cudaStreamDestroy(pl->s_comp);
  if (pl->s_out) cudaStreamDestroy(pl->s_out);
  delete pl;
}

int element_bytes(int32_t dt) {
  return dt == MOE_B200_FLOAT ? 4 : 2;
}

}  // namespace

extern "C" {

int moe_b200_pipeline_create(const moe_b200_problem* problem, const moe_b200_tensors* weights,
                             int32_t depth, moe_b200_pipeline** pipeline) {
  moe::clear_stale_cuda_error();
  if (problem == nullptr || weights == nullptr || pipeline == nullptr)
    return moe::set_error(MOE_B200_INVALID_ARGUMENT, "problem, weights and pipeline must be non-NULL");
  if (depth < 1 || depth > 8)
    return moe::set_error(MOE_B200_INVALID_ARGUMENT, "depth=%d must be in [1, 8]", depth);
  if (problem->num_rows < 1)
    return moe::set_error(MOE_B200_INVALID_ARGUMENT, "num_rows (the largest call) must be >= 1");
  // Workspace for every call size up to num_rows: the largest call's, and (QMoE) a
  // decode-sized call's, whose fp32 partial sums the prefill paths do not need.
  size_t ws = 0;
  int st = moe_b200_workspace_size(problem, &ws);
  if (st != MOE_B200_OK) return st;
  if (problem->attrs.expert_weight_bits != 0) {
    moe_b200_problem small = *problem;
    small.num_rows = std::min<int64_t>(problem->num_rows, 512 / problem->attrs.k);
    size_t ws_small = 0;
    if (small.num_rows > 0 && moe_b200_workspace_size(&small, &ws_small) == MOE_B200_OK)
      ws = std::max(ws, ws_small);
  }
  auto* pl = new moe_b200_pipeline();
  pl->problem = *problem;
  pl->weights = *weights;
  pl->weights.input = nullptr;
  pl->weights.router_probs = nullptr;
  pl->weights.output = nullptr;
  pl->depth = depth;
  const size_t es = static_cast<size_t>(element_bytes(problem->dtype));
  pl->in_bytes = es * static_cast<size_t>(problem->hidden_size);
  pl->lg_bytes = es * static_cast<size_t>(problem->num_experts);
  pl->out_bytes = pl->in_bytes;
  pl->ws_bytes = ws;
  auto fail = [&](cudaError_t e, const char* what) {
    const int code = cuda_fail(e, what);
    destroy(pl);
    return code;
  };
  cudaError_t e = cudaGetDevice(&pl->device);
  if (e != cudaSuccess) return fail(e, "cudaGetDevice");
  const size_t rows = static_cast<size_t>(problem->num_rows);
  if ((e = cudaStreamCreateWithFlags(&pl->s_in, cudaStreamNonBlocking)) != cudaSuccess ||
      (e = cudaStreamCreateWithFlags(&pl->s_comp, cudaStreamNonBlocking)) != cudaSuccess ||
      (e = cudaStreamCreateWithFlags(&pl->s_out, cudaStreamNonBlocking)) != cudaSuccess)
    return fail(e, "cudaStreamCreate");
  if ((e = cudaMalloc(&pl->workspace, ws)) != cudaSuccess) return fail(e, "workspace");
  pl->slots.resize(depth);
  for (auto& s : pl->slots) {
    if ((e = cudaMalloc(&s.x, rows * pl->in_bytes)) != cudaSuccess ||
        (e = cudaMalloc(&s.lg, rows * pl->lg_bytes)) != cudaSuccess ||
        (e = cudaMalloc(&s.out, rows * pl->out_bytes)) != cudaSuccess)
      return fail(e, "staging buffers");
    if ((e = cudaEventCreateWithFlags(&s.in_done, cudaEventDisableTiming)) != cudaSuccess ||
        (e = cudaEventCreateWithFlags(&s.comp_done, cudaEventDisableTiming)) != cudaSuccess ||
        (e = cudaEventCreateWithFlags(&s.out_done, cudaEventDisableTiming)) != cudaSuccess)
      return fail(e, "events");
  }
  *pipeline = pl;
  return MOE_B200_OK;
}

int moe_b200_pipeline_set_prepacked(moe_b200_pipeline* pl, moe_b200_prepacked* prepacked) {
  if (pl == nullptr) return moe::set_error(MOE_B200_INVALID_ARGUMENT, "pipeline is NULL");
  if (prepacked != nullptr && !moe::prepack_matches(*prepacked, pl->problem))
    return moe::set_error(MOE_B200_INVALID_ARGUMENT, "the prepack was made for other weight shapes");
  // Calls already submitted keep the weights they were enqueued with; the reference
  // dropped here is released only after them.
  if (pl->prepacked != nullptr) {
    cudaError_t e = cudaStreamSynchronize(pl->s_comp);
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
    moe_b200_prepack_release(pl->prepacked);
  }
  if (prepacked != nullptr) prepacked->refs.fetch_add(1);
  pl->prepacked = prepacked;
  return MOE_B200_OK;
}

int moe_b200_pipeline_submit(moe_b200_pipeline* pl, const void* host_input,
                             const void* host_router_probs, void* host_output,
                             int64_t num_rows) {
  moe::clear_stale_cuda_error();
  if (pl == nullptr) return moe::set_error(MOE_B200_INVALID_ARGUMENT, "pipeline is NULL");
  if (num_rows < 0 || num_rows > pl->problem.num_rows)
    return moe::set_error(MOE_B200_INVALID_ARGUMENT,
                          "num_rows=%lld outside [0, %lld] (the pipeline's largest call)",
                          (long long)num_rows, (long long)pl->problem.num_rows);
  if (num_rows > 0 && (host_input == nullptr || host_router_probs == nullptr ||
                       host_output == nullptr))
    return moe::set_error(MOE_B200_INVALID_ARGUMENT, "host buffers must be non-NULL");
  PL_CHECK(cudaSetDevice(pl->device), "cudaSetDevice");
  auto& s = pl->slots[pl->calls % pl->depth];
  const size_t n = static_cast<size_t>(num_rows);
  if (pl->calls >= pl->depth) PL_CHECK(cudaStreamWaitEvent(pl->s_in, s.comp_done, 0), "wait");
  PL_CHECK(cudaMemcpyAsync(s.x, host_input, n * pl->in_bytes, cudaMemcpyHostToDevice, pl->s_in),
           "H2D input");
  PL_CHECK(cudaMemcpyAsync(s.lg, host_router_probs, n * pl->lg_bytes, cudaMemcpyHostToDevice,
                           pl->s_in),
           "H2D router_probs");
  PL_CHECK(cudaEventRecord(s.in_done, pl->s_in), "record");

  PL_CHECK(cudaStreamWaitEvent(pl->s_comp, s.in_done, 0), "wait");
  if (pl->calls >= pl->depth) PL_CHECK(cudaStreamWaitEvent(pl->s_comp, s.out_done, 0), "wait");
  moe_b200_problem p = pl->problem;
  p.num_rows = num_rows;
  moe_b200_tensors t = pl->weights;
  t.input = s.x;
  t.router_probs = s.lg;
  t.output = s.out;
  const int st = moe_b200_forward_prepacked(&p, &t, pl->prepacked, pl->workspace, pl->ws_bytes,
                                            pl->s_comp, nullptr, 0);
  if (st != MOE_B200_OK) return st;
  PL_CHECK(cudaEventRecord(s.comp_done, pl->s_comp), "record");

  PL_CHECK(cudaStreamWaitEvent(pl->s_out, s.comp_done, 0), "wait");
  PL_CHECK(cudaMemcpyAsync(host_output, s.out, n * pl->out_bytes, cudaMemcpyDeviceToHost,
                           pl->s_out),
           "D2H output");
  PL_CHECK(cudaEventRecord(s.out_done, pl->s_out), "record");
  ++pl->calls;
  return MOE_B200_OK;
}

int moe_b200_pipeline_synchronize(moe_b200_pipeline* pl) {
  if (pl == nullptr) return moe::set_error(MOE_B200_INVALID_ARGUMENT, "pipeline is NULL");
  PL_CHECK(cudaSetDevice(pl->device), "cudaSetDevice");
  PL_CHECK(cudaStreamSynchronize(pl->s_in), "copy-in stream");
  PL_CHECK(cudaStreamSynchronize(pl->s_comp), "compute stream");
  PL_CHECK(cudaStreamSynchronize(pl->s_out), "copy-out stream");
  return MOE_B200_OK;
}

int moe_b200_pipeline_destroy(moe_b200_pipeline* pl) {
  if (pl == nullptr) return MOE_B200_OK;
  cudaSetDevice(pl->device);
  cudaStreamSynchronize(pl->s_in);
  cudaStreamSynchronize(pl->s_comp);
  cudaStreamSynchronize(pl->s_out);
  destroy(pl);
  return MOE_B200_OK;
}

}  // extern "C"
