// moe_b200_route_noalloc: the router with its scratch in a static device array.
//
// moe_b200_route needs a small scratch buffer (one expert histogram per 256-row
// chunk) and allocates it with stream-ordered cudaMallocAsync on every call.  Some
// callers cannot allocate device memory at the point where they route: an inference
// loop whose memory is planned up front and must not touch the allocator mid-run
// (allocation can synchronise or fail under memory pressure), or a host whose device
// memory is owned by an arena (ONNX Runtime's allocator policy) and that only hands a
// kernel its inputs and outputs.  This entry point gives them the same routing without
// any allocation: the scratch is the file-scope array below, which every GPU that
// loads the library holds until the process exits.
//
// Limits and sharing:
//   * at most kNoallocScratchInts histogram entries: ceil(num_rows / 256) * num_experts
//     <= 65536 (256 KiB), e.g. 65536 rows with 256 experts or 1M rows with 16 experts;
//     larger calls are rejected with MOE_B200_INVALID_ARGUMENT;
//   * every call on a device shares the one array, which keeps the last call's
//     contents; the router kernel writes every histogram entry it uses before it is
//     read, so nothing needs clearing between calls;
//   * calls that overlap on the GPU (two streams at once on the same device) race on
//     the array and must be serialised by the caller;
//   * the first call on each device looks up the array's device address
//     (cudaGetSymbolAddress, with that device current) and caches it, so make the
//     first call on a device before any stream capture.
#include <mutex>

#include "../../include/moe_b200.h"
#include "moe_kernels.h"

namespace {

constexpr int64_t kNoallocScratchInts = 65536;  // 256 KiB of int32

static __device__ __align__(256) int32_t g_route_scratch[kNoallocScratchInts];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {nullptr};

// Device address of g_route_scratch on the current device (set up once per device).
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t st = cudaGetDevice(&dev);
  if (st != cudaSuccess)
    return moe::set_error(MOE_B200_EP_FAIL, "cudaGetDevice: %s", cudaGetErrorString(st));
  if (dev < 0 || dev >= kMaxDevices)
    return moe::set_error(MOE_B200_EP_FAIL, "device %d is beyond the supported %d", dev,
                          kMaxDevices);
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    st = cudaGetSymbolAddress(&p, g_route_scratch);
    if (st != cudaSuccess || p == nullptr)
      return moe::set_error(MOE_B200_EP_FAIL, "cudaGetSymbolAddress(route scratch): %s",
                            cudaGetErrorString(st));
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return MOE_B200_OK;
}

}  // namespace

extern "C" int moe_b200_route_noalloc(const void* router_probs, int32_t dtype,
                                      int64_t num_rows, int64_t num_experts, int32_t k,
                                      int32_t normalize_routing_weights, int32_t* expert_idx,
                                      float* route_weight, void* stream) {
  moe::clear_stale_cuda_error();
  if (dtype != moe::kDtF32 && dtype != moe::kDtF16 && dtype != moe::kDtBF16)
    return moe::set_error(MOE_B200_NOT_IMPLEMENTED, "unsupported dtype %d", dtype);
  if (num_experts < 1 || num_experts > moe::kMaxExperts || k < 1 || k > num_experts ||
      k > moe::kMaxK || num_rows < 0)
    return moe::set_error(MOE_B200_INVALID_ARGUMENT, "invalid routing shape");
  if (normalize_routing_weights < 0 || normalize_routing_weights > moe::kRouteSparseMixer ||
      (normalize_routing_weights == moe::kRouteSparseMixer && k != 2))
    return moe::set_error(MOE_B200_INVALID_ARGUMENT,
                          "routing mode %d: 0, 1, or 2 (sparse mixer, k = 2)",
                          normalize_routing_weights);
  const int64_t need = static_cast<int64_t>(moe::num_route_chunks(num_rows)) * num_experts;
  if (need > kNoallocScratchInts)
    return moe::set_error(MOE_B200_INVALID_ARGUMENT,
                          "moe_b200_route_noalloc: ceil(num_rows/256) * num_experts = %lld "
                          "exceeds the static scratch of %lld entries; use moe_b200_route",
                          static_cast<long long>(need),
                          static_cast<long long>(kNoallocScratchInts));
  if (num_rows == 0) return MOE_B200_OK;
  void* scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc != MOE_B200_OK) return rc;
  cudaError_t st = moe::launch_route(dtype, router_probs, static_cast<int>(num_rows),
                                     static_cast<int>(num_experts), k,
                                     normalize_routing_weights, expert_idx, route_weight,
                                     static_cast<int32_t*>(scratch),
                                     static_cast<cudaStream_t>(stream));
  if (st != cudaSuccess)
    return moe::set_error(MOE_B200_EP_FAIL, "route: %s", cudaGetErrorString(st));
  return MOE_B200_OK;
}
