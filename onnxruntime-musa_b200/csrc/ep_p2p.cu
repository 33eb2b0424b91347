// Device-side expert parallelism over peer memory (NVLink P2P, one process per GPU).
//
// Every rank owns one "symmetric" device allocation with the same layout (EpLayout):
// a receive buffer for the rows routed to its experts, a return buffer for the FFN rows
// of its own tokens, a count matrix and phase flags.  The allocations are exchanged once
// as CUDA IPC handles; afterwards a layer call needs no host synchronisation and no
// collective library on its data path:
//   counts   each rank stores its per-expert counts into every rank's count matrix and
//            raises a flag; one CTA per rank waits for all flags (bounded) and derives
//            every offset table on the device;
//   rows     the dispatch gather writes each routed row straight into the receive
//            buffer of the rank that owns its expert (16-byte stores over NVLink);
//   return   the fc2 epilogue of the grouped GEMM stores each output row straight into
//            the return buffer of the rank that sent it (moe_api.cu: GemmArgs remap);
//   combine  reads the local return buffer.
// A flag is the call's epoch (a per-communicator counter), stored with release
// semantics at system scope after a system-scope fence; waiters poll with acquire
// loads for at most kWaitLimitNs and report kErrTimeoutPeer instead of hanging.
// No TMA multicast and no NVLink multicast object is involved: plain loads and stores.
//
// The reference EP has no multi-device path (one EP instance drives one device,
// musa/ep/src/ep_factory.cc:466-470); this is the dispatch / combine all-to-all of the
// MoE path, fused into the gather and into the fc2 epilogue.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

#include "../../include/moe_b200.h"
#include "ep_p2p.h"

namespace moe {

namespace {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_sys(int32_t* p, int32_t v) {
  asm volatile("st.relaxed.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int32_t ld_relaxed_sys(const int32_t* p) {
  int32_t v;
  asm volatile("ld.relaxed.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t* flag_ptr(uint8_t* base, const EpLayout& lay, int phase,
                                              int src) {
  return reinterpret_cast<uint32_t*>(base + lay.flags) + phase * kMaxEpRanks + src;
}

// Bounded wait of lane `src` for flag [phase][src] of this rank == epoch.
__device__ bool wait_flag(uint8_t* own, const EpLayout& lay, int phase, int src,
                          uint32_t epoch) {
  const uint32_t* f = flag_ptr(own, lay, phase, src);
  if (ld_acquire_sys(f) == epoch) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (ld_acquire_sys(f) == epoch) return true;
    if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
  }
}

struct CountsArgs {
  EpPeers peers;
  EpLayout lay;
  int rank, W, E;
  uint32_t epoch;
  const int32_t* myoff;
  EpTables tab;
  int* err;
};

constexpr int kCountsThreads = 256;

__global__ void __launch_bounds__(kCountsThreads) ep_exchange_counts_kernel(const CountsArgs a) {
  __shared__ int32_t sC[kMaxEpRanks * kMaxExperts];       // C[s][e]
  __shared__ int32_t sP[kMaxEpRanks * (kMaxExperts + 1)];  // prefix over e of row s
  __shared__ int32_t sQ[kMaxExperts + 1];                  // prefix over local experts of
                                                           // the column sums, per owner
  __shared__ int s_ok;
  const int tid = threadIdx.x;
  const int W = a.W, E = a.E, El = E / W, r = a.rank;
  const int par = static_cast<int>(a.epoch & 1u);
  uint8_t* own = a.peers.base[r];
  if (tid < kClearWords) a.err[tid] = 0;
  if (tid == 0) s_ok = 1;

  // 1. My counts into every rank's count matrix, row `r`.
  for (int e = tid; e < E; e += blockDim.x) {
    const int32_t c = a.myoff != nullptr ? a.myoff[e + 1] - a.myoff[e] : 0;
    for (int d = 0; d < W; ++d) {
      int32_t* dst = reinterpret_cast<int32_t*>(a.peers.base[d] + a.lay.cnt) +
                     (par * W + r) * E + e;
      st_relaxed_sys(dst, c);
    }
  }
  __syncthreads();
  if (tid < W) {
    __threadfence_system();
    st_release_sys(flag_ptr(a.peers.base[tid], a.lay, kEpCounts, r), a.epoch);
  }
  // 2. Every rank's counts of this call.
  if (tid < W && !wait_flag(own, a.lay, kEpCounts, tid, a.epoch)) {
    atomicExch(a.err, kErrTimeoutPeer);
    s_ok = 0;
  }
  __syncthreads();
  __threadfence_system();
  const int32_t* cnt = reinterpret_cast<const int32_t*>(own + a.lay.cnt) + par * W * E;
  for (int i = tid; i < W * E; i += blockDim.x) sC[i] = s_ok ? ld_relaxed_sys(cnt + i) : 0;
  __syncthreads();

  // 3. Prefixes: sP[s][e] = sum_{e' < e} C[s][e'] (source s's permuted offsets) and, per
  // owner d, sQ[d*El + j] = sum_{j' < j} sum_s C[s][d*El + j'] (receive offsets at d).
  if (tid < W) {
    int32_t acc = 0;
    for (int e = 0; e < E; ++e) {
      sP[tid * (E + 1) + e] = acc;
      acc += sC[tid * E + e];
    }
    sP[tid * (E + 1) + E] = acc;
  }
  if (tid >= 32 && tid - 32 < W) {
    const int d = tid - 32;
    int32_t acc = 0;
    for (int j = 0; j < El; ++j) {
      sQ[d * El + j] = acc;
      for (int s = 0; s < W; ++s) acc += sC[s * E + d * El + j];
    }
    if (d == r) sQ[E] = acc;  // rows this rank receives
  }
  __syncthreads();

  // 4. Send table: row p of expert e lands at row Q[e] + sum_{s<r} C[s][e] + (p - myoff[e])
  // of rank e / El.
  for (int e = tid; e < E; e += blockDim.x) {
    int32_t before = 0;
    for (int s = 0; s < r; ++s) before += sC[s * E + e];
    a.tab.send_base[e] = sQ[e] + before - sP[r * (E + 1) + e];
  }
  // 5. Receive layout: local expert j, then source s; segment (j, s) returns to row
  // P[s][r*El + j] of source s's return buffer.
  for (int q = tid; q < El * W; q += blockDim.x) {
    const int j = q / W, s = q % W;
    const int e = r * El + j;
    int32_t before = 0;
    for (int s2 = 0; s2 < s; ++s2) before += sC[s2 * E + e];
    a.tab.seg_start[q] = sQ[e] + before;
    a.tab.seg_dst[q] = sP[s * (E + 1) + e];
  }
  if (tid == 0) {
    int32_t o = 0, t1 = 0, t2 = 0, t3 = 0;
    for (int j = 0; j < El; ++j) {
      a.tab.eoff[j] = o;
      a.tab.t128[j] = t1;
      a.tab.t64[j] = t2;
      a.tab.t256[j] = t3;
      int32_t c = 0;
      for (int s = 0; s < W; ++s) c += sC[s * E + r * El + j];
      o += c;
      t1 += (c + 127) / 128;
      t2 += (c + 63) / 64;
      t3 += (c + 255) / 256;
    }
    a.tab.eoff[El] = o;
    a.tab.t128[El] = t1;
    a.tab.t64[El] = t2;
    a.tab.t256[El] = t3;
    a.tab.seg_start[El * W] = o;
  }
}

struct SendArgs {
  EpPeers peers;
  size_t recv_off;
  size_t tok_off, gidx_off;  // dedup: token buffer and gather index (tok_off 0: off)
  int rank;
  int64_t max_rows;
  int E, El;
  const uint8_t* x;
  int64_t row_bytes;
  int k;
  const int32_t* idx;
  const int32_t* src;
  int64_t rows;
  const int32_t* send_base;
  const int* err;
};

// One warp per routed row, 16-byte stores into the owner's receive buffer.
__global__ void __launch_bounds__(256) ep_send_rows_kernel(const SendArgs a) {
  if (*reinterpret_cast<const volatile int*>(a.err) != 0) return;  // counts never arrived
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t vecs = a.row_bytes / 16;
  for (int64_t p = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       p < a.rows; p += warps) {
    const int32_t sidx = a.src[p];
    const int e = a.idx[sidx];
    const int d = e / a.El;
    const int64_t drow = static_cast<int64_t>(a.send_base[e]) + p;
    const int t = sidx / a.k;
    const uint4* srow = reinterpret_cast<const uint4*>(a.x + t * a.row_bytes);
    if (a.tok_off != 0) {
      // Receive row drow is gathered from token row rank * max_rows + t at rank d; the
      // token itself travels once: with its first slot that rank d owns.
      const int64_t trow = static_cast<int64_t>(a.rank) * a.max_rows + t;
      if (lane == 0)
        reinterpret_cast<int32_t*>(a.peers.base[d] + a.gidx_off)[drow] = static_cast<int32_t>(trow);
      const int j = sidx - t * a.k;
      bool first = true;
      for (int j2 = 0; j2 < j; ++j2) first &= a.idx[t * a.k + j2] / a.El != d;
      if (!first) continue;
      uint4* trow_ptr = reinterpret_cast<uint4*>(a.peers.base[d] + a.tok_off + trow * a.row_bytes);
      for (int64_t i = lane; i < vecs; i += 32) trow_ptr[i] = srow[i];
      continue;
    }
    uint4* drow_ptr = reinterpret_cast<uint4*>(a.peers.base[d] + a.recv_off + drow * a.row_bytes);
    for (int64_t i = lane; i < vecs; i += 32) drow_ptr[i] = srow[i];
  }
}

// Receive row x = token row gidx[x] (own region), one warp per row, rows below the
// device-side count eoff_total[0].
__global__ void __launch_bounds__(256)
ep_gather_tokens_kernel(uint8_t* own, size_t recv_off, size_t tok_off, size_t gidx_off,
                        int64_t row_bytes, const int32_t* eoff_total, const int* err) {
  if (*reinterpret_cast<const volatile int*>(err) != 0) return;
  const int lane = threadIdx.x & 31;
  const int64_t total = *eoff_total;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t vecs = row_bytes / 16;
  const int32_t* gidx = reinterpret_cast<const int32_t*>(own + gidx_off);
  for (int64_t x = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       x < total; x += warps) {
    const int64_t trow = gidx[x];
    const uint4* src = reinterpret_cast<const uint4*>(own + tok_off + trow * row_bytes);
    uint4* dst = reinterpret_cast<uint4*>(own + recv_off + x * row_bytes);
    for (int64_t i = lane; i < vecs; i += 32) dst[i] = src[i];
  }
}

__global__ void ep_signal_kernel(const EpPeers peers, const EpLayout lay, int rank, int W,
                                 int phase, uint32_t epoch) {
  __threadfence_system();
  const int d = threadIdx.x;
  if (d < W) st_release_sys(flag_ptr(peers.base[d], lay, phase, rank), epoch);
}

__global__ void ep_wait_kernel(uint8_t* own, const EpLayout lay, int W, int phase, uint32_t epoch,
                               int* err) {
  const int s = threadIdx.x;
  if (s < W && !wait_flag(own, lay, phase, s, epoch)) atomicExch(err, kErrTimeoutPeer);
  __threadfence_system();
}

}  // namespace

cudaError_t launch_ep_exchange_counts(const EpPeers& peers, const EpLayout& lay, int rank,
                                      int W, int E, uint32_t epoch, const int32_t* myoff,
                                      const EpTables& tab, int* err, cudaStream_t s) {
  CountsArgs a{peers, lay, rank, W, E, epoch, myoff, tab, err};
  ep_exchange_counts_kernel<<<1, kCountsThreads, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_ep_send_rows(const EpPeers& peers, const EpLayout& lay, int rank, int W, int E,
                                const void* x, int64_t row_bytes, int k, const int32_t* idx,
                                const int32_t* src, int64_t rows, const int32_t* send_base,
                                int64_t max_rows, bool dedup, const int* err, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  if (dedup && lay.tok == 0) return cudaErrorInvalidValue;
  SendArgs a{peers, lay.recv, dedup ? lay.tok : 0, lay.gidx, rank, max_rows, E, E / W,
             static_cast<const uint8_t*>(x), row_bytes, k, idx, src, rows, send_base, err};
  const int64_t blocks = std::min<int64_t>((rows + 7) / 8, 148 * 8);
  ep_send_rows_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_ep_gather_tokens(uint8_t* own, const EpLayout& lay, int64_t row_bytes,
                                    const int32_t* eoff_total, int64_t cap_rows, const int* err,
                                    cudaStream_t s) {
  if (lay.tok == 0) return cudaErrorInvalidValue;
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((cap_rows + 7) / 8, 148 * 8));
  ep_gather_tokens_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(
      own, lay.recv, lay.tok, lay.gidx, row_bytes, eoff_total, err);
  return cudaGetLastError();
}

cudaError_t launch_ep_signal(const EpPeers& peers, const EpLayout& lay, int rank, int W,
                             int phase, uint32_t epoch, cudaStream_t s) {
  ep_signal_kernel<<<1, 32, 0, s>>>(peers, lay, rank, W, phase, epoch);
  return cudaGetLastError();
}

cudaError_t launch_ep_wait(uint8_t* own, const EpLayout& lay, int W, int phase, uint32_t epoch,
                           int* err, cudaStream_t s) {
  ep_wait_kernel<<<1, 32, 0, s>>>(own, lay, W, phase, epoch, err);
  return cudaGetLastError();
}

}  // namespace moe

// ---------------------------------------------------------------------------- C ABI
namespace {

size_t align256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

moe::EpLayout ep_layout(int64_t cap_rows, int64_t ret_rows, int64_t row_bytes, int W, int E,
                        int64_t tok_rows) {
  moe::EpLayout l{};
  size_t o = 0;
  l.recv = o;
  o = align256(o + static_cast<size_t>(cap_rows) * row_bytes);
  l.ret = o;
  o = align256(o + static_cast<size_t>(ret_rows) * row_bytes);
  l.cnt = o;
  o = align256(o + 2 * static_cast<size_t>(W) * E * sizeof(int32_t));
  l.flags = o;
  o = align256(o + 3 * moe::kMaxEpRanks * sizeof(uint32_t));
  if (tok_rows > 0) {
    l.tok = o;
    o = align256(o + static_cast<size_t>(tok_rows) * row_bytes);
    l.gidx = o;
    o = align256(o + static_cast<size_t>(cap_rows) * sizeof(int32_t));
  }
  l.total = o;
  return l;
}

int cuda_fail(cudaError_t st, const char* what) {
  return moe::set_error(MOE_B200_EP_FAIL, "%s: %s", what, cudaGetErrorString(st));
}

// Travels after the IPC handle: the parameters that fix a region's layout.  Peers store
// rows and flags at offsets computed from their own layout, so every rank must hold the
// same one; connect compares them before it opens any peer region.
struct EpHandleDesc {
  uint32_t magic;
  int32_t rank, world, k_max, num_experts, dtype;
  int64_t max_rows, hidden;
  uint64_t total;
};
constexpr uint32_t kEpHandleMagic = 0x4d4f4550u;  // "MOEP"

EpHandleDesc describe(const moe_b200_ep_comm* c) {
  EpHandleDesc d{};
  d.magic = kEpHandleMagic;
  d.rank = c->rank;
  d.world = c->world;
  d.k_max = c->k_max;
  d.num_experts = c->num_experts;
  d.dtype = c->dtype;
  d.max_rows = c->max_rows;
  d.hidden = c->hidden;
  d.total = c->lay.total;
  return d;
}

constexpr size_t kEpHandleBytes = sizeof(cudaIpcMemHandle_t) + sizeof(EpHandleDesc);

}  // namespace

extern "C" {

int moe_b200_ep_comm_create(int32_t rank, int32_t world, int64_t max_rows, int32_t k_max,
                            int64_t hidden_size, int64_t num_experts, int32_t dtype,
                            moe_b200_ep_comm** comm) {
  moe::clear_stale_cuda_error();
  if (comm == nullptr) return moe::set_error(MOE_B200_INVALID_ARGUMENT, "comm is NULL");
  if (world < 1 || world > moe::kMaxEpRanks || rank < 0 || rank >= world)
    return moe::set_error(MOE_B200_INVALID_ARGUMENT, "rank %d / world %d (world <= %d)", rank,
                          world, moe::kMaxEpRanks);
  if (dtype != MOE_B200_FLOAT16 && dtype != MOE_B200_BFLOAT16)
    return moe::set_error(MOE_B200_NOT_IMPLEMENTED,
                          "device-side expert parallelism runs fp16/bf16 layers");
  if (num_experts < world || num_experts % world != 0 || num_experts > moe::kMaxExperts)
    return moe::set_error(MOE_B200_INVALID_ARGUMENT, "%lld experts do not split over %d ranks",
                          (long long)num_experts, world);
  if (max_rows < 1 || k_max < 1 || hidden_size < 8 || hidden_size % 8 != 0)
    return moe::set_error(MOE_B200_INVALID_ARGUMENT,
                          "max_rows, k_max >= 1 and hidden_size a multiple of 8 required");
  auto* c = new moe_b200_ep_comm();
  c->rank = rank;
  c->world = world;
  c->max_rows = max_rows;
  c->k_max = k_max;
  c->hidden = hidden_size;
  c->num_experts = static_cast<int>(num_experts);
  c->dtype = dtype;
  c->cap_rows = static_cast<int64_t>(world) * max_rows * k_max;
  const int64_t row_bytes = hidden_size * 2;
  c->lay = ep_layout(c->cap_rows, max_rows * k_max, row_bytes, world,
                     static_cast<int>(num_experts),
                     k_max >= moe::kEpDedupMinK ? static_cast<int64_t>(world) * max_rows : 0);
  cudaError_t e = cudaGetDevice(&c->device);
  if (e == cudaSuccess) e = cudaMalloc(&c->sym, c->lay.total);
  if (e == cudaSuccess) e = cudaMemset(c->sym + c->lay.cnt, 0, c->lay.total - c->lay.cnt);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    if (c->sym) cudaFree(c->sym);
    delete c;
    return cuda_fail(e, "ep communicator buffers");
  }
  c->peers.base[rank] = c->sym;
  *comm = c;
  return MOE_B200_OK;
}

int moe_b200_ep_comm_handle_size(size_t* bytes) {
  if (bytes == nullptr) return moe::set_error(MOE_B200_INVALID_ARGUMENT, "bytes is NULL");
  *bytes = kEpHandleBytes;
  return MOE_B200_OK;
}

int moe_b200_ep_comm_get_handle(moe_b200_ep_comm* c, void* handle) {
  if (c == nullptr || handle == nullptr)
    return moe::set_error(MOE_B200_INVALID_ARGUMENT, "comm and handle must be non-NULL");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, c->sym);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  const EpHandleDesc d = describe(c);
  std::memcpy(handle, &h, sizeof(h));
  std::memcpy(static_cast<uint8_t*>(handle) + sizeof(h), &d, sizeof(d));
  return MOE_B200_OK;
}

int moe_b200_ep_comm_connect(moe_b200_ep_comm* c, const void* handles) {
  if (c == nullptr || handles == nullptr)
    return moe::set_error(MOE_B200_INVALID_ARGUMENT, "comm and handles must be non-NULL");
  if (c->connected) return moe::set_error(MOE_B200_INVALID_ARGUMENT, "already connected");
  const uint8_t* blob = static_cast<const uint8_t*>(handles);
  const EpHandleDesc mine = describe(c);
  for (int d = 0; d < c->world; ++d) {
    if (d == c->rank) continue;
    EpHandleDesc o;
    std::memcpy(&o, blob + d * kEpHandleBytes + sizeof(cudaIpcMemHandle_t), sizeof(o));
    if (o.magic != kEpHandleMagic || o.rank != d)
      return moe::set_error(MOE_B200_INVALID_ARGUMENT,
                            "handle %d is not a moe_b200_ep_comm handle of rank %d", d, d);
    if (o.world != mine.world || o.k_max != mine.k_max || o.num_experts != mine.num_experts ||
        o.dtype != mine.dtype || o.max_rows != mine.max_rows || o.hidden != mine.hidden ||
        o.total != mine.total)
      return moe::set_error(
          MOE_B200_INVALID_ARGUMENT,
          "rank %d's region differs from rank %d's (world %d/%d, max_rows %lld/%lld, k_max "
          "%d/%d, hidden %lld/%lld, experts %d/%d, dtype %d/%d): every rank must create its "
          "communicator with the same arguments",
          d, c->rank, o.world, mine.world, (long long)o.max_rows, (long long)mine.max_rows,
          o.k_max, mine.k_max, (long long)o.hidden, (long long)mine.hidden, o.num_experts,
          mine.num_experts, o.dtype, mine.dtype);
  }
  cudaError_t e = cudaSetDevice(c->device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  for (int d = 0; d < c->world; ++d) {
    if (d == c->rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, blob + d * kEpHandleBytes, sizeof(h));
    void* ptr = nullptr;
    e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
    c->peers.base[d] = static_cast<uint8_t*>(ptr);
    c->opened[d] = true;
  }
  c->connected = true;
  return MOE_B200_OK;
}

int moe_b200_ep_comm_destroy(moe_b200_ep_comm* c) {
  if (c == nullptr) return MOE_B200_OK;
  cudaSetDevice(c->device);
  cudaDeviceSynchronize();
  for (int d = 0; d < c->world; ++d)
    if (c->opened[d]) cudaIpcCloseMemHandle(c->peers.base[d]);
  cudaFree(c->sym);
  delete c;
  return MOE_B200_OK;
}

int moe_b200_ep_workspace_size(const moe_b200_ep_comm* c, const moe_b200_problem* problem,
                               size_t* bytes) {
  if (c == nullptr || problem == nullptr || bytes == nullptr)
    return moe::set_error(MOE_B200_INVALID_ARGUMENT, "comm, problem and bytes must be non-NULL");
  *bytes = moe::ep_workspace_bytes(c, *problem);
  return MOE_B200_OK;
}

int moe_b200_ep_forward(moe_b200_ep_comm* c, const moe_b200_problem* problem,
                        const moe_b200_tensors* t, void* workspace, size_t workspace_bytes,
                        void* stream) {
  moe::clear_stale_cuda_error();
  if (c == nullptr || problem == nullptr || t == nullptr)
    return moe::set_error(MOE_B200_INVALID_ARGUMENT, "comm, problem and tensors must be non-NULL");
  if (!c->connected) return moe::set_error(MOE_B200_INVALID_ARGUMENT, "comm is not connected");
  return moe::ep_forward_impl(c, *problem, *t, static_cast<uint8_t*>(workspace), workspace_bytes,
                              static_cast<cudaStream_t>(stream));
}

int moe_b200_ep_forward_staged(moe_b200_ep_comm* c, const moe_b200_problem* problem,
                               const moe_b200_tensors* t, void* workspace,
                               size_t workspace_bytes, void* stream, void* const* events,
                               int32_t num_events) {
  moe::clear_stale_cuda_error();
  if (c == nullptr || problem == nullptr || t == nullptr || events == nullptr ||
      num_events < moe::kEpNumPhases + 1)
    return moe::set_error(MOE_B200_INVALID_ARGUMENT,
                          "comm, problem, tensors non-NULL and >= %d events required",
                          moe::kEpNumPhases + 1);
  if (!c->connected) return moe::set_error(MOE_B200_INVALID_ARGUMENT, "comm is not connected");
  cudaEvent_t ev[moe::kEpNumPhases + 1];
  for (int i = 0; i <= moe::kEpNumPhases; ++i) ev[i] = static_cast<cudaEvent_t>(events[i]);
  return moe::ep_forward_impl(c, *problem, *t, static_cast<uint8_t*>(workspace), workspace_bytes,
                              static_cast<cudaStream_t>(stream), ev);
}

}  // extern "C"
