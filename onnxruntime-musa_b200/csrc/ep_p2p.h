// Device-side expert parallelism over peer memory: internal interface between the
// communicator (ep_p2p.cu) and the layer sequence (moe_api.cu).
#pragma once

#include "moe_kernels.h"

namespace moe {

// Offsets inside each rank's symmetric region (same on every rank).
struct EpLayout {
  size_t recv;    // [cap_rows, H]: rows routed to this rank's experts, by (local expert, source)
  size_t ret;     // [max_rows * k_max, H]: FFN rows of this rank's tokens, in its permuted order
  size_t cnt;     // int32 [2][W][E]: per-source expert counts (by call parity)
  size_t flags;   // uint32 [3][kMaxEpRanks]: phase flags (epoch of the last signal per source)
  // Deduplicated dispatch (k_max >= kEpDedupMinK): each token travels once per destination
  // rank into tok ([W * max_rows, H], source s's token t at row s * max_rows + t), and
  // gidx[x] (int32 [cap_rows]) names the tok row of receive row x; the receiver gathers
  // its expert-ordered rows locally.  0 when the region has no such buffers.
  size_t tok;
  size_t gidx;
  size_t total;
};

// Smallest k at which dispatch sends each token once per destination rank.
constexpr int kEpDedupMinK = 4;

enum EpPhase : int { kEpCounts = 0, kEpRows = 1, kEpReturn = 2 };

struct EpPeers {
  uint8_t* base[kMaxEpRanks];   // symmetric region of each rank (own included)
};

// Tables of one call, in the local workspace.
struct EpTables {
  int32_t* send_base;   // [E]: my permuted row p of expert e goes to row send_base[e] + p
                        // of rank e / El's receive buffer
  int32_t* eoff;        // [El+1] receive offsets per local expert
  int32_t* t128;        // [El+1] tile prefixes (128 / 64 / 256 rows)
  int32_t* t64;
  int32_t* t256;
  int32_t* seg_start;   // [El*W+1] receive row start of segment (j, s), q = j*W + s
  int32_t* seg_dst;     // [El*W] row in source s's return buffer
};

// Publishes this rank's per-expert counts (from `myoff`, E+1 offsets; nullptr = no rows)
// to every rank, waits (bounded) for all ranks' counts of this call and builds `tab`.
// Also clears the call's status block (err[0..kClearWords)).
cudaError_t launch_ep_exchange_counts(const EpPeers& peers, const EpLayout& lay, int rank,
                                      int W, int E, uint32_t epoch, const int32_t* myoff,
                                      const EpTables& tab, int* err, cudaStream_t s);
// Copies routed row p (token src[p] / k) into its expert's rank's receive buffer; with
// `dedup` (lay.tok set) it copies each token once per destination rank into that rank's
// token buffer (row rank * max_rows + t) and stores the receive row's tok row in gidx.
cudaError_t launch_ep_send_rows(const EpPeers& peers, const EpLayout& lay, int rank, int W, int E,
                                const void* x, int64_t row_bytes, int k, const int32_t* idx,
                                const int32_t* src, int64_t rows, const int32_t* send_base,
                                int64_t max_rows, bool dedup, const int* err, cudaStream_t s);
// Receiver side of the deduplicated dispatch: receive row x < eoff[El] (a device count)
// = token row gidx[x] of the own token buffer.
cudaError_t launch_ep_gather_tokens(uint8_t* own, const EpLayout& lay, int64_t row_bytes,
                                    const int32_t* eoff_total, int64_t cap_rows, const int* err,
                                    cudaStream_t s);
// After a system-scope fence, stores `epoch` into flag [phase][rank] of every rank.
cudaError_t launch_ep_signal(const EpPeers& peers, const EpLayout& lay, int rank, int W,
                             int phase, uint32_t epoch, cudaStream_t s);
// Waits (bounded) until every rank's flag [phase][*] in this rank's region equals `epoch`.
cudaError_t launch_ep_wait(uint8_t* own, const EpLayout& lay, int W, int phase, uint32_t epoch,
                           int* err, cudaStream_t s);

}  // namespace moe

// The communicator behind the C ABI's moe_b200_ep_comm.
struct moe_b200_ep_comm {
  int rank = 0, world = 1, device = 0;
  int64_t max_rows = 0;   // tokens per call per rank
  int k_max = 1;
  int64_t hidden = 0;
  int num_experts = 0;
  int dtype = 0;
  int64_t cap_rows = 0;   // world * max_rows * k_max
  moe::EpLayout lay{};
  uint8_t* sym = nullptr;
  moe::EpPeers peers{};
  bool opened[moe::kMaxEpRanks] = {};
  bool connected = false;
  uint32_t epoch = 0;
};

namespace moe {
// Layer call of the device-side expert-parallel path (moe_api.cu).
constexpr int kEpNumPhases = 8;
int ep_forward_impl(moe_b200_ep_comm* c, const moe_b200_problem& p, const moe_b200_tensors& t,
                    uint8_t* ws, size_t ws_bytes, cudaStream_t s, cudaEvent_t* ev = nullptr);
size_t ep_workspace_bytes(const moe_b200_ep_comm* c, const moe_b200_problem& p);
}  // namespace moe
