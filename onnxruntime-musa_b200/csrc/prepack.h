// QMoE weight prepack: dequantised copies of a node's expert weights, made once when
// the session is initialised and, on request, shared between nodes of equal content.
#pragma once

#include <atomic>
#include <cstddef>
#include <cstdint>

#include "../../include/moe_b200.h"

struct moe_b200_prepacked {
  std::atomic<int> refs{1};
  int device = 0;
  // Shape of the weights this prepack was made from (the problem's row count is not
  // part of it).
  int32_t dtype = 0;
  int64_t E = 0, H = 0, I = 0, n1 = 0;
  int32_t has_fc3 = 0, bits = 0, block = 0;
  bool shared = false;    // registered for sharing under `key`
  uint64_t key = 0;       // content hash of codes and scales
  void* base = nullptr;   // one device allocation holding w1, w2, w3
  size_t bytes = 0;
  const void* w1 = nullptr;
  const void* w2 = nullptr;
  const void* w3 = nullptr;
};

namespace moe {

// Routed rows (tokens x k) from which a QMoE call with a prepack runs the fp16/bf16
// tensor-core GEMMs on the prepacked weights (MOE_B200_PREPACK_MIN_ROWS overrides).
// Decode-sized calls always stream the packed codes (half or a quarter of the bytes).
// Above them the prepacked GEMMs were faster at every size measured on B200 (C5 shapes,
// int8 per-row: 0.46 vs 0.66 ms at 512 tokens, 1.27 vs 1.46 ms at 4096): the fp16
// kernel has swapped tail tiles for experts with few rows, and no conversion warps.
constexpr int64_t kPrepackMinRows = 0;

// True when `pk` was made from weights of the problem's shape.
bool prepack_matches(const moe_b200_prepacked& pk, const moe_b200_problem& p);

// True when a call of problem `p` takes the prepacked weights.
bool prepack_applies(const moe_b200_prepacked* pk, const moe_b200_problem& p);

}  // namespace moe
