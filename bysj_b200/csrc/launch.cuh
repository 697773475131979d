// Launch-shape helpers shared by the kernels' host code.
#pragma once

#include "common.cuh"

namespace bysj {

constexpr int kBlock = 256;           // 8 warps per CTA
constexpr int kWarpsPerBlock = kBlock / kWarp;

// Resident CTAs per SM for `kernel` at `threads` threads per CTA (cached per
// device).
int resident_blocks(const void* kernel, size_t dynamic_smem = 0, int threads = kBlock);
// Raises the kernel's dynamic shared memory limit to `bytes` (needed above
// 48 KB) once per kernel and device; BYSJ_OK or an error status.
int allow_dynamic_smem(const void* kernel, size_t bytes);

// Merge-path partitioning for a kernel whose warps each own one partition:
// one wave of resident warps, but never fewer than `min_items` items each.
struct PartitionPlan {
  int64_t parts = 1;
  int64_t ipc = 1;
  unsigned blocks = 1;
};

inline PartitionPlan plan_partitions(int64_t n_edges, int64_t n_nodes,
                                     int64_t resident_warps,
                                     int64_t min_items) {
  PartitionPlan plan;
  const int64_t total = n_edges + n_nodes;
  int64_t parts = resident_warps < 1 ? 1 : resident_warps;
  const int64_t cap = (total + min_items - 1) / min_items;
  if (parts > cap) parts = cap;
  if (parts < 1) parts = 1;
  plan.ipc = (total + parts - 1) / parts;
  if (plan.ipc < 1) plan.ipc = 1;
  plan.parts = (total + plan.ipc - 1) / plan.ipc;
  if (plan.parts < 1) plan.parts = 1;
  plan.blocks = static_cast<unsigned>((plan.parts + kWarpsPerBlock - 1) /
                                      kWarpsPerBlock);
  return plan;
}

inline int64_t next_pow2(int64_t v) {
  int64_t p = 1;
  while (p < v) p <<= 1;
  return p;
}

}  // namespace bysj
