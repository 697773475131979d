// Opt-in index guard (sm_100a): the checks the kernels do not make.
//
// Every operator trusts its index inputs (as the reference's native paths
// do, python/kernels/gie.py:80-81): an offsets array that is not a CSR prefix
// sum, an order that is not a permutation, or a slot table pointing past the
// radial slots would make a kernel read out of bounds.  This pass checks those
// invariants on the device and ORs a bit per violated invariant into a device
// error word, which the caller reads back -- the stand-in for a debug build
// that bounds-checks every index read (compute-sanitizer is not available on
// the target pool).  The Python layer runs it when grouping validation is
// asked for (check_grouping=True or DPA4_CHECK_GROUPING=1).
#include "launch.cuh"

namespace bysj {
namespace {

// offsets[0] == 0, offsets[n_nodes] == n_edges, 0 <= offsets[i] <= offsets[i+1].
__global__ void __launch_bounds__(kBlock)
    guard_offsets_kernel(const int64_t* __restrict__ offsets, int64_t n_nodes,
                         int64_t n_edges, uint32_t* error) {
  uint32_t bad = 0;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i <= n_nodes;
       i += stride) {
    const int64_t v = __ldg(offsets + i);
    if (v < 0 || v > n_edges) bad = 1;
    if (i == 0 && v != 0) bad = 1;
    if (i == n_nodes && v != n_edges) bad = 1;
    if (i < n_nodes && v > __ldg(offsets + i + 1)) bad = 1;
  }
  if (__any_sync(kFull, bad) && lane_id() == 0) atomicOr(error, BYSJ_INDEX_OFFSETS);
}

// order[e] in [0, n_edges), no value twice (so a permutation): one bit per
// edge in `seen` (zeroed by the caller); a bit found already set is a repeat.
__global__ void __launch_bounds__(kBlock)
    guard_order_kernel(const int64_t* __restrict__ order, int64_t n_edges,
                       unsigned* __restrict__ seen, uint32_t* error) {
  uint32_t bad = 0;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < n_edges;
       e += stride) {
    const int64_t v = __ldg(order + e);
    if (v < 0 || v >= n_edges) {
      bad = 1;
      continue;
    }
    const unsigned bit = 1u << (v & 31);
    if (atomicOr(seen + (v >> 5), bit) & bit) bad = 1;
  }
  if (__any_sync(kFull, bad) && lane_id() == 0) atomicOr(error, BYSJ_INDEX_ORDER);
}

// values[i] in [0, limit).
__global__ void __launch_bounds__(kBlock)
    guard_values_kernel(const int64_t* __restrict__ values, int64_t n, int64_t limit,
                        uint32_t* error) {
  uint32_t bad = 0;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += stride) {
    const int64_t v = __ldg(values + i);
    if (v < 0 || v >= limit) bad = 1;
  }
  if (__any_sync(kFull, bad) && lane_id() == 0) atomicOr(error, BYSJ_INDEX_VALUES);
}

unsigned guard_blocks(int64_t items) {
  int64_t blocks = (items + kBlock - 1) / kBlock;
  const int64_t cap = static_cast<int64_t>(current_device_info().sm_count) * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return static_cast<unsigned>(blocks);
}

}  // namespace
}  // namespace bysj

using namespace bysj;

extern "C" {

size_t bysj_check_indices_workspace_size(int64_t n_edges) {
  if (n_edges < 0) return 0;
  return sizeof(unsigned) * static_cast<size_t>((n_edges + 31) / 32 + 1);
}

int bysj_check_indices(const int64_t* offsets, int64_t n_nodes, int64_t n_edges,
                       const int64_t* order, const int64_t* values, int64_t n_values,
                       int64_t value_limit, uint32_t* error, void* workspace,
                       size_t workspace_bytes, void* stream) {
  clear_error();
  if (n_nodes < 0 || n_edges < 0 || n_values < 0)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "index guard: invalid sizes");
  if (error == nullptr) return fail(BYSJ_ERR_INVALID_ARGUMENT, "index guard: NULL error word");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int st = BYSJ_OK;
  if (offsets != nullptr) {
    guard_offsets_kernel<<<guard_blocks(n_nodes + 1), kBlock, 0, s>>>(offsets, n_nodes, n_edges,
                                                                      error);
    st = launch_check("guard_offsets_kernel");
    if (st) return st;
  }
  if (order != nullptr && n_edges > 0) {
    const size_t need = bysj_check_indices_workspace_size(n_edges);
    if (workspace == nullptr || workspace_bytes < need)
      return fail(BYSJ_ERR_WORKSPACE, "index guard: workspace of %zu bytes needed, %zu given",
                  need, workspace_bytes);
    st = cuda_check(cudaMemsetAsync(workspace, 0, need, s), "index guard: bitmap reset");
    if (st) return st;
    guard_order_kernel<<<guard_blocks(n_edges), kBlock, 0, s>>>(
        order, n_edges, static_cast<unsigned*>(workspace), error);
    st = launch_check("guard_order_kernel");
    if (st) return st;
  }
  if (values != nullptr && n_values > 0) {
    guard_values_kernel<<<guard_blocks(n_values), kBlock, 0, s>>>(values, n_values, value_limit,
                                                                  error);
    st = launch_check("guard_values_kernel");
  }
  return st;
}

}  // extern "C"
