// segment_offsets: exclusive prefix sum of the per-node edge counts.
//
// The reference (python/kernels/segment.py:46-57) does bincount + cumsum
// and a host-synchronising min/max range check.  Two integer-exact device
// paths replace it:
//
//  * sorted: for a destination-sorted edge list the offsets are the segment
//    boundaries, offsets[n] = first e with dst[e] >= n.  One pass validates
//    dst (flags for unsorted or out-of-range input) and writes the
//    boundaries from clamped values, so an unsorted list cannot make it loop
//    or write out of bounds (its offsets are then meaningless).
//  * histogram: any order.  Warp-aggregated integer atomics count the edges
//    per node (lanes holding the same destination are merged with
//    __match_any_sync first), then a three-phase exclusive scan.  Integer
//    addition is associative, so the result is exact and order-independent.
#include "launch.cuh"

namespace bysj {
namespace {

constexpr int kScanTile = 2048;  // elements per CTA in the scan

// The sorted path reads dst as 16-byte pairs (elements 2i, 2i+1), two pairs
// per thread per step so that four loads are in flight; the element before a
// pair comes from its own 8-byte load (an L1 hit: the neighbouring lane read
// it).  `dst` must be 16-byte aligned for the pair loads (the host checks).
constexpr int kPairsPerStep = 2;

__device__ __forceinline__ longlong2 ld_pair(const int64_t* dst, int64_t i) {
  return __ldg(reinterpret_cast<const longlong2*>(dst) + i);
}

// offsets[n] for the nodes in (dst[e-1], dst[e]] is e.
__device__ __forceinline__ void write_boundary(int64_t prev, int64_t cur, int64_t e,
                                               int64_t* __restrict__ offsets) {
  for (int64_t n = prev + 1; n <= cur; ++n) offsets[n] = e;
}

// One pass for a sorted list: validates dst and writes the boundaries in the
// same read of each pair.  Values are clamped to [-1, n_nodes] before a
// boundary is written, so an unsorted or out-of-range list (flagged, its
// offsets meaningless) still writes only offsets[0..n_nodes] and no loop runs
// longer than n_nodes + 1 steps.  For a valid list every offset is written
// exactly once, as by the two-pass form.
__device__ __forceinline__ int64_t clamp_node(int64_t v, int64_t n_nodes) {
  return v < -1 ? -1 : (v > n_nodes ? n_nodes : v);
}

__global__ void __launch_bounds__(kBlock)
    offsets_sorted_fused_kernel(const int64_t* __restrict__ dst, int64_t n_edges,
                                int64_t n_nodes, int64_t* __restrict__ offsets,
                                uint32_t* flags) {
  uint32_t local = 0;
  const int64_t pairs = n_edges / 2;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i0 < pairs;
       i0 += stride * kPairsPerStep) {
    longlong2 v[kPairsPerStep];
    int64_t before[kPairsPerStep];
#pragma unroll
    for (int k = 0; k < kPairsPerStep; ++k) {
      const int64_t i = i0 + k * stride;
      v[k] = i < pairs ? ld_pair(dst, i) : make_longlong2(0, 0);
      before[k] = (i < pairs && i > 0) ? __ldg(dst + 2 * i - 1) : -1;
    }
#pragma unroll
    for (int k = 0; k < kPairsPerStep; ++k) {
      const int64_t i = i0 + k * stride;
      if (i >= pairs) continue;
      const int64_t x = v[k].x, y = v[k].y;
      if (x < 0 || x >= n_nodes || y < 0 || y >= n_nodes) local |= BYSJ_FLAG_OUT_OF_RANGE;
      if (before[k] > x || x > y) local |= BYSJ_FLAG_UNSORTED;
      const int64_t xc = clamp_node(x, n_nodes), yc = clamp_node(y, n_nodes);
      write_boundary(clamp_node(before[k], n_nodes), xc, 2 * i, offsets);
      write_boundary(xc, yc, 2 * i + 1, offsets);
    }
  }
  // The odd last element and the end marker: nodes in (dst[E-1], N] start at E.
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    int64_t prev = n_edges >= 2 ? __ldg(dst + 2 * pairs - 1) : -1;
    if (n_edges & 1) {
      const int64_t last = __ldg(dst + n_edges - 1);
      if (last < 0 || last >= n_nodes) local |= BYSJ_FLAG_OUT_OF_RANGE;
      if (n_edges > 1 && prev > last) local |= BYSJ_FLAG_UNSORTED;
      write_boundary(clamp_node(prev, n_nodes), clamp_node(last, n_nodes), n_edges - 1,
                     offsets);
      prev = last;
    }
    write_boundary(clamp_node(prev, n_nodes), n_nodes, n_edges, offsets);
  }
  local = __reduce_or_sync(kFull, local);
  if (local && lane_id() == 0) atomicOr(flags, local);
}

// Scalar forms for a dst that is not 16-byte aligned.
__global__ void __launch_bounds__(kBlock)
    offsets_check_scalar_kernel(const int64_t* __restrict__ dst, int64_t n_edges,
                                int64_t n_nodes, uint32_t* flags) {
  uint32_t local = 0;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       e < n_edges; e += stride) {
    const int64_t d = __ldg(dst + e);
    if (d < 0 || d >= n_nodes) local |= BYSJ_FLAG_OUT_OF_RANGE;
    if (e > 0 && __ldg(dst + e - 1) > d) local |= BYSJ_FLAG_UNSORTED;
  }
  local = __reduce_or_sync(kFull, local);
  if (local && lane_id() == 0) atomicOr(flags, local);
}

__global__ void __launch_bounds__(kBlock)
    offsets_boundary_scalar_kernel(const int64_t* __restrict__ dst, int64_t n_edges,
                                   int64_t n_nodes, int64_t* __restrict__ offsets,
                                   const uint32_t* flags) {
  if (*flags != 0) return;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       e <= n_edges; e += stride) {
    const int64_t prev = e > 0 ? __ldg(dst + e - 1) : -1;
    const int64_t cur = e < n_edges ? __ldg(dst + e) : n_nodes;
    write_boundary(prev, cur, e, offsets);
  }
}

__global__ void __launch_bounds__(kBlock)
    offsets_histogram_kernel(const int64_t* __restrict__ dst, int64_t n_edges,
                             int64_t n_nodes,
                             unsigned long long* __restrict__ counts,
                             uint32_t* flags) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  uint32_t bad = 0;
  const int64_t begin = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  // Uniform trip count per warp so __match_any_sync sees all lanes.
  const int64_t warp_begin = begin - lane_id();
  for (int64_t base = warp_begin; base < n_edges; base += stride) {
    const int64_t e = base + lane_id();
    int64_t d = -1;
    if (e < n_edges) {
      d = __ldg(dst + e);
      if (d < 0 || d >= n_nodes) {
        bad = BYSJ_FLAG_OUT_OF_RANGE;
        d = -1;
      }
    }
    const unsigned peers = __match_any_sync(kFull, static_cast<unsigned long long>(d));
    const int leader = __ffs(peers) - 1;
    if (d >= 0 && lane_id() == leader)
      atomicAdd(counts + d, static_cast<unsigned long long>(__popc(peers)));
  }
  bad = __reduce_or_sync(kFull, bad);
  if (bad && lane_id() == 0) atomicOr(flags, bad);
}

// Inclusive scan of one int64 per thread across the CTA; returns the CTA total
// through *total.
__device__ int64_t block_inclusive_scan(int64_t v, int64_t* total) {
  __shared__ int64_t warp_sums[kWarpsPerBlock];
  const int lane = lane_id();
  const int warp = threadIdx.x >> 5;
  for (int s = 1; s < kWarp; s <<= 1) {
    const int64_t t = __shfl_up_sync(kFull, v, s);
    if (lane >= s) v += t;
  }
  if (lane == kWarp - 1) warp_sums[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int64_t w = lane < kWarpsPerBlock ? warp_sums[lane] : 0;
    for (int s = 1; s < kWarpsPerBlock; s <<= 1) {
      const int64_t t = __shfl_up_sync(kFull, w, s);
      if (lane >= s) w += t;
    }
    if (lane < kWarpsPerBlock) warp_sums[lane] = w;
  }
  __syncthreads();
  if (warp > 0) v += warp_sums[warp - 1];
  *total = warp_sums[kWarpsPerBlock - 1];
  __syncthreads();
  return v;
}

// Phase 1: per-tile sums of counts[0, n).
__global__ void __launch_bounds__(kBlock)
    scan_tile_sums_kernel(const unsigned long long* __restrict__ counts, int64_t n,
                          int64_t* __restrict__ tile_sums) {
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanTile;
  int64_t v = 0;
  for (int i = threadIdx.x; i < kScanTile; i += kBlock)
    if (base + i < n) v += static_cast<int64_t>(counts[base + i]);
  int64_t total = 0;
  block_inclusive_scan(v, &total);
  if (threadIdx.x == 0) tile_sums[blockIdx.x] = total;
}

// Phase 2: exclusive scan of the tile sums in one CTA.
__global__ void __launch_bounds__(kBlock)
    scan_tile_prefix_kernel(int64_t* __restrict__ tile_sums, int64_t tiles) {
  int64_t carry = 0;
  for (int64_t base = 0; base < tiles; base += kBlock) {
    const int64_t i = base + threadIdx.x;
    const int64_t v = i < tiles ? tile_sums[i] : 0;
    int64_t total = 0;
    const int64_t inc = block_inclusive_scan(v, &total);
    if (i < tiles) tile_sums[i] = carry + inc - v;
    carry += total;
  }
}

// Phase 3: offsets[i + 1] = prefix(tile) + inclusive scan inside the tile.
__global__ void __launch_bounds__(kBlock)
    scan_tile_apply_kernel(const unsigned long long* __restrict__ counts, int64_t n,
                           const int64_t* __restrict__ tile_prefix,
                           int64_t* __restrict__ offsets) {
  constexpr int kPer = kScanTile / kBlock;  // consecutive elements per thread
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanTile +
                       static_cast<int64_t>(threadIdx.x) * kPer;
  int64_t local[kPer];
  int64_t run = 0;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int64_t idx = base + i;
    run += idx < n ? static_cast<int64_t>(counts[idx]) : 0;
    local[i] = run;
  }
  int64_t total = 0;
  const int64_t inc = block_inclusive_scan(run, &total);
  const int64_t before = tile_prefix[blockIdx.x] + inc - run;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int64_t idx = base + i;
    if (idx < n) offsets[idx + 1] = before + local[i];
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) offsets[0] = 0;
}

unsigned stream_blocks(int64_t items) {
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

int bysj_segment_offsets_sorted(const int64_t* dst, int64_t n_edges,
                                int64_t n_nodes, int64_t* offsets,
                                uint32_t* flags, void* stream) {
  clear_error();
  if (n_edges < 0 || n_nodes < 0)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "segment offsets: invalid sizes");
  if (offsets == nullptr || flags == nullptr || (n_edges > 0 && dst == nullptr))
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "segment offsets: NULL pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n_edges == 0)
    return cuda_check(cudaMemsetAsync(offsets, 0, sizeof(int64_t) * (n_nodes + 1), s),
                      "segment offsets: zero fill");
  if (aligned16(dst)) {
    const unsigned blocks = stream_blocks((n_edges / 2 + kPairsPerStep - 1) / kPairsPerStep);
    offsets_sorted_fused_kernel<<<blocks, kBlock, 0, s>>>(dst, n_edges, n_nodes, offsets,
                                                          flags);
    return launch_check("offsets_sorted_fused_kernel");
  }
  offsets_check_scalar_kernel<<<stream_blocks(n_edges), kBlock, 0, s>>>(dst, n_edges, n_nodes,
                                                                        flags);
  int st = launch_check("offsets_check_scalar_kernel");
  if (st) return st;
  offsets_boundary_scalar_kernel<<<stream_blocks(n_edges + 1), kBlock, 0, s>>>(
      dst, n_edges, n_nodes, offsets, flags);
  return launch_check("offsets_boundary_scalar_kernel");
}

size_t bysj_segment_offsets_workspace_size(int64_t n_nodes) {
  if (n_nodes < 0) return 0;
  const int64_t tiles = (n_nodes + kScanTile - 1) / kScanTile;
  Carver carve(nullptr);
  carve.take<unsigned long long>(static_cast<size_t>(n_nodes) + 1);
  carve.take<int64_t>(static_cast<size_t>(tiles) + 1);
  return carve.need;
}

int bysj_segment_offsets_histogram(const int64_t* dst, int64_t n_edges,
                                   int64_t n_nodes, int64_t* offsets,
                                   uint32_t* flags, void* workspace,
                                   size_t workspace_bytes, void* stream) {
  clear_error();
  if (n_edges < 0 || n_nodes < 0)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "segment offsets: invalid sizes");
  if (offsets == nullptr || flags == nullptr || (n_edges > 0 && dst == nullptr))
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "segment offsets: NULL pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n_nodes == 0)
    return cuda_check(cudaMemsetAsync(offsets, 0, sizeof(int64_t), s),
                      "segment offsets: zero fill");
  const int64_t tiles = (n_nodes + kScanTile - 1) / kScanTile;
  Carver carve(workspace);
  unsigned long long* counts = carve.take<unsigned long long>(static_cast<size_t>(n_nodes) + 1);
  int64_t* tile_sums = carve.take<int64_t>(static_cast<size_t>(tiles) + 1);
  if (workspace == nullptr || workspace_bytes < carve.need)
    return fail(BYSJ_ERR_WORKSPACE,
                "segment offsets: workspace of %zu bytes needed, %zu given",
                carve.need, workspace_bytes);
  int st = cuda_check(cudaMemsetAsync(counts, 0, sizeof(unsigned long long) * n_nodes, s),
                      "segment offsets: zero counts");
  if (st) return st;
  if (n_edges > 0) {
    offsets_histogram_kernel<<<stream_blocks(n_edges), kBlock, 0, s>>>(
        dst, n_edges, n_nodes, counts, flags);
    st = launch_check("offsets_histogram_kernel");
    if (st) return st;
  }
  scan_tile_sums_kernel<<<static_cast<unsigned>(tiles), kBlock, 0, s>>>(counts, n_nodes,
                                                                        tile_sums);
  st = launch_check("scan_tile_sums_kernel");
  if (st) return st;
  scan_tile_prefix_kernel<<<1, kBlock, 0, s>>>(tile_sums, tiles);
  st = launch_check("scan_tile_prefix_kernel");
  if (st) return st;
  scan_tile_apply_kernel<<<static_cast<unsigned>(tiles), kBlock, 0, s>>>(
      counts, n_nodes, tile_sums, offsets);
  return launch_check("scan_tile_apply_kernel");
}

}  // extern "C"
