// Stable grouping of an edge list by an integer key (the source atom):
// order[] lists the edges of key 0, then key 1, ..., each group in ascending
// edge index, and offsets[] is the exclusive prefix sum of the group sizes.
//
// The reference (python/kernels/segment.py:60-71) runs a stable argsort of
// the int64 keys plus bincount/cumsum.  Here, all on the device:
//
//  1. offsets: warp-aggregated histogram + three-phase scan (offsets.cu);
//  2. scatter: each edge takes a slot in its key's group with a warp-
//     aggregated integer atomic (lanes of one warp instruction keep their
//     order, warps do not);
//  3. sort each group by edge index, which restores the stable order
//     exactly (edge indices are distinct, so the sorted group is unique and
//     the result does not depend on the scatter's interleaving):
//       <= 256 edges: one warp per group, bitonic network in registers;
//       <= 4096 edges: one CTA per group, bitonic network in shared memory;
//       larger groups: one CTA per group re-scans the keys in order with a
//       CTA-wide prefix count and writes the group directly.
// Integer work only, so the result is bit-exact and run-to-run identical.
#include "launch.cuh"

namespace bysj {
namespace {

constexpr int kWarpBucket = 256;   // largest group sorted by one warp
constexpr int kBlockBucket = 4096; // largest group sorted by one CTA in shared memory
constexpr int64_t kNoEdge = INT64_MAX;

__device__ __forceinline__ unsigned lanemask_lt() {
  return (1u << lane_id()) - 1u;
}

// order[offsets[k] + cursor[k]++] = e for every edge, lanes holding the same
// key merged by __match_any_sync.
__global__ void __launch_bounds__(kBlock)
    group_scatter_kernel(const int64_t* __restrict__ keys, int64_t n_edges, int64_t n_keys,
                         const int64_t* __restrict__ offsets, unsigned* __restrict__ cursor,
                         int64_t* __restrict__ order) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t warp_begin =
      static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x - lane_id();
  for (int64_t base = warp_begin; base < n_edges; base += stride) {  // warp-uniform
    const int64_t e = base + lane_id();
    int64_t k = -1;
    if (e < n_edges) {
      k = __ldg(keys + e);
      if (k < 0 || k >= n_keys) k = -1;
    }
    const unsigned peers = __match_any_sync(kFull, static_cast<unsigned long long>(k));
    const int leader = __ffs(peers) - 1;
    unsigned slot = 0;
    if (k >= 0 && lane_id() == leader) slot = atomicAdd(cursor + k, __popc(peers));
    slot = __shfl_sync(kFull, slot, leader);
    if (k >= 0) order[__ldg(offsets + k) + slot + __popc(peers & lanemask_lt())] = e;
  }
}

// Sorts seg[0, n) ascending, n <= 32 K, with one warp: element i = 32 k + lane
// lives in register a[k] of that lane; strides below 32 exchange across lanes,
// larger strides inside a lane.
template <int K>
__device__ __forceinline__ void warp_bitonic(int64_t* __restrict__ seg, int n) {
  const int lane = lane_id();
  int64_t a[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const int i = 32 * k + lane;
    a[k] = i < n ? seg[i] : kNoEdge;
  }
#pragma unroll
  for (int size = 2; size <= 32 * K; size <<= 1) {
#pragma unroll
    for (int stride = size / 2; stride > 0; stride >>= 1) {
      if (stride >= 32) {
        const int ks = stride / 32;
#pragma unroll
        for (int k = 0; k < K; ++k) {
          if ((k & ks) != 0) continue;
          const int k2 = k | ks;
          const bool up = ((32 * k + lane) & size) == 0;
          const int64_t lo = a[k] < a[k2] ? a[k] : a[k2];
          const int64_t hi = a[k] < a[k2] ? a[k2] : a[k];
          a[k] = up ? lo : hi;
          a[k2] = up ? hi : lo;
        }
      } else {
#pragma unroll
        for (int k = 0; k < K; ++k) {
          const int64_t other = __shfl_xor_sync(kFull, a[k], stride);
          const bool up = ((32 * k + lane) & size) == 0;
          const bool lower = (lane & stride) == 0;
          const int64_t lo = a[k] < other ? a[k] : other;
          const int64_t hi = a[k] < other ? other : a[k];
          a[k] = (lower == up) ? lo : hi;
        }
      }
    }
  }
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const int i = 32 * k + lane;
    if (i < n) seg[i] = a[k];
  }
}

struct GroupLists {
  int* block_groups;  // keys whose group needs a CTA sort
  int* scan_groups;   // keys whose group is re-scanned
  int* counts;        // [0]: block_groups used, [1]: scan_groups used
};

// One warp per key: sorts groups of up to 256 edges, lists the others.
__global__ void __launch_bounds__(kBlock)
    group_sort_warp_kernel(const int64_t* __restrict__ offsets, int64_t n_keys,
                           int64_t* __restrict__ order, GroupLists lists) {
  const int64_t warps = static_cast<int64_t>(gridDim.x) * kWarpsPerBlock;
  for (int64_t key = global_warp(); key < n_keys; key += warps) {
    const int64_t lo = __ldg(offsets + key);
    const int64_t n = __ldg(offsets + key + 1) - lo;
    if (n <= 1) continue;
    int64_t* seg = order + lo;
    const int m = static_cast<int>(n < kWarpBucket ? n : kWarpBucket);
    if (n <= 32) {
      warp_bitonic<1>(seg, m);
    } else if (n <= 64) {
      warp_bitonic<2>(seg, m);
    } else if (n <= 128) {
      warp_bitonic<4>(seg, m);
    } else if (n <= kWarpBucket) {
      warp_bitonic<8>(seg, m);
    } else if (lane_id() == 0) {
      if (n <= kBlockBucket)
        lists.block_groups[atomicAdd(lists.counts, 1)] = static_cast<int>(key);
      else
        lists.scan_groups[atomicAdd(lists.counts + 1, 1)] = static_cast<int>(key);
    }
  }
}

// One CTA per listed group of 257..4096 edges: bitonic sort in shared memory.
__global__ void __launch_bounds__(kBlock)
    group_sort_block_kernel(const int64_t* __restrict__ offsets, int64_t* __restrict__ order,
                            GroupLists lists) {
  __shared__ int64_t s[kBlockBucket];
  const int used = *reinterpret_cast<volatile int*>(lists.counts);
  for (int g = blockIdx.x; g < used; g += gridDim.x) {
    const int key = lists.block_groups[g];
    const int64_t lo = offsets[key];
    const int n = static_cast<int>(offsets[key + 1] - lo);
    int p = 1;
    while (p < n) p <<= 1;
    for (int i = threadIdx.x; i < p; i += blockDim.x) s[i] = i < n ? order[lo + i] : kNoEdge;
    __syncthreads();
    for (int size = 2; size <= p; size <<= 1) {
      for (int stride = size / 2; stride > 0; stride >>= 1) {
        for (int t = threadIdx.x; t < p / 2; t += blockDim.x) {
          const int i = 2 * stride * (t / stride) + (t % stride);
          const int j = i + stride;
          const bool up = (i & size) == 0;
          const int64_t x = s[i], y = s[j];
          if ((x > y) == up) {
            s[i] = y;
            s[j] = x;
          }
        }
        __syncthreads();
      }
    }
    for (int i = threadIdx.x; i < n; i += blockDim.x) order[lo + i] = s[i];
    __syncthreads();
  }
}

// Inclusive CTA-wide scan of one int per thread; *total gets the CTA sum.
__device__ int block_scan_int(int v, int* total) {
  __shared__ int warp_sums[kWarpsPerBlock];
  const int lane = lane_id();
  const int warp = threadIdx.x >> 5;
  for (int s = 1; s < kWarp; s <<= 1) {
    const int t = __shfl_up_sync(kFull, v, s);
    if (lane >= s) v += t;
  }
  if (lane == kWarp - 1) warp_sums[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int w = lane < kWarpsPerBlock ? warp_sums[lane] : 0;
    for (int s = 1; s < kWarpsPerBlock; s <<= 1) {
      const int t = __shfl_up_sync(kFull, w, s);
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

// One CTA per listed group of more than 4096 edges: scans all keys in edge
// order and writes the group's edges in that order.
__global__ void __launch_bounds__(kBlock)
    group_scan_kernel(const int64_t* __restrict__ keys, int64_t n_edges,
                      const int64_t* __restrict__ offsets, int64_t* __restrict__ order,
                      GroupLists lists) {
  constexpr int kPer = 4;  // consecutive edges per thread per step
  const int used = *reinterpret_cast<volatile int*>(lists.counts + 1);
  for (int g = blockIdx.x; g < used; g += gridDim.x) {
    const int64_t key = lists.scan_groups[g];
    int64_t out = offsets[key];
    for (int64_t base = 0; base < n_edges; base += static_cast<int64_t>(kBlock) * kPer) {
      const int64_t first = base + static_cast<int64_t>(threadIdx.x) * kPer;
      bool hit[kPer];
      int mine = 0;
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        hit[j] = first + j < n_edges && __ldg(keys + first + j) == key;
        mine += hit[j];
      }
      int total = 0;
      const int inclusive = block_scan_int(mine, &total);
      int64_t at = out + inclusive - mine;
#pragma unroll
      for (int j = 0; j < kPer; ++j)
        if (hit[j]) order[at++] = first + j;
      out += total;
    }
  }
}

unsigned grid_for(int64_t items, int64_t per_block, int64_t cap_per_sm) {
  int64_t blocks = (items + per_block - 1) / per_block;
  const int64_t cap = static_cast<int64_t>(current_device_info().sm_count) * cap_per_sm;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return static_cast<unsigned>(blocks);
}

struct GroupLayout {
  size_t offsets_ws = 0;
  size_t need = 0;
  void* offsets_workspace = nullptr;
  unsigned* cursor = nullptr;
  GroupLists lists{};
};

GroupLayout group_layout(int64_t n_keys, void* ws) {
  GroupLayout L;
  L.offsets_ws = bysj_segment_offsets_workspace_size(n_keys);
  Carver carve(ws);
  L.offsets_workspace = carve.take<char>(L.offsets_ws);
  L.cursor = carve.take<unsigned>(static_cast<size_t>(n_keys) + 1);
  L.lists.counts = carve.take<int>(2);
  L.lists.block_groups = carve.take<int>(static_cast<size_t>(n_keys) + 1);
  L.lists.scan_groups = carve.take<int>(static_cast<size_t>(n_keys) + 1);
  L.need = carve.need;
  return L;
}

}  // namespace
}  // namespace bysj

using namespace bysj;

extern "C" {

size_t bysj_group_by_key_workspace_size(int64_t n_edges, int64_t n_keys) {
  if (n_edges < 0 || n_keys < 0) return 0;
  return group_layout(n_keys, nullptr).need;
}

int bysj_group_by_key(const int64_t* keys, int64_t n_edges, int64_t n_keys, int64_t* order,
                      int64_t* offsets, uint32_t* flags, void* workspace,
                      size_t workspace_bytes, void* stream) {
  clear_error();
  if (n_edges < 0 || n_keys < 0)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "group by key: invalid sizes");
  if (n_keys > INT32_MAX - 1)
    return fail(BYSJ_ERR_TOO_LARGE, "group by key: more than 2^31 - 2 keys");
  if (offsets == nullptr || flags == nullptr ||
      (n_edges > 0 && (keys == nullptr || order == nullptr)))
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "group by key: NULL pointer");
  GroupLayout L = group_layout(n_keys, workspace);
  if (workspace == nullptr || workspace_bytes < L.need)
    return fail(BYSJ_ERR_WORKSPACE, "group by key: workspace of %zu bytes needed, %zu given",
                L.need, workspace_bytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int st = bysj_segment_offsets_histogram(keys, n_edges, n_keys, offsets, flags,
                                          L.offsets_workspace, L.offsets_ws, stream);
  if (st) return st;
  if (n_edges == 0 || n_keys == 0) return BYSJ_OK;
  st = cuda_check(cudaMemsetAsync(L.cursor, 0, sizeof(unsigned) * n_keys, s),
                  "group by key: zero cursors");
  if (st) return st;
  st = cuda_check(cudaMemsetAsync(L.lists.counts, 0, 2 * sizeof(int), s),
                  "group by key: zero list counts");
  if (st) return st;
  group_scatter_kernel<<<grid_for(n_edges, kBlock, 8), kBlock, 0, s>>>(keys, n_edges, n_keys,
                                                                      offsets, L.cursor, order);
  st = launch_check("group_scatter_kernel");
  if (st) return st;
  group_sort_warp_kernel<<<grid_for(n_keys, kWarpsPerBlock, 16), kBlock, 0, s>>>(
      offsets, n_keys, order, L.lists);
  st = launch_check("group_sort_warp_kernel");
  if (st) return st;
  const unsigned sms = static_cast<unsigned>(current_device_info().sm_count);
  group_sort_block_kernel<<<2 * sms, kBlock, 0, s>>>(offsets, order, L.lists);
  st = launch_check("group_sort_block_kernel");
  if (st) return st;
  group_scan_kernel<<<sms, kBlock, 0, s>>>(keys, n_edges, offsets, order, L.lists);
  return launch_check("group_scan_kernel");
}

}  // extern "C"
