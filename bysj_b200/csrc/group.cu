// Stable grouping of an edge list by an integer key (the source atom):
// order[] lists the edges of key 0, then key 1, ..., each group in ascending
// edge index, and offsets[] is the exclusive prefix sum of the group sizes.
//
// The reference (python/kernels/segment.py:60-71) runs a stable argsort of
// the int64 keys plus bincount/cumsum.  Here, all on the device:
//
//  1. count: each tile of edges is counted in a shared-memory hash table of
//     its keys, then one global atomic per distinct key reserves the tile's
//     slots; each edge keeps a distinct slot in its group (arrival order);
//     a three-phase scan turns the counts into offsets;
//  2. place: order[offsets[key] + slot] = edge, with no atomics;
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

// Pass 1: counts[k] = number of edges with key k, and rank[e] = a distinct
// slot of edge e in its group (arrival order; pass 3 sorts the groups).  A
// CTA takes tiles of kHashTile consecutive edges and counts each tile in a
// shared-memory hash table of its keys first: a tile of a dst-sorted
// neighbour list holds a few hundred distinct sources in ~4096 edges (their
// key range is wide -- Morton order wraps around a periodic box -- so a
// window would not do), and the table turns one returning global atomic per
// edge into one per distinct key per tile.  An edge whose key finds no free
// slot within kHashProbes probes takes its slot from the global counter
// directly.  Out-of-range keys are skipped and flagged.
constexpr int kHashTile = 4096;                 // edges per tile
constexpr int kHashPer = kHashTile / kBlock;    // edges per thread per tile
constexpr int kHashSlots = 2048;                // table size (a power of two)
constexpr int kHashProbes = 32;
constexpr uint32_t kHashEmpty = 0xffffffffu;    // no key: keys are < 2^31 - 1
constexpr int kSlotDirect = -1, kSlotSkip = -2;

__global__ void __launch_bounds__(kBlock)
    group_count_kernel(const int64_t* __restrict__ keys, int64_t n_edges, int64_t n_keys,
                       unsigned* __restrict__ counts, unsigned* __restrict__ rank,
                       uint32_t* flags) {
  __shared__ uint32_t s_key[kHashSlots];
  __shared__ unsigned s_cnt[kHashSlots];
  uint32_t bad = 0;
  for (int64_t tile = static_cast<int64_t>(blockIdx.x) * kHashTile; tile < n_edges;
       tile += static_cast<int64_t>(gridDim.x) * kHashTile) {
    for (int i = threadIdx.x; i < kHashSlots; i += kBlock) {
      s_key[i] = kHashEmpty;
      s_cnt[i] = 0;
    }
    __syncthreads();
    int slot[kHashPer];
    unsigned local[kHashPer];
#pragma unroll
    for (int j = 0; j < kHashPer; ++j) {
      const int64_t e = tile + j * kBlock + threadIdx.x;
      slot[j] = kSlotSkip;
      local[j] = 0;
      if (e >= n_edges) continue;
      const int64_t k = __ldg(keys + e);
      if (k < 0 || k >= n_keys) {
        bad = BYSJ_FLAG_OUT_OF_RANGE;
        continue;
      }
      const uint32_t key = static_cast<uint32_t>(k);
      uint32_t h = (key * 0x9e3779b1u) >> (32 - 11);  // 11 bits: kHashSlots
      slot[j] = kSlotDirect;
      for (int probe = 0; probe < kHashProbes; ++probe) {
        const uint32_t old = atomicCAS(s_key + h, kHashEmpty, key);
        if (old == kHashEmpty || old == key) {
          slot[j] = static_cast<int>(h);
          break;
        }
        h = (h + 1) & (kHashSlots - 1);
      }
      local[j] = slot[j] >= 0 ? atomicAdd(s_cnt + slot[j], 1u) : atomicAdd(counts + k, 1u);
    }
    __syncthreads();
    // One global atomic per distinct key of the tile: the tile's base slot.
    for (int i = threadIdx.x; i < kHashSlots; i += kBlock) {
      const uint32_t key = s_key[i];
      if (key != kHashEmpty) s_cnt[i] = atomicAdd(counts + key, s_cnt[i]);
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kHashPer; ++j) {
      const int64_t e = tile + j * kBlock + threadIdx.x;
      if (slot[j] == kSlotSkip) continue;
      rank[e] = slot[j] >= 0 ? s_cnt[slot[j]] + local[j] : local[j];
    }
    __syncthreads();  // the table is reset for the next tile
  }
  bad = __reduce_or_sync(kFull, bad);
  if (bad && lane_id() == 0) atomicOr(flags, bad);
}
static_assert(kHashSlots == 1 << 11, "the hash takes the top 11 bits");
static_assert(kHashTile % kBlock == 0, "whole edges per thread");

// Pass 2 (no atomics): order[offsets[k] + rank[e]] = e.
template <typename V>
__global__ void __launch_bounds__(kBlock)
    group_place_kernel(const int64_t* __restrict__ keys, int64_t n_edges, int64_t n_keys,
                       const int64_t* __restrict__ offsets, const unsigned* __restrict__ rank,
                       V* __restrict__ order) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < n_edges;
       e += stride) {
    const int64_t k = __ldg(keys + e);
    if (k < 0 || k >= n_keys) continue;
    order[__ldg(offsets + k) + __ldg(rank + e)] = static_cast<V>(e);
  }
}

// Inclusive CTA-wide scan of one int64 per thread; *total gets the CTA sum.
__device__ int64_t block_scan_i64(int64_t v, int64_t* total) {
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

constexpr int kScanTile = 2048;  // counts per CTA in the offsets scan

// Exclusive scan of counts[0, n) into offsets[0, n] in three phases.
__global__ void __launch_bounds__(kBlock)
    group_tile_sums_kernel(const unsigned* __restrict__ counts, int64_t n,
                           int64_t* __restrict__ tile_sums) {
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanTile;
  int64_t v = 0;
  for (int i = threadIdx.x; i < kScanTile; i += kBlock)
    if (base + i < n) v += counts[base + i];
  int64_t total = 0;
  block_scan_i64(v, &total);
  if (threadIdx.x == 0) tile_sums[blockIdx.x] = total;
}

__global__ void __launch_bounds__(kBlock)
    group_tile_prefix_kernel(int64_t* __restrict__ tile_sums, int64_t tiles) {
  int64_t carry = 0;
  for (int64_t base = 0; base < tiles; base += kBlock) {
    const int64_t i = base + threadIdx.x;
    const int64_t v = i < tiles ? tile_sums[i] : 0;
    int64_t total = 0;
    const int64_t inc = block_scan_i64(v, &total);
    if (i < tiles) tile_sums[i] = carry + inc - v;
    carry += total;
  }
}

__global__ void __launch_bounds__(kBlock)
    group_tile_apply_kernel(const unsigned* __restrict__ counts, int64_t n,
                            const int64_t* __restrict__ tile_prefix,
                            int64_t* __restrict__ offsets) {
  constexpr int kPer = kScanTile / kBlock;
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanTile +
                       static_cast<int64_t>(threadIdx.x) * kPer;
  int64_t local[kPer];
  int64_t run = 0;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    run += base + i < n ? counts[base + i] : 0;
    local[i] = run;
  }
  int64_t total = 0;
  const int64_t inc = block_scan_i64(run, &total);
  const int64_t before = tile_prefix[blockIdx.x] + inc - run;
#pragma unroll
  for (int i = 0; i < kPer; ++i)
    if (base + i < n) offsets[base + i + 1] = before + local[i];
  if (blockIdx.x == 0 && threadIdx.x == 0) offsets[0] = 0;
}

// Sorts seg[0, n) ascending, n <= 32 K, with one warp: element i = 32 k + lane
// lives in register a[k] of that lane; strides below 32 exchange across lanes,
// larger strides inside a lane.  V: the register type of an edge index
// (uint32_t when every index fits, else int64_t).
template <int K, typename V>
__device__ __forceinline__ void warp_bitonic(int64_t* __restrict__ seg, int n) {
  constexpr V kPad = ~V(0) > V(0) ? ~V(0) : V(INT64_MAX);
  const int lane = lane_id();
  V a[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const int i = 32 * k + lane;
    a[k] = i < n ? static_cast<V>(seg[i]) : kPad;
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
          const V lo = a[k] < a[k2] ? a[k] : a[k2];
          const V hi = a[k] < a[k2] ? a[k2] : a[k];
          a[k] = up ? lo : hi;
          a[k2] = up ? hi : lo;
        }
      } else {
#pragma unroll
        for (int k = 0; k < K; ++k) {
          const V other = __shfl_xor_sync(kFull, a[k], stride);
          const bool up = ((32 * k + lane) & size) == 0;
          const bool lower = (lane & stride) == 0;
          const V lo = a[k] < other ? a[k] : other;
          const V hi = a[k] < other ? other : a[k];
          a[k] = (lower == up) ? lo : hi;
        }
      }
    }
  }
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const int i = 32 * k + lane;
    if (i < n) seg[i] = static_cast<int64_t>(a[k]);
  }
}

struct GroupLists {
  int* block_groups;  // keys whose group needs a CTA sort
  int* scan_groups;   // keys whose group is re-scanned
  int* counts;        // [0]: block_groups used, [1]: scan_groups used
};

// One warp per key: sorts groups of up to 256 edges, lists the others.
template <typename V>
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
      warp_bitonic<1, V>(seg, m);
    } else if (n <= 64) {
      warp_bitonic<2, V>(seg, m);
    } else if (n <= 128) {
      warp_bitonic<4, V>(seg, m);
    } else if (n <= kWarpBucket) {
      warp_bitonic<8, V>(seg, m);
    } else if (lane_id() == 0) {
      if (n <= kBlockBucket)
        lists.block_groups[atomicAdd(lists.counts, 1)] = static_cast<int>(key);
      else
        lists.scan_groups[atomicAdd(lists.counts + 1, 1)] = static_cast<int>(key);
    }
  }
}

// The groups the warp pass listed, one CTA each: groups of 257..4096 edges
// are sorted by a bitonic network in shared memory; larger groups are
// rebuilt by scanning all keys in edge order with a CTA-wide prefix count.
template <typename V>
__global__ void __launch_bounds__(kBlock)
    group_sort_large_kernel(const int64_t* __restrict__ keys, int64_t n_edges,
                            const int64_t* __restrict__ offsets, int64_t* __restrict__ order,
                            GroupLists lists) {
  constexpr V kPad = ~V(0) > V(0) ? ~V(0) : V(INT64_MAX);
  constexpr int kPer = 4;  // consecutive edges per thread per scan step
  __shared__ V s[kBlockBucket];
  const int sorted = *reinterpret_cast<volatile int*>(lists.counts);
  const int scanned = *reinterpret_cast<volatile int*>(lists.counts + 1);
  for (int g = blockIdx.x; g < sorted + scanned; g += gridDim.x) {
    if (g < sorted) {
      const int key = lists.block_groups[g];
      const int64_t lo = offsets[key];
      const int n = static_cast<int>(offsets[key + 1] - lo);
      int p = 1;
      while (p < n) p <<= 1;
      for (int i = threadIdx.x; i < p; i += blockDim.x)
        s[i] = i < n ? static_cast<V>(order[lo + i]) : kPad;
      __syncthreads();
      for (int size = 2; size <= p; size <<= 1) {
        for (int stride = size / 2; stride > 0; stride >>= 1) {
          for (int t = threadIdx.x; t < p / 2; t += blockDim.x) {
            const int i = 2 * stride * (t / stride) + (t % stride);
            const int j = i + stride;
            const bool up = (i & size) == 0;
            const V x = s[i], y = s[j];
            if ((x > y) == up) {
              s[i] = y;
              s[j] = x;
            }
          }
          __syncthreads();
        }
      }
      for (int i = threadIdx.x; i < n; i += blockDim.x) order[lo + i] = static_cast<int64_t>(s[i]);
      __syncthreads();
    } else {
      const int64_t key = lists.scan_groups[g - sorted];
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
        int64_t total = 0;
        const int64_t inclusive = block_scan_i64(mine, &total);
        int64_t at = out + inclusive - mine;
#pragma unroll
        for (int j = 0; j < kPer; ++j)
          if (hit[j]) order[at++] = first + j;
        out += total;
      }
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
  size_t need = 0;
  int64_t tiles = 0;
  unsigned* counts = nullptr;   // [n_keys]
  unsigned* rank = nullptr;     // [n_edges]
  int64_t* tile_sums = nullptr; // [tiles + 1]
  GroupLists lists{};
};

GroupLayout group_layout(int64_t n_edges, int64_t n_keys, void* ws) {
  GroupLayout L;
  L.tiles = (n_keys + kScanTile - 1) / kScanTile;
  Carver carve(ws);
  L.counts = carve.take<unsigned>(static_cast<size_t>(n_keys) + 1);
  L.rank = carve.take<unsigned>(static_cast<size_t>(n_edges) + 1);
  L.tile_sums = carve.take<int64_t>(static_cast<size_t>(L.tiles) + 1);
  L.lists.counts = carve.take<int>(2);
  L.lists.block_groups = carve.take<int>(static_cast<size_t>(n_keys) + 1);
  L.lists.scan_groups = carve.take<int>(static_cast<size_t>(n_keys) + 1);
  L.need = carve.need;
  return L;
}

template <typename V>
int group_sorts(const int64_t* keys, int64_t n_edges, int64_t n_keys, const int64_t* offsets,
                int64_t* order, const GroupLayout& L, cudaStream_t s) {
  group_sort_warp_kernel<V><<<grid_for(n_keys, kWarpsPerBlock, 16), kBlock, 0, s>>>(
      offsets, n_keys, order, L.lists);
  int st = launch_check("group_sort_warp_kernel");
  if (st) return st;
  const unsigned sms = static_cast<unsigned>(current_device_info().sm_count);
  group_sort_large_kernel<V><<<2 * sms, kBlock, 0, s>>>(keys, n_edges, offsets, order, L.lists);
  return launch_check("group_sort_large_kernel");
}

}  // namespace
}  // namespace bysj

using namespace bysj;

extern "C" {

size_t bysj_group_by_key_workspace_size(int64_t n_edges, int64_t n_keys) {
  if (n_edges < 0 || n_keys < 0) return 0;
  return group_layout(n_edges, n_keys, nullptr).need;
}

int bysj_group_by_key(const int64_t* keys, int64_t n_edges, int64_t n_keys, int64_t* order,
                      int64_t* offsets, uint32_t* flags, void* workspace,
                      size_t workspace_bytes, void* stream) {
  clear_error();
  if (n_edges < 0 || n_keys < 0)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "group by key: invalid sizes");
  if (n_keys > INT32_MAX - 1 || n_edges > static_cast<int64_t>(UINT32_MAX))
    return fail(BYSJ_ERR_TOO_LARGE, "group by key: more than 2^31 - 2 keys or 2^32 - 1 edges");
  if (offsets == nullptr || flags == nullptr ||
      (n_edges > 0 && (keys == nullptr || order == nullptr)))
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "group by key: NULL pointer");
  GroupLayout L = group_layout(n_edges, n_keys, workspace);
  if (workspace == nullptr || workspace_bytes < L.need)
    return fail(BYSJ_ERR_WORKSPACE, "group by key: workspace of %zu bytes needed, %zu given",
                L.need, workspace_bytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n_keys == 0)
    return cuda_check(cudaMemsetAsync(offsets, 0, sizeof(int64_t), s), "group by key: offsets");
  int st = cuda_check(cudaMemsetAsync(L.counts, 0, sizeof(unsigned) * n_keys, s),
                      "group by key: zero counts");
  if (st) return st;
  st = cuda_check(cudaMemsetAsync(L.lists.counts, 0, 2 * sizeof(int), s),
                  "group by key: zero list counts");
  if (st) return st;
  if (n_edges > 0) {
    group_count_kernel<<<grid_for(n_edges, kHashTile, 8), kBlock, 0, s>>>(
        keys, n_edges, n_keys, L.counts, L.rank, flags);
    st = launch_check("group_count_kernel");
    if (st) return st;
  }
  group_tile_sums_kernel<<<static_cast<unsigned>(L.tiles), kBlock, 0, s>>>(L.counts, n_keys,
                                                                          L.tile_sums);
  st = launch_check("group_tile_sums_kernel");
  if (st) return st;
  group_tile_prefix_kernel<<<1, kBlock, 0, s>>>(L.tile_sums, L.tiles);
  st = launch_check("group_tile_prefix_kernel");
  if (st) return st;
  group_tile_apply_kernel<<<static_cast<unsigned>(L.tiles), kBlock, 0, s>>>(
      L.counts, n_keys, L.tile_sums, offsets);
  st = launch_check("group_tile_apply_kernel");
  if (st || n_edges == 0) return st;
  group_place_kernel<int64_t><<<grid_for(n_edges, kBlock, 8), kBlock, 0, s>>>(
      keys, n_edges, n_keys, offsets, L.rank, order);
  st = launch_check("group_place_kernel");
  if (st) return st;
  // Sorting 32-bit edge indices halves the register and shuffle traffic.
  if (n_edges <= static_cast<int64_t>(UINT32_MAX) - 1)
    return group_sorts<uint32_t>(keys, n_edges, n_keys, offsets, order, L, s);
  return group_sorts<int64_t>(keys, n_edges, n_keys, offsets, order, L, s);
}

}  // extern "C"
