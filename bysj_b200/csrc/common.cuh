// Shared device and host helpers for the sm_100a segmented-operator kernels.
//
// The kernels are HBM-bound integer/float streaming work: they use 16-byte
// vector loads on the read-only path, warp-level shuffles for reductions and
// no floating-point atomics, so every result is reproducible bit for bit.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstddef>

#include "../../include/bysj_b200.h"

namespace bysj {

constexpr int kWarp = 32;
constexpr unsigned kFull = 0xffffffffu;

// ---------------------------------------------------------------------------
// Host side: error reporting, device properties, workspace carving.
// ---------------------------------------------------------------------------

// Records a human-readable failure for bysj_last_error() and returns `status`.
int fail(int status, const char* fmt, ...);
// Clears the thread's last error.
void clear_error();
// Checks a CUDA runtime result; returns BYSJ_OK or BYSJ_ERR_CUDA with detail.
int cuda_check(cudaError_t err, const char* what);
// Checks cudaGetLastError after a launch.
int launch_check(const char* kernel);

struct DeviceInfo {
  int device = 0;
  int sm_count = 148;
  int max_threads_per_sm = 2048;
};
// Properties of the current device (cached per device).
const DeviceInfo& current_device_info();

// Bump allocator over a caller-provided workspace.  Every region is aligned
// to 256 bytes; `need` accumulates the total so the same code path computes
// the workspace size (base == nullptr) and carves the buffer.
struct Carver {
  char* base;
  size_t need = 0;
  explicit Carver(void* b) : base(static_cast<char*>(b)) {}
  template <typename T>
  T* take(size_t count) {
    size_t off = (need + 255) & ~size_t(255);
    need = off + count * sizeof(T);
    return base ? reinterpret_cast<T*>(base + off) : nullptr;
  }
};

inline bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}
inline bool aligned8(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 7u) == 0;
}

// ---------------------------------------------------------------------------
// Device side: loads.
// ---------------------------------------------------------------------------

// 16-byte streaming load through the non-coherent path without L1
// allocation: edge rows are read once, so keeping them out of L1 leaves room
// for the small per-segment data (logits, scales) that is re-read.
__device__ __forceinline__ float4 ld_stream_f4(const float* p) {
  float4 v;
  asm("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
      : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
      : "l"(p));
  return v;
}

__device__ __forceinline__ uint4 ld_stream_u4(const void* p) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p));
  return v;
}

// Asks the TMA unit to bring `bytes` at `p` into L2 (no shared memory, no
// registers, no completion to wait for).  `p` 16-byte aligned, `bytes` a
// multiple of 16.  Used to put the next loop step's rows in flight while this
// step's loads are still outstanding.
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// bf16 -> fp32 is exact: the bf16 bits are the high half of the fp32 word.
__device__ __forceinline__ float bf16_lo(uint32_t w) {
  return __uint_as_float(w << 16);
}
__device__ __forceinline__ float bf16_hi(uint32_t w) {
  return __uint_as_float(w & 0xffff0000u);
}

// Vector of VEC consecutive row elements, kept in its loaded (raw) form so
// that a bf16 vector occupies 4 registers while in flight; get(i) converts one
// element to fp32 (i is a compile-time constant after unrolling).
template <typename T, int VEC>
struct RowVec;

template <>
struct RowVec<float, 4> {
  float4 r;
  __device__ __forceinline__ void load(const float* row, int64_t j) {
    r = ld_stream_f4(row + j * 4);
  }
  __device__ __forceinline__ float get(int i) const {
    return i == 0 ? r.x : i == 1 ? r.y : i == 2 ? r.z : r.w;
  }
};

template <>
struct RowVec<float, 1> {
  float r;
  __device__ __forceinline__ void load(const float* row, int64_t j) {
    r = __ldg(row + j);
  }
  __device__ __forceinline__ float get(int) const { return r; }
};

template <>
struct RowVec<__nv_bfloat16, 8> {
  uint4 r;
  __device__ __forceinline__ void load(const __nv_bfloat16* row, int64_t j) {
    r = ld_stream_u4(row + j * 8);
  }
  __device__ __forceinline__ float get(int i) const {
    const uint32_t w = (i >> 1) == 0 ? r.x : (i >> 1) == 1 ? r.y
                     : (i >> 1) == 2 ? r.z : r.w;
    return (i & 1) ? bf16_hi(w) : bf16_lo(w);
  }
};

template <>
struct RowVec<__nv_bfloat16, 1> {
  unsigned short r;
  __device__ __forceinline__ void load(const __nv_bfloat16* row, int64_t j) {
    r = __ldg(reinterpret_cast<const unsigned short*>(row) + j);
  }
  __device__ __forceinline__ float get(int) const {
    return __uint_as_float(static_cast<uint32_t>(r) << 16);
  }
};

// Store VEC fp32 values to an fp32 destination (16-byte store when VEC == 4).
template <int VEC>
__device__ __forceinline__ void store_f32(float* dst, const float (&v)[VEC]) {
  if constexpr (VEC == 4) {
    *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
  } else if constexpr (VEC == 8) {
    reinterpret_cast<float4*>(dst)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(dst)[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) dst[i] = v[i];
  }
}

// Coherent (L2) vector reads for partial results written by other warps.
template <int VEC>
__device__ __forceinline__ void load_cg(const float* src, float (&v)[VEC]) {
  if constexpr (VEC % 4 == 0) {
#pragma unroll
    for (int i = 0; i < VEC; i += 4) {
      float4 t = __ldcg(reinterpret_cast<const float4*>(src + i));
      v[i] = t.x; v[i + 1] = t.y; v[i + 2] = t.z; v[i + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) v[i] = __ldcg(src + i);
  }
}

template <int VEC>
__device__ __forceinline__ void store_cg(float* dst, const float (&v)[VEC]) {
  if constexpr (VEC % 4 == 0) {
#pragma unroll
    for (int i = 0; i < VEC; i += 4)
      __stcg(reinterpret_cast<float4*>(dst + i),
             make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]));
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) __stcg(dst + i, v[i]);
  }
}

// ---------------------------------------------------------------------------
// Device side: warp helpers.
// ---------------------------------------------------------------------------

__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }

__device__ __forceinline__ int64_t global_warp() {
  return (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
}

// Asynchronous global -> shared copies (LDGSTS) of 16 or 4 bytes, committed
// in groups and waited on by group count.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   static_cast<unsigned>(__cvta_generic_to_shared(smem))),
               "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(
                   static_cast<unsigned>(__cvta_generic_to_shared(smem))),
               "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Packed pairs of fp32 (add/sub/mul .f32x2, sm_100: two IEEE
// round-to-nearest operations per instruction, so a pair gives the same bits
// as two scalar operations) and 2^t by the approximate PTX ex2.approx.ftz.f32.
__device__ __forceinline__ uint64_t pk2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float2 upk2(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float ex2_ftz(float t) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(t));
  return r;
}

// Butterfly sum over the lanes that differ in bits [lo_bit, 5).  Every
// participating lane ends with the same value: each step adds two operands
// in either order, and fp32 addition is commutative.
__device__ __forceinline__ float xor_sum(float v, int first_stride) {
  for (int s = first_stride; s < kWarp; s <<= 1)
    v += __shfl_xor_sync(kFull, v, s);
  return v;
}
__device__ __forceinline__ double xor_sum(double v, int first_stride) {
  for (int s = first_stride; s < kWarp; s <<= 1)
    v += __shfl_xor_sync(kFull, v, s);
  return v;
}
__device__ __forceinline__ float xor_max(float v, int first_stride) {
  for (int s = first_stride; s < kWarp; s <<= 1)
    v = fmaxf(v, __shfl_xor_sync(kFull, v, s));
  return v;
}
// Butterfly over the low bits [0, log2(width)): reduces within aligned groups
// of `width` lanes.
__device__ __forceinline__ float group_sum(float v, int width) {
  for (int s = 1; s < width; s <<= 1) v += __shfl_xor_sync(kFull, v, s);
  return v;
}
__device__ __forceinline__ double group_sum(double v, int width) {
  for (int s = 1; s < width; s <<= 1) v += __shfl_xor_sync(kFull, v, s);
  return v;
}

// Effective logit of the gated softmax: l = logit + 2 ln(env) for env > 0,
// -inf (no mass) otherwise.  A NULL envelope means every edge is kept.
__device__ __forceinline__ float gated_logit(float logit, const float* env,
                                             int64_t edge) {
  if (env == nullptr) return logit;
  const float g = __ldg(env + edge);
  if (!(g > 0.0f)) return -INFINITY;
  return logit + 2.0f * logf(g);
}

// exp(x - m) with the convention exp(-inf - m) = 0 and a -inf maximum giving 0.
__device__ __forceinline__ float shifted_exp(float x, float m) {
  return (x == -INFINITY || m == -INFINITY) ? 0.0f : expf(x - m);
}

// exp(x - m) by the __expf intrinsic (one ex2 on the transcendental pipe).
// CUDA documents its error as 2 + floor(|1.173 (x - m)|) ulp; outputs of a
// softmax matter to an absolute 1e-6 only for x - m >= -14, where that is at
// most 18 ulp (~1.1e-6 relative), well inside rtol 1e-5.  For kernels whose
// time goes to the exponentials rather than to HBM.
__device__ __forceinline__ float shifted_exp_fast(float x, float m) {
  return (x == -INFINITY || m == -INFINITY) ? 0.0f : __expf(x - m);
}

// ---------------------------------------------------------------------------
// Merge-path partition of a CSR segment list.
//
// The work of a segmented reduction is the merged sequence of the E edge
// slots and the N segment ends: segment a occupies positions
// [offsets[a] + a, offsets[a+1] + a], its end marker being the last one.
// Partition p owns positions [p*ipc, (p+1)*ipc), so every warp gets the same
// number of items whatever the degree distribution.  A segment that crosses a
// partition boundary is "split": each partition that holds some of it writes
// a partial result into its head or tail slot, and the last one to finish
// (an integer ticket) combines the partials in partition order.
// ---------------------------------------------------------------------------

struct MergePath {
  const int64_t* offsets;
  int64_t n_nodes;
  int64_t n_edges;
  int64_t ipc;  // items per partition
  int64_t parts;

  // Number of segment ends strictly before merged position d (warp-wide;
  // every lane returns the same value).  32-ary search: log32(N) rounds.
  __device__ __forceinline__ int64_t ends_before(int64_t d) const {
    const int lane = lane_id();
    int64_t lo = d > n_edges ? d - n_edges : 0;
    int64_t hi = d < n_nodes ? d : n_nodes;
    while (hi - lo > kWarp) {
      const int64_t step = (hi - lo + kWarp - 1) / kWarp;
      const int64_t probe = lo + lane * step;
      const bool before = probe < hi && (__ldg(offsets + probe + 1) + probe < d);
      const int cnt = __popc(__ballot_sync(kFull, before));
      if (cnt == 0) return lo;
      const int64_t new_lo = lo + (cnt - 1) * step + 1;
      const int64_t new_hi = lo + cnt * step;
      lo = new_lo;
      hi = new_hi < hi ? new_hi : hi;
    }
    const int64_t probe = lo + lane;
    const bool before = probe < hi && (__ldg(offsets + probe + 1) + probe < d);
    return lo + __popc(__ballot_sync(kFull, before));
  }

  // Number of segments whose start diagonal offsets[n] + n lies below d
  // (warp-wide; every lane returns the same value).  Partition p of a
  // whole-segment kernel owns segments [starts_before(p ipc),
  // starts_before((p + 1) ipc)): every segment exactly once, never split.
  __device__ __forceinline__ int64_t starts_before(int64_t d) const {
    const int lane = lane_id();
    if (d > n_edges + n_nodes) d = n_edges + n_nodes;  // the last partition's end
    int64_t lo = d > n_edges ? d - n_edges : 0;
    int64_t hi = d < n_nodes ? d : n_nodes;
    while (hi - lo > kWarp) {
      const int64_t step = (hi - lo + kWarp - 1) / kWarp;
      const int64_t probe = lo + lane * step;
      const bool before = probe < hi && (__ldg(offsets + probe) + probe < d);
      const int cnt = __popc(__ballot_sync(kFull, before));
      if (cnt == 0) return lo;
      const int64_t new_lo = lo + (cnt - 1) * step + 1;
      const int64_t new_hi = lo + cnt * step;
      lo = new_lo;
      hi = new_hi < hi ? new_hi : hi;
    }
    const int64_t probe = lo + lane;
    const bool before = probe < hi && (__ldg(offsets + probe) + probe < d);
    return lo + __popc(__ballot_sync(kFull, before));
  }

  __device__ __forceinline__ int64_t part_of_first_edge(int64_t a) const {
    return (__ldg(offsets + a) + a) / ipc;
  }
  __device__ __forceinline__ int64_t part_of_end(int64_t a) const {
    return (__ldg(offsets + a + 1) + a) / ipc;
  }
};

// One partition's share: segment ends [a0, a1) and edge slots [b0, b1).
struct PartRange {
  int64_t a0, a1, b0, b1;
};

__device__ __forceinline__ PartRange part_range(const MergePath& mp,
                                                int64_t p) {
  const int64_t total = mp.n_edges + mp.n_nodes;
  int64_t d0 = p * mp.ipc;
  int64_t d1 = d0 + mp.ipc;
  if (d0 > total) d0 = total;
  if (d1 > total) d1 = total;
  PartRange r;
  r.a0 = mp.ends_before(d0);
  r.a1 = mp.ends_before(d1);
  r.b0 = d0 - r.a0;
  r.b1 = d1 - r.a1;
  return r;
}

// Role of a segment inside one partition.
enum SegKind : int { kWhole = 0, kHead = 1, kTail = 2 };

// Iterates over the segments touched by a partition.  Usage:
//   SegCursor cur(mp, range);
//   while (cur.next()) { ... cur.node, cur.lo, cur.hi, cur.kind ... }
struct SegCursor {
  const MergePath* mp;  // a pointer, so that a cursor can be copied and reassigned
  PartRange r;
  int64_t node, lo, hi, e;
  int kind;
  __device__ SegCursor(const MergePath& m, const PartRange& range)
      : mp(&m), r(range), node(range.a0 - 1), lo(0), hi(0), e(range.b0),
        kind(kWhole) {}
  __device__ __forceinline__ bool next() {
    ++node;
    if (node > r.a1) return false;
    if (node == r.a1) {
      // Trailing segment without its end marker: a tail, if non-empty.
      if (e >= r.b1) return false;
      lo = e;
      hi = r.b1;
      kind = kTail;
      e = hi;
      return true;
    }
    lo = e;
    hi = __ldg(mp->offsets + node + 1);
    kind = (__ldg(mp->offsets + node) >= r.b0) ? kWhole : kHead;
    e = hi;
    return true;
  }
};

// Partial-result slots: two per partition (head, tail), `stride` floats each.
struct SplitSlots {
  float* slots;     // [parts][2][stride]
  int* tickets;     // [parts * tiles], zeroed before the launch
  int64_t stride;
  int tiles;
  __device__ __forceinline__ float* slot(int64_t part, int kind) const {
    return slots + (part * 2 + (kind == kHead ? 0 : 1)) * stride;
  }
};

// Publishes this warp's partial (already stored by all lanes) and returns
// true on the warp that arrives last for segment `node`; that warp must then
// combine the partials of parts [first, last] in order.  Memory ordering:
// every lane fences its own stores before the warp barrier, the ticket is
// taken by lane 0, and the combining warp fences again before reading the
// other warps' partials through L2.
__device__ __forceinline__ bool arrive_last(const SplitSlots& ss,
                                            int64_t first, int64_t last,
                                            int tile) {
  __threadfence();
  __syncwarp();
  int ticket = 0;
  if (lane_id() == 0)
    ticket = atomicAdd(ss.tickets + last * ss.tiles + tile, 1);
  ticket = __shfl_sync(kFull, ticket, 0);
  const bool is_last = ticket == static_cast<int>(last - first);
  if (is_last) __threadfence();
  return is_last;
}

}  // namespace bysj
