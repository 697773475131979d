// Force and per-atom virial assembly from per-edge energy gradients (sm_100a).
//
//   F_k = sum_{dst(e)=k} g_e - sum_{src(e)=k} g_e
//   W_k = - sum_{src(e)=k} g_e (x) v_e          (row-major 3x3)
//
// Contract and fp64 accumulation follow the reference's
// csrc/force_assembly.cpp:64-96 (products double(g) * v, summed in double).
//
// The working set (grad_edge, edge_vec, src_order: ~73 MB at 2.2 M edges) is
// small and the source side is a gather: the rows g_e, v_e of the edges
// leaving atom k lie in ~90 different destination segments, each in its own
// cache line.  What limits the kernel is therefore the number of L1 requests
// per gathered row and the number of dependent round trips per atom, not
// DRAM bandwidth.  Layout: one warp per atom, lanes 3T + r form ten
// "triplets" T = 0..9 with component r = 0..2, lanes 30-31 idle.  A triplet
// takes every tenth edge; its three lanes load the three components of the
// same 12-byte row with one warp instruction (one request per row and array),
// exchange the edge vector's components by shuffle, and each lane accumulates
// its row r of the virial (g_r v_c, c = 0..2) and force component r in fp64.
// All K source slots, their gathers and K destination rows of a lane are
// issued as one burst, so a typical atom (<= 10 K edges per side) costs three
// dependent round trips: offsets, src_order, rows.  The ten triplets' sums
// are folded through shared memory in triplet order, so repeated runs are
// bit-identical.
#include "launch.cuh"

namespace bysj {
namespace {

constexpr int kTriplets = 10;          // lanes 0..29 in use
constexpr int kSlotsPerLane = 6;       // K: edges per triplet per burst (even)
constexpr int kForceMinBlocks = 4;
constexpr int kChunk = kTriplets * kSlotsPerLane;

// Lanes per atom and atoms per warp of the destination-add kernel below.
constexpr int kLanesPerAtom = 8;
constexpr int kAtomsPerWarp = kWarp / kLanesPerAtom;

enum Mode : int { kAssemble = 0, kSrcPartial = 1 };

// Edge bounds of one atom on both sides.
template <typename I>
struct AtomSpan {
  I s0 = 0, s1 = 0, d0 = 0, d1 = 0;
};

template <int MODE, typename I>
__device__ __forceinline__ AtomSpan<I> atom_span(const int64_t* __restrict__ dst_offsets,
                                                 const int64_t* __restrict__ src_offsets,
                                                 int64_t atom, int64_t n_nodes) {
  AtomSpan<I> a;
  if (atom < n_nodes) {
    a.s0 = static_cast<I>(__ldg(src_offsets + atom));
    a.s1 = static_cast<I>(__ldg(src_offsets + atom + 1));
    if constexpr (MODE == kAssemble) {
      a.d0 = static_cast<I>(__ldg(dst_offsets + atom));
      a.d1 = static_cast<I>(__ldg(dst_offsets + atom + 1));
    }
  }
  return a;
}

// Accumulates slots [base, base + 10 K) of both sides of one atom: triplet T
// takes slots base + T + 10 k, k < K.
template <int MODE, typename I, int K>
__device__ __forceinline__ void force_chunk(const float* __restrict__ grad_edge,
                                            const float* __restrict__ edge_vec,
                                            const int64_t* __restrict__ src_order,
                                            const AtomSpan<I>& cur, I base, bool active,
                                            int T, int r, int src_lane, double& af,
                                            double& aw0, double& aw1, double& aw2) {
  const I ns = cur.s1 - cur.s0;
  const I nd = cur.d1 - cur.d0;
  const I first = base + T;
  I edge[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const I j = first + k * kTriplets;
    edge[k] = (active && j < ns) ? static_cast<I>(__ldg(src_order + (cur.s0 + j))) : I(-1);
  }
  float dg[K];
  if constexpr (MODE == kAssemble) {
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const I j = first + k * kTriplets;
      dg[k] = (active && j < nd) ? __ldg(grad_edge + (3 * (cur.d0 + j) + r)) : 0.0f;
    }
  }
  float gr[K], vr[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    gr[k] = 0.0f;
    vr[k] = 0.0f;
    if (edge[k] >= 0) {
      const I at = 3 * edge[k] + r;
      gr[k] = __ldg(grad_edge + at);
      vr[k] = __ldg(edge_vec + at);
    }
  }
  if constexpr (MODE == kAssemble) {
#pragma unroll
    for (int k = 0; k < K; ++k) af += static_cast<double>(dg[k]);
  }
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const float v0 = __shfl_sync(kFull, vr[k], src_lane);
    const float v1 = __shfl_sync(kFull, vr[k], src_lane + 1);
    const float v2 = __shfl_sync(kFull, vr[k], src_lane + 2);
    if (edge[k] >= 0) {
      const double g = static_cast<double>(gr[k]);
      af -= g;
      aw0 -= g * static_cast<double>(v0);
      aw1 -= g * static_cast<double>(v1);
      aw2 -= g * static_cast<double>(v2);
    }
  }
}

// I: index type of edge arithmetic -- int32_t when 3 * n_edges fits, else
// int64_t (the host picks).  The next atom's offsets are loaded while the
// current atom's rows are in flight.  Chunks of 60, 30 or 10 slots per side
// are picked by what is left, so a ~90-edge atom runs 60 + 30.
template <int MODE, typename I>
__global__ void __launch_bounds__(kBlock, kForceMinBlocks)
    force_assembly_kernel(const float* __restrict__ grad_edge,
                          const float* __restrict__ edge_vec,
                          const int64_t* __restrict__ dst_offsets,
                          const int64_t* __restrict__ src_offsets,
                          const int64_t* __restrict__ src_order,
                          int64_t n_nodes, float* __restrict__ force,
                          float* __restrict__ virial,
                          double* __restrict__ partial) {
  __shared__ double fold[kWarpsPerBlock][kTriplets * 12];
  const int lane = lane_id();
  const int T = lane / 3;
  const int r = lane - 3 * T;
  const bool active = T < kTriplets;
  const int src_lane = 3 * (active ? T : 0);
  double* mine = fold[threadIdx.x >> 5];
  const int64_t warps = static_cast<int64_t>(gridDim.x) * kWarpsPerBlock;
  int64_t atom = global_warp();
  AtomSpan<I> cur = atom_span<MODE, I>(dst_offsets, src_offsets, atom, n_nodes);
  for (; atom < n_nodes; atom += warps) {
    const AtomSpan<I> next = atom_span<MODE, I>(dst_offsets, src_offsets, atom + warps, n_nodes);
    double af = 0.0, aw0 = 0.0, aw1 = 0.0, aw2 = 0.0;
    const I ns = cur.s1 - cur.s0;
    const I nd = cur.d1 - cur.d0;
    const I span = ns > nd ? ns : nd;
    for (I base = 0; base < span;) {  // warp-uniform
      const I left = span - base;
      if (left > kChunk / 2) {
        force_chunk<MODE, I, kSlotsPerLane>(grad_edge, edge_vec, src_order, cur, base, active, T,
                                            r, src_lane, af, aw0, aw1, aw2);
        base += kChunk;
      } else if (left > kTriplets) {
        force_chunk<MODE, I, kSlotsPerLane / 2>(grad_edge, edge_vec, src_order, cur, base, active,
                                                T, r, src_lane, af, aw0, aw1, aw2);
        base += kChunk / 2;
      } else {
        force_chunk<MODE, I, 1>(grad_edge, edge_vec, src_order, cur, base, active, T, r,
                                src_lane, af, aw0, aw1, aw2);
        base += kTriplets;
      }
    }
    // Fold the ten triplets: column j of the 12-vector is summed by lane j
    // in triplet order.
    if (active) {
      mine[T * 12 + r] = af;
      mine[T * 12 + 3 + 3 * r] = aw0;
      mine[T * 12 + 4 + 3 * r] = aw1;
      mine[T * 12 + 5 + 3 * r] = aw2;
    }
    __syncwarp();
    if (lane < 12) {
      double v = 0.0;
#pragma unroll
      for (int t = 0; t < kTriplets; ++t) v += mine[t * 12 + lane];
      if constexpr (MODE == kAssemble) {
        if (lane < 3) force[atom * 3 + lane] = static_cast<float>(v);
        else if (virial) virial[atom * 9 + (lane - 3)] = static_cast<float>(v);
      } else {
        partial[atom * 12 + lane] = v;
      }
    }
    __syncwarp();
    cur = next;
  }
}

// 32-bit edge arithmetic is exact when 3 * n_edges + 3 < 2^31.
bool force_index32(int64_t n_edges) { return n_edges < (int64_t{1} << 31) / 3 - 1; }

// force[k] = sum_{dst(e)=k} g_e + summed[k, 0:3];  virial[k] = summed[k, 3:12]
// (summed in fp64: the partials of all ranks, added before one rounding)
__global__ void __launch_bounds__(kBlock)
    force_dst_add_kernel(const float* __restrict__ grad_edge,
                         const int64_t* __restrict__ dst_offsets,
                         int64_t n_local, const double* __restrict__ summed,
                         float* __restrict__ force, float* __restrict__ virial) {
  const int lane = lane_id();
  const int sub = lane & (kLanesPerAtom - 1);
  const int64_t stride =
      static_cast<int64_t>(gridDim.x) * kWarpsPerBlock * kAtomsPerWarp;
  for (int64_t base = global_warp() * kAtomsPerWarp; base < n_local;
       base += stride) {
    const int64_t atom = base + (lane / kLanesPerAtom);
    const bool valid = atom < n_local;
    double acc[3] = {0.0, 0.0, 0.0};
    if (valid) {
      const int64_t d0 = __ldg(dst_offsets + atom);
      const int64_t d1 = __ldg(dst_offsets + atom + 1);
      for (int64_t e = d0 + sub; e < d1; e += kLanesPerAtom) {
        acc[0] += __ldg(grad_edge + e * 3);
        acc[1] += __ldg(grad_edge + e * 3 + 1);
        acc[2] += __ldg(grad_edge + e * 3 + 2);
      }
    }
#pragma unroll
    for (int c = 0; c < 3; ++c) acc[c] = group_sum(acc[c], kLanesPerAtom);
    if (!valid) continue;
    if (sub < 3) {
      const double v = sub == 0 ? acc[0] : sub == 1 ? acc[1] : acc[2];
      force[atom * 3 + sub] =
          static_cast<float>(v + summed[atom * 12 + sub]);
    }
    if (virial) {
      virial[atom * 9 + sub] = static_cast<float>(summed[atom * 12 + 3 + sub]);
      if (sub == 0) virial[atom * 9 + 8] = static_cast<float>(summed[atom * 12 + 11]);
    }
  }
}

unsigned atom_blocks(int64_t n_nodes) {
  const int64_t per_block = static_cast<int64_t>(kWarpsPerBlock) * kAtomsPerWarp;
  int64_t blocks = (n_nodes + per_block - 1) / per_block;
  const int64_t cap = static_cast<int64_t>(current_device_info().sm_count) * 64;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return static_cast<unsigned>(blocks);
}

// One warp per atom, at most one wave of resident warps (grid-stride beyond).
unsigned warp_per_atom_blocks(int64_t n_nodes) {
  int64_t blocks = (n_nodes + kWarpsPerBlock - 1) / kWarpsPerBlock;
  const int64_t cap =
      static_cast<int64_t>(current_device_info().sm_count) * kForceMinBlocks;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return static_cast<unsigned>(blocks);
}

}  // namespace
}  // namespace bysj

using namespace bysj;

extern "C" {

int bysj_force_assembly(const float* grad_edge, const float* edge_vec,
                        const int64_t* dst_offsets, const int64_t* src_offsets,
                        const int64_t* src_order, int64_t n_edges,
                        int64_t n_nodes, float* force, float* virial,
                        void* stream) {
  clear_error();
  if (n_edges < 0 || n_nodes < 0)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "force assembly: invalid sizes");
  if (n_nodes == 0) return BYSJ_OK;
  if (dst_offsets == nullptr || src_offsets == nullptr || force == nullptr ||
      (n_edges > 0 && (grad_edge == nullptr || edge_vec == nullptr ||
                       src_order == nullptr)))
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "force assembly: NULL pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (force_index32(n_edges))
    force_assembly_kernel<kAssemble, int32_t><<<warp_per_atom_blocks(n_nodes), kBlock, 0, s>>>(
        grad_edge, edge_vec, dst_offsets, src_offsets, src_order, n_nodes, force, virial,
        nullptr);
  else
    force_assembly_kernel<kAssemble, int64_t><<<warp_per_atom_blocks(n_nodes), kBlock, 0, s>>>(
        grad_edge, edge_vec, dst_offsets, src_offsets, src_order, n_nodes, force, virial,
        nullptr);
  return launch_check("force_assembly_kernel");
}

int bysj_force_assembly_src_partial(const float* grad_edge,
                                    const float* edge_vec,
                                    const int64_t* src_offsets,
                                    const int64_t* src_order, int64_t n_edges,
                                    int64_t n_nodes, double* partial,
                                    void* stream) {
  clear_error();
  if (n_edges < 0 || n_nodes < 0)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "force partial: invalid sizes");
  if (n_nodes == 0) return BYSJ_OK;
  if (src_offsets == nullptr || partial == nullptr ||
      (n_edges > 0 && (grad_edge == nullptr || edge_vec == nullptr ||
                       src_order == nullptr)))
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "force partial: NULL pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (force_index32(n_edges))
    force_assembly_kernel<kSrcPartial, int32_t><<<warp_per_atom_blocks(n_nodes), kBlock, 0, s>>>(
        grad_edge, edge_vec, nullptr, src_offsets, src_order, n_nodes, nullptr, nullptr,
        partial);
  else
    force_assembly_kernel<kSrcPartial, int64_t><<<warp_per_atom_blocks(n_nodes), kBlock, 0, s>>>(
        grad_edge, edge_vec, nullptr, src_offsets, src_order, n_nodes, nullptr, nullptr,
        partial);
  return launch_check("force_assembly_kernel<src partial>");
}

int bysj_force_assembly_dst_add(const float* grad_edge,
                                const int64_t* dst_offsets, int64_t n_local,
                                const double* summed_partial, float* force,
                                float* virial, void* stream) {
  clear_error();
  if (n_local < 0)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "force dst add: invalid sizes");
  if (n_local == 0) return BYSJ_OK;
  if (dst_offsets == nullptr || summed_partial == nullptr || force == nullptr)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "force dst add: NULL pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  force_dst_add_kernel<<<atom_blocks(n_local), kBlock, 0, s>>>(
      grad_edge, dst_offsets, n_local, summed_partial, force, virial);
  return launch_check("force_dst_add_kernel");
}

}  // extern "C"
