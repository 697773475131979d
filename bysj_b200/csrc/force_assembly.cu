// Force and per-atom virial assembly from per-edge energy gradients (sm_100a).
//
//   F_k = sum_{dst(e)=k} g_e - sum_{src(e)=k} g_e
//   W_k = - sum_{src(e)=k} g_e (x) v_e          (row-major 3x3)
//
// Contract and fp64 accumulation follow the reference's
// csrc/force_assembly.cpp:64-96.  The whole working set (grad_edge, edge_vec,
// src_order: ~73 MB at 2.2 M edges) is small, so the kernel is bound by
// memory latency rather than bandwidth; it maximises loads in flight: eight
// lanes cooperate on one atom (four atoms per warp), each lane taking every
// eighth edge of both CSR lists and issuing its loads in bursts, and the
// twelve fp64 sums are folded with a 3-step butterfly inside the 8-lane
// group.  The summation order is fixed, so repeated runs are bit-identical.
#include "launch.cuh"

namespace bysj {
namespace {

constexpr int kLanesPerAtom = 8;
constexpr int kAtomsPerWarp = kWarp / kLanesPerAtom;

enum Mode : int { kAssemble = 0, kSrcPartial = 1 };

// Loads of one lane are issued in bursts so that an atom costs a handful of
// dependent memory round trips, not one per edge: up to kSlots source slots
// (src_order) are fetched at once, then their grad/vec rows in batches of
// kBatch, and the destination rows in batches of kBatch while those are in
// flight.
constexpr int kSlots = 12;
constexpr int kBatch = 6;

// Row e of an [E, 3] float array with two loads: the 8-byte-aligned pair
// (components 0-1 for even e, 1-2 for odd e) and the remaining single.
// Needs an 8-byte-aligned base; PAIR = false falls back to three loads.
template <bool PAIR>
__device__ __forceinline__ void load_row3(const float* __restrict__ base, int64_t e,
                                          float (&v)[3]) {
  const float* p = base + 3 * e;
  if constexpr (PAIR) {
    const bool odd = (e & 1) != 0;
    const float2 pair = __ldg(reinterpret_cast<const float2*>(p + (odd ? 1 : 0)));
    const float single = __ldg(p + (odd ? 0 : 2));
    v[0] = odd ? single : pair.x;
    v[1] = odd ? pair.x : pair.y;
    v[2] = odd ? pair.y : single;
  } else {
    v[0] = __ldg(p);
    v[1] = __ldg(p + 1);
    v[2] = __ldg(p + 2);
  }
}

template <bool PAIR>
__device__ __forceinline__ void add_src_rows(const float* __restrict__ grad_edge,
                                             const float* __restrict__ edge_vec,
                                             const int64_t (&edge)[kBatch], int count,
                                             double (&acc)[12]) {
  float g[kBatch][3], v[kBatch][3];
#pragma unroll
  for (int b = 0; b < kBatch; ++b) {
    if (b < count) {
      load_row3<PAIR>(grad_edge, edge[b], g[b]);
      load_row3<PAIR>(edge_vec, edge[b], v[b]);
    }
  }
#pragma unroll
  for (int b = 0; b < kBatch; ++b) {
    if (b < count) {
#pragma unroll
      for (int r = 0; r < 3; ++r) {
        acc[r] -= g[b][r];
#pragma unroll
        for (int c = 0; c < 3; ++c) acc[3 + r * 3 + c] -= static_cast<double>(g[b][r]) * v[b][c];
      }
    }
  }
}

template <int MODE, bool PAIR>
__global__ void __launch_bounds__(kBlock, 2)
    force_assembly_kernel(const float* __restrict__ grad_edge,
                          const float* __restrict__ edge_vec,
                          const int64_t* __restrict__ dst_offsets,
                          const int64_t* __restrict__ src_offsets,
                          const int64_t* __restrict__ src_order,
                          int64_t n_nodes, float* __restrict__ force,
                          float* __restrict__ virial,
                          float* __restrict__ partial) {
  const int lane = lane_id();
  const int sub = lane & (kLanesPerAtom - 1);
  const int64_t stride =
      static_cast<int64_t>(gridDim.x) * kWarpsPerBlock * kAtomsPerWarp;
  for (int64_t base = global_warp() * kAtomsPerWarp; base < n_nodes;
       base += stride) {
    const int64_t atom = base + (lane / kLanesPerAtom);
    const bool valid = atom < n_nodes;
    double acc[12];
#pragma unroll
    for (int c = 0; c < 12; ++c) acc[c] = 0.0;
    if (valid) {
      int64_t d0 = 0, d1 = 0;
      if constexpr (MODE == kAssemble) {
        d0 = __ldg(dst_offsets + atom) + sub;
        d1 = __ldg(dst_offsets + atom + 1);
      }
      const int64_t s1 = __ldg(src_offsets + atom + 1);
      for (int64_t s = __ldg(src_offsets + atom) + sub; s < s1;
           s += static_cast<int64_t>(kSlots) * kLanesPerAtom) {
        // Burst 1: this lane's next kSlots source slots.
        int64_t edge[kSlots];
        int count = 0;
#pragma unroll
        for (int t = 0; t < kSlots; ++t) {
          const int64_t slot = s + static_cast<int64_t>(t) * kLanesPerAtom;
          if (slot < s1) {
            edge[t] = __ldg(src_order + slot);
            count = t + 1;
          }
        }
        // Destination rows of this round (contiguous), issued before the
        // gathers are consumed.
        float dg[kBatch][3];
        int dcount = 0;
        if constexpr (MODE == kAssemble) {
#pragma unroll
          for (int b = 0; b < kBatch; ++b) {
            const int64_t e = d0 + static_cast<int64_t>(b) * kLanesPerAtom;
            if (e < d1) {
              load_row3<PAIR>(grad_edge, e, dg[b]);
              dcount = b + 1;
            }
          }
          d0 += static_cast<int64_t>(kBatch) * kLanesPerAtom;
        }
        // Bursts 2 and 3: the gathered rows, kBatch slots at a time.
#pragma unroll
        for (int h = 0; h < kSlots / kBatch; ++h) {
          int64_t part[kBatch];
#pragma unroll
          for (int b = 0; b < kBatch; ++b) part[b] = edge[h * kBatch + b];
          const int c = count - h * kBatch;
          if (c > 0) add_src_rows<PAIR>(grad_edge, edge_vec, part, c < kBatch ? c : kBatch, acc);
        }
        if constexpr (MODE == kAssemble) {
#pragma unroll
          for (int b = 0; b < kBatch; ++b)
            if (b < dcount) {
              acc[0] += dg[b][0];
              acc[1] += dg[b][1];
              acc[2] += dg[b][2];
            }
        }
      }
      // Destination rows left over when an atom has more targets than sources.
      if constexpr (MODE == kAssemble) {
        for (; d0 < d1; d0 += kLanesPerAtom) {
          float row[3];
          load_row3<PAIR>(grad_edge, d0, row);
          acc[0] += row[0];
          acc[1] += row[1];
          acc[2] += row[2];
        }
      }
    }
#pragma unroll
    for (int c = 0; c < 12; ++c) acc[c] = group_sum(acc[c], kLanesPerAtom);
    if (!valid) continue;
    // Lane `sub` stores component sub, and sub + 8 when that exists.
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int c = sub + half * kLanesPerAtom;
      if (c >= 12) break;
      double v = 0.0;
#pragma unroll
      for (int t = 0; t < 12; ++t) v = (t == c) ? acc[t] : v;
      if constexpr (MODE == kAssemble) {
        if (c < 3) force[atom * 3 + c] = static_cast<float>(v);
        else if (virial) virial[atom * 9 + (c - 3)] = static_cast<float>(v);
      } else {
        partial[atom * 12 + c] = static_cast<float>(v);
      }
    }
  }
}

// force[k] = sum_{dst(e)=k} g_e + summed[k, 0:3];  virial[k] = summed[k, 3:12]
__global__ void __launch_bounds__(kBlock)
    force_dst_add_kernel(const float* __restrict__ grad_edge,
                         const int64_t* __restrict__ dst_offsets,
                         int64_t n_local, const float* __restrict__ summed,
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
          static_cast<float>(v + static_cast<double>(summed[atom * 12 + sub]));
    }
    if (virial) {
      virial[atom * 9 + sub] = summed[atom * 12 + 3 + sub];
      if (sub == 0) virial[atom * 9 + 8] = summed[atom * 12 + 11];
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
  if (aligned8(grad_edge) && aligned8(edge_vec))
    force_assembly_kernel<kAssemble, true><<<atom_blocks(n_nodes), kBlock, 0, s>>>(
        grad_edge, edge_vec, dst_offsets, src_offsets, src_order, n_nodes, force,
        virial, nullptr);
  else
    force_assembly_kernel<kAssemble, false><<<atom_blocks(n_nodes), kBlock, 0, s>>>(
        grad_edge, edge_vec, dst_offsets, src_offsets, src_order, n_nodes, force,
        virial, nullptr);
  return launch_check("force_assembly_kernel");
}

int bysj_force_assembly_src_partial(const float* grad_edge,
                                    const float* edge_vec,
                                    const int64_t* src_offsets,
                                    const int64_t* src_order, int64_t n_edges,
                                    int64_t n_nodes, float* partial,
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
  if (aligned8(grad_edge) && aligned8(edge_vec))
    force_assembly_kernel<kSrcPartial, true><<<atom_blocks(n_nodes), kBlock, 0, s>>>(
        grad_edge, edge_vec, nullptr, src_offsets, src_order, n_nodes, nullptr,
        nullptr, partial);
  else
    force_assembly_kernel<kSrcPartial, false><<<atom_blocks(n_nodes), kBlock, 0, s>>>(
        grad_edge, edge_vec, nullptr, src_offsets, src_order, n_nodes, nullptr,
        nullptr, partial);
  return launch_check("force_assembly_kernel<src partial>");
}

int bysj_force_assembly_dst_add(const float* grad_edge,
                                const int64_t* dst_offsets, int64_t n_local,
                                const float* summed_partial, float* force,
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
