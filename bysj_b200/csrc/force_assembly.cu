// Force and per-atom virial assembly from per-edge energy gradients (sm_100a).
//
//   F_k = sum_{dst(e)=k} g_e - sum_{src(e)=k} g_e
//   W_k = - sum_{src(e)=k} g_e (x) v_e          (row-major 3x3)
//
// Contract and fp64 accumulation follow the reference's
// csrc/force_assembly.cpp:64-96.  The whole working set (grad_edge, edge_vec,
// src_order: ~73 MB at 2.2 M edges) is small, so the kernel is bound by
// memory latency rather than bandwidth; it maximises loads in flight: eight
// lanes cooperate on one atom (four atoms per warp), each lane walking every
// eighth edge of both CSR lists with independent loads, and the twelve fp64
// sums are folded with a 3-step butterfly inside the 8-lane group.  The
// summation order is fixed, so repeated runs are bit-identical.
#include "launch.cuh"

namespace bysj {
namespace {

constexpr int kLanesPerAtom = 8;
constexpr int kAtomsPerWarp = kWarp / kLanesPerAtom;

enum Mode : int { kAssemble = 0, kSrcPartial = 1 };

template <int MODE>
__global__ void __launch_bounds__(kBlock)
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
      if constexpr (MODE == kAssemble) {
        const int64_t d0 = __ldg(dst_offsets + atom);
        const int64_t d1 = __ldg(dst_offsets + atom + 1);
        int64_t e = d0 + sub;
        for (; e + kLanesPerAtom < d1; e += 2 * kLanesPerAtom) {
          const float* g0 = grad_edge + e * 3;
          const float* g1 = grad_edge + (e + kLanesPerAtom) * 3;
          const float a0 = __ldg(g0), a1 = __ldg(g0 + 1), a2 = __ldg(g0 + 2);
          const float b0 = __ldg(g1), b1 = __ldg(g1 + 1), b2 = __ldg(g1 + 2);
          acc[0] += a0; acc[1] += a1; acc[2] += a2;
          acc[0] += b0; acc[1] += b1; acc[2] += b2;
        }
        if (e < d1) {
          const float* g0 = grad_edge + e * 3;
          acc[0] += __ldg(g0); acc[1] += __ldg(g0 + 1); acc[2] += __ldg(g0 + 2);
        }
      }
      const int64_t s0 = __ldg(src_offsets + atom);
      const int64_t s1 = __ldg(src_offsets + atom + 1);
      int64_t s = s0 + sub;
      for (; s + kLanesPerAtom < s1; s += 2 * kLanesPerAtom) {
        const int64_t ea = __ldg(src_order + s);
        const int64_t eb = __ldg(src_order + s + kLanesPerAtom);
        float ga[3], va[3], gb[3], vb[3];
#pragma unroll
        for (int r = 0; r < 3; ++r) {
          ga[r] = __ldg(grad_edge + ea * 3 + r);
          va[r] = __ldg(edge_vec + ea * 3 + r);
          gb[r] = __ldg(grad_edge + eb * 3 + r);
          vb[r] = __ldg(edge_vec + eb * 3 + r);
        }
#pragma unroll
        for (int r = 0; r < 3; ++r) {
          acc[r] -= ga[r];
#pragma unroll
          for (int c = 0; c < 3; ++c)
            acc[3 + r * 3 + c] -= static_cast<double>(ga[r]) * va[c];
        }
#pragma unroll
        for (int r = 0; r < 3; ++r) {
          acc[r] -= gb[r];
#pragma unroll
          for (int c = 0; c < 3; ++c)
            acc[3 + r * 3 + c] -= static_cast<double>(gb[r]) * vb[c];
        }
      }
      if (s < s1) {
        const int64_t ea = __ldg(src_order + s);
        float ga[3], va[3];
#pragma unroll
        for (int r = 0; r < 3; ++r) {
          ga[r] = __ldg(grad_edge + ea * 3 + r);
          va[r] = __ldg(edge_vec + ea * 3 + r);
        }
#pragma unroll
        for (int r = 0; r < 3; ++r) {
          acc[r] -= ga[r];
#pragma unroll
          for (int c = 0; c < 3; ++c)
            acc[3 + r * 3 + c] -= static_cast<double>(ga[r]) * va[c];
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
  force_assembly_kernel<kAssemble><<<atom_blocks(n_nodes), kBlock, 0, s>>>(
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
  force_assembly_kernel<kSrcPartial><<<atom_blocks(n_nodes), kBlock, 0, s>>>(
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
