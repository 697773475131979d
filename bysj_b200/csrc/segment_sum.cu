// Destination-segmented sum (forward and backward) for sm_100a.
//
//   out[n, c] = node_scale[n] * sum_{slot in seg(n)} edge_scale[e] * src[e, c]
//
// Same contract as the reference's csrc/segment_sum.cpp:77-183, built the
// B200 way: the (edges + segment ends) sequence is cut into equal merge-path
// partitions, one per warp, so a skewed degree distribution cannot leave one
// warp with a giant segment.  Lanes read edge rows with 16-byte streaming
// loads, several rows in flight per lane; narrow rows pack several edges into
// one warp (lane groups) and fold them with a fixed butterfly.  A segment cut
// by a partition boundary is finished by the last partition to reach it,
// which sums the partials in partition order: results are bit-identical from
// run to run and no floating-point atomic is used.
#include "launch.cuh"

namespace bysj {
namespace {

struct SumArgs {
  const void* src;
  int64_t channels;
  int64_t lv;  // row width in vectors
  const float* edge_scale;
  const float* node_scale;
  const int64_t* order;
  float* out;
  MergePath mp;
  SplitSlots ss;
};

// G lane groups of LPG = 32/G lanes; each lane holds NV vectors of VEC
// elements of the row; U edges per group are loaded before they are used.
template <typename T, int VEC, int NV, int G>
struct SumShape {
  static constexpr int LPG = kWarp / G;
  static constexpr int TV = LPG * NV;  // vectors per column tile
  // 128-256 bytes of row data in flight per lane, within a register budget
  // that keeps 16 (wide rows) or 24 warps resident per SM.
  static constexpr int U = (NV * VEC >= 64)   ? 1
                           : (NV * VEC >= 16) ? 2
                           : (8 / NV < 1 ? 1 : 8 / NV);
  static constexpr int kMinBlocks = (NV * VEC >= 32) ? 2 : 3;
};

template <typename T, int VEC, int NV, int G>
__device__ __forceinline__ void sum_edges(const SumArgs& a, int64_t lo,
                                          int64_t hi, int g, int64_t j0,
                                          float (&acc)[NV][VEC]) {
  using S = SumShape<T, VEC, NV, G>;
  const T* src = static_cast<const T*>(a.src);
  const int64_t C = a.channels;
  // Lanes past the end of the row re-read its last vector (same sectors as a
  // neighbouring lane, so no extra traffic) and never store what they sum;
  // this keeps the loads unpredicated.
  int64_t jl[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int64_t j = j0 + k * S::LPG;
    jl[k] = j < a.lv ? j : a.lv - 1;
  }
  int64_t s = lo + g;
  for (; s + (S::U - 1) * G < hi; s += S::U * G) {
    const T* row[S::U];
    float w[S::U];
#pragma unroll
    for (int u = 0; u < S::U; ++u) {
      const int64_t slot = s + u * G;
      const int64_t edge = a.order ? __ldg(a.order + slot) : slot;
      row[u] = src + edge * C;
      w[u] = a.edge_scale ? __ldg(a.edge_scale + edge) : 1.0f;
    }
    RowVec<T, VEC> buf[S::U][NV];
#pragma unroll
    for (int u = 0; u < S::U; ++u)
#pragma unroll
      for (int k = 0; k < NV; ++k) buf[u][k].load(row[u], jl[k]);
#pragma unroll
    for (int u = 0; u < S::U; ++u)
#pragma unroll
      for (int k = 0; k < NV; ++k)
#pragma unroll
        for (int i = 0; i < VEC; ++i)
          acc[k][i] = fmaf(w[u], buf[u][k].get(i), acc[k][i]);
  }
  for (; s < hi; s += G) {
    const int64_t edge = a.order ? __ldg(a.order + s) : s;
    const float w = a.edge_scale ? __ldg(a.edge_scale + edge) : 1.0f;
    const T* row = src + edge * C;
    RowVec<T, VEC> buf[NV];
#pragma unroll
    for (int k = 0; k < NV; ++k) buf[k].load(row, jl[k]);
#pragma unroll
    for (int k = 0; k < NV; ++k)
#pragma unroll
      for (int i = 0; i < VEC; ++i)
        acc[k][i] = fmaf(w, buf[k].get(i), acc[k][i]);
  }
}

template <typename T, int VEC, int NV, int G>
__global__ void __launch_bounds__(kBlock, SumShape<T, VEC, NV, G>::kMinBlocks)
    segment_sum_fwd_kernel(SumArgs a) {
  using S = SumShape<T, VEC, NV, G>;
  const int64_t p = global_warp();
  if (p >= a.mp.parts) return;
  const int tile = blockIdx.y;
  const int lane = lane_id();
  const int g = lane / S::LPG;
  const int64_t jt = static_cast<int64_t>(tile) * S::TV;  // tile start
  const int64_t j0 = jt + lane % S::LPG;                  // lane's first vector
  const int64_t C = a.channels;

  SegCursor cur(a.mp, part_range(a.mp, p));
  while (cur.next()) {
    float acc[NV][VEC];
#pragma unroll
    for (int k = 0; k < NV; ++k)
#pragma unroll
      for (int i = 0; i < VEC; ++i) acc[k][i] = 0.0f;
    sum_edges<T, VEC, NV, G>(a, cur.lo, cur.hi, g, j0, acc);
    if constexpr (G > 1) {
#pragma unroll
      for (int k = 0; k < NV; ++k)
#pragma unroll
        for (int i = 0; i < VEC; ++i) acc[k][i] = xor_sum(acc[k][i], S::LPG);
    }
    const int64_t n = cur.node;
    if (cur.kind == kWhole) {
      const float scale = a.node_scale ? __ldg(a.node_scale + n) : 1.0f;
      if (g == 0) {
#pragma unroll
        for (int k = 0; k < NV; ++k) {
          const int64_t j = j0 + k * S::LPG;
          if (j < a.lv) {
            float v[VEC];
#pragma unroll
            for (int i = 0; i < VEC; ++i) v[i] = acc[k][i] * scale;
            store_f32<VEC>(a.out + n * C + j * VEC, v);
          }
        }
      }
      continue;
    }
    // Split segment: publish the partial, the last contributor combines.
    float* mine = a.ss.slot(p, cur.kind);
    if (g == 0) {
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const int64_t j = j0 + k * S::LPG;
        if (j < a.lv) store_cg<VEC>(mine + j * VEC, acc[k]);
      }
    }
    const int64_t first = a.mp.part_of_first_edge(n);
    const int64_t last = a.mp.part_of_end(n);
    if (!arrive_last(a.ss, first, last, tile)) continue;
    const float scale = a.node_scale ? __ldg(a.node_scale + n) : 1.0f;
    for (int64_t jj = lane; jj < S::TV; jj += kWarp) {
      const int64_t j = jt + jj;
      if (j >= a.lv) break;
      float sum[VEC];
#pragma unroll
      for (int i = 0; i < VEC; ++i) sum[i] = 0.0f;
      for (int64_t q = first; q <= last; ++q) {
        float part[VEC];
        load_cg<VEC>(a.ss.slot(q, q == last ? kHead : kTail) + j * VEC, part);
#pragma unroll
        for (int i = 0; i < VEC; ++i) sum[i] += part[i];
      }
#pragma unroll
      for (int i = 0; i < VEC; ++i) sum[i] *= scale;
      store_f32<VEC>(a.out + n * C + j * VEC, sum);
    }
  }
}

// ---------------------------------------------------------------------------
// Backward: grad_src is an element-wise gather of the node rows.
// ---------------------------------------------------------------------------
template <int VEC>
__global__ void __launch_bounds__(kBlock)
    segment_sum_grad_src_kernel(const float* __restrict__ grad_out,
                                const float* __restrict__ edge_scale,
                                const float* __restrict__ node_scale,
                                const int64_t* __restrict__ dst,
                                float* __restrict__ grad_src, int64_t n_edges,
                                int64_t channels) {
  const int64_t lv = channels / VEC;
  const int64_t total = n_edges * lv;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x +
                     threadIdx.x;
       idx < total; idx += stride) {
    const int64_t e = idx / lv;
    const int64_t j = idx - e * lv;
    const int64_t n = __ldg(dst + e);
    float scale = edge_scale ? __ldg(edge_scale + e) : 1.0f;
    if (node_scale) scale *= __ldg(node_scale + n);
    float v[VEC];
    if constexpr (VEC == 4) {
      const float4 t = __ldg(reinterpret_cast<const float4*>(
          grad_out + n * channels + j * 4));
      v[0] = t.x * scale; v[1] = t.y * scale;
      v[2] = t.z * scale; v[3] = t.w * scale;
    } else {
      v[0] = __ldg(grad_out + n * channels + j) * scale;
    }
    store_f32<VEC>(grad_src + e * channels + j * VEC, v);
  }
}

// grad_node_scale[n] = sum_c grad_out[n, c] * sum_{e in n} w_e src[e, c]
// computed as sum_e w_e <grad_out[n], src[e]>; one scalar per segment, so
// split segments combine scalars.
struct NodeScaleGradArgs {
  const void* src;
  int64_t channels;
  const float* grad_out;
  const float* edge_scale;
  const int64_t* order;
  float* grad_node_scale;
  MergePath mp;
  SplitSlots ss;
};

// grad_src for 16-byte rows over merge-path partitions: a warp loads the
// node's grad_out row (its NV vectors per lane) once per piece and streams
// row * (edge_scale[e] * node_scale[n]) to the piece's edges (the reference's
// scale order, csrc/segment_sum.cpp:136-149).  Pieces of a split segment are
// independent, so nothing is combined.
template <int NV>
__global__ void __launch_bounds__(kBlock)
    segment_sum_grad_src_rows_kernel(const float* __restrict__ grad_out,
                                     const float* __restrict__ edge_scale,
                                     const float* __restrict__ node_scale,
                                     const int64_t* __restrict__ order, MergePath mp,
                                     int64_t channels, float* __restrict__ grad_src) {
  constexpr int TV = kWarp * NV;
  const int64_t p = global_warp();
  if (p >= mp.parts) return;
  const int lane = lane_id();
  const int64_t lv = channels / 4;
  const int64_t j0 = static_cast<int64_t>(blockIdx.y) * TV + lane;
  SegCursor cur(mp, part_range(mp, p));
  while (cur.next()) {
    if (cur.lo >= cur.hi) continue;
    const int64_t n = cur.node;
    const float sn = node_scale ? __ldg(node_scale + n) : 1.0f;
    float4 row[NV];
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int64_t j = j0 + k * kWarp;
      row[k] = j < lv ? __ldg(reinterpret_cast<const float4*>(grad_out + n * channels) + j)
                      : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    for (int64_t slot = cur.lo; slot < cur.hi; ++slot) {
      const int64_t e = order ? __ldg(order + slot) : slot;
      const float scale = (edge_scale ? __ldg(edge_scale + e) : 1.0f) * sn;
      float4* out = reinterpret_cast<float4*>(grad_src + e * channels);
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const int64_t j = j0 + k * kWarp;
        if (j < lv)
          __stcs(out + j, make_float4(row[k].x * scale, row[k].y * scale, row[k].z * scale,
                                      row[k].w * scale));
      }
    }
  }
}

// grad_node_scale[n] = sum_{e in n} edge_scale[e] * <grad_out[n], src[e]>:
// lanes over the row's vectors, edges in slot order, merge-path pieces
// combined in partition order.
template <typename T, int VEC, bool kVecG = false>
__global__ void __launch_bounds__(kBlock)
    segment_sum_grad_scale_kernel(NodeScaleGradArgs a) {
  const int64_t p = global_warp();
  if (p >= a.mp.parts) return;
  const int lane = lane_id();
  const T* src = static_cast<const T*>(a.src);
  const int64_t C = a.channels;
  const int64_t lv = C / VEC;
  SegCursor cur(a.mp, part_range(a.mp, p));
  while (cur.next()) {
    const int64_t n = cur.node;
    const float* g = a.grad_out + n * C;
    float acc = 0.0f;
    for (int64_t s = cur.lo; s < cur.hi; ++s) {
      const int64_t e = a.order ? __ldg(a.order + s) : s;
      float dot = 0.0f;
      for (int64_t j = lane; j < lv; j += kWarp) {
        RowVec<T, VEC> v;
        v.load(src + e * C, j);
        float gv[VEC];
        if constexpr (kVecG) {  // 16-byte loads of the grad_out row (L1)
#pragma unroll
          for (int i = 0; i < VEC; i += 4) {
            const float4 t = __ldg(reinterpret_cast<const float4*>(g + j * VEC + i));
            gv[i] = t.x; gv[i + 1] = t.y; gv[i + 2] = t.z; gv[i + 3] = t.w;
          }
        } else {
#pragma unroll
          for (int i = 0; i < VEC; ++i) gv[i] = __ldg(g + j * VEC + i);
        }
#pragma unroll
        for (int i = 0; i < VEC; ++i) dot = fmaf(gv[i], v.get(i), dot);
      }
      const float w = a.edge_scale ? __ldg(a.edge_scale + e) : 1.0f;
      acc = fmaf(w, dot, acc);
    }
    acc = xor_sum(acc, 1);
    if (cur.kind == kWhole) {
      if (lane == 0) a.grad_node_scale[n] = acc;
      continue;
    }
    if (lane == 0) __stcg(a.ss.slot(p, cur.kind), acc);
    const int64_t first = a.mp.part_of_first_edge(n);
    const int64_t last = a.mp.part_of_end(n);
    if (!arrive_last(a.ss, first, last, 0)) continue;
    if (lane == 0) {
      float sum = 0.0f;
      for (int64_t q = first; q <= last; ++q)
        sum += __ldcg(a.ss.slot(q, q == last ? kHead : kTail));
      a.grad_node_scale[n] = sum;
    }
  }
}

// grad_src and grad_node_scale in one pass, for fp32 src rows of at most
// 32 NV float4 (one tile; used up to 256 channels): a warp holds the node's grad_out row in registers;
// per edge it loads the src row, adds edge_scale * <grad_out, src> to its
// lane's partial (the lanes' vectors and the order of the products are those
// of segment_sum_grad_scale_kernel, so grad_node_scale has the same bits) and
// stores grad_out * (edge_scale * node_scale) (as the rows kernel).  Two
// edges' src rows are in flight per iteration.  Same partitions, slots and
// in-order combination of split segments as segment_sum_grad_scale_kernel.
template <int NV>
__device__ __forceinline__ float row_dot(const float4 (&row)[NV], const float4 (&v)[NV]) {
  float dot = 0.0f;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    dot = fmaf(row[k].x, v[k].x, dot);
    dot = fmaf(row[k].y, v[k].y, dot);
    dot = fmaf(row[k].z, v[k].z, dot);
    dot = fmaf(row[k].w, v[k].w, dot);
  }
  return dot;
}

template <int NV>
__global__ void __launch_bounds__(kBlock)
    segment_sum_bwd_fused_kernel(NodeScaleGradArgs a, const float* __restrict__ node_scale,
                                 float* __restrict__ grad_src) {
  const int64_t p = global_warp();
  if (p >= a.mp.parts) return;
  const int lane = lane_id();
  const int64_t C = a.channels;
  const int64_t lv = C / 4;
  const float* src = static_cast<const float*>(a.src);
  SegCursor cur(a.mp, part_range(a.mp, p));
  while (cur.next()) {
    const int64_t n = cur.node;
    const float sn = node_scale ? __ldg(node_scale + n) : 1.0f;
    float4 row[NV];
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int64_t j = lane + k * kWarp;
      row[k] = j < lv ? __ldg(reinterpret_cast<const float4*>(a.grad_out + n * C) + j)
                      : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    float acc = 0.0f;
    auto load = [&](int64_t e, float4 (&v)[NV]) {
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const int64_t j = lane + k * kWarp;
        v[k] = j < lv ? ld_stream_f4(src + e * C + 4 * j) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      }
    };
    auto store = [&](int64_t e, float w) {
      const float scale = w * sn;
      float4* out = reinterpret_cast<float4*>(grad_src + e * C);
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const int64_t j = lane + k * kWarp;
        if (j < lv)
          __stcs(out + j, make_float4(row[k].x * scale, row[k].y * scale, row[k].z * scale,
                                      row[k].w * scale));
      }
    };
    int64_t sl = cur.lo;
    for (; sl + 1 < cur.hi; sl += 2) {
      const int64_t e0 = a.order ? __ldg(a.order + sl) : sl;
      const int64_t e1 = a.order ? __ldg(a.order + sl + 1) : sl + 1;
      float4 v0[NV], v1[NV];
      load(e0, v0);
      load(e1, v1);
      const float w0 = a.edge_scale ? __ldg(a.edge_scale + e0) : 1.0f;
      const float w1 = a.edge_scale ? __ldg(a.edge_scale + e1) : 1.0f;
      acc = fmaf(w0, row_dot<NV>(row, v0), acc);
      acc = fmaf(w1, row_dot<NV>(row, v1), acc);
      store(e0, w0);
      store(e1, w1);
    }
    if (sl < cur.hi) {
      const int64_t e0 = a.order ? __ldg(a.order + sl) : sl;
      float4 v0[NV];
      load(e0, v0);
      const float w0 = a.edge_scale ? __ldg(a.edge_scale + e0) : 1.0f;
      acc = fmaf(w0, row_dot<NV>(row, v0), acc);
      store(e0, w0);
    }
    acc = xor_sum(acc, 1);
    if (cur.kind == kWhole) {
      if (lane == 0) a.grad_node_scale[n] = acc;
      continue;
    }
    if (lane == 0) __stcg(a.ss.slot(p, cur.kind), acc);
    const int64_t first = a.mp.part_of_first_edge(n);
    const int64_t last = a.mp.part_of_end(n);
    if (!arrive_last(a.ss, first, last, 0)) continue;
    if (lane == 0) {
      float sum = 0.0f;
      for (int64_t q = first; q <= last; ++q)
        sum += __ldcg(a.ss.slot(q, q == last ? kHead : kTail));
      a.grad_node_scale[n] = sum;
    }
  }
}

// ---------------------------------------------------------------------------
// Host dispatch.
// ---------------------------------------------------------------------------
using FwdKernel = void (*)(SumArgs);

struct SumConfig {
  FwdKernel kernel = nullptr;
  int vec = 1, nv = 1, g = 1;
  int64_t lv = 0, tv = 0, tiles = 1;
};

template <typename T, int VEC>
SumConfig pick_for(int64_t lv) {
  SumConfig c;
  c.vec = VEC;
  c.lv = lv;
  if (lv >= 256) {
    c.kernel = segment_sum_fwd_kernel<T, VEC, 8, 1>; c.nv = 8; c.g = 1;
  } else if (lv > 64) {
    if (lv > 128) { c.kernel = segment_sum_fwd_kernel<T, VEC, 8, 1>; c.nv = 8; }
    else { c.kernel = segment_sum_fwd_kernel<T, VEC, 4, 1>; c.nv = 4; }
  } else if (lv > 32) {
    c.kernel = segment_sum_fwd_kernel<T, VEC, 2, 1>; c.nv = 2;
  } else {
    const int64_t w = next_pow2(lv);
    c.nv = 1;
    switch (w) {
      case 32: c.kernel = segment_sum_fwd_kernel<T, VEC, 1, 1>; c.g = 1; break;
      case 16: c.kernel = segment_sum_fwd_kernel<T, VEC, 1, 2>; c.g = 2; break;
      case 8: c.kernel = segment_sum_fwd_kernel<T, VEC, 1, 4>; c.g = 4; break;
      case 4: c.kernel = segment_sum_fwd_kernel<T, VEC, 1, 8>; c.g = 8; break;
      case 2: c.kernel = segment_sum_fwd_kernel<T, VEC, 1, 16>; c.g = 16; break;
      default: c.kernel = segment_sum_fwd_kernel<T, VEC, 1, 32>; c.g = 32; break;
    }
  }
  c.tv = static_cast<int64_t>(kWarp / c.g) * c.nv;
  c.tiles = (lv + c.tv - 1) / c.tv;
  return c;
}

SumConfig pick_sum(bool vec_ok, int dtype, int64_t channels) {
  if (dtype == BYSJ_BF16) {
    if (vec_ok && channels % 8 == 0)
      return pick_for<__nv_bfloat16, 8>(channels / 8);
    return pick_for<__nv_bfloat16, 1>(channels);
  }
  if (vec_ok && channels % 4 == 0) return pick_for<float, 4>(channels / 4);
  return pick_for<float, 1>(channels);
}

struct SumLayout {
  SumConfig cfg;
  PartitionPlan plan;
  int64_t stride = 0;
  size_t bytes = 0;
};

SumLayout layout_sum(bool vec_ok, int dtype, int64_t n_edges,
                     int64_t n_nodes, int64_t channels, void* ws,
                     SplitSlots* ss) {
  SumLayout L;
  L.cfg = pick_sum(vec_ok, dtype, channels);
  const DeviceInfo& dev = current_device_info();
  const int64_t resident =
      static_cast<int64_t>(dev.sm_count) *
      resident_blocks(reinterpret_cast<const void*>(L.cfg.kernel)) *
      kWarpsPerBlock;
  int64_t warps = resident / L.cfg.tiles;
  if (warps < 1) warps = 1;
  L.plan = plan_partitions(n_edges, n_nodes, warps, 16);
  L.stride = (channels + 7) / 8 * 8;
  Carver carve(ws);
  float* slots = carve.take<float>(static_cast<size_t>(L.plan.parts) * 2 *
                                   L.stride);
  int* tickets = carve.take<int>(static_cast<size_t>(L.plan.parts) *
                                 L.cfg.tiles);
  L.bytes = carve.need;
  if (ss) {
    ss->slots = slots;
    ss->tickets = tickets;
    ss->stride = L.stride;
    ss->tiles = static_cast<int>(L.cfg.tiles);
  }
  return L;
}

int check_common(int64_t n_edges, int64_t n_nodes, int64_t channels,
                 const int64_t* offsets) {
  if (n_edges < 0 || n_nodes < 0 || channels <= 0)
    return fail(BYSJ_ERR_INVALID_ARGUMENT,
                "segment sum: invalid sizes (edges %lld, nodes %lld, "
                "channels %lld)",
                (long long)n_edges, (long long)n_nodes, (long long)channels);
  if (n_nodes > 0 && offsets == nullptr)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "segment sum: offsets is NULL");
  return BYSJ_OK;
}

int sum_bwd_fused(const float* grad_out, const void* src, const int64_t* offsets,
                  int64_t n_edges, int64_t n_nodes, int64_t channels, const float* edge_scale,
                  const float* node_scale, const int64_t* order, float* grad_src,
                  float* grad_node_scale, void* workspace, size_t workspace_bytes,
                  cudaStream_t s) {
  const DeviceInfo& dev = current_device_info();
  const int64_t resident = static_cast<int64_t>(dev.sm_count) * 8 * kWarpsPerBlock;
  const PartitionPlan plan = plan_partitions(n_edges, n_nodes, resident, 16);
  Carver carve(workspace);
  float* slots = carve.take<float>(static_cast<size_t>(plan.parts) * 2);
  int* tickets = carve.take<int>(static_cast<size_t>(plan.parts));
  if (workspace == nullptr || workspace_bytes < carve.need)
    return fail(BYSJ_ERR_WORKSPACE,
                "segment sum backward: workspace of %zu bytes needed, %zu given", carve.need,
                workspace_bytes);
  int st = cuda_check(cudaMemsetAsync(tickets, 0, sizeof(int) * plan.parts, s),
                      "segment sum backward: ticket reset");
  if (st) return st;
  NodeScaleGradArgs a;
  a.src = src;
  a.channels = channels;
  a.grad_out = grad_out;
  a.edge_scale = edge_scale;
  a.order = order;
  a.grad_node_scale = grad_node_scale;
  a.mp = MergePath{offsets, n_nodes, n_edges, plan.ipc, plan.parts};
  a.ss = SplitSlots{slots, tickets, 1, 1};
  const int64_t lv = channels / 4;  // <= 64
  if (lv > kWarp)
    segment_sum_bwd_fused_kernel<2><<<plan.blocks, kBlock, 0, s>>>(a, node_scale, grad_src);
  else
    segment_sum_bwd_fused_kernel<1><<<plan.blocks, kBlock, 0, s>>>(a, node_scale, grad_src);
  return launch_check("segment_sum_bwd_fused_kernel");
}

}  // namespace
}  // namespace bysj

using namespace bysj;

extern "C" {

size_t bysj_segment_sum_workspace_size(int64_t n_edges, int64_t n_nodes,
                                       int64_t channels, int src_dtype) {
  if (n_edges < 0 || n_nodes <= 0 || channels <= 0) return 0;
  // The pointers' alignment decides between the vector and scalar kernels;
  // size for whichever of the two needs more.
  const size_t a = layout_sum(true, src_dtype, n_edges, n_nodes, channels,
                              nullptr, nullptr).bytes;
  const size_t b = layout_sum(false, src_dtype, n_edges, n_nodes, channels,
                              nullptr, nullptr).bytes;
  return a > b ? a : b;
}

int bysj_segment_sum_forward(const void* src, int src_dtype, int64_t n_edges,
                             int64_t channels, const int64_t* offsets,
                             int64_t n_nodes, const float* edge_scale,
                             const float* node_scale, const int64_t* order,
                             float* out, void* workspace,
                             size_t workspace_bytes, void* stream) {
  clear_error();
  int st = check_common(n_edges, n_nodes, channels, offsets);
  if (st) return st;
  if (src_dtype != BYSJ_F32 && src_dtype != BYSJ_BF16)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "segment sum: unknown dtype %d",
                src_dtype);
  if (n_nodes == 0) return BYSJ_OK;
  if (out == nullptr || (n_edges > 0 && src == nullptr))
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "segment sum: NULL src/out");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  SplitSlots ss{};
  // The vector path loads and stores 16-byte chunks of the rows.
  const bool vec_ok = aligned16(src) && aligned16(out);
  SumLayout L = layout_sum(vec_ok, src_dtype, n_edges, n_nodes, channels,
                           workspace, &ss);
  if (workspace == nullptr || workspace_bytes < L.bytes)
    return fail(BYSJ_ERR_WORKSPACE,
                "segment sum: workspace of %zu bytes needed, %zu given",
                L.bytes, workspace_bytes);
  st = cuda_check(cudaMemsetAsync(ss.tickets, 0,
                                  sizeof(int) * L.plan.parts * L.cfg.tiles, s),
                  "segment sum: ticket reset");
  if (st) return st;
  SumArgs a;
  a.src = src;
  a.channels = channels;
  a.lv = L.cfg.lv;
  a.edge_scale = edge_scale;
  a.node_scale = node_scale;
  a.order = order;
  a.out = out;
  a.mp = MergePath{offsets, n_nodes, n_edges, L.plan.ipc, L.plan.parts};
  a.ss = ss;
  dim3 grid(L.plan.blocks, static_cast<unsigned>(L.cfg.tiles));
  L.cfg.kernel<<<grid, kBlock, 0, s>>>(a);
  return launch_check("segment_sum_fwd_kernel");
}

size_t bysj_segment_sum_backward_workspace_size(int64_t n_edges,
                                                int64_t n_nodes,
                                                int64_t channels,
                                                int src_dtype) {
  (void)channels;
  (void)src_dtype;
  if (n_edges < 0 || n_nodes <= 0) return 0;
  const DeviceInfo& dev = current_device_info();
  const int64_t resident = static_cast<int64_t>(dev.sm_count) * 8 *
                           kWarpsPerBlock;
  PartitionPlan plan = plan_partitions(n_edges, n_nodes, resident, 16);
  Carver carve(nullptr);
  carve.take<float>(static_cast<size_t>(plan.parts) * 2);
  carve.take<int>(static_cast<size_t>(plan.parts));
  return carve.need;
}

int bysj_segment_sum_backward(const float* grad_out, const void* src,
                              int src_dtype, const int64_t* dst,
                              const int64_t* offsets, int64_t n_edges,
                              int64_t n_nodes, int64_t channels,
                              const float* edge_scale, const float* node_scale,
                              const int64_t* order, float* grad_src,
                              float* grad_node_scale, void* workspace,
                              size_t workspace_bytes, void* stream) {
  clear_error();
  int st = check_common(n_edges, n_nodes, channels, offsets);
  if (st) return st;
  if (n_edges > 0 && (grad_out == nullptr || dst == nullptr ||
                      grad_src == nullptr))
    return fail(BYSJ_ERR_INVALID_ARGUMENT,
                "segment sum backward: NULL grad_out/dst/grad_src");
  if (grad_node_scale != nullptr && node_scale == nullptr)
    return fail(BYSJ_ERR_INVALID_ARGUMENT,
                "segment sum backward: a node_scale gradient needs node_scale");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Both gradients in one pass for fp32 rows of up to 256 channels (measured
  // faster there; from 512 channels on the two separate streams are).
  const bool fused = grad_node_scale != nullptr && n_edges > 0 && src_dtype != BYSJ_BF16 &&
                     channels % 4 == 0 && channels <= 256 && aligned16(grad_out) &&
                     aligned16(grad_src) && aligned16(src);
  if (fused) return sum_bwd_fused(grad_out, src, offsets, n_edges, n_nodes, channels,
                                  edge_scale, node_scale, order, grad_src, grad_node_scale,
                                  workspace, workspace_bytes, s);
  if (n_edges > 0 && channels % 4 == 0 && aligned16(grad_out) && aligned16(grad_src)) {
    const int64_t lv = channels / 4;
    const int nv = lv > 128 ? 8 : lv > 64 ? 4 : lv > 32 ? 2 : 1;
    const int64_t tiles = (lv + kWarp * nv - 1) / (kWarp * nv);
    const DeviceInfo& dev = current_device_info();
    const int64_t resident = static_cast<int64_t>(dev.sm_count) * 8 * kWarpsPerBlock;
    int64_t warps = resident / tiles;
    if (warps < 1) warps = 1;
    const PartitionPlan plan = plan_partitions(n_edges, n_nodes, warps, 16);
    const MergePath mp{offsets, n_nodes, n_edges, plan.ipc, plan.parts};
    const dim3 grid(plan.blocks, static_cast<unsigned>(tiles));
    switch (nv) {
      case 8:
        segment_sum_grad_src_rows_kernel<8><<<grid, kBlock, 0, s>>>(
            grad_out, edge_scale, node_scale, order, mp, channels, grad_src);
        break;
      case 4:
        segment_sum_grad_src_rows_kernel<4><<<grid, kBlock, 0, s>>>(
            grad_out, edge_scale, node_scale, order, mp, channels, grad_src);
        break;
      case 2:
        segment_sum_grad_src_rows_kernel<2><<<grid, kBlock, 0, s>>>(
            grad_out, edge_scale, node_scale, order, mp, channels, grad_src);
        break;
      default:
        segment_sum_grad_src_rows_kernel<1><<<grid, kBlock, 0, s>>>(
            grad_out, edge_scale, node_scale, order, mp, channels, grad_src);
    }
    st = launch_check("segment_sum_grad_src_rows_kernel");
    if (st) return st;
  } else if (n_edges > 0) {
    // Unaligned or narrow rows: one element per thread, node from dst.
    const int64_t total = n_edges * channels;
    const DeviceInfo& dev = current_device_info();
    int64_t blocks = (total + kBlock - 1) / kBlock;
    const int64_t cap = static_cast<int64_t>(dev.sm_count) * 16;
    if (blocks > cap) blocks = cap;
    segment_sum_grad_src_kernel<1><<<static_cast<unsigned>(blocks), kBlock, 0, s>>>(
        grad_out, edge_scale, node_scale, dst, grad_src, n_edges, channels);
    st = launch_check("segment_sum_grad_src_kernel");
    if (st) return st;
  }
  if (grad_node_scale == nullptr || n_nodes == 0) return BYSJ_OK;
  const DeviceInfo& dev = current_device_info();
  const int64_t resident = static_cast<int64_t>(dev.sm_count) * 8 *
                           kWarpsPerBlock;
  PartitionPlan plan = plan_partitions(n_edges, n_nodes, resident, 16);
  Carver carve(workspace);
  float* slots = carve.take<float>(static_cast<size_t>(plan.parts) * 2);
  int* tickets = carve.take<int>(static_cast<size_t>(plan.parts));
  if (workspace == nullptr || workspace_bytes < carve.need)
    return fail(BYSJ_ERR_WORKSPACE,
                "segment sum backward: workspace of %zu bytes needed, %zu "
                "given",
                carve.need, workspace_bytes);
  st = cuda_check(cudaMemsetAsync(tickets, 0, sizeof(int) * plan.parts, s),
                  "segment sum backward: ticket reset");
  if (st) return st;
  NodeScaleGradArgs a;
  a.src = src;
  a.channels = channels;
  a.grad_out = grad_out;
  a.edge_scale = edge_scale;
  a.order = order;
  a.grad_node_scale = grad_node_scale;
  a.mp = MergePath{offsets, n_nodes, n_edges, plan.ipc, plan.parts};
  a.ss = SplitSlots{slots, tickets, 1, 1};
  const bool bf16 = src_dtype == BYSJ_BF16;
  const bool vec = bf16 ? (channels % 8 == 0 && aligned16(src))
                        : (channels % 4 == 0 && aligned16(src));
  const bool vec_g = vec && aligned16(grad_out);
  if (bf16) {
    if (vec_g)
      segment_sum_grad_scale_kernel<__nv_bfloat16, 8, true><<<plan.blocks, kBlock, 0, s>>>(a);
    else if (vec)
      segment_sum_grad_scale_kernel<__nv_bfloat16, 8><<<plan.blocks, kBlock, 0, s>>>(a);
    else
      segment_sum_grad_scale_kernel<__nv_bfloat16, 1><<<plan.blocks, kBlock, 0, s>>>(a);
  } else {
    if (vec_g)
      segment_sum_grad_scale_kernel<float, 4, true><<<plan.blocks, kBlock, 0, s>>>(a);
    else if (vec)
      segment_sum_grad_scale_kernel<float, 4><<<plan.blocks, kBlock, 0, s>>>(a);
    else
      segment_sum_grad_scale_kernel<float, 1><<<plan.blocks, kBlock, 0, s>>>(a);
  }
  return launch_check("segment_sum_grad_scale_kernel");
}

}  // extern "C"
