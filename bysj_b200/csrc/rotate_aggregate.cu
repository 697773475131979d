// Fused rotate-back aggregation (the flash seam of DeepMD's SO(2) block) for
// sm_100a.
//
//   out[n, l*l + b, c] = sum_{dst(e)=n} alpha[e, c / dh] * rescale[e] *
//                        sum_a D_{e,l}[a, b] * x_local[e, l*l + a, c]
//
// x_local [E, (L+1)^2, C] holds each edge's message in the edge's local frame;
// rotation [E, sum_l (2l+1)^2] packs the block-diagonal rotation of each edge
// per degree (block l row-major, x_local = D x_global, so rotating back is the
// transpose).  The argument list is the one the reference records for
// DeepMD's _flash_atten_fn (docs/deepmd-fused-dispatch.md:127-128), where the
// rotated messages would otherwise be materialised, weighted and scattered
// with index_add_.  Here the rotated message never reaches HBM: one pass reads
// each edge's message row (16 x 64 fp32 = 4 KB at L = 3, C = 64), its 84
// rotation coefficients and its attention row, and accumulates the rotated,
// weighted row in registers per destination segment.
//
// Work decomposition: the merge path over (edge slots, segment ends) shared
// by the segmented kernels, one partition per warp; a segment cut by a
// partition boundary publishes its partial and the last piece to arrive sums
// the pieces in partition order (integer ticket, no spin), so results are
// bit-identical run to run.  Lane layout: lane L owns the VEC consecutive
// channels of group L (+ 32 per column tile) for every component; the edge's
// rotation coefficients are staged in the warp's shared memory and read by
// broadcast, so each lane performs sum_l (2l+1)^2 * VEC fused multiply-adds
// per edge out of registers.  The rotation is not a GEMM worth a tensor core
// (a 16 x 16 block-diagonal with 84 non-zeros per edge, against 4 KB of
// message bytes): the kernel is HBM-bound.
#include "launch.cuh"

namespace bysj {
namespace {

constexpr int kRotMaxL = 3;

struct RotArgs {
  const float* x;        // [E, S, C]
  const float* rot;      // [E, R]
  const float* rescale;  // [E] or NULL
  const float* alpha;    // [E, H]
  const int64_t* order;  // [E] slot -> edge, or NULL
  float* out;            // [N, S, C]
  int heads;
  int64_t channels;      // C
  int64_t dh;            // C / H
  int64_t groups;        // C / VEC
  MergePath mp;
  SplitSlots ss;         // slots of S * C floats
};

template <int L>
struct RotShape {
  static constexpr int S = (L + 1) * (L + 1);
  static constexpr int R = (L + 1) * (2 * L + 1) * (2 * L + 3) / 3;  // sum_l (2l+1)^2
  static __device__ __forceinline__ constexpr int off(int l) {
    return l * (2 * l - 1) * (2 * l + 1) / 3;
  }
};

template <int VEC>
__device__ __forceinline__ void load_vec(const float* p, float (&v)[VEC]) {
  if constexpr (VEC == 4) {
    const float4 t = ld_stream_f4(p);
    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
  } else if constexpr (VEC == 2) {
    const float2 t = __ldg(reinterpret_cast<const float2*>(p));
    v[0] = t.x; v[1] = t.y;
  } else {
    v[0] = __ldg(p);
  }
}

template <int VEC>
__device__ __forceinline__ void store_vec(float* p, const float (&v)[VEC]) {
  if constexpr (VEC == 4) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  } else if constexpr (VEC == 2) {
    *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
  } else {
    p[0] = v[0];
  }
}

// acc[l*l + b][v] += sum_a d[off(l) + a*m + b] * w * x[l*l + a][v], every
// degree (x is scaled by w in place: it is dead afterwards).
template <int L, int VEC>
__device__ __forceinline__ void rot_accumulate(const float* __restrict__ d,
                                               float (&x)[RotShape<L>::S][VEC], float w,
                                               float (&acc)[RotShape<L>::S][VEC]) {
  constexpr int S = RotShape<L>::S;
#pragma unroll
  for (int j = 0; j < S; ++j)
#pragma unroll
    for (int v = 0; v < VEC; ++v) x[j][v] *= w;
#pragma unroll
  for (int l = 0; l <= L; ++l) {
    const int m = 2 * l + 1;
    const int base = l * l;
    const int off = RotShape<L>::off(l);
#pragma unroll
    for (int aa = 0; aa < m; ++aa)
#pragma unroll
      for (int b = 0; b < m; ++b) {
        const float dd = d[off + aa * m + b];
#pragma unroll
        for (int v = 0; v < VEC; ++v)
          acc[base + b][v] = fmaf(dd, x[base + aa][v], acc[base + b][v]);
      }
  }
}

// Edges whose message rows are in flight together: two while two rows of
// S * VEC floats fit beside the accumulators, else one (a 4 KB row per warp
// is then in flight, 16 warps per SM: enough bytes to cover the latency).
template <int L, int VEC>
struct RotStep {
  static constexpr int U = (RotShape<L>::S * VEC >= 32) ? 1 : 2;
};

template <int L, int VEC>
__global__ void __launch_bounds__(kBlock, 2) rotate_aggregate_kernel(RotArgs a) {
  constexpr int S = RotShape<L>::S;
  constexpr int R = RotShape<L>::R;
  constexpr int U = RotStep<L, VEC>::U;
  constexpr int kCoefLoads = (2 * R + kWarp - 1) / kWarp;
  __shared__ float s_rot[kWarpsPerBlock][2 * R];
  const int64_t p = global_warp();
  if (p >= a.mp.parts) return;
  float* srot = s_rot[threadIdx.x >> 5];
  const int lane = lane_id();
  const int tile = blockIdx.y;
  const int64_t gidx = static_cast<int64_t>(tile) * kWarp + lane;  // channel group
  const bool active = gidx < a.groups;
  const int64_t C = a.channels;
  const int64_t c0 = (active ? gidx : 0) * VEC;
  const int head = static_cast<int>(c0 / a.dh);
  const float* x = a.x + c0;

  SegCursor cur(a.mp, part_range(a.mp, p));
  while (cur.next()) {
    float acc[S][VEC];
#pragma unroll
    for (int j = 0; j < S; ++j)
#pragma unroll
      for (int v = 0; v < VEC; ++v) acc[j][v] = 0.0f;
    for (int64_t s = cur.lo; s < cur.hi; s += U) {
      const bool two = U == 2 && s + 1 < cur.hi;  // warp-uniform
      const int64_t e0 = a.order ? __ldg(a.order + s) : s;
      const int64_t e1 = two ? (a.order ? __ldg(a.order + s + 1) : s + 1) : e0;
      float x0[S][VEC], x1[S][VEC];
#pragma unroll
      for (int j = 0; j < S; ++j) load_vec<VEC>(x + (e0 * S + j) * C, x0[j]);
      if (two) {
#pragma unroll
        for (int j = 0; j < S; ++j) load_vec<VEC>(x + (e1 * S + j) * C, x1[j]);
      }
      float w0 = __ldg(a.alpha + e0 * a.heads + head);
      float w1 = two ? __ldg(a.alpha + e1 * a.heads + head) : 0.0f;
      if (a.rescale) {
        w0 *= __ldg(a.rescale + e0);
        if (two) w1 *= __ldg(a.rescale + e1);
      }
      __syncwarp();  // the previous step's coefficients have been read
#pragma unroll
      for (int t = 0; t < kCoefLoads; ++t) {
        const int idx = lane + t * kWarp;
        if (idx < R) srot[idx] = __ldg(a.rot + e0 * R + idx);
        else if (idx < 2 * R && two) srot[idx] = __ldg(a.rot + e1 * R + (idx - R));
      }
      __syncwarp();
      rot_accumulate<L, VEC>(srot, x0, w0, acc);
      if (two) rot_accumulate<L, VEC>(srot + R, x1, w1, acc);
    }

    const int64_t n = cur.node;
    if (cur.kind == kWhole) {
      if (active) {
#pragma unroll
        for (int j = 0; j < S; ++j) store_vec<VEC>(a.out + (n * S + j) * C + c0, acc[j]);
      }
      continue;
    }
    // Split segment: publish the partial; the last piece sums them in order.
    float* mine = a.ss.slot(p, cur.kind);
    if (active) {
#pragma unroll
      for (int j = 0; j < S; ++j)
#pragma unroll
        for (int v = 0; v < VEC; ++v) __stcg(mine + j * C + c0 + v, acc[j][v]);
    }
    const int64_t first = a.mp.part_of_first_edge(n);
    const int64_t last = a.mp.part_of_end(n);
    if (!arrive_last(a.ss, first, last, tile)) continue;
    if (!active) continue;
#pragma unroll
    for (int j = 0; j < S; ++j) {
      float sum[VEC];
#pragma unroll
      for (int v = 0; v < VEC; ++v) sum[v] = 0.0f;
      for (int64_t q = first; q <= last; ++q) {
        const float* sq = a.ss.slot(q, q == last ? kHead : kTail) + j * C + c0;
#pragma unroll
        for (int v = 0; v < VEC; ++v) sum[v] += __ldcg(sq + v);
      }
      store_vec<VEC>(a.out + (n * S + j) * C + c0, sum);
    }
  }
}

using RotKernel = void (*)(RotArgs);

template <int L>
RotKernel rot_kernel_for(int vec) {
  if constexpr (L < 3) {  // rot_vec never picks 4 channels per lane at lmax 3
    if (vec == 4) return rotate_aggregate_kernel<L, 4>;
  }
  if (vec == 2) return rotate_aggregate_kernel<L, 2>;
  return rotate_aggregate_kernel<L, 1>;
}

RotKernel rot_kernel(int lmax, int vec) {
  switch (lmax) {
    case 0: return rot_kernel_for<0>(vec);
    case 1: return rot_kernel_for<1>(vec);
    case 2: return rot_kernel_for<2>(vec);
    default: return rot_kernel_for<3>(vec);
  }
}

// Channels per lane: the widest of 4, 2, 1 that divides the channels and the
// head width, keeps at least one full warp of channel groups when the channels
// allow it, fits the registers (no 4 at lmax 3) and (for 2 and 4) finds
// x_local and out aligned.
int rot_vec(int lmax, int64_t channels, int64_t dh, bool aligned16_ok, bool aligned8_ok) {
  for (int v : {4, 2}) {
    if (v == 4 && lmax >= 3) continue;  // 16 x 4 accumulators and a row exceed the registers
    if (channels % v || dh % v) continue;
    if (channels / v < kWarp && channels >= kWarp) continue;
    if (v == 4 && !aligned16_ok) continue;
    if (v == 2 && !aligned8_ok) continue;
    return v;
  }
  return 1;
}

struct RotLayout {
  RotKernel kernel = nullptr;
  int vec = 1;
  int64_t groups = 0, tiles = 1;
  PartitionPlan plan;
  size_t bytes = 0;
};

RotLayout rot_layout(int lmax, int vec, int64_t n_edges, int64_t n_nodes, int64_t channels,
                     void* ws, SplitSlots* ss) {
  RotLayout L;
  L.vec = vec;
  L.kernel = rot_kernel(lmax, vec);
  L.groups = channels / vec;
  L.tiles = (L.groups + kWarp - 1) / kWarp;
  const int64_t comps = static_cast<int64_t>(lmax + 1) * (lmax + 1);
  const DeviceInfo& dev = current_device_info();
  int64_t warps = static_cast<int64_t>(dev.sm_count) *
                  resident_blocks(reinterpret_cast<const void*>(L.kernel)) * kWarpsPerBlock /
                  L.tiles;
  if (warps < 1) warps = 1;
  L.plan = plan_partitions(n_edges, n_nodes, warps, 16);
  const int64_t stride = comps * channels;
  Carver carve(ws);
  float* slots = carve.take<float>(static_cast<size_t>(L.plan.parts) * 2 * stride);
  int* tickets = carve.take<int>(static_cast<size_t>(L.plan.parts) * L.tiles);
  L.bytes = carve.need;
  if (ss) *ss = SplitSlots{slots, tickets, stride, static_cast<int>(L.tiles)};
  return L;
}

int rot_check(int64_t n_edges, int64_t n_nodes, int64_t lmax, int64_t heads,
              int64_t channels) {
  if (n_edges < 0 || n_nodes < 0 || channels <= 0 || heads <= 0)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "rotate-back aggregate: invalid sizes");
  if (lmax < 0 || lmax > kRotMaxL)
    return fail(BYSJ_ERR_UNSUPPORTED, "rotate-back aggregate: lmax %lld outside [0, %d]",
                (long long)lmax, kRotMaxL);
  if (channels % heads)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "rotate-back aggregate: heads must divide channels");
  return BYSJ_OK;
}

}  // namespace
}  // namespace bysj

using namespace bysj;

extern "C" {

size_t bysj_rotate_back_aggregate_workspace_size(int64_t n_edges, int64_t n_nodes,
                                                 int64_t lmax, int64_t heads,
                                                 int64_t channels) {
  if (n_edges < 0 || n_nodes <= 0 || lmax < 0 || lmax > kRotMaxL || heads <= 0 ||
      channels <= 0 || channels % heads)
    return 0;
  size_t most = 0;
  for (int v : {4, 2, 1}) {
    if (channels % v || (channels / heads) % v || (v == 4 && lmax >= 3)) continue;
    const size_t b = rot_layout(static_cast<int>(lmax), v, n_edges, n_nodes, channels, nullptr,
                                nullptr).bytes;
    if (b > most) most = b;
  }
  return most;
}

int bysj_rotate_back_aggregate(const float* x_local, const float* rotation,
                               const float* rescale, const float* alpha,
                               const int64_t* offsets, const int64_t* order, int64_t n_edges,
                               int64_t n_nodes, int64_t lmax, int64_t heads, int64_t channels,
                               float* out, void* workspace, size_t workspace_bytes,
                               void* stream) {
  clear_error();
  int st = rot_check(n_edges, n_nodes, lmax, heads, channels);
  if (st) return st;
  if (n_nodes == 0) return BYSJ_OK;
  if (offsets == nullptr || out == nullptr ||
      (n_edges > 0 && (x_local == nullptr || rotation == nullptr || alpha == nullptr)))
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "rotate-back aggregate: NULL pointer");
  const int64_t dh = channels / heads;
  const int vec = rot_vec(static_cast<int>(lmax), channels, dh,
                          aligned16(x_local) && aligned16(out),
                          aligned8(x_local) && aligned8(out));
  SplitSlots ss{};
  RotLayout L = rot_layout(static_cast<int>(lmax), vec, n_edges, n_nodes, channels, workspace,
                           &ss);
  if (workspace == nullptr || workspace_bytes < L.bytes)
    return fail(BYSJ_ERR_WORKSPACE,
                "rotate-back aggregate: workspace of %zu bytes needed, %zu given", L.bytes,
                workspace_bytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  st = cuda_check(cudaMemsetAsync(ss.tickets, 0, sizeof(int) * L.plan.parts * L.tiles, s),
                  "rotate-back aggregate: ticket reset");
  if (st) return st;
  RotArgs a;
  a.x = x_local;
  a.rot = rotation;
  a.rescale = rescale;
  a.alpha = alpha;
  a.order = order;
  a.out = out;
  a.heads = static_cast<int>(heads);
  a.channels = channels;
  a.dh = dh;
  a.groups = L.groups;
  a.mp = MergePath{offsets, n_nodes, n_edges, L.plan.ipc, L.plan.parts};
  a.ss = ss;
  dim3 grid(L.plan.blocks, static_cast<unsigned>(L.tiles));
  L.kernel<<<grid, kBlock, 0, s>>>(a);
  return launch_check("rotate_aggregate_kernel");
}

}  // extern "C"
