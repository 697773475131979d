// Fused gated segment softmax + weighted segment sum for sm_100a.
//
//   alpha[e, h]     = softmax over the edges of seg(n) of l[e, h]
//                     (l = logit + 2 ln env, env <= 0 excluded, optional
//                      per-node null logit, as in the reference's
//                      csrc/segment_softmax.cpp:16-23)
//   out[n, h, s, k] = sum_e alpha[e, h] * value[e, s, h*dh + k]   (dh = C / H)
//
// The reference composes this from segment_softmax (writes alpha to HBM)
// and segment_sum (reads it back with the values).  Here one warp owns one
// merge-path partition; for each segment it first reduces the tiny logit
// rows (H floats per edge, read from L2/L1) to the per-head maximum and
// denominator, then streams the value rows exactly once with 16-byte loads,
// weighting each by alpha recomputed in registers.  alpha never reaches HBM.
// Segments cut by a partition boundary are combined like split-K attention:
// each piece keeps its local maximum m_q, denominator d_q and unnormalised
// sum; the last piece to finish rescales them by exp(m_q - m) in partition
// order, so results are deterministic.
#include <mutex>
#include <utility>

#include "launch.cuh"

namespace bysj {
namespace {

constexpr int kMaxHeads = 32;

struct AttnArgs {
  const float* logit;       // [E, H]
  const void* value;        // [E, S, C]
  const float* env;         // [E] or NULL
  const float* null_logit;  // [N, H] or NULL
  const int64_t* order;
  float* out;               // [N, H, S, dh]
  int heads;
  int hp;                   // heads rounded up to a power of two
  int64_t comps;            // S
  int64_t channels;         // C
  int64_t dh;               // C / H
  int64_t row;              // S * C elements per edge
  int64_t lv;               // row / VEC
  int64_t stats_off;        // offset of (m, d) inside a split slot
  MergePath mp;
  SplitSlots ss;
};

template <typename T, int VEC, int NV>
struct AttnShape {
  static constexpr int TV = kWarp * NV;
  static constexpr int U = (NV * VEC >= 64)   ? 1
                           : (NV * VEC >= 16) ? 2
                           : (8 / NV < 1 ? 1 : 8 / NV);
  static constexpr int kMinBlocks = (NV * VEC >= 32) ? 2 : 3;
  // 2 KB rows with 16-byte vectors (bf16 [16, 64], fp32 [16, 32]): the rows
  // of the edges `kAhead` slots ahead (the next loop step) are prefetched
  // into L2 by one bulk request each, so that two steps of row loads are in
  // flight without more registers (C3 bf16: 856 -> 799 us; fp32 at C = 32:
  // 801 -> 769 us).  4 KB fp32 rows already keep enough bytes in flight;
  // prefetching them only competes for L2 there.
  static constexpr int kAhead = (VEC * sizeof(T) == 16 && kWarp * NV * VEC * sizeof(T) == 2048) ? 2 : 0;
};

// Per-head maximum and denominator over slots [lo, hi).  Whole segments
// include the null logit and return the reciprocal of the denominator;
// pieces of a split segment return their local (m, d) and inv = 1.
// Results land in the warp's shared-memory stats arrays.
__device__ __forceinline__ void head_stats(const AttnArgs& a, int64_t node,
                                           int64_t lo, int64_t hi,
                                           bool whole, float* sm_m,
                                           float* sm_inv, float* sm_d) {
  const int lane = lane_id();
  const int h = lane % a.hp;
  const int gs = lane / a.hp;
  const int groups = kWarp / a.hp;
  const bool valid = h < a.heads;
  float mx = -INFINITY;
  if (valid) {
    for (int64_t s = lo + gs; s < hi; s += groups) {
      const int64_t e = a.order ? __ldg(a.order + s) : s;
      mx = fmaxf(mx, gated_logit(__ldg(a.logit + e * a.heads + h), a.env, e));
    }
  }
  mx = xor_max(mx, a.hp);
  float nl = -INFINITY;
  if (whole && valid && a.null_logit) nl = __ldg(a.null_logit + node * a.heads + h);
  const float m = fmaxf(mx, nl);
  float d = 0.0f;
  if (valid) {
    for (int64_t s = lo + gs; s < hi; s += groups) {
      const int64_t e = a.order ? __ldg(a.order + s) : s;
      d += shifted_exp(gated_logit(__ldg(a.logit + e * a.heads + h), a.env, e), m);
    }
  }
  d = xor_sum(d, a.hp);
  float inv = 1.0f;
  if (whole) {
    d += shifted_exp(nl, m);
    inv = d > 0.0f ? 1.0f / d : 0.0f;
  }
  if (gs == 0 && valid) {
    sm_m[h] = m;
    sm_inv[h] = inv;
    sm_d[h] = d;
  }
  __syncwarp();
}

template <typename T, int VEC, int NV, bool kHeadConst>
__global__ void __launch_bounds__(kBlock, AttnShape<T, VEC, NV>::kMinBlocks)
    segment_attention_kernel(AttnArgs a) {
  using S = AttnShape<T, VEC, NV>;
  __shared__ float s_stats[kWarpsPerBlock][3][kMaxHeads];
  const int64_t p = global_warp();
  if (p >= a.mp.parts) return;
  const int wib = threadIdx.x >> 5;
  float* sm_m = s_stats[wib][0];
  float* sm_inv = s_stats[wib][1];
  float* sm_d = s_stats[wib][2];
  const int tile = blockIdx.y;
  const int lane = lane_id();
  const int64_t jt = static_cast<int64_t>(tile) * S::TV;
  const T* value = static_cast<const T*>(a.value);

  // Per-vector head and output offset inside the node's [H, S, dh] block.
  int head[NV];
  int64_t jl[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int64_t j = jt + lane + k * kWarp;
    jl[k] = j < a.lv ? j : a.lv - 1;
    const int64_t c = (jl[k] * VEC) % a.channels;
    head[k] = static_cast<int>(c / a.dh);
  }

  SegCursor cur(a.mp, part_range(a.mp, p));
  while (cur.next()) {
    const int64_t n = cur.node;
    const bool whole = cur.kind == kWhole;
    head_stats(a, n, cur.lo, cur.hi, whole, sm_m, sm_inv, sm_d);
    float mk[NV], ik[NV];
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      mk[k] = sm_m[kHeadConst ? head[0] : head[k]];
      ik[k] = sm_inv[kHeadConst ? head[0] : head[k]];
    }
    __syncwarp();  // stats read before the next segment overwrites them

    float acc[NV][VEC];
#pragma unroll
    for (int k = 0; k < NV; ++k)
#pragma unroll
      for (int i = 0; i < VEC; ++i) acc[k][i] = 0.0f;

    int64_t s = cur.lo;
    for (; s + S::U <= cur.hi; s += S::U) {
      if constexpr (S::kAhead > 0) {
        const int64_t t = s + S::kAhead + lane;
        if (lane < S::U && t < cur.r.b1)
          prefetch_l2_bulk(value + (a.order ? __ldg(a.order + t) : t) * a.row,
                           static_cast<uint32_t>(a.row * sizeof(T)));
      }
      const T* rowp[S::U];
      float w[S::U][kHeadConst ? 1 : NV];
#pragma unroll
      for (int u = 0; u < S::U; ++u) {
        const int64_t e = a.order ? __ldg(a.order + s + u) : s + u;
        rowp[u] = value + e * a.row;
        if constexpr (kHeadConst) {
          const float l = gated_logit(__ldg(a.logit + e * a.heads + head[0]), a.env, e);
          w[u][0] = shifted_exp(l, mk[0]) * ik[0];
        } else {
#pragma unroll
          for (int k = 0; k < NV; ++k) {
            const float l = gated_logit(__ldg(a.logit + e * a.heads + head[k]), a.env, e);
            w[u][k] = shifted_exp(l, mk[k]) * ik[k];
          }
        }
      }
      RowVec<T, VEC> buf[S::U][NV];
#pragma unroll
      for (int u = 0; u < S::U; ++u)
#pragma unroll
        for (int k = 0; k < NV; ++k) buf[u][k].load(rowp[u], jl[k]);
#pragma unroll
      for (int u = 0; u < S::U; ++u)
#pragma unroll
        for (int k = 0; k < NV; ++k)
#pragma unroll
          for (int i = 0; i < VEC; ++i)
            acc[k][i] = fmaf(w[u][kHeadConst ? 0 : k], buf[u][k].get(i), acc[k][i]);
    }
    for (; s < cur.hi; ++s) {
      if constexpr (S::kAhead > 0) {
        const int64_t t = s + S::kAhead;
        if (lane == 0 && t < cur.r.b1)
          prefetch_l2_bulk(value + (a.order ? __ldg(a.order + t) : t) * a.row,
                           static_cast<uint32_t>(a.row * sizeof(T)));
      }
      const int64_t e = a.order ? __ldg(a.order + s) : s;
      const T* rowp = value + e * a.row;
      RowVec<T, VEC> buf[NV];
#pragma unroll
      for (int k = 0; k < NV; ++k) buf[k].load(rowp, jl[k]);
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const int hh = kHeadConst ? head[0] : head[k];
        const float l = gated_logit(__ldg(a.logit + e * a.heads + hh), a.env, e);
        const float w = shifted_exp(l, mk[k]) * ik[k];
#pragma unroll
        for (int i = 0; i < VEC; ++i) acc[k][i] = fmaf(w, buf[k].get(i), acc[k][i]);
      }
    }

    if (whole) {
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const int64_t j = jt + lane + k * kWarp;
        if (j < a.lv) {
          const int64_t x = j * VEC;
          const int64_t i = x / a.channels;
          const int64_t kk = (x % a.channels) % a.dh;
          store_f32<VEC>(a.out + n * a.row + (head[k] * a.comps + i) * a.dh + kk,
                         acc[k]);
        }
      }
      continue;
    }

    // Split segment: publish (unnormalised sum, local m, local d).
    float* mine = a.ss.slot(p, cur.kind);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int64_t j = jt + lane + k * kWarp;
      if (j < a.lv) store_cg<VEC>(mine + j * VEC, acc[k]);
    }
    if (lane < a.heads) {
      __stcg(mine + a.stats_off + lane, sm_m[lane]);
      __stcg(mine + a.stats_off + kMaxHeads + lane, sm_d[lane]);
    }
    const int64_t first = a.mp.part_of_first_edge(n);
    const int64_t last = a.mp.part_of_end(n);
    __syncwarp();
    if (!arrive_last(a.ss, first, last, tile)) continue;

    // Final per-head maximum and reciprocal denominator.
    if (lane < a.heads) {
      const float nl = a.null_logit ? __ldg(a.null_logit + n * a.heads + lane)
                                    : -INFINITY;
      float m = nl;
      for (int64_t q = first; q <= last; ++q)
        m = fmaxf(m, __ldcg(a.ss.slot(q, q == last ? kHead : kTail) +
                            a.stats_off + lane));
      float d = shifted_exp(nl, m);
      for (int64_t q = first; q <= last; ++q) {
        const float* sq = a.ss.slot(q, q == last ? kHead : kTail) + a.stats_off;
        d += shifted_exp(__ldcg(sq + lane), m) * __ldcg(sq + kMaxHeads + lane);
      }
      sm_m[lane] = m;
      sm_inv[lane] = d > 0.0f ? 1.0f / d : 0.0f;
    }
    __syncwarp();
    for (int64_t jj = lane; jj < S::TV; jj += kWarp) {
      const int64_t j = jt + jj;
      if (j >= a.lv) continue;
      const int64_t x = j * VEC;
      const int hh = static_cast<int>((x % a.channels) / a.dh);
      const float m = sm_m[hh];
      float sum[VEC];
#pragma unroll
      for (int i = 0; i < VEC; ++i) sum[i] = 0.0f;
      for (int64_t q = first; q <= last; ++q) {
        const float* sq = a.ss.slot(q, q == last ? kHead : kTail);
        const float scale = shifted_exp(__ldcg(sq + a.stats_off + hh), m);
        float part[VEC];
        load_cg<VEC>(sq + x, part);
#pragma unroll
        for (int i = 0; i < VEC; ++i) sum[i] = fmaf(scale, part[i], sum[i]);
      }
      const float inv = sm_inv[hh];
#pragma unroll
      for (int i = 0; i < VEC; ++i) sum[i] *= inv;
      const int64_t i = x / a.channels;
      const int64_t kk = (x % a.channels) % a.dh;
      store_f32<VEC>(a.out + n * a.row + (hh * a.comps + i) * a.dh + kk, sum);
    }
    __syncwarp();
  }
}

using AttnKernel = void (*)(AttnArgs);

struct AttnConfig {
  AttnKernel kernel = nullptr;
  int vec = 1, nv = 1;
  int64_t lv = 0, tv = 0, tiles = 1;
};

template <typename T, int VEC, bool kHC>
AttnConfig attn_pick(int64_t lv) {
  AttnConfig c;
  c.vec = VEC;
  c.lv = lv;
  if (lv > 128) { c.kernel = segment_attention_kernel<T, VEC, 8, kHC>; c.nv = 8; }
  else if (lv > 64) { c.kernel = segment_attention_kernel<T, VEC, 4, kHC>; c.nv = 4; }
  else if (lv > 32) { c.kernel = segment_attention_kernel<T, VEC, 2, kHC>; c.nv = 2; }
  else { c.kernel = segment_attention_kernel<T, VEC, 1, kHC>; c.nv = 1; }
  c.tv = static_cast<int64_t>(kWarp) * c.nv;
  c.tiles = (lv + c.tv - 1) / c.tv;
  return c;
}

template <typename T, int VEC>
AttnConfig attn_pick_hc(int64_t lv, bool head_const) {
  return head_const ? attn_pick<T, VEC, true>(lv) : attn_pick<T, VEC, false>(lv);
}

AttnConfig attn_config(bool vec_ok, int dtype, int64_t channels, int64_t dh,
                       int64_t row) {
  if (dtype == BYSJ_BF16) {
    if (vec_ok && dh % 8 == 0)
      return attn_pick_hc<__nv_bfloat16, 8>(row / 8, (kWarp * 8) % channels == 0);
    return attn_pick_hc<__nv_bfloat16, 1>(row, kWarp % channels == 0);
  }
  if (vec_ok && dh % 4 == 0)
    return attn_pick_hc<float, 4>(row / 4, (kWarp * 4) % channels == 0);
  return attn_pick_hc<float, 1>(row, kWarp % channels == 0);
}

struct AttnLayout {
  AttnConfig cfg;
  PartitionPlan plan;
  int64_t stride = 0, stats_off = 0;
  size_t bytes = 0;
};

AttnLayout attn_layout(bool vec_ok, int dtype, int64_t n_edges,
                       int64_t n_nodes, int64_t heads, int64_t comps,
                       int64_t channels, void* ws, SplitSlots* ss) {
  AttnLayout L;
  const int64_t row = comps * channels;
  L.cfg = attn_config(vec_ok, dtype, channels, channels / heads, row);
  const DeviceInfo& dev = current_device_info();
  const int64_t resident =
      static_cast<int64_t>(dev.sm_count) *
      resident_blocks(reinterpret_cast<const void*>(L.cfg.kernel)) *
      kWarpsPerBlock;
  int64_t warps = resident / L.cfg.tiles;
  if (warps < 1) warps = 1;
  L.plan = plan_partitions(n_edges, n_nodes, warps, 16);
  L.stats_off = (row + 7) / 8 * 8;
  L.stride = L.stats_off + 2 * kMaxHeads;
  Carver carve(ws);
  float* slots =
      carve.take<float>(static_cast<size_t>(L.plan.parts) * 2 * L.stride);
  int* tickets =
      carve.take<int>(static_cast<size_t>(L.plan.parts) * L.cfg.tiles);
  L.bytes = carve.need;
  if (ss) *ss = SplitSlots{slots, tickets, L.stride, static_cast<int>(L.cfg.tiles)};
  return L;
}

}  // namespace
}  // namespace bysj

using namespace bysj;

extern "C" {

size_t bysj_segment_attention_workspace_size(int64_t n_edges, int64_t n_nodes,
                                             int64_t heads,
                                             int64_t components,
                                             int64_t channels,
                                             int value_dtype) {
  if (n_edges < 0 || n_nodes <= 0 || heads <= 0 || heads > kMaxHeads ||
      components <= 0 || channels <= 0 || channels % heads != 0)
    return 0;
  const size_t a = attn_layout(true, value_dtype, n_edges, n_nodes, heads,
                               components, channels, nullptr, nullptr).bytes;
  const size_t b = attn_layout(false, value_dtype, n_edges, n_nodes, heads,
                               components, channels, nullptr, nullptr).bytes;
  return a > b ? a : b;
}

int bysj_segment_attention_forward(const float* logit, const void* value,
                                   int value_dtype, const float* env,
                                   const float* null_logit,
                                   const int64_t* offsets,
                                   const int64_t* order, int64_t n_edges,
                                   int64_t n_nodes, int64_t heads,
                                   int64_t components, int64_t channels,
                                   float* out, void* workspace,
                                   size_t workspace_bytes, void* stream) {
  clear_error();
  if (n_edges < 0 || n_nodes < 0 || heads <= 0 || components <= 0 ||
      channels <= 0)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "segment attention: invalid sizes");
  if (heads > kMaxHeads)
    return fail(BYSJ_ERR_UNSUPPORTED,
                "segment attention: at most %d heads are supported, got %lld",
                kMaxHeads, (long long)heads);
  if (channels % heads != 0)
    return fail(BYSJ_ERR_INVALID_ARGUMENT,
                "segment attention: heads (%lld) must divide channels (%lld)",
                (long long)heads, (long long)channels);
  if (value_dtype != BYSJ_F32 && value_dtype != BYSJ_BF16)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "segment attention: unknown dtype");
  if (n_nodes == 0) return BYSJ_OK;
  if (offsets == nullptr || out == nullptr ||
      (n_edges > 0 && (logit == nullptr || value == nullptr)))
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "segment attention: NULL pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool vec_ok = aligned16(value) && aligned16(out);
  SplitSlots ss{};
  AttnLayout L = attn_layout(vec_ok, value_dtype, n_edges, n_nodes, heads,
                             components, channels, workspace, &ss);
  if (workspace == nullptr || workspace_bytes < L.bytes)
    return fail(BYSJ_ERR_WORKSPACE,
                "segment attention: workspace of %zu bytes needed, %zu given",
                L.bytes, workspace_bytes);
  int st = cuda_check(
      cudaMemsetAsync(ss.tickets, 0, sizeof(int) * L.plan.parts * L.cfg.tiles, s),
      "segment attention: ticket reset");
  if (st) return st;
  AttnArgs a;
  a.logit = logit;
  a.value = value;
  a.env = env;
  a.null_logit = null_logit;
  a.order = order;
  a.out = out;
  a.heads = static_cast<int>(heads);
  a.hp = static_cast<int>(next_pow2(heads));
  a.comps = components;
  a.channels = channels;
  a.dh = channels / heads;
  a.row = components * channels;
  a.lv = L.cfg.lv;
  a.stats_off = L.stats_off;
  a.mp = MergePath{offsets, n_nodes, n_edges, L.plan.ipc, L.plan.parts};
  a.ss = ss;
  dim3 grid(L.plan.blocks, static_cast<unsigned>(L.cfg.tiles));
  L.cfg.kernel<<<grid, kBlock, 0, s>>>(a);
  return launch_check("segment_attention_kernel");
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free entry point.
//
// Some callers cannot hand this library a workspace: a plugin hook that only
// receives input/output pointers and a stream (a molecular-dynamics engine's
// pair-style callback, a serving runtime that forbids allocation after its
// warm-up so its memory footprint stays fixed), or code on a hot path where
// cudaMalloc would synchronise the whole device.  For them the split-segment
// scratch of the fused attention lives in one file-scope device array of
// BYSJ_ATTENTION_NOALLOC_SCRATCH_BYTES (16 MiB), which every GPU that loads
// this library keeps until the process exits.
// ---------------------------------------------------------------------------

static __device__ __align__(256) unsigned char
    bysj_attention_noalloc_scratch[BYSJ_ATTENTION_NOALLOC_SCRATCH_BYTES];

namespace bysj {
namespace {

std::mutex g_noalloc_mutex;
struct NoallocSlot {
  unsigned long long context = 0;  // unique id of the context the address belongs to
  void* address = nullptr;
};
NoallocSlot g_noalloc_slot[64];

// Unique id of the calling thread's current CUDA context (0 if none or if the
// driver entry points are unavailable).  Context ids are never reused within a
// process, so an address cached under one stays valid exactly as long as that
// context: after cudaDeviceReset the runtime creates a new context on the
// next call, the library's module is loaded again and the array may move.
// The driver functions are looked up through the runtime, so the library needs
// no link-time dependency on the driver library.
unsigned long long current_context_id() {
  using GetCurrent = int (*)(void**);
  using GetId = int (*)(void*, unsigned long long*);
  static const std::pair<GetCurrent, GetId> fns = [] {
    void* cur = nullptr;
    void* id = nullptr;
    cudaDriverEntryPointQueryResult q1 = cudaDriverEntryPointSymbolNotFound;
    cudaDriverEntryPointQueryResult q2 = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &cur, 12000, cudaEnableDefault,
                                         &q1) != cudaSuccess ||
        q1 != cudaDriverEntryPointSuccess)
      cur = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &id, 12000, cudaEnableDefault, &q2) !=
            cudaSuccess ||
        q2 != cudaDriverEntryPointSuccess)
      id = nullptr;
    return std::make_pair(reinterpret_cast<GetCurrent>(cur), reinterpret_cast<GetId>(id));
  }();
  if (fns.first == nullptr || fns.second == nullptr) return 0;
  void* ctx = nullptr;
  if (fns.first(&ctx) != 0 || ctx == nullptr) return 0;
  unsigned long long id = 0;
  if (fns.second(ctx, &id) != 0) return 0;
  return id;
}

// Device address of the scratch array in the current device's context.  In
// host code the array's name is only a host-side handle, so the address is
// looked up (with the device current) once per device and context and cached.
int noalloc_scratch_address(void** address) {
  int device = 0;
  int st = cuda_check(cudaGetDevice(&device), "segment attention (no-alloc): current device");
  if (st) return st;
  if (device < 0 || device >= 64)
    return fail(BYSJ_ERR_UNSUPPORTED, "segment attention (no-alloc): device %d", device);
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  NoallocSlot& slot = g_noalloc_slot[device];
  const unsigned long long ctx = current_context_id();
  if (slot.address == nullptr || ctx == 0 || ctx != slot.context) {
    void* ptr = nullptr;
    st = cuda_check(cudaGetSymbolAddress(&ptr, bysj_attention_noalloc_scratch),
                    "segment attention (no-alloc): scratch address");
    if (st) return st;
    slot.address = ptr;
    slot.context = current_context_id();  // the lookup made the context current
  }
  *address = slot.address;
  return BYSJ_OK;
}

// Same tiling as attn_layout, with the partition count capped so that the
// split slots and tickets fit in the fixed scratch array.
int noalloc_layout(bool vec_ok, int dtype, int64_t n_edges, int64_t n_nodes,
                   int64_t heads, int64_t comps, int64_t channels, void* base,
                   AttnLayout* L, SplitSlots* ss) {
  const int64_t row = comps * channels;
  L->cfg = attn_config(vec_ok, dtype, channels, channels / heads, row);
  L->stats_off = (row + 7) / 8 * 8;
  L->stride = L->stats_off + 2 * kMaxHeads;
  const size_t slack = 2 * 256;  // alignment of the two carved regions
  const size_t per_part = 2 * sizeof(float) * static_cast<size_t>(L->stride) +
                          sizeof(int) * static_cast<size_t>(L->cfg.tiles);
  const size_t capacity = BYSJ_ATTENTION_NOALLOC_SCRATCH_BYTES;
  if (per_part + slack > capacity)
    return fail(BYSJ_ERR_TOO_LARGE,
                "segment attention (no-alloc): a value row of %lld elements needs %zu "
                "bytes of scratch per partition; the fixed scratch holds %zu bytes "
                "(use bysj_segment_attention_forward with a workspace)",
                (long long)row, per_part, capacity);
  const int64_t cap = static_cast<int64_t>((capacity - slack) / per_part);
  const DeviceInfo& dev = current_device_info();
  int64_t warps = static_cast<int64_t>(dev.sm_count) *
                  resident_blocks(reinterpret_cast<const void*>(L->cfg.kernel)) *
                  kWarpsPerBlock / L->cfg.tiles;
  if (warps > cap) warps = cap;
  if (warps < 1) warps = 1;
  L->plan = plan_partitions(n_edges, n_nodes, warps, 16);
  Carver carve(base);
  float* slots = carve.take<float>(static_cast<size_t>(L->plan.parts) * 2 * L->stride);
  int* tickets = carve.take<int>(static_cast<size_t>(L->plan.parts) * L->cfg.tiles);
  L->bytes = carve.need;
  if (L->bytes > capacity)
    return fail(BYSJ_ERR_TOO_LARGE, "segment attention (no-alloc): scratch plan overflow");
  *ss = SplitSlots{slots, tickets, L->stride, static_cast<int>(L->cfg.tiles)};
  return BYSJ_OK;
}

}  // namespace
}  // namespace bysj

extern "C" int bysj_segment_attention_forward_noalloc(
    const float* logit, const void* value, int value_dtype, const float* env,
    const float* null_logit, const int64_t* offsets, const int64_t* order, int64_t n_edges,
    int64_t n_nodes, int64_t heads, int64_t components, int64_t channels, float* out,
    void* stream) {
  clear_error();
  if (n_edges < 0 || n_nodes < 0 || heads <= 0 || components <= 0 || channels <= 0)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "segment attention (no-alloc): invalid sizes");
  if (heads > kMaxHeads)
    return fail(BYSJ_ERR_UNSUPPORTED,
                "segment attention (no-alloc): at most %d heads are supported", kMaxHeads);
  if (channels % heads != 0)
    return fail(BYSJ_ERR_INVALID_ARGUMENT,
                "segment attention (no-alloc): heads must divide channels");
  if (value_dtype != BYSJ_F32 && value_dtype != BYSJ_BF16)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "segment attention (no-alloc): unknown dtype");
  const bool vec_ok = aligned16(value) && aligned16(out);
  AttnLayout L;
  SplitSlots ss{};
  // Size check first, so an oversized row is rejected whatever the counts.
  int st = noalloc_layout(vec_ok, value_dtype, n_edges, n_nodes, heads, components, channels,
                          nullptr, &L, &ss);
  if (st) return st;
  if (n_nodes == 0) return BYSJ_OK;
  if (offsets == nullptr || out == nullptr ||
      (n_edges > 0 && (logit == nullptr || value == nullptr)))
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "segment attention (no-alloc): NULL pointer");
  void* base = nullptr;
  st = noalloc_scratch_address(&base);
  if (st) return st;
  st = noalloc_layout(vec_ok, value_dtype, n_edges, n_nodes, heads, components, channels, base,
                      &L, &ss);
  if (st) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The array keeps the previous call's contents; only the tickets must
  // start at zero (partial slots are always written before they are read).
  st = cuda_check(cudaMemsetAsync(ss.tickets, 0, sizeof(int) * L.plan.parts * L.cfg.tiles, s),
                  "segment attention (no-alloc): ticket reset");
  if (st) return st;
  AttnArgs a;
  a.logit = logit;
  a.value = value;
  a.env = env;
  a.null_logit = null_logit;
  a.order = order;
  a.out = out;
  a.heads = static_cast<int>(heads);
  a.hp = static_cast<int>(next_pow2(heads));
  a.comps = components;
  a.channels = channels;
  a.dh = channels / heads;
  a.row = components * channels;
  a.lv = L.cfg.lv;
  a.stats_off = L.stats_off;
  a.mp = MergePath{offsets, n_nodes, n_edges, L.plan.ipc, L.plan.parts};
  a.ss = ss;
  dim3 grid(L.plan.blocks, static_cast<unsigned>(L.cfg.tiles));
  L.cfg.kernel<<<grid, kBlock, 0, s>>>(a);
  return launch_check("segment_attention_kernel (no-alloc)");
}
