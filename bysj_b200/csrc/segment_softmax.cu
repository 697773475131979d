// Gated destination-segmented softmax, forward and backward, for sm_100a.
//
// Mathematics (reference csrc/segment_softmax.cpp:16-32), per segment n and
// channel c, with l_e = logit[e,c] + 2 ln env[e] for env[e] > 0:
//   m = max(null[n,c], max_e l_e),  D = exp(null - m) + sum_e exp(l_e - m)
//   alpha[e,c] = exp(l_e - m) / D,  null_alpha[n,c] = exp(null - m) / D
// backward, from the stored weights:
//   S = sum_e alpha*g + null_alpha*g0
//   grad_logit = alpha (g - S), grad_null = null_alpha (g0 - S)
//   grad_env[e] = (sum_c grad_logit[e,c]) * 2 / env[e]   (0 if env <= 0)
//
// Work split: merge-path partitions, one per warp.  A narrow channel count
// packs G = 32 / next_pow2(C) edges side by side in a warp.  Whole segments
// run max / sum / write back to back while the segment's rows are still in
// L1.  For a segment cut by partition boundaries, the pieces publish their
// partial statistics, the last piece to finish combines them in partition
// order into a final-statistics slot, and a second, equally partitioned
// kernel writes the per-edge outputs of those segments.  The forward pass
// for C = 4, 8 or 16 with rows in storage order (the attention widths)
// instead gives each warp whole segments (segment_softmax_whole_kernel): no
// split, no second pass.
#include <atomic>

#include "launch.cuh"

namespace bysj {
namespace {

struct SmxArgs {
  // forward inputs / backward "alpha" and "grad_alpha"
  const float* x;        // forward: logit   | backward: alpha
  const float* y;        // forward: unused  | backward: grad_alpha
  const float* env;
  const float* xn;       // forward: null_logit | backward: null_alpha
  const float* yn;       // backward: grad_null_alpha
  const int64_t* order;
  float* out;            // forward: alpha  | backward: grad_logit
  float* out_null;       // forward: null_alpha | backward: grad_null_logit
  float* out_env;        // backward: grad_env (NULL: computed elsewhere)
  int64_t channels;
  int64_t cpad;          // channels rounded up to a multiple of 4
  MergePath mp;
  SplitSlots ss;         // partial statistics  [parts][2][2*cpad]
  float* final_stats;    // combined statistics [parts][2*cpad]
  int* big_split;        // set when a split segment is left to the second pass
  int64_t* hub_slot;     // whole forward: per partition, the hub segment it left
                         // to segment_softmax_hub_kernel, or -1 (NULL: no hubs)
  int64_t hub_rows;      // segments longer than this are hubs
  float* hub_stats;      // [parts][2][2*cpad]: (max, sum) of a partition's slice of
                         // the hub it starts (kind 0) and of the one it continues (1)
  unsigned long long* hub_flag;  // == epoch when this call met a hub
  unsigned long long epoch;      // unique per call
};

// Split segments up to this many edges are written by the piece that
// combines them; longer ones by the second, equally partitioned pass.
constexpr int64_t kSelfWrite = 4096;

template <int NC, int G>
struct SmxShape {
  static constexpr int LPG = kWarp / G;  // channel lanes per group
  static constexpr int TC = LPG * NC;    // channels per tile
};

template <int NC, int G>
__device__ __forceinline__ int64_t lane_channel(int lane, int tile, int k) {
  using S = SmxShape<NC, G>;
  return static_cast<int64_t>(tile) * S::TC + lane % S::LPG + k * S::LPG;
}

// ---- forward --------------------------------------------------------------

template <int NC, int G>
__device__ __forceinline__ void smx_fwd_write(const SmxArgs& a, int64_t lo,
                                              int64_t hi, int g,
                                              const int64_t (&ch)[NC],
                                              const bool (&ok)[NC],
                                              const float (&m)[NC],
                                              const float (&inv)[NC]) {
  const int64_t C = a.channels;
  for (int64_t s = lo + g; s < hi; s += G) {
    const int64_t e = a.order ? __ldg(a.order + s) : s;
#pragma unroll
    for (int k = 0; k < NC; ++k)
      if (ok[k]) {
        const float l = gated_logit(__ldg(a.x + e * C + ch[k]), a.env, e);
        a.out[e * C + ch[k]] = shifted_exp(l, m[k]) * inv[k];
      }
  }
}

template <int NC, int G>
__global__ void __launch_bounds__(kBlock) segment_softmax_fwd_kernel(SmxArgs a) {
  using S = SmxShape<NC, G>;
  const int64_t p = global_warp();
  if (p >= a.mp.parts) return;
  const int lane = lane_id();
  const int tile = blockIdx.y;
  const int g = lane / S::LPG;
  const int64_t C = a.channels;
  int64_t ch[NC];
  bool ok[NC];
#pragma unroll
  for (int k = 0; k < NC; ++k) {
    ch[k] = lane_channel<NC, G>(lane, tile, k);
    ok[k] = ch[k] < C;
  }
  SegCursor cur(a.mp, part_range(a.mp, p));
  while (cur.next()) {
    const int64_t n = cur.node;
    const bool whole = cur.kind == kWhole;
    float m[NC];
#pragma unroll
    for (int k = 0; k < NC; ++k) m[k] = -INFINITY;
    for (int64_t s = cur.lo + g; s < cur.hi; s += G) {
      const int64_t e = a.order ? __ldg(a.order + s) : s;
#pragma unroll
      for (int k = 0; k < NC; ++k)
        if (ok[k]) m[k] = fmaxf(m[k], gated_logit(__ldg(a.x + e * C + ch[k]), a.env, e));
    }
    float nl[NC];
#pragma unroll
    for (int k = 0; k < NC; ++k) {
      m[k] = xor_max(m[k], S::LPG);
      nl[k] = (whole && ok[k] && a.xn) ? __ldg(a.xn + n * C + ch[k]) : -INFINITY;
      m[k] = fmaxf(m[k], nl[k]);
    }
    float d[NC];
#pragma unroll
    for (int k = 0; k < NC; ++k) d[k] = 0.0f;
    for (int64_t s = cur.lo + g; s < cur.hi; s += G) {
      const int64_t e = a.order ? __ldg(a.order + s) : s;
#pragma unroll
      for (int k = 0; k < NC; ++k)
        if (ok[k])
          d[k] += shifted_exp(gated_logit(__ldg(a.x + e * C + ch[k]), a.env, e), m[k]);
    }
#pragma unroll
    for (int k = 0; k < NC; ++k) d[k] = xor_sum(d[k], S::LPG);

    if (whole) {
      float inv[NC];
#pragma unroll
      for (int k = 0; k < NC; ++k) {
        const float w0 = shifted_exp(nl[k], m[k]);
        const float total = d[k] + w0;
        inv[k] = total > 0.0f ? 1.0f / total : 0.0f;
        if (g == 0 && ok[k] && a.out_null) a.out_null[n * C + ch[k]] = w0 * inv[k];
      }
      smx_fwd_write<NC, G>(a, cur.lo, cur.hi, g, ch, ok, m, inv);
      continue;
    }
    float* mine = a.ss.slot(p, cur.kind);
    if (g == 0) {
#pragma unroll
      for (int k = 0; k < NC; ++k)
        if (ok[k]) {
          __stcg(mine + ch[k], m[k]);
          __stcg(mine + a.cpad + ch[k], d[k]);
        }
    }
    const int64_t first = a.mp.part_of_first_edge(n);
    const int64_t last = a.mp.part_of_end(n);
    if (!arrive_last(a.ss, first, last, tile)) continue;
    if (g == 0) {
      float* fin = a.final_stats + last * 2 * a.cpad;
#pragma unroll
      for (int k = 0; k < NC; ++k) {
        if (!ok[k]) continue;
        const float n0 = a.xn ? __ldg(a.xn + n * C + ch[k]) : -INFINITY;
        float mm = n0;
        for (int64_t q = first; q <= last; ++q)
          mm = fmaxf(mm, __ldcg(a.ss.slot(q, q == last ? kHead : kTail) + ch[k]));
        float total = shifted_exp(n0, mm);
        for (int64_t q = first; q <= last; ++q) {
          const float* sq = a.ss.slot(q, q == last ? kHead : kTail);
          total += shifted_exp(__ldcg(sq + ch[k]), mm) * __ldcg(sq + a.cpad + ch[k]);
        }
        const float inv = total > 0.0f ? 1.0f / total : 0.0f;
        if (a.out_null) a.out_null[n * C + ch[k]] = shifted_exp(n0, mm) * inv;
        __stcg(fin + ch[k], mm);
        __stcg(fin + a.cpad + ch[k], inv);
      }
    }
  }
}

// Writes alpha for the edges of split segments once their statistics are final.
template <int NC, int G>
__global__ void __launch_bounds__(kBlock) segment_softmax_fwd_split_kernel(SmxArgs a) {
  using S = SmxShape<NC, G>;
  const int64_t p = global_warp();
  if (p >= a.mp.parts) return;
  const int lane = lane_id();
  const int tile = blockIdx.y;
  const int g = lane / S::LPG;
  int64_t ch[NC];
  bool ok[NC];
#pragma unroll
  for (int k = 0; k < NC; ++k) {
    ch[k] = lane_channel<NC, G>(lane, tile, k);
    ok[k] = ch[k] < a.channels;
  }
  SegCursor cur(a.mp, part_range(a.mp, p));
  while (cur.next()) {
    if (cur.kind == kWhole) continue;
    const int64_t last = a.mp.part_of_end(cur.node);
    const float* fin = a.final_stats + last * 2 * a.cpad;
    float m[NC], inv[NC];
#pragma unroll
    for (int k = 0; k < NC; ++k) {
      m[k] = ok[k] ? __ldcg(fin + ch[k]) : 0.0f;
      inv[k] = ok[k] ? __ldcg(fin + a.cpad + ch[k]) : 0.0f;
    }
    smx_fwd_write<NC, G>(a, cur.lo, cur.hi, g, ch, ok, m, inv);
  }
}

// ---- forward, quad-vector form (C % 4 == 0, C <= 128) ------------------------
// Lanes of a warp are (edge group g, channel quad q): LP = pow2(C/4) lanes per
// edge row, G = 32/LP rows side by side, T rows per lane per chunk.  A chunk
// of G*T rows is loaded in one burst of 16-byte loads; each lane keeps a
// running (max, denominator) per channel, rescaled when the max grows, and
// the G groups are merged with a fixed butterfly.  A segment that fits in
// one chunk is written straight from registers (one read, one write of the
// logits); longer segments re-read their rows (from L1/L2) for the write.
template <int LP>
struct QuadSmx {
  static constexpr int G = kWarp / LP;
  static constexpr int T = 8;
  static constexpr int CHUNK = G * T;
};

__device__ __forceinline__ float quad_get(const float4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

__device__ __forceinline__ void quad_set(float4& v, int i, float x) {
  if (i == 0) v.x = x; else if (i == 1) v.y = x; else if (i == 2) v.z = x; else v.w = x;
}

// Rows of slots base + g + t*G (t < TT) that lie below `hi`.
template <int LP, int TT>
__device__ __forceinline__ int quad_rows_n(int64_t base, int64_t hi, int g) {
  using Q = QuadSmx<LP>;
  const int64_t left = hi - base - g;
  if (left <= 0) return 0;
  const int64_t r = (left + Q::G - 1) / Q::G;
  return r < TT ? static_cast<int>(r) : TT;
}
template <int LP>
__device__ __forceinline__ int quad_rows(int64_t base, int64_t hi, int g) {
  return quad_rows_n<LP, QuadSmx<LP>::T>(base, hi, g);
}

// Loads the gated logits of slots base + g + t*G (t < T) into x (-inf past
// `hi` and for masked edges).  The envelope shift 2 ln env of a row is
// computed once, by lane (t mod LP) of the row's group, and shuffled to the
// other LP - 1 lanes of that row.
template <int LP, bool kEnv>
__device__ __forceinline__ void quad_load(const SmxArgs& a, int64_t base, int64_t hi, int g,
                                          int q, bool qok, float4 (&x)[QuadSmx<LP>::T]) {
  using Q = QuadSmx<LP>;
  constexpr int kOwn = (Q::T + LP - 1) / LP;  // rows whose envelope this lane takes
  const int64_t cq = a.channels / 4;
  const int64_t first = base + g;
  const int rows = quad_rows<LP>(base, hi, g);
  float sh[kOwn];
  if constexpr (kEnv) {
#pragma unroll
    for (int j = 0; j < kOwn; ++j) {
      const int t = q + j * LP;
      float v = -INFINITY;
      if (t < rows) {
        const int64_t s = first + static_cast<int64_t>(t) * Q::G;
        const float env = __ldg(a.env + (a.order ? __ldg(a.order + s) : s));
        if (env > 0.0f) v = 2.0f * __logf(env);
      }
      sh[j] = v;
    }
  }
  const int mine = qok ? rows : 0;
  const float4* row = reinterpret_cast<const float4*>(a.x) + q;
#pragma unroll
  for (int t = 0; t < Q::T; ++t) {
    float shift = 0.0f;
    if constexpr (kEnv) {
      if constexpr (LP == 1) {
        shift = sh[t];
      } else {
        shift = __shfl_sync(kFull, sh[t / LP], g * LP + (t % LP));
      }
    }
    float4 v = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    if (t < mine) {
      const int64_t slot = first + static_cast<int64_t>(t) * Q::G;
      const float4 raw = __ldg(row + (a.order ? __ldg(a.order + slot) : slot) * cq);
      if (!kEnv || shift != -INFINITY)
        v = make_float4(raw.x + shift, raw.y + shift, raw.z + shift, raw.w + shift);
    }
    x[t] = v;
  }
}

// Stores x[t] as the out row of slot base + g + t*G for the rows below `hi`.
template <int LP>
__device__ __forceinline__ void quad_store(const SmxArgs& a, int64_t base, int64_t hi, int g,
                                           int q, bool qok, const float4 (&x)[QuadSmx<LP>::T]) {
  using Q = QuadSmx<LP>;
  const int mine = qok ? quad_rows<LP>(base, hi, g) : 0;
  const int64_t cq = a.channels / 4;
  const int64_t first = base + g;
  float4* row = reinterpret_cast<float4*>(a.out) + q;
#pragma unroll
  for (int t = 0; t < Q::T; ++t) {
    if (t >= mine) break;
    const int64_t slot = first + static_cast<int64_t>(t) * Q::G;
    row[(a.order ? __ldg(a.order + slot) : slot) * cq] = x[t];
  }
}

// x[t] <- exp(x[t] - m) * inv, per channel of the quad.
template <int LP>
__device__ __forceinline__ void quad_weights(float4 (&x)[QuadSmx<LP>::T], const float (&m)[4],
                                             const float (&inv)[4]) {
#pragma unroll
  for (int t = 0; t < QuadSmx<LP>::T; ++t)
#pragma unroll
    for (int i = 0; i < 4; ++i) quad_set(x[t], i, shifted_exp_fast(quad_get(x[t], i), m[i]) * inv[i]);
}

template <int LP>
__device__ __forceinline__ void quad_write(const SmxArgs& a, int64_t base, int64_t hi, int g,
                                           int q, bool qok, float4 (&x)[QuadSmx<LP>::T],
                                           const float (&m)[4], const float (&inv)[4]) {
  quad_weights<LP>(x, m, inv);
  quad_store<LP>(a, base, hi, g, q, qok, x);
}

// Reads of a staged chunk through explicit shared-memory addresses (the
// buffers are picked at run time, which would otherwise leave generic loads).
// volatile: kept in order with the cp.async waits above them.
__device__ __forceinline__ float4 lds_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr));
  return v;
}
__device__ __forceinline__ float lds_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ int64_t lds_i64(uint32_t addr) {
  int64_t v;
  asm volatile("ld.shared.s64 %0, [%1];" : "=l"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async8(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_addr(smem)), "l"(gmem)
               : "memory");
}

// Shared-memory staging of one chunk of a warp: lane (g, q) copies the quad
// q of rows base + g + t*G into buf[32 t + lane] (the place it reads it from
// later), and lane q == 0 of each group the row's envelope into
// env[t G + g].  4 KB of rows + G*T floats of envelope per buffer.
template <int LP>
struct QuadStage {
  static constexpr int kRowsF4 = QuadSmx<LP>::T * kWarp;
  static constexpr int kEnvF = QuadSmx<LP>::CHUNK;
  static constexpr size_t kBytes = sizeof(float4) * kRowsF4 + sizeof(float) * kEnvF;
  static constexpr size_t kWarpBytes = 2 * kBytes;  // double buffer
};

template <int LP, bool kEnv>
__device__ __forceinline__ void quad_stage(const SmxArgs& a, int64_t base, int64_t hi, int g,
                                           int q, bool qok, float4* buf, float* env) {
  using Q = QuadSmx<LP>;
  const int rows = quad_rows<LP>(base, hi, g);
  const int64_t C = a.channels;
  const int lane = g * LP + q;
#pragma unroll
  for (int t = 0; t < Q::T; ++t) {
    if (t >= rows) break;
    const int64_t slot = base + g + static_cast<int64_t>(t) * Q::G;
    const int64_t e = a.order ? __ldg(a.order + slot) : slot;
    if (qok) cp_async16(buf + t * kWarp + lane, a.x + e * C + 4 * q);
    if (kEnv && q == 0) cp_async4(env + t * Q::G + g, a.env + e);
  }
}

// quad_load from a staged chunk.
template <int LP, bool kEnv>
__device__ __forceinline__ void quad_load_smem(const float4* buf, const float* envs,
                                               int64_t base, int64_t hi, int g, int q, bool qok,
                                               float4 (&x)[QuadSmx<LP>::T]) {
  using Q = QuadSmx<LP>;
  constexpr int kOwn = (Q::T + LP - 1) / LP;
  const int rows = quad_rows<LP>(base, hi, g);
  const int lane = g * LP + q;
  const uint32_t rows_s = smem_addr(buf) + 16u * lane;
  const uint32_t env_s = smem_addr(envs) + 4u * g;
  float sh[kOwn];
  if constexpr (kEnv) {
#pragma unroll
    for (int j = 0; j < kOwn; ++j) {
      const int t = q + j * LP;
      float v = -INFINITY;
      if (t < rows) {
        const float env = lds_f32(env_s + 4u * t * Q::G);
        if (env > 0.0f) v = 2.0f * __logf(env);
      }
      sh[j] = v;
    }
  }
  const int mine = qok ? rows : 0;
#pragma unroll
  for (int t = 0; t < Q::T; ++t) {
    float shift = 0.0f;
    if constexpr (kEnv) {
      if constexpr (LP == 1) {
        shift = sh[t];
      } else {
        shift = __shfl_sync(kFull, sh[t / LP], g * LP + (t % LP));
      }
    }
    float4 v = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    if (t < mine) {
      const float4 raw = lds_f4(rows_s + 16u * t * kWarp);
      if (!kEnv || shift != -INFINITY)
        v = make_float4(raw.x + shift, raw.y + shift, raw.z + shift, raw.w + shift);
    }
    x[t] = v;
  }
}

// The segment piece a cursor stands on.
struct Piece {
  int64_t node, lo, hi;
  int kind;
};
__device__ __forceinline__ Piece piece_of(const SegCursor& c) {
  return Piece{c.node, c.lo, c.hi, c.kind};
}

// One segment piece of the quad kernel (`staged`: its rows in shared memory,
// or nullptr to read them from global memory).
template <int LP, bool kSplitPass, bool kEnv>
__device__ __forceinline__ void quad_segment(const SmxArgs& a, int64_t p, const Piece& cur,
                                             int lane, int g, int q, bool qok,
                                             const float4* staged, const float* staged_env) {
  using Q = QuadSmx<LP>;
  const int64_t C = a.channels;
  const int64_t n = cur.node;
  const bool whole = cur.kind == kWhole;
  float4 x[Q::T];
  float m[4], inv[4];
  if constexpr (kSplitPass) {
    if (whole) return;
    if (__ldg(a.mp.offsets + n + 1) - __ldg(a.mp.offsets + n) <= kSelfWrite) return;
    const float* fin = a.final_stats + a.mp.part_of_end(n) * 2 * a.cpad;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      m[i] = qok ? __ldcg(fin + 4 * q + i) : 0.0f;
      inv[i] = qok ? __ldcg(fin + a.cpad + 4 * q + i) : 0.0f;
    }
    #pragma unroll 1
    for (int64_t base = cur.lo; base < cur.hi; base += Q::CHUNK) {
      quad_load<LP, kEnv>(a, base, cur.hi, g, q, qok, x);
      quad_write<LP>(a, base, cur.hi, g, q, qok, x, m, inv);
    }
    return;
  } else {
    float d[4];
    const bool one_chunk = cur.hi - cur.lo <= Q::CHUNK;
    float nl[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    if (whole && a.xn && qok) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(a.xn + n * C) + q);
      nl[0] = v.x; nl[1] = v.y; nl[2] = v.z; nl[3] = v.w;
    }
    if (one_chunk) {
      // Exact two-step form: maximum first, then each exponential once;
      // x keeps exp(l - m) for the write.
      if (staged != nullptr)
        quad_load_smem<LP, kEnv>(staged, staged_env, cur.lo, cur.hi, g, q, qok, x);
      else
        quad_load<LP, kEnv>(a, cur.lo, cur.hi, g, q, qok, x);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float cm = -INFINITY;
#pragma unroll
        for (int t = 0; t < Q::T; ++t) cm = fmaxf(cm, quad_get(x[t], i));
        for (int st = LP; st < kWarp; st <<= 1) cm = fmaxf(cm, __shfl_xor_sync(kFull, cm, st));
        m[i] = fmaxf(cm, nl[i]);
        // With m = -inf every row is -inf too; shifting by 0 keeps
        // exp(-inf) = 0 and avoids -inf - -inf.
        const float ms = m[i] == -INFINITY ? 0.0f : m[i];
        float acc = 0.0f;
#pragma unroll
        for (int t = 0; t < Q::T; ++t) {
          const float w = __expf(quad_get(x[t], i) - ms);
          quad_set(x[t], i, w);
          acc += w;
        }
        for (int st = LP; st < kWarp; st <<= 1) acc += __shfl_xor_sync(kFull, acc, st);
        d[i] = acc;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) { m[i] = -INFINITY; d[i] = 0.0f; }
      #pragma unroll 1
      for (int64_t base = cur.lo; base < cur.hi; base += Q::CHUNK) {
        quad_load<LP, kEnv>(a, base, cur.hi, g, q, qok, x);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float cm = -INFINITY;
#pragma unroll
          for (int t = 0; t < Q::T; ++t) cm = fmaxf(cm, quad_get(x[t], i));
          const float mn = fmaxf(m[i], cm);
          float acc = d[i] * shifted_exp(m[i], mn);
#pragma unroll
          for (int t = 0; t < Q::T; ++t) acc += shifted_exp_fast(quad_get(x[t], i), mn);
          d[i] = acc;
          m[i] = mn;
        }
      }
      // Merge the G edge groups (fixed butterfly; every lane ends equal).
      for (int st = LP; st < kWarp; st <<= 1) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float mo = __shfl_xor_sync(kFull, m[i], st);
          const float dd = __shfl_xor_sync(kFull, d[i], st);
          const float mn = fmaxf(m[i], mo);
          d[i] = d[i] * shifted_exp(m[i], mn) + dd * shifted_exp(mo, mn);
          m[i] = mn;
        }
      }
    }
    if (whole) {
      float w0[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        // one_chunk: m already includes the null logit and x holds
        // exp(l - m); otherwise rescale the running sum to the final max.
        const float mm = fmaxf(m[i], nl[i]);
        w0[i] = shifted_exp(nl[i], mm);
        const float total = (one_chunk ? d[i] : d[i] * shifted_exp(m[i], mm)) + w0[i];
        inv[i] = total > 0.0f ? 1.0f / total : 0.0f;
        m[i] = mm;
      }
      if (g == 0 && qok && a.out_null) {
        reinterpret_cast<float4*>(a.out_null + n * C)[q] =
            make_float4(w0[0] * inv[0], w0[1] * inv[1], w0[2] * inv[2], w0[3] * inv[3]);
      }
      if (one_chunk) {
#pragma unroll
        for (int t = 0; t < Q::T; ++t)
          x[t] = make_float4(x[t].x * inv[0], x[t].y * inv[1], x[t].z * inv[2], x[t].w * inv[3]);
        quad_store<LP>(a, cur.lo, cur.hi, g, q, qok, x);
      } else {
        #pragma unroll 1
        for (int64_t base = cur.lo; base < cur.hi; base += Q::CHUNK) {
          quad_load<LP, kEnv>(a, base, cur.hi, g, q, qok, x);
          quad_write<LP>(a, base, cur.hi, g, q, qok, x, m, inv);
        }
      }
      return;
    }
    // Split segment: publish per-channel (m, d); the last piece combines.
    float* mine = a.ss.slot(p, cur.kind);
    if (g == 0 && qok) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        __stcg(mine + 4 * q + i, m[i]);
        __stcg(mine + a.cpad + 4 * q + i, d[i]);
      }
    }
    const int64_t first = a.mp.part_of_first_edge(n);
    const int64_t last = a.mp.part_of_end(n);
    if (!arrive_last(a.ss, first, last, 0)) return;
    // Every lane combines its own channel quad (the G copies agree).
    if (a.xn && qok) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(a.xn + n * C) + q);
      nl[0] = v.x; nl[1] = v.y; nl[2] = v.z; nl[3] = v.w;
    }
    float* fin = a.final_stats + last * 2 * a.cpad;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t c = 4 * q + i;
      float mm = nl[i];
      float total = 0.0f;
      if (qok) {
        for (int64_t qq = first; qq <= last; ++qq)
          mm = fmaxf(mm, __ldcg(a.ss.slot(qq, qq == last ? kHead : kTail) + c));
        total = shifted_exp(nl[i], mm);
        for (int64_t qq = first; qq <= last; ++qq) {
          const float* sq = a.ss.slot(qq, qq == last ? kHead : kTail);
          total += shifted_exp(__ldcg(sq + c), mm) * __ldcg(sq + a.cpad + c);
        }
      }
      const float iv = total > 0.0f ? 1.0f / total : 0.0f;
      m[i] = mm;
      inv[i] = iv;
      if (g == 0 && qok) {
        if (a.out_null) a.out_null[n * C + c] = shifted_exp(nl[i], mm) * iv;
        __stcg(fin + c, mm);
        __stcg(fin + a.cpad + c, iv);
      }
    }
    const int64_t seg_lo = __ldg(a.mp.offsets + n);
    const int64_t seg_hi = __ldg(a.mp.offsets + n + 1);
    if (seg_hi - seg_lo <= kSelfWrite) {
      #pragma unroll 1
      for (int64_t base = seg_lo; base < seg_hi; base += Q::CHUNK) {
        quad_load<LP, kEnv>(a, base, seg_hi, g, q, qok, x);
        quad_write<LP>(a, base, seg_hi, g, q, qok, x, m, inv);
      }
    } else if (lane == 0) {
      atomicExch(a.big_split, 1);
    }
  }
}

// ---- forward, lean form: C == 4 LP exactly, rows in storage order --------
// The common case of the pipelined widths (H = 4 or 8 heads, no storage
// order): a row is exactly LP quads, so every row address is one base plus a
// compile-time stride, and the envelope shift of a row is taken by both of
// its lanes (no shuffle).  Same staging layout as quad_stage and the same
// arithmetic as quad_segment's one-chunk path for a whole segment.

template <int LP, bool kEnv, int TT = QuadSmx<LP>::T>
__device__ __forceinline__ void lean_stage(const SmxArgs& a, int64_t lo, int64_t hi, int g,
                                           int q, float4* buf, float* env) {
  using Q = QuadSmx<LP>;
  const int rows = quad_rows_n<LP, TT>(lo, hi, g);
  const int lane = g * LP + q;
  const float4* src = reinterpret_cast<const float4*>(a.x) + (lo + g) * LP + q;
#pragma unroll
  for (int t = 0; t < TT; ++t)
    if (t < rows) cp_async16(buf + t * kWarp + lane, src + t * Q::G * LP);
  if constexpr (kEnv) {
    const float* es = a.env + lo + g;
#pragma unroll
    for (int j = 0; j < TT / LP; ++j) {
      const int t = q + j * LP;
      if (t < rows) cp_async4(env + t * Q::G + g, es + t * Q::G);
    }
  }
}

// A no-op for the refill hook of the staged segment passes: a caller with a
// single stage buffer passes a functor that stages the next segment once the
// buffer has been read into registers.
struct NoRefill {
  __device__ __forceinline__ void operator()() const {}
};

template <int LP, bool kEnv, int TT = QuadSmx<LP>::T, typename Refill = NoRefill>
__device__ __forceinline__ void lean_whole(const SmxArgs& a, int64_t n, int64_t lo, int64_t hi,
                                           int g, int q, const float4* buf, const float* envs,
                                           const int64_t* idx = nullptr,
                                           Refill refill = Refill{}) {
  using Q = QuadSmx<LP>;
  constexpr int C = 4 * LP;
  const int rows = quad_rows_n<LP, TT>(lo, hi, g);
  const int lane = g * LP + q;
  const uint32_t rows_s = smem_addr(buf) + 16u * lane;
  const uint32_t env_s = smem_addr(envs) + 4u * g;
  uint64_t x[TT][2];  // channel pairs (0,1), (2,3)
  const uint64_t ninf = pk2(-INFINITY, -INFINITY);
#pragma unroll
  for (int t = 0; t < TT; ++t) {
    float shift = 0.0f;
    bool keep = t < rows;
    if constexpr (kEnv) {
      const float e = keep ? lds_f32(env_s + 4u * t * Q::G) : 0.0f;
      keep = keep && e > 0.0f;
      shift = keep ? 2.0f * __logf(e) : 0.0f;
    }
    x[t][0] = ninf;
    x[t][1] = ninf;
    if (keep) {
      const float4 raw = lds_f4(rows_s + 16u * t * kWarp);
      const uint64_t sh = pk2(shift, shift);
      x[t][0] = add2(pk2(raw.x, raw.y), sh);
      x[t][1] = add2(pk2(raw.z, raw.w), sh);
    }
  }
  refill();  // the rows are in registers (the index buffer is read below)
  float nl[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
  if (a.xn) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(a.xn + n * C) + q);
    nl[0] = v.x; nl[1] = v.y; nl[2] = v.z; nl[3] = v.w;
  }
  float m[4], ms[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float cm = -INFINITY;
#pragma unroll
    for (int t = 0; t < TT; ++t) {
      const float2 v = upk2(x[t][i >> 1]);
      cm = fmaxf(cm, (i & 1) ? v.y : v.x);
    }
#pragma unroll
    for (int st = LP; st < kWarp; st <<= 1) cm = fmaxf(cm, __shfl_xor_sync(kFull, cm, st));
    m[i] = fmaxf(cm, nl[i]);
    ms[i] = m[i] == -INFINITY ? 0.0f : m[i];
  }
  // w = exp(y), y = x - ms <= 0, written as 2^(y log2 e) (base conversion),
  // two channels per instruction.  The product adds at most |y| log2 e 2^-24
  // to the exponent (< 1.3e-6 for the y >= -14 whose weights matter to an
  // absolute 1e-6), ex2.approx adds a few ulp, and weights below 2^-126 flush
  // to zero; on the C3 frame the results equal __expf(y) bit for bit.  The
  // tests hold them to rtol 1e-5 against float64.
  const uint64_t l2e = pk2(1.4426950408889634f, 1.4426950408889634f);
  uint64_t acc[2] = {pk2(0.0f, 0.0f), pk2(0.0f, 0.0f)};
#pragma unroll
  for (int pr = 0; pr < 2; ++pr) {
    const uint64_t msp = pk2(ms[2 * pr], ms[2 * pr + 1]);
#pragma unroll
    for (int t = 0; t < TT; ++t) {
      const float2 y = upk2(mul2(sub2(x[t][pr], msp), l2e));
      const uint64_t w = pk2(ex2_ftz(y.x), ex2_ftz(y.y));
      x[t][pr] = w;
      acc[pr] = add2(acc[pr], w);
    }
  }
  float w0[4], inv[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 ap = upk2(acc[i >> 1]);
    float s = (i & 1) ? ap.y : ap.x;
#pragma unroll
    for (int st = LP; st < kWarp; st <<= 1) s += __shfl_xor_sync(kFull, s, st);
    w0[i] = shifted_exp(nl[i], m[i]);
    const float total = s + w0[i];
    inv[i] = total > 0.0f ? __frcp_rn(total) : 0.0f;
  }
  if (g == 0 && a.out_null) {
    reinterpret_cast<float4*>(a.out_null + n * C)[q] =
        make_float4(w0[0] * inv[0], w0[1] * inv[1], w0[2] * inv[2], w0[3] * inv[3]);
  }
  const uint64_t inv01 = pk2(inv[0], inv[1]), inv23 = pk2(inv[2], inv[3]);
  auto out_row = [&](int t) {
    const float2 lo2 = upk2(mul2(x[t][0], inv01));
    const float2 hi2 = upk2(mul2(x[t][1], inv23));
    return make_float4(lo2.x, lo2.y, hi2.x, hi2.y);
  };
  if (idx != nullptr) {  // rows in storage order: row of slot lo + i is idx[i]
    const uint32_t idx_s = smem_addr(idx) + 8u * g;
#pragma unroll
    for (int t = 0; t < TT; ++t)
      if (t < rows) {
        const int64_t e = lds_i64(idx_s + 8u * t * Q::G);
        reinterpret_cast<float4*>(a.out)[e * LP + q] = out_row(t);
      }
    return;
  }
  float4* dst = reinterpret_cast<float4*>(a.out) + (lo + g) * LP + q;
#pragma unroll
  for (int t = 0; t < TT; ++t)
    if (t < rows) dst[t * Q::G * LP] = out_row(t);
}

// Channel counts up to 8 (LP <= 2) hold a typical segment (<= 128 rows) in
// one chunk, so the main pass stages the next piece in shared memory while
// computing the current one (2 CTAs per SM: 72 KB of buffers each).  Wider
// rows do not fit a chunk; their main pass reads global memory directly.
template <int LP>
constexpr bool quad_pipelined() {
  return LP <= 2;
}

template <int LP, bool kSplitPass, bool kEnv>
__global__ void __launch_bounds__(kBlock, quad_pipelined<LP>() ? 2 : 3)
    segment_softmax_quad_kernel(SmxArgs a) {
  using Q = QuadSmx<LP>;
  using S = QuadStage<LP>;
  extern __shared__ float4 quad_smem[];
  const int64_t p = global_warp();
  if (p >= a.mp.parts) return;
  const int lane = lane_id();
  const int g = lane / LP;
  const int q = lane % LP;
  const bool qok = 4 * q < a.channels;
  if constexpr (kSplitPass || !quad_pipelined<LP>()) {
    if constexpr (kSplitPass) {
      if (*reinterpret_cast<volatile int*>(a.big_split) == 0) return;
    }
    SegCursor cur(a.mp, part_range(a.mp, p));
    while (cur.next())
      quad_segment<LP, kSplitPass, kEnv>(a, p, piece_of(cur), lane, g, q, qok, nullptr, nullptr);
  } else {
    // Double-buffered pipeline: the next piece's rows (when it fits one
    // chunk) are copied into shared memory while this one is computed.
    char* mine = reinterpret_cast<char*>(quad_smem) + (threadIdx.x >> 5) * S::kWarpBytes;
    float4* bufs[2] = {reinterpret_cast<float4*>(mine),
                       reinterpret_cast<float4*>(mine + S::kBytes)};
    SegCursor ahead(a.mp, part_range(a.mp, p));  // one piece ahead of `cur`
    bool have = ahead.next();
    Piece cur = piece_of(ahead);
    int b = 0;
    if (have && cur.hi - cur.lo <= Q::CHUNK)
      quad_stage<LP, kEnv>(a, cur.lo, cur.hi, g, q, qok, bufs[0],
                           reinterpret_cast<float*>(bufs[0] + S::kRowsF4));
    cp_async_commit();
    while (have) {
      const bool have_next = ahead.next();
      const Piece nxt = piece_of(ahead);
      if (have_next && nxt.hi - nxt.lo <= Q::CHUNK)
        quad_stage<LP, kEnv>(a, nxt.lo, nxt.hi, g, q, qok, bufs[b ^ 1],
                             reinterpret_cast<float*>(bufs[b ^ 1] + S::kRowsF4));
      cp_async_commit();
      cp_async_wait<1>();  // this piece's copies have landed
      __syncwarp();
      const bool staged = cur.hi - cur.lo <= Q::CHUNK;
      quad_segment<LP, false, kEnv>(a, p, cur, lane, g, q, qok, staged ? bufs[b] : nullptr,
                                    staged ? reinterpret_cast<float*>(bufs[b] + S::kRowsF4)
                                           : nullptr);
      __syncwarp();  // every lane is done with bufs[b] before it is refilled
      cur = nxt;
      have = have_next;
      b ^= 1;
    }
    cp_async_wait<0>();
  }
}

// ---- forward, whole-segment partitions (lean widths) -----------------------
// For the lean widths the merge-path partitions are used only to balance the
// work: warp p takes every segment whose first merge-path item (diagonal
// offsets[n] + n) lies in its partition, whole.  No segment is split, so
// there are no partial statistics, tickets or second pass; the imbalance is
// at most one segment (<= CHUNK rows in the pipelined case).

// A whole segment longer than one chunk: running (max, sum) per channel over
// chunks read from global memory, merged over the edge groups, then a second
// read for the weights (as quad_segment's multi-chunk whole path).  The three
// steps are separate so that a CTA can share one long segment among its warps
// (segment_softmax_hub_kernel): pass 1 and pass 2 walk the chunks
// lo + first, lo + first + step, ...

// Pass 1: this warp's running (max, sum) per channel of its quad, merged over
// the edge groups (every lane of quad q ends with the same values).
template <int LP, bool kEnv>
__device__ __forceinline__ void lean_stats(const SmxArgs& a, int64_t lo, int64_t hi,
                                           int64_t first, int64_t step, int g, int q,
                                           float (&m)[4], float (&d)[4]) {
  using Q = QuadSmx<LP>;
  float4 x[Q::T];
#pragma unroll
  for (int i = 0; i < 4; ++i) { m[i] = -INFINITY; d[i] = 0.0f; }
  #pragma unroll 1
  for (int64_t base = lo + first; base < hi; base += step) {
    quad_load<LP, kEnv>(a, base, hi, g, q, true, x);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float cm = -INFINITY;
#pragma unroll
      for (int t = 0; t < Q::T; ++t) cm = fmaxf(cm, quad_get(x[t], i));
      const float mn = fmaxf(m[i], cm);
      float acc = d[i] * shifted_exp(m[i], mn);
#pragma unroll
      for (int t = 0; t < Q::T; ++t) acc += shifted_exp_fast(quad_get(x[t], i), mn);
      d[i] = acc;
      m[i] = mn;
    }
  }
  for (int st = LP; st < kWarp; st <<= 1) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float mo = __shfl_xor_sync(kFull, m[i], st);
      const float dd = __shfl_xor_sync(kFull, d[i], st);
      const float mn = fmaxf(m[i], mo);
      d[i] = d[i] * shifted_exp(m[i], mn) + dd * shifted_exp(mo, mn);
      m[i] = mn;
    }
  }
}

// Folds in the null logit: m becomes the final shift, inv the reciprocal
// denominator; the null weight is written when `write_null` (group 0).
template <int LP>
__device__ __forceinline__ void lean_norm(const SmxArgs& a, int64_t n, int g, int q,
                                          bool write_null, float (&m)[4], const float (&d)[4],
                                          float (&inv)[4]) {
  constexpr int C = 4 * LP;
  float nl[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
  if (a.xn) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(a.xn + n * C) + q);
    nl[0] = v.x; nl[1] = v.y; nl[2] = v.z; nl[3] = v.w;
  }
  float w0[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float mm = fmaxf(m[i], nl[i]);
    w0[i] = shifted_exp(nl[i], mm);
    const float total = d[i] * shifted_exp(m[i], mm) + w0[i];
    inv[i] = total > 0.0f ? 1.0f / total : 0.0f;
    m[i] = mm;
  }
  if (write_null && g == 0 && a.out_null)
    reinterpret_cast<float4*>(a.out_null + n * C)[q] =
        make_float4(w0[0] * inv[0], w0[1] * inv[1], w0[2] * inv[2], w0[3] * inv[3]);
}

// Pass 2: the weights of this warp's chunks.
template <int LP, bool kEnv>
__device__ __forceinline__ void lean_emit(const SmxArgs& a, int64_t lo, int64_t hi,
                                          int64_t first, int64_t step, int g, int q,
                                          const float (&m)[4], const float (&inv)[4]) {
  using Q = QuadSmx<LP>;
  float4 x[Q::T];
  float mm[4], ii[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) { mm[i] = m[i]; ii[i] = inv[i]; }
  #pragma unroll 1
  for (int64_t base = lo + first; base < hi; base += step) {
    quad_load<LP, kEnv>(a, base, hi, g, q, true, x);
    quad_write<LP>(a, base, hi, g, q, true, x, mm, ii);
  }
}

template <int LP, bool kEnv>
__device__ __forceinline__ void lean_big(const SmxArgs& a, int64_t n, int64_t lo, int64_t hi,
                                         int g, int q) {
  using Q = QuadSmx<LP>;
  float m[4], d[4], inv[4];
  lean_stats<LP, kEnv>(a, lo, hi, 0, Q::CHUNK, g, q, m, d);
  lean_norm<LP>(a, n, g, q, true, m, d, inv);
  lean_emit<LP, kEnv>(a, lo, hi, 0, Q::CHUNK, g, q, m, inv);
}

// Rows per lane and CTA shape of the whole kernel: a 128-row chunk at every
// width (4, 8 or 16 rows per lane at LP = 1, 2, 4), so that a typical segment
// (~90 edges) fits one chunk without lanes idling over most of it.  One
// stage buffer per warp (the next segment is staged once this one is in
// registers), four-warp CTAs; LP <= 2: five per SM (102 registers; C3, H = 8:
// 37.9 us with a double buffer and three eight-warp CTAs at 80 registers,
// 35.9 us single-buffered at the same shape, 33.8 us at this one; two or six
// CTAs per SM measured 37.0 / 35.9 us); LP = 4: three per SM.  (At LP = 1, 4
// rows per lane measured 1.3x faster than 8.)
template <int LP>
struct WholeShape {
  static constexpr int T = LP >= 4 ? 16 : LP == 2 ? 8 : 4;
  static constexpr int G = kWarp / LP;
  static constexpr int CHUNK = G * T;
  static constexpr int kRowsF4 = T * kWarp;
  static constexpr size_t kBytes = sizeof(float4) * kRowsF4 + sizeof(float) * CHUNK;
  static constexpr size_t kWarpBytes = kBytes;  // one stage buffer per warp
  static constexpr int kThreads = 128;
  static constexpr int kMinBlocks = LP >= 4 ? 3 : 5;
  static_assert(kBytes % 16 == 0, "stage buffers must stay 16-byte aligned");
};

// Running (max, sum) per channel of this lane's quad over one staged chunk
// [lo, hi) (rows and envelopes as lean_stage leaves them).
template <int LP, bool kEnv, int TT, typename Refill = NoRefill>
__device__ __forceinline__ void staged_stats(const float4* buf, const float* envs, int64_t lo,
                                             int64_t hi, int g, int q, float (&m)[4],
                                             float (&d)[4], Refill refill = Refill{}) {
  constexpr int G = WholeShape<LP>::G;
  const int rows = quad_rows_n<LP, TT>(lo, hi, g);
  const int lane = g * LP + q;
  const uint32_t rows_s = smem_addr(buf) + 16u * lane;
  const uint32_t env_s = smem_addr(envs) + 4u * g;
  float4 x[TT];
#pragma unroll
  for (int t = 0; t < TT; ++t) {
    float shift = 0.0f;
    bool keep = t < rows;
    if constexpr (kEnv) {
      const float e = keep ? lds_f32(env_s + 4u * t * G) : 0.0f;
      keep = keep && e > 0.0f;
      shift = keep ? 2.0f * __logf(e) : 0.0f;
    }
    float4 v = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    if (keep) {
      const float4 raw = lds_f4(rows_s + 16u * t * kWarp);
      v = make_float4(raw.x + shift, raw.y + shift, raw.z + shift, raw.w + shift);
    }
    x[t] = v;
  }
  refill();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float cm = -INFINITY;
#pragma unroll
    for (int t = 0; t < TT; ++t) cm = fmaxf(cm, quad_get(x[t], i));
    const float mn = fmaxf(m[i], cm);
    float acc = d[i] * shifted_exp(m[i], mn);
#pragma unroll
    for (int t = 0; t < TT; ++t) acc += shifted_exp_fast(quad_get(x[t], i), mn);
    d[i] = acc;
    m[i] = mn;
  }
}

// (max, sum) per channel of rows [lo, hi) of a hub segment, stored as
// max[C] | sum[C] (C = 4 LP) at `slot` by the lanes of edge group 0.  The
// rows go through the warp's stage buffer (cp.async; the next chunk is staged
// as soon as this one is in registers), as the whole kernel's segments do.
template <int LP, bool kEnv>
__device__ __forceinline__ void hub_slice(const SmxArgs& a, int64_t lo, int64_t hi, int g, int q,
                                          float4* smem, float* slot) {
  using S = WholeShape<LP>;
  constexpr int TT = S::T;
  constexpr int64_t kChunk = S::CHUNK;
  float4* const buf =
      reinterpret_cast<float4*>(reinterpret_cast<char*>(smem) + (threadIdx.x >> 5) * S::kWarpBytes);
  float* const envs = reinterpret_cast<float*>(buf + S::kRowsF4);
  float m[4], d[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) { m[i] = -INFINITY; d[i] = 0.0f; }
  lean_stage<LP, kEnv, TT>(a, lo, lo + kChunk < hi ? lo + kChunk : hi, g, q, buf, envs);
  cp_async_commit();
  #pragma unroll 1
  for (int64_t base = lo; base < hi; base += kChunk) {
    const int64_t next = base + kChunk;
    cp_async_wait<0>();
    __syncwarp();
    const auto refill = [&] {
      __syncwarp();  // every lane has read the buffer
      if (next < hi)
        lean_stage<LP, kEnv, TT>(a, next, next + kChunk < hi ? next + kChunk : hi, g, q, buf,
                                 envs);
      cp_async_commit();
    };
    staged_stats<LP, kEnv, TT>(buf, envs, base, next < hi ? next : hi, g, q, m, d, refill);
  }
  cp_async_wait<0>();
  for (int st = LP; st < kWarp; st <<= 1) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float mo = __shfl_xor_sync(kFull, m[i], st);
      const float dd = __shfl_xor_sync(kFull, d[i], st);
      const float mn = fmaxf(m[i], mo);
      d[i] = d[i] * shifted_exp(m[i], mn) + dd * shifted_exp(mo, mn);
      m[i] = mn;
    }
  }
  if (g == 0) {
    reinterpret_cast<float4*>(slot)[q] = make_float4(m[0], m[1], m[2], m[3]);
    reinterpret_cast<float4*>(slot + 4 * LP)[q] = make_float4(d[0], d[1], d[2], d[3]);
  }
}

template <int LP, bool kEnv>
__global__ void __launch_bounds__(WholeShape<LP>::kThreads, WholeShape<LP>::kMinBlocks)
    segment_softmax_whole_kernel(SmxArgs a) {
  using Q = WholeShape<LP>;
  using S = WholeShape<LP>;
  constexpr int TT = S::T;
  // A segment that fits TS < TT rows per lane takes an instantiation with
  // TS row slots: the max, exponent and sum then skip the empty slots of a
  // typical ~90-row segment (they would add exact zeros, so the bits are the
  // same).  C3: H = 8 36.6 -> 34.8 us with TS = 7 (112 rows; 6 spills
  // registers), H = 16 63.6 -> 60.4 us and H = 4 28.7 -> 28.1 us with TS =
  // 3/4 TT (96 rows).
  constexpr int TS = LP == 2 ? TT * 7 / 8 : TT * 3 / 4;
  extern __shared__ float4 quad_smem[];
  const int64_t p = global_warp();
  if (p >= a.mp.parts) return;
  const int lane = lane_id();
  const int g = lane / LP;
  const int q = lane % LP;
  const int64_t n0 = a.mp.starts_before(p * a.mp.ipc);
  const int64_t n1 = a.mp.starts_before((p + 1) * a.mp.ipc);
  // Every partition records the hub segment it starts, or -1 (at most one: a
  // hub is longer than a partition, so its start is the only segment start in
  // the partition's range).  A partition whose range begins inside a hub's
  // edges computes the (max, sum) of that slice for the hub pass: the
  // partitions a hub spans share its statistics, as a split segment's
  // pieces do, and nothing is idle while the hub pass waits.
  if (a.hub_slot != nullptr) {
    if (lane == 0) a.hub_slot[p] = -1;
    if (n0 >= 1) {
      const int64_t c = n0 - 1;
      const int64_t clo = __ldg(a.mp.offsets + c), chi = __ldg(a.mp.offsets + c + 1);
      const int64_t e0 = p * a.mp.ipc - c;  // edge at this partition's first position
      if (chi - clo > a.hub_rows && e0 < chi)
        hub_slice<LP, kEnv>(a, e0, e0 + a.mp.ipc < chi ? e0 + a.mp.ipc : chi, g, q, quad_smem,
                            a.hub_stats + (2 * p + 1) * 2 * a.cpad);
    }
  }
  if (n0 >= n1) return;
  float4* const buf = reinterpret_cast<float4*>(reinterpret_cast<char*>(quad_smem) +
                                                (threadIdx.x >> 5) * S::kWarpBytes);
  float* const envs = reinterpret_cast<float*>(buf + S::kRowsF4);
  const int64_t* off = a.mp.offsets;
  // Segment n is [lo, hi); the next one ends at nhi.  One stage buffer per
  // warp: once segment n's rows are in registers the buffer takes segment
  // n+1's copies, which land while segment n is computed.
  int64_t lo = __ldg(off + n0), hi = __ldg(off + n0 + 1);
  int64_t nhi = n0 + 1 < n1 ? __ldg(off + n0 + 2) : hi;
  if (hi - lo <= Q::CHUNK) lean_stage<LP, kEnv, TT>(a, lo, hi, g, q, buf, envs);
  cp_async_commit();
  bool owns_hub = false;
  for (int64_t n = n0; n < n1; ++n) {
    const int64_t nnhi = n + 2 < n1 ? __ldg(off + n + 3) : nhi;
    cp_async_wait<0>();  // this segment's copies have landed
    __syncwarp();
    const auto refill = [&] {
      __syncwarp();  // every lane has read the buffer
      if (n + 1 < n1 && nhi - hi <= Q::CHUNK) lean_stage<LP, kEnv, TT>(a, hi, nhi, g, q, buf, envs);
      cp_async_commit();
    };
    if (hi - lo <= TS * S::G) {
      lean_whole<LP, kEnv, TS>(a, n, lo, hi, g, q, buf, envs, nullptr, refill);
    } else if (hi - lo <= Q::CHUNK) {
      lean_whole<LP, kEnv, TT>(a, n, lo, hi, g, q, buf, envs, nullptr, refill);
    } else if (a.hub_slot != nullptr && hi - lo > a.hub_rows) {
      // the hub pass writes its weights; this partition's slice statistics
      // are computed after the loop (the partition index is recomputed
      // rather than kept live through the loop)
      refill();
      if (lane == 0) {
        a.hub_slot[global_warp()] = n;
        *reinterpret_cast<volatile unsigned long long*>(a.hub_flag) = a.epoch;
      }
      owns_hub = true;
    } else {
      refill();
      lean_big<LP, kEnv>(a, n, lo, hi, g, q);
    }
    lo = hi;
    hi = nhi;
    nhi = nnhi;
  }
  cp_async_wait<0>();
  if (owns_hub) {  // the slice of the hub from its first row to this partition's end
    __syncwarp();
    const int64_t pp = global_warp();
    const int64_t n = *reinterpret_cast<volatile int64_t*>(a.hub_slot + pp);
    const int64_t hlo = __ldg(off + n), hhi = __ldg(off + n + 1);
    const int64_t end = (pp + 1) * a.mp.ipc - n;
    hub_slice<LP, kEnv>(a, hlo, end < hhi ? end : hhi, g, q, quad_smem,
                        a.hub_stats + 2 * pp * 2 * a.cpad);
  }
  // This warp's slots are written: the dependent hub pass may be scheduled.
  asm volatile("griddepcontrol.launch_dependents;");
}

// ---- forward, hub segments of the whole kernel -----------------------------
// A segment longer than hub_rows (and than a partition) would keep one warp
// of the whole kernel busy for all of its rows (a 100,000-edge hub: 8 ms).
// Instead every partition the hub spans computes the (max, sum) of its slice
// inside the whole kernel (hub_slice), and this pass -- launched as a
// programmatic dependent of the whole kernel, one CTA per SM -- merges the
// slices in partition order (deterministic: the same slices, the same order,
// every call) and writes the weights, the hub's chunks dealt over every warp
// of the grid.  Every CTA merges the statistics itself, so no CTA waits on
// another.  A call without hubs reads one word (the flag the whole kernel sets
// to this call's epoch when it meets a hub) and returns.
constexpr int kHubWarps = 16;
constexpr int64_t kHubRows = 4096;

template <int LP, bool kEnv>
__global__ void __launch_bounds__(kHubWarps * kWarp, 1) segment_softmax_hub_kernel(SmxArgs a) {
  using Q = QuadSmx<LP>;
  constexpr int C = 4 * LP;
  constexpr int kThreads = kHubWarps * kWarp;
  __shared__ float s_m[kHubWarps][C];
  __shared__ float s_d[kHubWarps][C];
  __shared__ float s_fm[C], s_fd[C];
  constexpr int kScan = 8;  // hub slots read per thread per sweep, all in flight
  __shared__ int64_t s_list[kThreads * kScan];
  __shared__ int s_count;
  const int lane = lane_id();
  const int w = threadIdx.x >> 5;
  const int g = lane / LP;
  const int q = lane % LP;
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the whole kernel is complete
  if (*reinterpret_cast<volatile unsigned long long*>(a.hub_flag) != a.epoch) return;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * kHubWarps;
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * kHubWarps + w;
  const int64_t stride = 2 * a.cpad;
  for (int64_t base = 0; base < a.mp.parts; base += kThreads * kScan) {
    int64_t found[kScan];
#pragma unroll
    for (int k = 0; k < kScan; ++k) {
      const int64_t p = base + k * kThreads + threadIdx.x;
      found[k] = p < a.mp.parts ? __ldcg(a.hub_slot + p) : -1;
    }
    if (threadIdx.x == 0) s_count = 0;
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kScan; ++k)  // each hub is computed on its own: any order
      if (found[k] >= 0) s_list[atomicAdd(&s_count, 1)] = found[k];
    __syncthreads();
    const int hubs = s_count;
    for (int k = 0; k < hubs; ++k) {
      const int64_t n = s_list[k];
      const int64_t lo = __ldg(a.mp.offsets + n), hi = __ldg(a.mp.offsets + n + 1);
      const int64_t pa = (lo + n) / a.mp.ipc, pb = (hi - 1 + n) / a.mp.ipc;
      // Slices pa (kind 0), pa+1 .. pb (kind 1): warp w takes the run
      // [w*per, (w+1)*per) of them, its lanes as R = 32 / C rows of C
      // channels, row r merging slices r, r + R, ...; the rows are then
      // merged by a butterfly, whose row 0 is kept, and the warps' results in
      // warp order.  A fixed pattern for a given slice count: the same bits
      // every call.
      constexpr int R = kWarp / C;
      const int ch = lane % C, r = lane / C;
      const int64_t count = pb - pa + 1;
      const int64_t per = (count + kHubWarps - 1) / kHubWarps;
      const int64_t j1 = (w + 1) * per < count ? (w + 1) * per : count;
      float mm = -INFINITY, dd = 0.0f;
#pragma unroll 4
      for (int64_t j = w * per + r; j < j1; j += R) {
        const float* slot = a.hub_stats + (2 * (pa + j) + (j == 0 ? 0 : 1)) * stride;
        const float mo = __ldcg(slot + ch), dk = __ldcg(slot + C + ch);
        const float mn = fmaxf(mm, mo);
        dd = dd * shifted_exp(mm, mn) + dk * shifted_exp(mo, mn);
        mm = mn;
      }
#pragma unroll
      for (int st = C; st < kWarp; st <<= 1) {
        const float mo = __shfl_xor_sync(kFull, mm, st), dk = __shfl_xor_sync(kFull, dd, st);
        const float mn = fmaxf(mm, mo);
        dd = dd * shifted_exp(mm, mn) + dk * shifted_exp(mo, mn);
        mm = mn;
      }
      if (r == 0) {
        s_m[w][ch] = mm;
        s_d[w][ch] = dd;
      }
      __syncthreads();
      if (w == 0 && lane < C) {  // the warps' results, in warp order
        float fm = -INFINITY, fd = 0.0f;
        for (int k2 = 0; k2 < kHubWarps; ++k2) {
          const float mo = s_m[k2][lane], dk = s_d[k2][lane];
          const float mn = fmaxf(fm, mo);
          fd = fd * shifted_exp(fm, mn) + dk * shifted_exp(mo, mn);
          fm = mn;
        }
        s_fm[lane] = fm;
        s_fd[lane] = fd;
      }
      __syncthreads();
      float m[4], d[4], inv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        m[i] = s_fm[4 * q + i];
        d[i] = s_fd[4 * q + i];
      }
      lean_norm<LP>(a, n, g, q, gw == 0, m, d, inv);
      lean_emit<LP, kEnv>(a, lo, hi, gw * Q::CHUNK, warps * Q::CHUNK, g, q, m, inv);
      __syncthreads();  // s_m / s_d are reused by the next hub
    }
    __syncthreads();  // s_count / s_list are reused by the next sweep
  }
}

// ---- forward, whole segments in a permuted storage order (C = 4 or 8) -----
// The rows of segment n sit at storage rows order[lo..hi): a gather.  A lane
// that had to load order[slot] before issuing its row copy would wait a full
// memory round trip; so the warp runs three stages: segment n+2's contiguous
// order[lo..hi) slice is copied into one of three index buffers, and as soon
// as segment n's rows are in registers, segment n+1's rows and envelopes are
// gathered into the warp's one row buffer (cp.async, indices read from
// shared memory) while segment n is computed.  Outputs go to the staged
// storage rows.  Arithmetic as the whole kernel; segments longer than a
// chunk take lean_big (global, through order).  One row buffer per warp:
// five four-warp CTAs per SM (C3 permuted, H = 8: 78.0 -> 75.1 us against
// two row buffers).
constexpr int kGatherBlock = 128;  // four-warp CTAs
constexpr int kGatherMinBlocks = 5;

template <int LP>
struct GatherStage {
  using Q = QuadSmx<LP>;
  static constexpr size_t kRows = sizeof(float4) * Q::T * kWarp;
  static constexpr size_t kEnv = sizeof(float) * Q::CHUNK;
  static constexpr size_t kIdx = sizeof(int64_t) * Q::CHUNK;
  static constexpr size_t kWarpBytes = (kRows + kEnv) + 3 * kIdx;  // one row buffer
  static_assert((kRows + kEnv) % 16 == 0 && kIdx % 16 == 0, "16-byte aligned buffers");
};

template <int LP, bool kEnv>
__global__ void __launch_bounds__(kGatherBlock, kGatherMinBlocks)
    segment_softmax_gather_kernel(SmxArgs a) {
  using Q = QuadSmx<LP>;
  using S = GatherStage<LP>;
  // Row slots per lane for a segment within 7/8 (C = 8) or 3/8 (C = 4) of
  // the chunk: a typical ~90-row segment then skips the empty slots (same
  // bits; C3 permuted, H = 4: 80.9 -> 73.9 us, H = 8 unchanged).
  constexpr int kGatherShort = LP == 2 ? 7 : 3;
  extern __shared__ float4 quad_smem[];
  const int64_t p = global_warp();
  if (p >= a.mp.parts) return;
  const int lane = lane_id();
  const int g = lane / LP;
  const int q = lane % LP;
  const int64_t n0 = a.mp.starts_before(p * a.mp.ipc);
  const int64_t n1 = a.mp.starts_before((p + 1) * a.mp.ipc);
  if (n0 >= n1) return;
  char* mine = reinterpret_cast<char*>(quad_smem) + (threadIdx.x >> 5) * S::kWarpBytes;
  float4* const rbuf = reinterpret_cast<float4*>(mine);
  float* const ebuf = reinterpret_cast<float*>(mine + S::kRows);
  auto idx_buf = [&](int k) {
    return reinterpret_cast<int64_t*>(mine + (S::kRows + S::kEnv) + k * S::kIdx);
  };
  // order[lo..hi) -> index buffer k (if the segment fits a chunk).
  auto stage_idx = [&](int64_t lo, int64_t hi, int k) {
    if (hi - lo > Q::CHUNK) return;
    int64_t* dst = idx_buf(k);
    for (int64_t i = lane; i < hi - lo; i += kWarp) cp_async8(dst + i, a.order + lo + i);
  };
  // Rows (and envelopes) of a staged segment, gathered by its staged indices.
  auto stage_rows = [&](int64_t lo, int64_t hi, int k) {
    if (hi - lo > Q::CHUNK) return;
    const int rows = quad_rows<LP>(lo, hi, g);
    const int64_t* idx = idx_buf(k);
    float4* rb = rbuf;
#pragma unroll
    for (int t = 0; t < Q::T; ++t)
      if (t < rows) {
        const int64_t e = idx[g + t * Q::G];
        cp_async16(rb + t * kWarp + lane, a.x + e * (4 * LP) + 4 * q);
      }
    if constexpr (kEnv) {
      float* eb = ebuf;
#pragma unroll
      for (int j = 0; j < Q::T / LP; ++j) {
        const int t = q + j * LP;
        if (t < rows) cp_async4(eb + t * Q::G + g, a.env + idx[g + t * Q::G]);
      }
    }
  };
  const int64_t* off = a.mp.offsets;
  // o[0..3] = offsets[n .. n+3] (clamped at the partition's last end).
  int64_t o0 = __ldg(off + n0), o1 = __ldg(off + n0 + 1);
  int64_t o2 = n0 + 1 < n1 ? __ldg(off + n0 + 2) : o1;
  int64_t o3 = n0 + 2 < n1 ? __ldg(off + n0 + 3) : o2;
  stage_idx(o0, o1, 0);
  cp_async_commit();
  cp_async_wait<0>();
  __syncwarp();
  if (n0 + 1 < n1) stage_idx(o1, o2, 1);
  stage_rows(o0, o1, 0);
  cp_async_commit();
  int kb = 0;  // index buffer of segment n
  for (int64_t n = n0; n < n1; ++n) {
    cp_async_wait<0>();  // segment n's rows, segment n+1's indices
    __syncwarp();
    const int64_t o4 = n + 3 < n1 ? __ldg(off + n + 4) : o3;
    const int k1 = kb == 2 ? 0 : kb + 1;
    const int k2 = k1 == 2 ? 0 : k1 + 1;
    if (n + 2 < n1) stage_idx(o2, o3, k2);
    cp_async_commit();
    // One row buffer: segment n+1's rows are gathered into it as soon as
    // segment n's are in registers.
    const auto refill = [&] {
      __syncwarp();  // every lane has read the row buffer
      if (n + 1 < n1) stage_rows(o1, o2, k1);
      cp_async_commit();
    };
    if (o1 - o0 <= kGatherShort * Q::G) {
      lean_whole<LP, kEnv, kGatherShort>(a, n, o0, o1, g, q, rbuf, ebuf, idx_buf(kb), refill);
    } else if (o1 - o0 <= Q::CHUNK) {
      lean_whole<LP, kEnv>(a, n, o0, o1, g, q, rbuf, ebuf, idx_buf(kb), refill);
    } else {
      refill();
      lean_big<LP, kEnv>(a, n, o0, o1, g, q);
    }
    __syncwarp();  // segment n's index buffer is free for segment n+3
    o0 = o1;
    o1 = o2;
    o2 = o3;
    o3 = o4;
    kb = k1;
  }
  cp_async_wait<0>();
}

// ---- backward -------------------------------------------------------------

// grad_logit for slots [lo, hi) given the final S; also grad_env when one
// warp covers all channels (out_env != NULL).
template <int NC, int G>
__device__ __forceinline__ void smx_bwd_write(const SmxArgs& a, int64_t lo,
                                              int64_t hi, int g,
                                              const int64_t (&ch)[NC],
                                              const bool (&ok)[NC],
                                              const float (&S)[NC]) {
  using Sh = SmxShape<NC, G>;
  const int64_t C = a.channels;
  // Lanes of one group handle the same edge, so the trip count is uniform
  // within a group; groups may differ by one iteration, hence the explicit
  // group-level mask for the channel reduction.
  const int64_t count = hi - lo;
  const int64_t iters = (count + G - 1) / G;
  for (int64_t t = 0; t < iters; ++t) {
    const int64_t s = lo + g + t * G;
    const bool live = s < hi;
    float rowsum = 0.0f;
    int64_t e = 0;
    if (live) {
      e = a.order ? __ldg(a.order + s) : s;
#pragma unroll
      for (int k = 0; k < NC; ++k)
        if (ok[k]) {
          const int64_t idx = e * C + ch[k];
          const float gl = __ldg(a.x + idx) * (__ldg(a.y + idx) - S[k]);
          a.out[idx] = gl;
          rowsum += gl;
        }
    }
    if (a.out_env) {
      rowsum = group_sum(rowsum, Sh::LPG);
      if (live && lane_id() % Sh::LPG == 0) {
        const float env = a.env ? __ldg(a.env + e) : 1.0f;
        a.out_env[e] = env > 0.0f ? rowsum * 2.0f / env : 0.0f;
      }
    }
  }
}

template <int NC, int G>
__global__ void __launch_bounds__(kBlock) segment_softmax_bwd_kernel(SmxArgs a) {
  using S = SmxShape<NC, G>;
  const int64_t p = global_warp();
  if (p >= a.mp.parts) return;
  const int lane = lane_id();
  const int tile = blockIdx.y;
  const int g = lane / S::LPG;
  const int64_t C = a.channels;
  int64_t ch[NC];
  bool ok[NC];
#pragma unroll
  for (int k = 0; k < NC; ++k) {
    ch[k] = lane_channel<NC, G>(lane, tile, k);
    ok[k] = ch[k] < C;
  }
  SegCursor cur(a.mp, part_range(a.mp, p));
  while (cur.next()) {
    const int64_t n = cur.node;
    const bool whole = cur.kind == kWhole;
    float sum[NC];
#pragma unroll
    for (int k = 0; k < NC; ++k) sum[k] = 0.0f;
    for (int64_t s = cur.lo + g; s < cur.hi; s += G) {
      const int64_t e = a.order ? __ldg(a.order + s) : s;
#pragma unroll
      for (int k = 0; k < NC; ++k)
        if (ok[k]) {
          const int64_t idx = e * C + ch[k];
          sum[k] = fmaf(__ldg(a.x + idx), __ldg(a.y + idx), sum[k]);
        }
    }
#pragma unroll
    for (int k = 0; k < NC; ++k) sum[k] = xor_sum(sum[k], S::LPG);
    if (whole) {
#pragma unroll
      for (int k = 0; k < NC; ++k)
        if (a.xn && ok[k]) {
          const float a0 = __ldg(a.xn + n * C + ch[k]);
          const float g0 = __ldg(a.yn + n * C + ch[k]);
          sum[k] = fmaf(a0, g0, sum[k]);
          if (g == 0) a.out_null[n * C + ch[k]] = a0 * (g0 - sum[k]);
        }
      smx_bwd_write<NC, G>(a, cur.lo, cur.hi, g, ch, ok, sum);
      continue;
    }
    float* mine = a.ss.slot(p, cur.kind);
    if (g == 0) {
#pragma unroll
      for (int k = 0; k < NC; ++k)
        if (ok[k]) __stcg(mine + ch[k], sum[k]);
    }
    const int64_t first = a.mp.part_of_first_edge(n);
    const int64_t last = a.mp.part_of_end(n);
    if (!arrive_last(a.ss, first, last, tile)) continue;
    if (g == 0) {
      float* fin = a.final_stats + last * 2 * a.cpad;
#pragma unroll
      for (int k = 0; k < NC; ++k) {
        if (!ok[k]) continue;
        float total = 0.0f;
        for (int64_t q = first; q <= last; ++q)
          total += __ldcg(a.ss.slot(q, q == last ? kHead : kTail) + ch[k]);
        if (a.xn) {
          const float a0 = __ldg(a.xn + n * C + ch[k]);
          const float g0 = __ldg(a.yn + n * C + ch[k]);
          total = fmaf(a0, g0, total);
          a.out_null[n * C + ch[k]] = a0 * (g0 - total);
        }
        __stcg(fin + ch[k], total);
      }
    }
  }
}

template <int NC, int G>
__global__ void __launch_bounds__(kBlock) segment_softmax_bwd_split_kernel(SmxArgs a) {
  using S = SmxShape<NC, G>;
  const int64_t p = global_warp();
  if (p >= a.mp.parts) return;
  const int lane = lane_id();
  const int tile = blockIdx.y;
  const int g = lane / S::LPG;
  int64_t ch[NC];
  bool ok[NC];
#pragma unroll
  for (int k = 0; k < NC; ++k) {
    ch[k] = lane_channel<NC, G>(lane, tile, k);
    ok[k] = ch[k] < a.channels;
  }
  SegCursor cur(a.mp, part_range(a.mp, p));
  while (cur.next()) {
    if (cur.kind == kWhole) continue;
    const int64_t last = a.mp.part_of_end(cur.node);
    const float* fin = a.final_stats + last * 2 * a.cpad;
    float sum[NC];
#pragma unroll
    for (int k = 0; k < NC; ++k) sum[k] = ok[k] ? __ldcg(fin + ch[k]) : 0.0f;
    smx_bwd_write<NC, G>(a, cur.lo, cur.hi, g, ch, ok, sum);
  }
}

// ---- backward, quad-vector form (C % 4 == 0, C <= 128) -----------------------
// Same lane layout as the forward quad kernel (LP lanes per row, G rows side
// by side, T rows per lane per chunk).  Per segment: S[c] = sum_e alpha g
// (+ null_alpha g0) from 16-byte loads of alpha and grad_alpha, a butterfly
// over the G groups, then grad_logit = alpha (g - S) and, per row,
// grad_env = 2 / env * sum_c grad_logit (a butterfly over the row's LP lanes).
// A piece that fits one chunk keeps its rows in registers between the sum
// and the write.  Split segments publish partial S; the last piece combines
// them and writes segments of up to kSelfWrite edges itself, longer ones in
// the equally partitioned second pass.
template <int LP, int TT = QuadSmx<LP>::T>
__device__ __forceinline__ void quad_bwd_load(const SmxArgs& a, int64_t base, int64_t hi, int g,
                                              int q, bool qok, float4 (&al)[TT],
                                              float4 (&gr)[TT]) {
  using Q = QuadSmx<LP>;
  const int mine = qok ? quad_rows_n<LP, TT>(base, hi, g) : 0;
  const int64_t cq = a.channels / 4;
#pragma unroll
  for (int t = 0; t < TT; ++t) {
    al[t] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    gr[t] = al[t];
    if (t < mine) {
      const int64_t slot = base + g + static_cast<int64_t>(t) * Q::G;
      const int64_t e = a.order ? __ldg(a.order + slot) : slot;
      al[t] = __ldg(reinterpret_cast<const float4*>(a.x) + e * cq + q);
      gr[t] = __ldg(reinterpret_cast<const float4*>(a.y) + e * cq + q);
    }
  }
}

// Writes grad_logit (and grad_env) of slots base + g + t G from rows in registers.
template <int LP, int TT = QuadSmx<LP>::T>
__device__ __forceinline__ void quad_bwd_store(const SmxArgs& a, int64_t base, int64_t hi, int g,
                                               int q, bool qok, const float4 (&al)[TT],
                                               const float4 (&gr)[TT], const float (&S)[4]) {
  using Q = QuadSmx<LP>;
  const int rows = quad_rows_n<LP, TT>(base, hi, g);
  const int64_t cq = a.channels / 4;
#pragma unroll
  for (int t = 0; t < TT; ++t) {
    const int64_t slot = base + g + static_cast<int64_t>(t) * Q::G;
    const bool live = t < rows;
    const int64_t e = live ? (a.order ? __ldg(a.order + slot) : slot) : 0;
    float4 gl = make_float4(al[t].x * (gr[t].x - S[0]), al[t].y * (gr[t].y - S[1]),
                            al[t].z * (gr[t].z - S[2]), al[t].w * (gr[t].w - S[3]));
    if (!qok) gl = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (live && qok) reinterpret_cast<float4*>(a.out)[e * cq + q] = gl;
    if (a.out_env) {
      float rowsum = (gl.x + gl.y) + (gl.z + gl.w);
      if constexpr (LP > 1) rowsum = group_sum(rowsum, LP);
      if (live && q == 0) {
        const float env = a.env ? __ldg(a.env + e) : 1.0f;
        a.out_env[e] = env > 0.0f ? rowsum * 2.0f / env : 0.0f;
      }
    }
  }
}

template <int LP, bool kSplitPass>
__global__ void __launch_bounds__(kBlock, 2) segment_softmax_quad_bwd_kernel(SmxArgs a) {
  using Q = QuadSmx<LP>;
  const int64_t p = global_warp();
  if (p >= a.mp.parts) return;
  const int lane = lane_id();
  const int g = lane / LP;
  const int q = lane % LP;
  const int64_t C = a.channels;
  const bool qok = 4 * q < C;
  if constexpr (kSplitPass) {
    if (*reinterpret_cast<volatile int*>(a.big_split) == 0) return;
  }
  SegCursor cur(a.mp, part_range(a.mp, p));
  while (cur.next()) {
    const int64_t n = cur.node;
    const bool whole = cur.kind == kWhole;
    float4 al[Q::T], gr[Q::T];
    float S[4];
    if constexpr (kSplitPass) {
      if (whole) continue;
      if (__ldg(a.mp.offsets + n + 1) - __ldg(a.mp.offsets + n) <= kSelfWrite) continue;
      const float* fin = a.final_stats + a.mp.part_of_end(n) * 2 * a.cpad;
#pragma unroll
      for (int i = 0; i < 4; ++i) S[i] = qok ? __ldcg(fin + 4 * q + i) : 0.0f;
#pragma unroll 1
      for (int64_t base = cur.lo; base < cur.hi; base += Q::CHUNK) {
        quad_bwd_load<LP>(a, base, cur.hi, g, q, qok, al, gr);
        quad_bwd_store<LP>(a, base, cur.hi, g, q, qok, al, gr, S);
      }
      continue;
    } else {
      const bool one_chunk = cur.hi - cur.lo <= Q::CHUNK;
#pragma unroll
      for (int i = 0; i < 4; ++i) S[i] = 0.0f;
#pragma unroll 1
      for (int64_t base = cur.lo; base < cur.hi; base += Q::CHUNK) {
        quad_bwd_load<LP>(a, base, cur.hi, g, q, qok, al, gr);
#pragma unroll
        for (int t = 0; t < Q::T; ++t) {
          S[0] = fmaf(al[t].x, gr[t].x, S[0]);
          S[1] = fmaf(al[t].y, gr[t].y, S[1]);
          S[2] = fmaf(al[t].z, gr[t].z, S[2]);
          S[3] = fmaf(al[t].w, gr[t].w, S[3]);
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
        for (int st = LP; st < kWarp; st <<= 1) S[i] += __shfl_xor_sync(kFull, S[i], st);
      if (whole) {
        if (a.xn && qok) {
          const float4 a0 = __ldg(reinterpret_cast<const float4*>(a.xn + n * C) + q);
          const float4 g0 = __ldg(reinterpret_cast<const float4*>(a.yn + n * C) + q);
          S[0] = fmaf(a0.x, g0.x, S[0]);
          S[1] = fmaf(a0.y, g0.y, S[1]);
          S[2] = fmaf(a0.z, g0.z, S[2]);
          S[3] = fmaf(a0.w, g0.w, S[3]);
          if (g == 0)
            reinterpret_cast<float4*>(a.out_null + n * C)[q] =
                make_float4(a0.x * (g0.x - S[0]), a0.y * (g0.y - S[1]), a0.z * (g0.z - S[2]),
                            a0.w * (g0.w - S[3]));
        }
        if (one_chunk) {
          quad_bwd_store<LP>(a, cur.lo, cur.hi, g, q, qok, al, gr, S);
        } else {
#pragma unroll 1
          for (int64_t base = cur.lo; base < cur.hi; base += Q::CHUNK) {
            quad_bwd_load<LP>(a, base, cur.hi, g, q, qok, al, gr);
            quad_bwd_store<LP>(a, base, cur.hi, g, q, qok, al, gr, S);
          }
        }
        continue;
      }
      // Split segment: publish the partial S; the last piece combines.
      float* mine = a.ss.slot(p, cur.kind);
      if (g == 0 && qok) {
#pragma unroll
        for (int i = 0; i < 4; ++i) __stcg(mine + 4 * q + i, S[i]);
      }
      const int64_t first = a.mp.part_of_first_edge(n);
      const int64_t last = a.mp.part_of_end(n);
      if (!arrive_last(a.ss, first, last, 0)) continue;
      float* fin = a.final_stats + last * 2 * a.cpad;
      float total[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      if (qok) {
        for (int64_t qq = first; qq <= last; ++qq) {
          const float* sq = a.ss.slot(qq, qq == last ? kHead : kTail);
#pragma unroll
          for (int i = 0; i < 4; ++i) total[i] += __ldcg(sq + 4 * q + i);
        }
        if (a.xn) {
          const float4 a0 = __ldg(reinterpret_cast<const float4*>(a.xn + n * C) + q);
          const float4 g0 = __ldg(reinterpret_cast<const float4*>(a.yn + n * C) + q);
          total[0] = fmaf(a0.x, g0.x, total[0]);
          total[1] = fmaf(a0.y, g0.y, total[1]);
          total[2] = fmaf(a0.z, g0.z, total[2]);
          total[3] = fmaf(a0.w, g0.w, total[3]);
          if (g == 0)
            reinterpret_cast<float4*>(a.out_null + n * C)[q] =
                make_float4(a0.x * (g0.x - total[0]), a0.y * (g0.y - total[1]),
                            a0.z * (g0.z - total[2]), a0.w * (g0.w - total[3]));
        }
        if (g == 0) {
#pragma unroll
          for (int i = 0; i < 4; ++i) __stcg(fin + 4 * q + i, total[i]);
        }
      }
      const int64_t seg_lo = __ldg(a.mp.offsets + n);
      const int64_t seg_hi = __ldg(a.mp.offsets + n + 1);
      if (seg_hi - seg_lo <= kSelfWrite) {
#pragma unroll 1
        for (int64_t base = seg_lo; base < seg_hi; base += Q::CHUNK) {
          quad_bwd_load<LP>(a, base, seg_hi, g, q, qok, al, gr);
          quad_bwd_store<LP>(a, base, seg_hi, g, q, qok, al, gr, total);
        }
      } else if (lane == 0) {
        atomicExch(a.big_split, 1);
      }
    }
  }
}

// Adds the null term to S (S += null_alpha g0) and writes grad_null_logit.
template <int LP>
__device__ __forceinline__ void bwd_null(const SmxArgs& a, int64_t n, int g, int q, bool qok,
                                         float (&S)[4]) {
  if (!a.xn || !qok) return;
  const int64_t C = a.channels;
  const float4 a0 = __ldg(reinterpret_cast<const float4*>(a.xn + n * C) + q);
  const float4 g0 = __ldg(reinterpret_cast<const float4*>(a.yn + n * C) + q);
  S[0] = fmaf(a0.x, g0.x, S[0]);
  S[1] = fmaf(a0.y, g0.y, S[1]);
  S[2] = fmaf(a0.z, g0.z, S[2]);
  S[3] = fmaf(a0.w, g0.w, S[3]);
  if (g == 0)
    reinterpret_cast<float4*>(a.out_null + n * C)[q] =
        make_float4(a0.x * (g0.x - S[0]), a0.y * (g0.y - S[1]), a0.z * (g0.z - S[2]),
                    a0.w * (g0.w - S[3]));
}

// Backward over whole-segment partitions (as the forward whole kernel): warp
// p takes every segment whose start diagonal lies in its partition, so no
// partial S is published and there is no second pass.  A segment of up to one
// chunk keeps its rows in registers between the sum and the write; a longer
// one reads its rows twice (the second time from L1).

// Rows per lane per chunk of the register form.  Four rows, at four CTAs per
// SM (64 registers), measured faster than eight rows kept in registers at
// two or three CTAs: the kernel waits on memory, and a longer segment
// re-reads its rows from L1 in the second pass.
constexpr int kBwdT = 4;

// One whole segment [lo, hi) from global memory (register form).
template <int LP, int TT>
__device__ __forceinline__ void bwd_segment_global(const SmxArgs& a, int64_t n, int64_t lo,
                                                   int64_t hi, int g, int q, bool qok) {
  using Q = QuadSmx<LP>;
  constexpr int64_t kChunk = static_cast<int64_t>(Q::G) * TT;
  float4 al[TT], gr[TT];
  float S[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 1
  for (int64_t base = lo; base < hi; base += kChunk) {
    quad_bwd_load<LP, TT>(a, base, hi, g, q, qok, al, gr);
#pragma unroll
    for (int t = 0; t < TT; ++t) {
      S[0] = fmaf(al[t].x, gr[t].x, S[0]);
      S[1] = fmaf(al[t].y, gr[t].y, S[1]);
      S[2] = fmaf(al[t].z, gr[t].z, S[2]);
      S[3] = fmaf(al[t].w, gr[t].w, S[3]);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
    for (int st = LP; st < kWarp; st <<= 1) S[i] += __shfl_xor_sync(kFull, S[i], st);
  bwd_null<LP>(a, n, g, q, qok, S);
  if (hi - lo <= kChunk) {
    quad_bwd_store<LP, TT>(a, lo, hi, g, q, qok, al, gr, S);
  } else {
#pragma unroll 1
    for (int64_t base = lo; base < hi; base += kChunk) {
      quad_bwd_load<LP, TT>(a, base, hi, g, q, qok, al, gr);
      quad_bwd_store<LP, TT>(a, base, hi, g, q, qok, al, gr, S);
    }
  }
}

template <int LP>
__global__ void __launch_bounds__(kBlock, 4) segment_softmax_whole_bwd_kernel(SmxArgs a) {
  const int64_t p = global_warp();
  if (p >= a.mp.parts) return;
  const int lane = lane_id();
  const int g = lane / LP;
  const int q = lane % LP;
  const bool qok = 4 * q < a.channels;
  const int64_t n0 = a.mp.starts_before(p * a.mp.ipc);
  const int64_t n1 = a.mp.starts_before((p + 1) * a.mp.ipc);
  if (n0 >= n1) return;
  const int64_t* off = a.mp.offsets;
  int64_t lo = __ldg(off + n0);
  int64_t hi = __ldg(off + n0 + 1);
  for (int64_t n = n0; n < n1; ++n) {
    const int64_t nhi = n + 1 < n1 ? __ldg(off + n + 2) : hi;
    bwd_segment_global<LP, kBwdT>(a, n, lo, hi, g, q, qok);
    lo = hi;
    hi = nhi;
  }
}

// Backward for C = 4 LP exactly (LP <= 2) with shared-memory staging, as the
// forward whole kernel: a segment's alpha, grad_alpha and envelope rows are
// staged (cp.async), the first pass reads them into registers (S), the warp's
// one stage buffer is refilled with the next segment at once, and the second
// pass (grad_logit, grad_env) runs from registers while those copies land.
// The rows of a lane are summed in the same order as in the register form,
// so both give the same bits.  Segments longer than a chunk take the
// register form.  Four-warp CTAs, 8.7 KB of buffer per warp at LP = 2 (the
// width it is used for), four CTAs per SM.
constexpr int kStagedBwdBlock = 128;
constexpr int kStagedBwdMinBlocks = 4;

template <int LP>
struct BwdStage {
  static constexpr int G = kWarp / LP;
  static constexpr int T = 8;
  static constexpr int CHUNK = G * T;
  static constexpr int kRowsF4 = T * kWarp;  // float4 per staged array
  static constexpr size_t kBytes = 2 * sizeof(float4) * kRowsF4 + sizeof(float) * CHUNK;
  static constexpr size_t kWarpBytes = 2 * kBytes;
  static_assert(kBytes % 16 == 0, "stage buffers must stay 16-byte aligned");
};
constexpr int kBwdShort = 6;  // row slots per lane for segments within 3/4 of a chunk

template <int LP>
__device__ __forceinline__ void bwd_stage(const SmxArgs& a, int64_t lo, int64_t hi, int g, int q,
                                          char* buf, const int64_t* idx = nullptr) {
  using B = BwdStage<LP>;
  constexpr int C = 4 * LP;
  const int rows = quad_rows_n<LP, B::T>(lo, hi, g);
  const int lane = g * LP + q;
  float4* al = reinterpret_cast<float4*>(buf);
  float4* gr = al + B::kRowsF4;
  float* env = reinterpret_cast<float*>(gr + B::kRowsF4);
#pragma unroll
  for (int t = 0; t < B::T; ++t) {
    if (t < rows) {
      const int64_t slot = lo + g + static_cast<int64_t>(t) * B::G;
      const int64_t e = idx ? idx[g + t * B::G] : a.order ? __ldg(a.order + slot) : slot;
      cp_async16(al + t * kWarp + lane, a.x + e * C + 4 * q);
      cp_async16(gr + t * kWarp + lane, a.y + e * C + 4 * q);
      if (a.env && q == 0) cp_async4(env + t * B::G + g, a.env + e);
    }
  }
}

// TT row slots per lane (<= BwdStage<LP>::T): a segment that fits fewer
// slots skips the empty ones (they add nothing, so the bits are the same).
// The rows (and envelopes) go to registers in the first pass; `refill` runs
// once the stage buffer has been read (a single-buffer caller stages the next
// segment into it there, while this one's second pass runs).
template <int LP, int TT = BwdStage<LP>::T, typename Refill = NoRefill>
__device__ __forceinline__ void bwd_segment_staged(const SmxArgs& a, int64_t n, int64_t lo,
                                                   int64_t hi, int g, int q, const char* buf,
                                                   const int64_t* idx = nullptr,
                                                   Refill refill = Refill{}) {
  using B = BwdStage<LP>;
  const int rows = quad_rows_n<LP, TT>(lo, hi, g);
  const int lane = g * LP + q;
  const uint32_t al_s = smem_addr(buf) + 16u * lane;
  const uint32_t gr_s = al_s + 16u * B::kRowsF4;
  const uint32_t env_s = smem_addr(buf) + 32u * B::kRowsF4 + 4u * g;
  float S[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  float4 ah[TT], gh[TT];  // the rows, held for the second pass
  float eh[TT];
  int64_t ih[TT];
#pragma unroll
  for (int t = 0; t < TT; ++t) {
    ah[t] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    gh[t] = ah[t];
    eh[t] = 1.0f;
    ih[t] = 0;
    if (t < rows) {
      ah[t] = lds_f4(al_s + 16u * t * kWarp);
      gh[t] = lds_f4(gr_s + 16u * t * kWarp);
      if (a.env && a.out_env && q == 0) eh[t] = lds_f32(env_s + 4u * t * B::G);
      if (idx) ih[t] = lds_i64(smem_addr(idx) + 8u * (g + t * B::G));
      S[0] = fmaf(ah[t].x, gh[t].x, S[0]);
      S[1] = fmaf(ah[t].y, gh[t].y, S[1]);
      S[2] = fmaf(ah[t].z, gh[t].z, S[2]);
      S[3] = fmaf(ah[t].w, gh[t].w, S[3]);
    }
  }
  refill();
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int st = LP; st < kWarp; st <<= 1) S[i] += __shfl_xor_sync(kFull, S[i], st);
  bwd_null<LP>(a, n, g, q, true, S);
#pragma unroll
  for (int t = 0; t < TT; ++t) {
    const bool live = t < rows;
    const float4 al = ah[t], gr = gh[t];
    const float4 gl = make_float4(al.x * (gr.x - S[0]), al.y * (gr.y - S[1]),
                                  al.z * (gr.z - S[2]), al.w * (gr.w - S[3]));
    const int64_t slot = lo + g + static_cast<int64_t>(t) * B::G;
    const int64_t e = !live ? 0 : idx ? ih[t] : a.order ? __ldg(a.order + slot) : slot;
    if (live) reinterpret_cast<float4*>(a.out)[e * LP + q] = gl;
    if (a.out_env) {
      float rowsum = (gl.x + gl.y) + (gl.z + gl.w);
      if constexpr (LP > 1) rowsum = group_sum(rowsum, LP);
      if (live && q == 0) {
        const float env = eh[t];
        a.out_env[e] = env > 0.0f ? rowsum * 2.0f / env : 0.0f;
      }
    }
  }
}

// One stage buffer per warp: segment n's rows are read into registers, the
// buffer is refilled with segment n+1 at once, and segment n's second pass
// runs while those copies are in flight.  Half the shared memory of a double
// buffer, so four CTAs per SM (register-bound) instead of three.
template <int LP>
__global__ void __launch_bounds__(kStagedBwdBlock, kStagedBwdMinBlocks)
    segment_softmax_staged_bwd_kernel(SmxArgs a) {
  using B = BwdStage<LP>;
  extern __shared__ float4 quad_smem[];
  const int64_t p = global_warp();
  if (p >= a.mp.parts) return;
  const int lane = lane_id();
  const int g = lane / LP;
  const int q = lane % LP;
  const int64_t n0 = a.mp.starts_before(p * a.mp.ipc);
  const int64_t n1 = a.mp.starts_before((p + 1) * a.mp.ipc);
  if (n0 >= n1) return;
  char* buf = reinterpret_cast<char*>(quad_smem) + (threadIdx.x >> 5) * B::kBytes;
  const int64_t* off = a.mp.offsets;
  // Segment n is [lo, hi); the next one ends at nhi.
  int64_t lo = __ldg(off + n0), hi = __ldg(off + n0 + 1);
  int64_t nhi = n0 + 1 < n1 ? __ldg(off + n0 + 2) : hi;
  if (hi - lo <= B::CHUNK) bwd_stage<LP>(a, lo, hi, g, q, buf);
  cp_async_commit();
  for (int64_t n = n0; n < n1; ++n) {
    const int64_t nnhi = n + 2 < n1 ? __ldg(off + n + 3) : nhi;
    cp_async_wait<0>();  // this segment's copies have landed
    __syncwarp();
    const auto refill = [&] {
      __syncwarp();  // every lane has read the buffer
      if (n + 1 < n1 && nhi - hi <= B::CHUNK) bwd_stage<LP>(a, hi, nhi, g, q, buf);
      cp_async_commit();
    };
    // Segments that fit 3/4 of the chunk take 6 row slots per lane instead
    // of 8 (same bits).
    if (hi - lo <= kBwdShort * B::G) {
      bwd_segment_staged<LP, kBwdShort>(a, n, lo, hi, g, q, buf, nullptr, refill);
    } else if (hi - lo <= B::CHUNK) {
      bwd_segment_staged<LP>(a, n, lo, hi, g, q, buf, nullptr, refill);
    } else {
      refill();
      bwd_segment_global<LP, kBwdT>(a, n, lo, hi, g, q, true);
    }
    lo = hi;
    hi = nhi;
    nhi = nnhi;
  }
  cp_async_wait<0>();
}

// Staged backward with a permuted storage order (C = 8): the three-stage
// pipeline of the forward gather kernel (order slice two segments ahead,
// gathered alpha / grad_alpha / envelope rows one segment ahead in the
// warp's one row buffer, refilled once the first pass has the rows in
// registers; outputs scattered through the staged indices).
template <int LP>
struct GatherBwdStage {
  using B = BwdStage<LP>;
  static constexpr size_t kIdx = sizeof(int64_t) * B::CHUNK;
  static constexpr size_t kWarpBytes = B::kBytes + 3 * kIdx;  // one row buffer
};

template <int LP>
__global__ void __launch_bounds__(kStagedBwdBlock, 3)
    segment_softmax_gather_bwd_kernel(SmxArgs a) {
  using B = BwdStage<LP>;
  using S = GatherBwdStage<LP>;
  extern __shared__ float4 quad_smem[];
  const int64_t p = global_warp();
  if (p >= a.mp.parts) return;
  const int lane = lane_id();
  const int g = lane / LP;
  const int q = lane % LP;
  const int64_t n0 = a.mp.starts_before(p * a.mp.ipc);
  const int64_t n1 = a.mp.starts_before((p + 1) * a.mp.ipc);
  if (n0 >= n1) return;
  char* mine = reinterpret_cast<char*>(quad_smem) + (threadIdx.x >> 5) * S::kWarpBytes;
  char* const buf = mine;
  auto idx_buf = [&](int k) {
    return reinterpret_cast<int64_t*>(mine + B::kBytes + k * S::kIdx);
  };
  auto stage_idx = [&](int64_t lo, int64_t hi, int k) {
    if (hi - lo > B::CHUNK) return;
    int64_t* dst = idx_buf(k);
    for (int64_t i = lane; i < hi - lo; i += kWarp) cp_async8(dst + i, a.order + lo + i);
  };
  const int64_t* off = a.mp.offsets;
  int64_t o0 = __ldg(off + n0), o1 = __ldg(off + n0 + 1);
  int64_t o2 = n0 + 1 < n1 ? __ldg(off + n0 + 2) : o1;
  int64_t o3 = n0 + 2 < n1 ? __ldg(off + n0 + 3) : o2;
  stage_idx(o0, o1, 0);
  cp_async_commit();
  cp_async_wait<0>();
  __syncwarp();
  if (n0 + 1 < n1) stage_idx(o1, o2, 1);
  if (o1 - o0 <= B::CHUNK) bwd_stage<LP>(a, o0, o1, g, q, buf, idx_buf(0));
  cp_async_commit();
  int kb = 0;
  for (int64_t n = n0; n < n1; ++n) {
    cp_async_wait<0>();  // segment n's rows, segment n+1's indices
    __syncwarp();
    const int64_t o4 = n + 3 < n1 ? __ldg(off + n + 4) : o3;
    const int k1 = kb == 2 ? 0 : kb + 1;
    const int k2 = k1 == 2 ? 0 : k1 + 1;
    if (n + 2 < n1) stage_idx(o2, o3, k2);
    cp_async_commit();
    // One row buffer: segment n+1's rows are gathered into it as soon as
    // segment n's are in registers.
    const auto refill = [&] {
      __syncwarp();  // every lane has read the row buffer
      if (n + 1 < n1 && o2 - o1 <= B::CHUNK) bwd_stage<LP>(a, o1, o2, g, q, buf, idx_buf(k1));
      cp_async_commit();
    };
    if (o1 - o0 <= kBwdShort * B::G) {
      bwd_segment_staged<LP, kBwdShort>(a, n, o0, o1, g, q, buf, idx_buf(kb), refill);
    } else if (o1 - o0 <= B::CHUNK) {
      bwd_segment_staged<LP>(a, n, o0, o1, g, q, buf, idx_buf(kb), refill);
    } else {
      refill();
      bwd_segment_global<LP, kBwdT>(a, n, o0, o1, g, q, true);
    }
    __syncwarp();  // segment n's index buffer is free for segment n+3
    o0 = o1;
    o1 = o2;
    o2 = o3;
    o3 = o4;
    kb = k1;
  }
  cp_async_wait<0>();
}

// grad_env for channel counts wider than one warp tile.
__global__ void __launch_bounds__(kBlock)
    segment_softmax_env_kernel(const float* __restrict__ grad_logit,
                               const float* __restrict__ env,
                               float* __restrict__ grad_env, int64_t n_edges,
                               int64_t channels) {
  const int64_t warps = static_cast<int64_t>(gridDim.x) * kWarpsPerBlock;
  for (int64_t e = global_warp(); e < n_edges; e += warps) {
    float sum = 0.0f;
    for (int64_t c = lane_id(); c < channels; c += kWarp)
      sum += __ldg(grad_logit + e * channels + c);
    sum = xor_sum(sum, 1);
    if (lane_id() == 0) {
      const float g = env ? __ldg(env + e) : 1.0f;
      grad_env[e] = g > 0.0f ? sum * 2.0f / g : 0.0f;
    }
  }
}

// ---- host -----------------------------------------------------------------

using SmxKernel = void (*)(SmxArgs);
struct SmxConfig {
  SmxKernel main = nullptr, split = nullptr;
  SmxKernel hub = nullptr;  // whole forward: the dependent pass over hub segments
  int64_t tc = 0, tiles = 1;
  size_t main_smem = 0;  // dynamic shared memory of the main launch
  int block = kBlock;    // threads per CTA of the main launch
};

template <int NC, int G>
SmxConfig smx_make(bool backward) {
  SmxConfig c;
  c.main = backward ? segment_softmax_bwd_kernel<NC, G> : segment_softmax_fwd_kernel<NC, G>;
  c.split = backward ? segment_softmax_bwd_split_kernel<NC, G>
                     : segment_softmax_fwd_split_kernel<NC, G>;
  c.tc = SmxShape<NC, G>::TC;
  return c;
}

template <int LP, bool kEnv, bool kLean = false>
SmxConfig quad_make_env() {
  SmxConfig c;
  if constexpr (kLean) {
    c.main = segment_softmax_whole_kernel<LP, kEnv>;
    c.split = nullptr;  // no segment is split
    c.hub = segment_softmax_hub_kernel<LP, kEnv>;
    c.block = WholeShape<LP>::kThreads;
  } else {
    c.main = segment_softmax_quad_kernel<LP, false, kEnv>;
    c.split = segment_softmax_quad_kernel<LP, true, kEnv>;
  }
  c.tc = 4 * LP;
  c.tiles = 1;
  if constexpr (kLean)
    c.main_smem = (WholeShape<LP>::kThreads / kWarp) * WholeShape<LP>::kWarpBytes;
  else
    c.main_smem = quad_pipelined<LP>() ? kWarpsPerBlock * QuadStage<LP>::kWarpBytes : 0;
  return c;
}

template <int LP>
SmxConfig quad_make(bool env) {
  return env ? quad_make_env<LP, true>() : quad_make_env<LP, false>();
}

// C == 4 LP with a permuted storage order (C = 4 or 8): the gather kernel.
template <int LP, bool kEnv>
SmxConfig gather_make_env() {
  SmxConfig c;
  c.main = segment_softmax_gather_kernel<LP, kEnv>;
  c.split = nullptr;  // no segment is split
  c.tc = 4 * LP;
  c.tiles = 1;
  c.block = kGatherBlock;
  c.main_smem = (kGatherBlock / kWarp) * GatherStage<LP>::kWarpBytes;
  return c;
}
template <int LP>
SmxConfig gather_make(bool env) {
  return env ? gather_make_env<LP, true>() : gather_make_env<LP, false>();
}

// C == 4 LP with rows in storage order (C = 4, 8 or 16): whole-segment
// partitions.
template <int LP>
SmxConfig quad_make_lean(bool env) {
  return env ? quad_make_env<LP, true, true>() : quad_make_env<LP, false, true>();
}

template <int LP>
SmxConfig staged_bwd_make() {
  SmxConfig c;
  c.main = segment_softmax_staged_bwd_kernel<LP>;
  c.split = nullptr;  // no segment is split
  c.tc = 4 * LP;
  c.tiles = 1;
  c.block = kStagedBwdBlock;
  c.main_smem = (kStagedBwdBlock / kWarp) * BwdStage<LP>::kBytes;
  return c;
}

template <int LP>
SmxConfig gather_bwd_make() {
  SmxConfig c = staged_bwd_make<LP>();
  c.main = segment_softmax_gather_bwd_kernel<LP>;
  c.main_smem = (kStagedBwdBlock / kWarp) * GatherBwdStage<LP>::kWarpBytes;
  return c;
}

template <int LP>
SmxConfig quad_bwd_make() {
  SmxConfig c;
  c.main = segment_softmax_whole_bwd_kernel<LP>;
  c.split = nullptr;  // no segment is split
  c.tc = 4 * LP;
  c.tiles = 1;
  return c;
}

SmxConfig smx_config(int64_t channels, bool backward, bool quad_ok, bool env = true,
                     bool lean = false, bool gather = false) {
  SmxConfig c;
  if (!backward && quad_ok && gather) {
    if (channels == 4) return gather_make<1>(env);
    if (channels == 8) return gather_make<2>(env);
  }
  if (!backward && quad_ok && lean) {
    if (channels == 4) return quad_make_lean<1>(env);
    if (channels == 8) return quad_make_lean<2>(env);
    if (channels == 16) return quad_make_lean<4>(env);
  }
  // Staged backward at C = 8 (at C = 4 the register form measured faster);
  // with a storage order, its gather form.
  if (backward && quad_ok && channels == 8) return gather ? gather_bwd_make<2>() : staged_bwd_make<2>();
  if (backward && quad_ok && channels % 4 == 0 && channels <= 128) {
    switch (next_pow2(channels / 4)) {
      case 1: return quad_bwd_make<1>();
      case 2: return quad_bwd_make<2>();
      case 4: return quad_bwd_make<4>();
      case 8: return quad_bwd_make<8>();
      case 16: return quad_bwd_make<16>();
      default: return quad_bwd_make<32>();
    }
  }
  if (!backward && quad_ok && channels % 4 == 0 && channels <= 128) {
    switch (next_pow2(channels / 4)) {
      case 1: return quad_make<1>(env);
      case 2: return quad_make<2>(env);
      case 4: return quad_make<4>(env);
      case 8: return quad_make<8>(env);
      case 16: return quad_make<16>(env);
      default: return quad_make<32>(env);
    }
  }
  if (channels > 128) c = smx_make<8, 1>(backward);
  else if (channels > 64) c = smx_make<4, 1>(backward);
  else if (channels > 32) c = smx_make<2, 1>(backward);
  else {
    switch (next_pow2(channels)) {
      case 32: c = smx_make<1, 1>(backward); break;
      case 16: c = smx_make<1, 2>(backward); break;
      case 8: c = smx_make<1, 4>(backward); break;
      case 4: c = smx_make<1, 8>(backward); break;
      case 2: c = smx_make<1, 16>(backward); break;
      default: c = smx_make<1, 32>(backward); break;
    }
  }
  c.tiles = (channels + c.tc - 1) / c.tc;
  return c;
}

struct SmxLayout {
  SmxConfig cfg;
  PartitionPlan plan;
  int64_t cpad = 0;
  size_t bytes = 0;
  SplitSlots ss{};
  float* final_stats = nullptr;
  int64_t* hub_slot = nullptr;
  float* hub_stats = nullptr;
  unsigned long long* hub_flag = nullptr;
  int smem_status = BYSJ_OK;
};

SmxLayout smx_layout(int64_t n_edges, int64_t n_nodes, int64_t channels,
                     bool backward, void* ws, bool quad_ok = true, bool env = true,
                     bool lean = false, bool gather = false) {
  SmxLayout L;
  L.cfg = smx_config(channels, backward, quad_ok, env, lean, gather);
  const DeviceInfo& dev = current_device_info();
  L.smem_status = allow_dynamic_smem(reinterpret_cast<const void*>(L.cfg.main), L.cfg.main_smem);
  const int64_t warps_per_block = L.cfg.block / kWarp;
  const int64_t resident =
      static_cast<int64_t>(dev.sm_count) *
      resident_blocks(reinterpret_cast<const void*>(L.cfg.main), L.cfg.main_smem, L.cfg.block) *
      warps_per_block;
  int64_t warps = resident / L.cfg.tiles;
  if (warps < 1) warps = 1;
  L.plan = plan_partitions(n_edges, n_nodes, warps, 32);
  L.plan.blocks = static_cast<unsigned>((L.plan.parts + warps_per_block - 1) / warps_per_block);
  L.cpad = (channels + 3) / 4 * 4;
  Carver carve(ws);
  float* slots = carve.take<float>(static_cast<size_t>(L.plan.parts) * 2 * 2 * L.cpad);
  int* tickets = carve.take<int>(static_cast<size_t>(L.plan.parts) * L.cfg.tiles + 1);
  L.final_stats = carve.take<float>(static_cast<size_t>(L.plan.parts) * 2 * L.cpad);
  if (L.cfg.hub != nullptr) {
    L.hub_slot = carve.take<int64_t>(static_cast<size_t>(L.plan.parts));
    L.hub_stats = carve.take<float>(static_cast<size_t>(L.plan.parts) * 2 * 2 * L.cpad);
    L.hub_flag = carve.take<unsigned long long>(1);
  }
  L.bytes = carve.need;
  L.ss = SplitSlots{slots, tickets, 2 * L.cpad, static_cast<int>(L.cfg.tiles)};
  return L;
}

// A value per call that the hub flag (left in the workspace by earlier use)
// is unlikely to hold already; if it does, the hub pass only scans the
// partitions' hub slots, which the whole kernel always rewrites.
unsigned long long next_hub_epoch() {
  static std::atomic<unsigned long long> counter{0x9e3779b97f4a7c15ull};
  return counter.fetch_add(0x9e3779b97f4a7c15ull, std::memory_order_relaxed);
}

int smx_run(SmxArgs& a, const SmxLayout& L, int64_t n_edges, int64_t n_nodes,
            const int64_t* offsets, cudaStream_t s, const char* name) {
  // Tickets and the big-split flag after them start at zero (kernels that
  // split no segment have no second pass and use neither).
  int st = BYSJ_OK;
  if (L.cfg.split != nullptr)
    st = cuda_check(
        cudaMemsetAsync(L.ss.tickets, 0, sizeof(int) * (L.plan.parts * L.cfg.tiles + 1), s),
        "segment softmax: ticket reset");
  if (st) return st;
  a.mp = MergePath{offsets, n_nodes, n_edges, L.plan.ipc, L.plan.parts};
  a.ss = L.ss;
  a.final_stats = L.final_stats;
  a.big_split = L.ss.tickets + L.plan.parts * L.cfg.tiles;
  a.cpad = L.cpad;
  a.hub_slot = L.hub_slot;
  a.hub_stats = L.hub_stats;
  a.hub_flag = L.hub_flag;
  a.epoch = next_hub_epoch();
  // A hub is longer than a partition (so a partition owns at most one) and
  // than kHubRows rows (so short-segment frames never use the hub pass).
  a.hub_rows = L.plan.ipc > kHubRows ? L.plan.ipc : kHubRows;
  if (L.smem_status != BYSJ_OK) return L.smem_status;
  dim3 grid(L.plan.blocks, static_cast<unsigned>(L.cfg.tiles));
  L.cfg.main<<<grid, L.cfg.block, L.cfg.main_smem, s>>>(a);
  st = launch_check(name);
  if (st) return st;
  if (L.cfg.hub != nullptr && n_edges > kHubRows) {  // no hub fits a smaller frame
    // A programmatic dependent launch: the hub kernel's launch is processed
    // while the whole kernel drains, and its griddepcontrol.wait orders it
    // after the whole kernel (the usual frame has no hub, so this launch is
    // all it costs).
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(current_device_info().sm_count));
    cfg.blockDim = dim3(kHubWarps * kWarp);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    st = cuda_check(cudaLaunchKernelEx(&cfg, L.cfg.hub, a), "segment softmax: hub pass");
    if (st) return st;
    st = launch_check(name);
  }
  if (st || L.cfg.split == nullptr) return st;
  L.cfg.split<<<grid, kBlock, 0, s>>>(a);
  return launch_check(name);
}

int smx_check(int64_t n_edges, int64_t n_nodes, int64_t channels,
              const int64_t* offsets) {
  if (n_edges < 0 || n_nodes < 0 || channels <= 0)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "segment softmax: invalid sizes");
  if (n_nodes > 0 && offsets == nullptr)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "segment softmax: offsets is NULL");
  return BYSJ_OK;
}

}  // namespace
}  // namespace bysj

using namespace bysj;

extern "C" {

size_t bysj_segment_softmax_workspace_size(int64_t n_edges, int64_t n_nodes,
                                           int64_t channels) {
  if (n_edges < 0 || n_nodes <= 0 || channels <= 0) return 0;
  // Pointer alignment, `env` and `order` pick the kernel (and with it the
  // partition count); size for every choice.
  size_t need = smx_layout(n_edges, n_nodes, channels, false, nullptr, false).bytes;
  for (int env = 0; env < 2; ++env)
    for (int form = 0; form < 3; ++form) {  // merge path, lean, gather
      const size_t b = smx_layout(n_edges, n_nodes, channels, false, nullptr, true, env,
                                  form == 1, form == 2)
                           .bytes;
      if (b > need) need = b;
    }
  return need;
}

int bysj_segment_softmax_forward(const float* logit, const float* env,
                                 const int64_t* offsets, int64_t n_edges,
                                 int64_t n_nodes, int64_t channels,
                                 const float* null_logit,
                                 const int64_t* order, float* alpha,
                                 float* null_alpha, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  clear_error();
  int st = smx_check(n_edges, n_nodes, channels, offsets);
  if (st) return st;
  if ((null_logit == nullptr) != (null_alpha == nullptr))
    return fail(BYSJ_ERR_INVALID_ARGUMENT,
                "segment softmax: null_logit and null_alpha go together");
  if (n_nodes == 0) return BYSJ_OK;
  if (n_edges > 0 && (logit == nullptr || alpha == nullptr))
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "segment softmax: NULL logit/alpha");
  const bool quad_ok = aligned16(logit) && aligned16(alpha) &&
                       (null_logit == nullptr || aligned16(null_logit)) &&
                       (null_alpha == nullptr || aligned16(null_alpha));
  SmxLayout L = smx_layout(n_edges, n_nodes, channels, false, workspace, quad_ok,
                           env != nullptr, order == nullptr, order != nullptr);
  if (workspace == nullptr || workspace_bytes < L.bytes)
    return fail(BYSJ_ERR_WORKSPACE,
                "segment softmax: workspace of %zu bytes needed, %zu given",
                L.bytes, workspace_bytes);
  SmxArgs a{};
  a.x = logit;
  a.env = env;
  a.xn = null_logit;
  a.order = order;
  a.out = alpha;
  a.out_null = null_alpha;
  a.channels = channels;
  return smx_run(a, L, n_edges, n_nodes, offsets,
                 static_cast<cudaStream_t>(stream), "segment_softmax_fwd");
}

size_t bysj_segment_softmax_backward_workspace_size(int64_t n_edges,
                                                    int64_t n_nodes,
                                                    int64_t channels) {
  if (n_edges < 0 || n_nodes <= 0 || channels <= 0) return 0;
  // Pointer alignment and `order` pick the kernel; size for every choice.
  size_t need = smx_layout(n_edges, n_nodes, channels, true, nullptr, false).bytes;
  for (int gather = 0; gather < 2; ++gather) {
    const size_t b =
        smx_layout(n_edges, n_nodes, channels, true, nullptr, true, true, false, gather).bytes;
    if (b > need) need = b;
  }
  return need;
}

int bysj_segment_softmax_backward(const float* alpha, const float* grad_alpha,
                                  const float* env, const int64_t* offsets,
                                  int64_t n_edges, int64_t n_nodes,
                                  int64_t channels, const float* null_alpha,
                                  const float* grad_null_alpha,
                                  const int64_t* order, float* grad_logit,
                                  float* grad_null_logit, float* grad_env,
                                  void* workspace, size_t workspace_bytes,
                                  void* stream) {
  clear_error();
  int st = smx_check(n_edges, n_nodes, channels, offsets);
  if (st) return st;
  const int nulls = (null_alpha != nullptr) + (grad_null_alpha != nullptr) +
                    (grad_null_logit != nullptr);
  if (nulls != 0 && nulls != 3)
    return fail(BYSJ_ERR_INVALID_ARGUMENT,
                "segment softmax backward: null_alpha, grad_null_alpha and "
                "grad_null_logit go together");
  if (n_nodes == 0) return BYSJ_OK;
  if (n_edges > 0 && (alpha == nullptr || grad_alpha == nullptr ||
                      grad_logit == nullptr))
    return fail(BYSJ_ERR_INVALID_ARGUMENT,
                "segment softmax backward: NULL alpha/grad_alpha/grad_logit");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool quad_ok = aligned16(alpha) && aligned16(grad_alpha) && aligned16(grad_logit) &&
                       (null_alpha == nullptr || aligned16(null_alpha)) &&
                       (grad_null_alpha == nullptr || aligned16(grad_null_alpha)) &&
                       (grad_null_logit == nullptr || aligned16(grad_null_logit));
  SmxLayout L = smx_layout(n_edges, n_nodes, channels, true, workspace, quad_ok, true, false,
                           order != nullptr);
  if (workspace == nullptr || workspace_bytes < L.bytes)
    return fail(BYSJ_ERR_WORKSPACE,
                "segment softmax backward: workspace of %zu bytes needed, %zu "
                "given",
                L.bytes, workspace_bytes);
  const bool env_in_warp = L.cfg.tiles == 1;
  SmxArgs a{};
  a.x = alpha;
  a.y = grad_alpha;
  a.env = env;
  a.xn = null_alpha;
  a.yn = grad_null_alpha;
  a.order = order;
  a.out = grad_logit;
  a.out_null = grad_null_logit;
  a.out_env = env_in_warp ? grad_env : nullptr;
  a.channels = channels;
  st = smx_run(a, L, n_edges, n_nodes, offsets, s, "segment_softmax_bwd");
  if (st || env_in_warp || grad_env == nullptr || n_edges == 0) return st;
  const DeviceInfo& dev = current_device_info();
  int64_t blocks = (n_edges + kWarpsPerBlock - 1) / kWarpsPerBlock;
  if (blocks > dev.sm_count * 8) blocks = dev.sm_count * 8;
  segment_softmax_env_kernel<<<static_cast<unsigned>(blocks), kBlock, 0, s>>>(
      grad_logit, env, grad_env, n_edges, channels);
  return launch_check("segment_softmax_env_kernel");
}

}  // extern "C"
