// GIE zonal scatter, forward and backward, for sm_100a.
//
//   out[n, 0, :]   = 0
//   out[n, r+1, c] = inv[n] * sum_{e in seg(n)} zonal[e, r] * radial[e, slot[r], c]
//
// Contract of the reference's csrc/gie.cpp:68-228 (normalise after the
// destination sum).  The reference scatters with one float atomicAdd per
// (edge, row, channel) and scales in a second pass; here the edges are read
// in destination (CSR) order, one merge-path partition per warp, each lane
// owning a slice of the node's [rows, channels] block in registers, and the
// normalisation is folded into the single store.  No atomics: repeated runs
// are bit-identical.  The backward writes the per-edge gradients directly
// (each edge reads only its own node's upstream row) and reduces the
// inverse-degree gradient per segment from the same unnormalised sums.
#include "launch.cuh"

namespace bysj {
namespace {

struct GieArgs {
  const float* zonal;    // [E, R]
  const float* radial;   // [E, NR, C]
  const int64_t* order;
  const int64_t* slot;   // [R]
  const float* inv;      // [N]
  const float* grad;     // backward: [N, R+1, C]
  const int64_t* dst;    // backward: [E]
  float* out;            // forward: [N, R+1, C] | backward: grad_inv [N]
  float* grad_zonal;     // [E, R]
  float* grad_radial;    // [E, NR, C]
  int64_t rows, n_radial, channels;
  int64_t lv;            // R*C/VEC
  int64_t skip_degrees;  // generic kernels: > 0 = return if slot[] is the degree table of that L
  const uint32_t* gate;  // non-NULL: every kernel returns at once if *gate != 0
  MergePath mp;
  SplitSlots ss;
};

template <int VEC>
__device__ __forceinline__ void ld_l1(const float* p, float (&v)[VEC]) {
  if constexpr (VEC == 4) {
    const float4 t = __ldg(reinterpret_cast<const float4*>(p));
    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) v[i] = __ldg(p + i);
  }
}

// True when slot[0..R), R = (L+1)^2 - 1, is the degree-grouped table
// slot[r] = l(r) + base, l(r) = floor(sqrt(r + 1)), with degrees 1..L inside
// the n_radial slots; sets base.  It is the test the host applies before it
// calls the degree entry points itself; the generic entry points, which are
// handed a slot table they do not read back, launch both kernels and let
// every warp of each make it (R <= 15 loads that hit L2).
__device__ __forceinline__ bool degree_table(const int64_t* slot, int degrees,
                                             int64_t n_radial, int64_t& base) {
  const int rows = (degrees + 1) * (degrees + 1) - 1;
  base = __ldg(slot) - 1;
  bool ok = base >= -1 && base + degrees <= n_radial - 1;
  int l = 1;
  for (int r = 0; r < rows; ++r) {
    if ((l + 1) * (l + 1) <= r + 1) ++l;
    ok = ok && __ldg(slot + r) == l + base;
  }
  return ok;
}

// slot_base value that tells a degree kernel to take its base from a.slot
// (and to do nothing unless a.slot is the degree table).
constexpr int64_t kSlotBaseOnDevice = INT64_MIN;

// Per-lane geometry of vector k: output row r, radial offset slot*C + c.
template <int VEC, int NV>
struct LaneMap {
  int64_t j[NV];     // vector index (clamped into range)
  bool ok[NV];
  int r[NV];
  int64_t roff[NV];  // slot[r] * C + c
  int64_t ooff[NV];  // (r + 1) * C + c inside the node block
  __device__ __forceinline__ void init(const GieArgs& a, int64_t jt, int lane) {
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int64_t jj = jt + lane + k * kWarp;
      ok[k] = jj < a.lv;
      j[k] = ok[k] ? jj : a.lv - 1;
      const int64_t x = j[k] * VEC;
      r[k] = static_cast<int>(x / a.channels);
      const int64_t c = x - r[k] * a.channels;
      roff[k] = __ldg(a.slot + r[k]) * a.channels + c;
      ooff[k] = (r[k] + 1) * a.channels + c;
    }
  }
};

template <int VEC, int NV>
__device__ __forceinline__ void gie_accumulate(const GieArgs& a, const LaneMap<VEC, NV>& L,
                                               int64_t lo, int64_t hi,
                                               float (&acc)[NV][VEC]) {
  for (int64_t s = lo; s < hi; ++s) {
    const int64_t e = a.order ? __ldg(a.order + s) : s;
    const float* zr = a.zonal + e * a.rows;
    const float* rr = a.radial + e * a.n_radial * a.channels;
    float z[NV];
    float rv[NV][VEC];
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      z[k] = __ldg(zr + L.r[k]);
      ld_l1<VEC>(rr + L.roff[k], rv[k]);
    }
#pragma unroll
    for (int k = 0; k < NV; ++k)
#pragma unroll
      for (int i = 0; i < VEC; ++i) acc[k][i] = fmaf(z[k], rv[k][i], acc[k][i]);
  }
}

template <int VEC, int NV>
__global__ void __launch_bounds__(kBlock, 2) gie_fwd_kernel(GieArgs a) {
  if (a.gate != nullptr && *a.gate != 0) return;  // the CSR view was not built
  constexpr int TV = kWarp * NV;
  const int64_t p = global_warp();
  if (p >= a.mp.parts) return;
  if (a.skip_degrees > 0) {
    int64_t base;
    if (degree_table(a.slot, static_cast<int>(a.skip_degrees), a.n_radial, base)) return;
  }
  const int lane = lane_id();
  const int tile = blockIdx.y;
  const int64_t jt = static_cast<int64_t>(tile) * TV;
  const int64_t block = (a.rows + 1) * a.channels;
  LaneMap<VEC, NV> L;
  L.init(a, jt, lane);
  SegCursor cur(a.mp, part_range(a.mp, p));
  while (cur.next()) {
    const int64_t n = cur.node;
    float acc[NV][VEC];
#pragma unroll
    for (int k = 0; k < NV; ++k)
#pragma unroll
      for (int i = 0; i < VEC; ++i) acc[k][i] = 0.0f;
    gie_accumulate<VEC, NV>(a, L, cur.lo, cur.hi, acc);
    float* on = a.out + n * block;
    if (cur.kind == kWhole) {
      const float inv = __ldg(a.inv + n);
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        if (!L.ok[k]) continue;
        float v[VEC];
#pragma unroll
        for (int i = 0; i < VEC; ++i) v[i] = acc[k][i] * inv;
        store_f32<VEC>(on + L.ooff[k], v);
      }
      if (tile == 0)
        for (int64_t c = lane; c < a.channels; c += kWarp) on[c] = 0.0f;
      continue;
    }
    float* mine = a.ss.slot(p, cur.kind);
#pragma unroll
    for (int k = 0; k < NV; ++k)
      if (L.ok[k]) store_cg<VEC>(mine + L.j[k] * VEC, acc[k]);
    const int64_t first = a.mp.part_of_first_edge(n);
    const int64_t last = a.mp.part_of_end(n);
    if (!arrive_last(a.ss, first, last, tile)) continue;
    const float inv = __ldg(a.inv + n);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      if (!L.ok[k]) continue;
      float sum[VEC];
#pragma unroll
      for (int i = 0; i < VEC; ++i) sum[i] = 0.0f;
      for (int64_t q = first; q <= last; ++q) {
        float part[VEC];
        load_cg<VEC>(a.ss.slot(q, q == last ? kHead : kTail) + L.j[k] * VEC, part);
#pragma unroll
        for (int i = 0; i < VEC; ++i) sum[i] += part[i];
      }
#pragma unroll
      for (int i = 0; i < VEC; ++i) sum[i] *= inv;
      store_f32<VEC>(on + L.ooff[k], sum);
    }
    if (tile == 0)
      for (int64_t c = lane; c < a.channels; c += kWarp) on[c] = 0.0f;
  }
}

// Forward for the degree-grouped row layout of DPA4's GIE: rows r = 0..R-1
// with R = (L+1)^2 - 1, row r has degree l(r) = floor(sqrt(r+1)) and reads
// radial slot l(r) + slot_base.  A lane owns one 4-channel column quad for
// all R rows (LPE = C/4 lanes per edge, EG = 32/LPE edges side by side), so
// per edge it streams each degree's radial quad once (L 16-byte loads), and
// the row -> slot choice is resolved at compile time.  The R zonal
// coefficients of an edge are the same for its LPE lanes: each warp stages
// them for 32 edges at a time in shared memory with coalesced loads, and the
// lanes read them back as broadcasts.  The radial quads go through a ring of
// kFwdStages step buffers in shared memory (cp.async): step j (EG edges, one
// per edge group) is computed while steps j+1 .. j+kFwdAhead are in flight,
// so the loads of several steps overlap without registers for them (C3 op
// with its CSR view, C = 32: 257 -> 231 us, C = 64: 362 -> 346 us; the
// register form kept two edges per lane in flight and was latency-bound, 8
// long-scoreboard stalls per issued instruction).  With
// L = 3 the 15 x 4 accumulators take 60 registers, so two CTAs per SM (also
// for L = 2); three for L = 1.
constexpr int kZonalChunk = 32;  // edges whose zonal rows a warp stages at once
constexpr int kFwdStages = 4;    // radial step buffers per warp
constexpr int kFwdAhead = kFwdStages - 1;

template <int L>
constexpr size_t gie_fwd_smem_bytes() {
  return static_cast<size_t>(kWarpsPerBlock) * kFwdStages * kWarp * L * sizeof(float4);
}

template <int LPE, int L>
__global__ void __launch_bounds__(kBlock, L >= 2 ? 2 : 3)
    gie_fwd_degree_kernel(GieArgs a, int64_t slot_base) {
  if (a.gate != nullptr && *a.gate != 0) return;  // the CSR view was not built
  constexpr int R = (L + 1) * (L + 1) - 1;
  constexpr int EG = kWarp / LPE;
  constexpr int kStepQuads = kWarp * L;  // EG edges x L degrees x LPE lanes
  __shared__ float zstage[kWarpsPerBlock][kZonalChunk * R];
  extern __shared__ float4 gie_fwd_ring[];
  const int64_t p = global_warp();
  if (p >= a.mp.parts) return;
  if (slot_base == kSlotBaseOnDevice && !degree_table(a.slot, L, a.n_radial, slot_base)) return;
  float* zb = zstage[threadIdx.x >> 5];
  float4* ring = gie_fwd_ring + (threadIdx.x >> 5) * kFwdStages * kStepQuads;
  const int lane = lane_id();
  const int eg = lane / LPE;
  const int c4 = lane % LPE;
  const int64_t C = a.channels;
  const int64_t block = (R + 1) * C;
  const int64_t radial_row = a.n_radial * C;
  SegCursor cur(a.mp, part_range(a.mp, p));
  while (cur.next()) {
    const int64_t n = cur.node;
    float acc[R][4];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[r][i] = 0.0f;
    // The radial quads of the step whose first edge is `base` into ring slot
    // b; a lane past the piece's end copies the step's first edge (in range),
    // so the quads it never uses are finite.  Each lane reads back only the
    // quads it copied itself.
    const auto radial_issue = [&](int64_t base, int b) {
      const int64_t k = base + eg < cur.hi ? base + eg : base;
      const int64_t e = a.order ? __ldg(a.order + k) : k;
      const float* rr = a.radial + e * radial_row + slot_base * C + 4 * c4;
      float4* dst = ring + b * kStepQuads + eg * L * LPE + c4;
#pragma unroll
      for (int l = 1; l <= L; ++l) cp_async16(dst + (l - 1) * LPE, rr + l * C);
    };
    __syncwarp();  // the previous piece's reads of the ring are done
#pragma unroll
    for (int j = 0; j < kFwdAhead; ++j) {
      if (cur.lo + j * EG < cur.hi) radial_issue(cur.lo + j * EG, j);
      cp_async_commit();
    }
    int slot = 0;  // ring slot of the step being computed
    for (int64_t lo = cur.lo; lo < cur.hi; lo += kZonalChunk) {  // warp-uniform
      const int rows = static_cast<int>(cur.hi - lo < kZonalChunk ? cur.hi - lo : kZonalChunk);
      __syncwarp();  // the previous chunk's reads are done
      if (a.order == nullptr) {
        const float* src = a.zonal + lo * R;
        for (int i = lane; i < rows * R; i += kWarp) zb[i] = __ldg(src + i);
      } else {
        for (int i = lane; i < rows * R; i += kWarp) {
          const int k = i / R;
          zb[i] = __ldg(a.zonal + __ldg(a.order + lo + k) * R + (i - k * R));
        }
      }
      __syncwarp();
      for (int k0 = 0; k0 < rows; k0 += EG) {  // warp-uniform
        const int64_t next = lo + k0 + kFwdAhead * EG;
        const int refill = slot == 0 ? kFwdStages - 1 : slot - 1;  // read one step ago
        if (next < cur.hi) radial_issue(next, refill);
        cp_async_commit();
        cp_async_wait<kFwdAhead>();  // this step's quads have landed
        const int k = k0 + eg;
        const bool valid = k < rows;
        const float* z = zb + (valid ? k : 0) * R;
        const float4* qs = ring + slot * kStepQuads + eg * L * LPE + c4;
#pragma unroll
        for (int l = 1; l <= L; ++l) {
          const float4 q = qs[(l - 1) * LPE];
#pragma unroll
          for (int r = l * l - 1; r < (l + 1) * (l + 1) - 1; ++r) {
            const float zr = valid ? z[r] : 0.0f;
            acc[r][0] = fmaf(zr, q.x, acc[r][0]);
            acc[r][1] = fmaf(zr, q.y, acc[r][1]);
            acc[r][2] = fmaf(zr, q.z, acc[r][2]);
            acc[r][3] = fmaf(zr, q.w, acc[r][3]);
          }
        }
        slot = slot == kFwdStages - 1 ? 0 : slot + 1;
      }
    }
    cp_async_wait<0>();  // no copy of this piece is left in flight
    if constexpr (EG > 1) {
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[r][i] = xor_sum(acc[r][i], LPE);
    }
    float* on = a.out + n * block;
    if (cur.kind == kWhole) {
      if (eg == 0) {
        const float inv = __ldg(a.inv + n);
        reinterpret_cast<float4*>(on)[c4] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
        for (int r = 0; r < R; ++r)
          reinterpret_cast<float4*>(on + (r + 1) * C)[c4] =
              make_float4(acc[r][0] * inv, acc[r][1] * inv, acc[r][2] * inv, acc[r][3] * inv);
      }
      continue;
    }
    float* mine = a.ss.slot(p, cur.kind);
    if (eg == 0) {
#pragma unroll
      for (int r = 0; r < R; ++r) store_cg<4>(mine + r * C + 4 * c4, acc[r]);
    }
    const int64_t first = a.mp.part_of_first_edge(n);
    const int64_t last = a.mp.part_of_end(n);
    if (!arrive_last(a.ss, first, last, 0)) continue;
    if (eg == 0) {
      const float inv = __ldg(a.inv + n);
      reinterpret_cast<float4*>(on)[c4] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        float sum[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int64_t q = first; q <= last; ++q) {
          float part[4];
          load_cg<4>(a.ss.slot(q, q == last ? kHead : kTail) + r * C + 4 * c4, part);
#pragma unroll
          for (int i = 0; i < 4; ++i) sum[i] += part[i];
        }
        reinterpret_cast<float4*>(on + (r + 1) * C)[c4] =
            make_float4(sum[0] * inv, sum[1] * inv, sum[2] * inv, sum[3] * inv);
      }
    }
  }
}

// Backward for the degree row layout (C = 4 LPE, LPE <= 16 lanes per edge,
// EG = 32 / LPE edges side by side).  With gi = g[n, 1:] * inv[n]:
//   grad_radial[e, base + l, c] = sum_{r of degree l} gi[r, c] zonal[e, r]
//   grad_radial[e, other slots, c] = 0
//   grad_zonal[e, r] = sum_c gi[r, c] radial[e, base + l(r), c]
//   grad_inv[n] = <g[n, 1:], pre[n]>,  pre[n, r, c] = sum_e zonal[e, r] radial[e, base + l(r), c]
// Per warp, shared memory holds gi of the current segment (R x C floats),
// the zonal rows of 32 edges, and a 32 x 17 tile through which each lane's
// 4-channel share of grad_zonal is summed over the LPE lanes of its edge (in
// lane order).  pre is summed over all the segment's edges (edge groups
// merged, split pieces combined) before the single dot product, as the
// forward normalises after its sum.  The radial rows of the next step
// (32 / LPE edges) are copied into a shared double buffer (cp.async) while
// the current step is computed.
constexpr int kTilePitch = 17;  // floats per lane row of the fold tile

template <int LPE, int L>
struct GieBwdSmem {
  static constexpr int R = (L + 1) * (L + 1) - 1;
  static constexpr size_t kG = sizeof(float4) * R * LPE;
  static constexpr size_t kZ = sizeof(float) * kZonalChunk * R;
  static constexpr size_t kT = sizeof(float) * kWarp * kTilePitch;
  // Radial quads of one step (32 / LPE edges x L degrees x LPE lanes), two
  // steps: the next step's rows are copied in while this step is computed.
  static constexpr int kRadQuads = kWarp * L;
  static constexpr size_t kRad = 2 * sizeof(float4) * kRadQuads;
  static constexpr size_t kWarpBytes = (kG + kZ + kT + kRad + 15) / 16 * 16;
};

template <int LPE, int L>
__global__ void __launch_bounds__(kBlock, 2)
    gie_bwd_degree_kernel(GieArgs a, int64_t slot_base) {
  if (a.gate != nullptr && *a.gate != 0) return;  // the CSR view was not built
  using M = GieBwdSmem<LPE, L>;
  constexpr int R = M::R;
  constexpr int EG = kWarp / LPE;
  static_assert(LPE <= 16 && R <= 16, "degree backward needs C <= 64 and L <= 3");
  extern __shared__ float4 gie_bwd_smem[];
  const int64_t p = global_warp();
  if (p >= a.mp.parts) return;
  if (slot_base == kSlotBaseOnDevice && !degree_table(a.slot, L, a.n_radial, slot_base)) return;
  char* mine_smem = reinterpret_cast<char*>(gie_bwd_smem) + (threadIdx.x >> 5) * M::kWarpBytes;
  float4* gq = reinterpret_cast<float4*>(mine_smem);
  float* zb = reinterpret_cast<float*>(mine_smem + M::kG);
  float* tile = reinterpret_cast<float*>(mine_smem + M::kG + M::kZ);
  float4* rbuf = reinterpret_cast<float4*>(mine_smem + M::kG + M::kZ + M::kT);
  const int lane = lane_id();
  const int eg = lane / LPE;
  const int c4 = lane % LPE;
  const int64_t C = a.channels;
  const int64_t block = (R + 1) * C;
  const int64_t radial_row = a.n_radial * C;
  SegCursor cur(a.mp, part_range(a.mp, p));
  while (cur.next()) {
    const int64_t n = cur.node;
    const float inv = __ldg(a.inv + n);
    const float4* gn = reinterpret_cast<const float4*>(a.grad + n * block + C);  // rows 1..R
    __syncwarp();  // the previous piece's reads of gq are done
    for (int i = lane; i < R * LPE; i += kWarp) {
      const float4 v = __ldg(gn + i);
      gq[i] = make_float4(v.x * inv, v.y * inv, v.z * inv, v.w * inv);
    }
    float acc[R][4];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[r][i] = 0.0f;
    // Copies the radial quads of the step whose first edge is `base` into
    // buffer b; a lane past the segment's end copies the step's first edge
    // (in range), so its unused quads are finite.
    auto radial_issue = [&](int64_t base, int b) {
      const int64_t k = base + eg < cur.hi ? base + eg : base;
      const int64_t e = a.order ? __ldg(a.order + k) : k;
      const float* rr = a.radial + e * radial_row + slot_base * C + 4 * c4;
      float4* dst = rbuf + b * M::kRadQuads + eg * L * LPE + c4;
#pragma unroll
      for (int l = 1; l <= L; ++l) cp_async16(dst + (l - 1) * LPE, rr + l * C);
    };
    int rb = 0;
    if (cur.lo < cur.hi) radial_issue(cur.lo, rb);  // an empty piece copies nothing
    cp_async_commit();
    for (int64_t lo = cur.lo; lo < cur.hi; lo += kZonalChunk) {  // warp-uniform
      const int rows = static_cast<int>(cur.hi - lo < kZonalChunk ? cur.hi - lo : kZonalChunk);
      __syncwarp();
      if (a.order == nullptr) {
        const float* src = a.zonal + lo * R;
        for (int i = lane; i < rows * R; i += kWarp) zb[i] = __ldg(src + i);
      } else {
        for (int i = lane; i < rows * R; i += kWarp) {
          const int k = i / R;
          zb[i] = __ldg(a.zonal + __ldg(a.order + lo + k) * R + (i - k * R));
        }
      }
      __syncwarp();
      for (int k0 = 0; k0 < rows; k0 += EG) {  // warp-uniform
        if (lo + k0 + EG < cur.hi) radial_issue(lo + k0 + EG, rb ^ 1);
        cp_async_commit();
        cp_async_wait<1>();  // this step's radial quads have landed
        __syncwarp();
        const int k = k0 + eg;
        const bool valid = k < rows;
        const int kk = valid ? k : 0;
        const int64_t slot = lo + kk;
        const int64_t e = a.order ? __ldg(a.order + slot) : slot;
        const float* z = zb + kk * R;
        const float4* qs = rbuf + rb * M::kRadQuads + eg * L * LPE + c4;
        rb ^= 1;
#pragma unroll
        for (int l = 1; l <= L; ++l) {
          const float4 q = qs[(l - 1) * LPE];
          float4 gr = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
          for (int r = l * l - 1; r < (l + 1) * (l + 1) - 1; ++r) {
            const float zr = valid ? z[r] : 0.0f;
            const float4 g = gq[r * LPE + c4];
            acc[r][0] = fmaf(zr, q.x, acc[r][0]);
            acc[r][1] = fmaf(zr, q.y, acc[r][1]);
            acc[r][2] = fmaf(zr, q.z, acc[r][2]);
            acc[r][3] = fmaf(zr, q.w, acc[r][3]);
            tile[lane * kTilePitch + r] = fmaf(g.x, q.x, fmaf(g.y, q.y, fmaf(g.z, q.z, g.w * q.w)));
            gr.x = fmaf(g.x, zr, gr.x);
            gr.y = fmaf(g.y, zr, gr.y);
            gr.z = fmaf(g.z, zr, gr.z);
            gr.w = fmaf(g.w, zr, gr.w);
          }
          if (valid)
            reinterpret_cast<float4*>(a.grad_radial + e * radial_row + (slot_base + l) * C)[c4] =
                gr;
        }
        if (valid) {
          for (int64_t sl = 0; sl < a.n_radial; ++sl) {
            if (sl >= slot_base + 1 && sl <= slot_base + L) continue;
            reinterpret_cast<float4*>(a.grad_radial + e * radial_row + sl * C)[c4] =
                make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          }
        }
        __syncwarp();
        if (valid) {
          for (int r = c4; r < R; r += LPE) {
            float sum = 0.0f;
#pragma unroll
            for (int t = 0; t < LPE; ++t) sum += tile[(eg * LPE + t) * kTilePitch + r];
            a.grad_zonal[e * R + r] = sum;
          }
        }
        __syncwarp();  // the tile is read before the next edge overwrites it
      }
    }
    cp_async_wait<0>();
    if constexpr (EG > 1) {
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[r][i] = xor_sum(acc[r][i], LPE);
    }
    if (cur.kind != kWhole) {
      float* mine = a.ss.slot(p, cur.kind);
      if (eg == 0) {
#pragma unroll
        for (int r = 0; r < R; ++r) store_cg<4>(mine + r * C + 4 * c4, acc[r]);
      }
      const int64_t first = a.mp.part_of_first_edge(n);
      const int64_t last = a.mp.part_of_end(n);
      if (!arrive_last(a.ss, first, last, 0)) continue;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        float sum[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int64_t q = first; q <= last; ++q) {
          float piece[4];
          load_cg<4>(a.ss.slot(q, q == last ? kHead : kTail) + r * C + 4 * c4, piece);
#pragma unroll
          for (int i = 0; i < 4; ++i) sum[i] += piece[i];
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[r][i] = sum[i];
      }
    }
    float dot = 0.0f;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float4 g = __ldg(gn + r * LPE + c4);
      dot = fmaf(g.x, acc[r][0], fmaf(g.y, acc[r][1], fmaf(g.z, acc[r][2], fmaf(g.w, acc[r][3], dot))));
    }
    if constexpr (LPE > 1) dot = group_sum(dot, LPE);
    if (lane == 0) a.out[n] = dot;
  }
}

// Backward.  Per edge, with gi = g[n] * inv[n] (g rows are re-read from L1):
//   grad_zonal[e, r]     = sum_c gi[r, c] * radial[e, slot r, c]
//   grad_radial[e, s, c] = sum_{r: slot r = s} gi[r, c] * zonal[e, r]
// and per segment grad_inv[n] = <g[n], pre[n]>, where pre is the
// unnormalised forward sum accumulated exactly as the forward does (sum over
// the edges first, then one dot product), so cancellation inside the sum is
// resolved before the upstream weight is applied.
template <int VEC, int NV>
__global__ void __launch_bounds__(kBlock, 2) gie_bwd_kernel(GieArgs a) {
  if (a.gate != nullptr && *a.gate != 0) return;  // the CSR view was not built
  constexpr int TV = kWarp * NV;
  extern __shared__ float s_dot[];  // [warps][TV]
  const int64_t p = global_warp();
  if (p >= a.mp.parts) return;
  if (a.skip_degrees > 0) {
    int64_t base;
    if (degree_table(a.slot, static_cast<int>(a.skip_degrees), a.n_radial, base)) return;
  }
  float* sdot = s_dot + (threadIdx.x >> 5) * TV;
  const int lane = lane_id();
  const int64_t block = (a.rows + 1) * a.channels;
  const int64_t vpr = a.channels / VEC;  // vectors per output row
  const int64_t radial_row = a.n_radial * a.channels;
  LaneMap<VEC, NV> L;
  L.init(a, 0, lane);
  SegCursor cur(a.mp, part_range(a.mp, p));
  while (cur.next()) {
    const int64_t n = cur.node;
    const float inv = __ldg(a.inv + n);
    const float* gn = a.grad + n * block;
    float acc[NV][VEC];
#pragma unroll
    for (int k = 0; k < NV; ++k)
#pragma unroll
      for (int i = 0; i < VEC; ++i) acc[k][i] = 0.0f;
    for (int64_t s = cur.lo; s < cur.hi; ++s) {
      const int64_t e = a.order ? __ldg(a.order + s) : s;
      const float* zr = a.zonal + e * a.rows;
      const float* rr = a.radial + e * radial_row;
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        float rv[VEC], g[VEC];
        ld_l1<VEC>(rr + L.roff[k], rv);
        ld_l1<VEC>(gn + L.ooff[k], g);
        const float z = __ldg(zr + L.r[k]);
        float d = 0.0f;
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
          d = fmaf(g[i] * inv, rv[i], d);
          acc[k][i] = fmaf(z, rv[i], acc[k][i]);
        }
        if (L.ok[k]) sdot[lane + k * kWarp] = d;
      }
      __syncwarp();
      for (int64_t r = lane; r < a.rows; r += kWarp) {
        float sum = 0.0f;
        for (int64_t v = 0; v < vpr; ++v) sum += sdot[r * vpr + v];
        a.grad_zonal[e * a.rows + r] = sum;
      }
      for (int64_t v = lane; v < radial_row / VEC; v += kWarp) {
        const int64_t x = v * VEC;
        const int64_t sl = x / a.channels;
        const int64_t c = x - sl * a.channels;
        float gr[VEC];
#pragma unroll
        for (int i = 0; i < VEC; ++i) gr[i] = 0.0f;
        for (int64_t r = 0; r < a.rows; ++r) {
          if (__ldg(a.slot + r) != sl) continue;
          const float z = __ldg(zr + r);
          float g[VEC];
          ld_l1<VEC>(gn + (r + 1) * a.channels + c, g);
#pragma unroll
          for (int i = 0; i < VEC; ++i) gr[i] = fmaf(g[i] * inv, z, gr[i]);
        }
        store_f32<VEC>(a.grad_radial + e * radial_row + x, gr);
      }
      __syncwarp();
    }
    if (cur.kind != kWhole) {
      float* mine = a.ss.slot(p, cur.kind);
#pragma unroll
      for (int k = 0; k < NV; ++k)
        if (L.ok[k]) store_cg<VEC>(mine + L.j[k] * VEC, acc[k]);
      const int64_t first = a.mp.part_of_first_edge(n);
      const int64_t last = a.mp.part_of_end(n);
      if (!arrive_last(a.ss, first, last, 0)) continue;
#pragma unroll
      for (int k = 0; k < NV; ++k) {
#pragma unroll
        for (int i = 0; i < VEC; ++i) acc[k][i] = 0.0f;
        if (!L.ok[k]) continue;
        for (int64_t q = first; q <= last; ++q) {
          float part[VEC];
          load_cg<VEC>(a.ss.slot(q, q == last ? kHead : kTail) + L.j[k] * VEC, part);
#pragma unroll
          for (int i = 0; i < VEC; ++i) acc[k][i] += part[i];
        }
      }
    }
    float dot = 0.0f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      if (!L.ok[k]) continue;
      float g[VEC];
      ld_l1<VEC>(gn + L.ooff[k], g);
#pragma unroll
      for (int i = 0; i < VEC; ++i) dot = fmaf(g[i], acc[k][i], dot);
    }
    dot = xor_sum(dot, 1);
    if (lane == 0) a.out[n] = dot;
  }
}

using GieKernel = void (*)(GieArgs);

struct GieConfig {
  GieKernel kernel = nullptr;
  int vec = 1, nv = 1;
  int64_t lv = 0, tiles = 1;
};

template <int VEC>
GieConfig gie_pick(int64_t lv, bool backward) {
  GieConfig c;
  c.vec = VEC;
  c.lv = lv;
  if (lv > 128) { c.nv = 8; c.kernel = backward ? gie_bwd_kernel<VEC, 8> : gie_fwd_kernel<VEC, 8>; }
  else if (lv > 64) { c.nv = 4; c.kernel = backward ? gie_bwd_kernel<VEC, 4> : gie_fwd_kernel<VEC, 4>; }
  else if (lv > 32) { c.nv = 2; c.kernel = backward ? gie_bwd_kernel<VEC, 2> : gie_fwd_kernel<VEC, 2>; }
  else { c.nv = 1; c.kernel = backward ? gie_bwd_kernel<VEC, 1> : gie_fwd_kernel<VEC, 1>; }
  c.tiles = (lv + kWarp * c.nv - 1) / (kWarp * c.nv);
  return c;
}

struct GieLayout {
  GieConfig cfg;
  PartitionPlan plan;
  size_t bytes = 0;
  SplitSlots ss{};
};

GieLayout gie_layout(bool vec_ok, int64_t n_edges, int64_t n_nodes,
                     int64_t rows, int64_t channels, bool backward, void* ws) {
  GieLayout L;
  const int64_t cells = rows * channels;
  L.cfg = (vec_ok && channels % 4 == 0) ? gie_pick<4>(cells / 4, backward)
                                        : gie_pick<1>(cells, backward);
  const DeviceInfo& dev = current_device_info();
  const size_t smem = backward ? sizeof(float) * kBlock * L.cfg.nv : 0;
  const int64_t resident =
      static_cast<int64_t>(dev.sm_count) *
      resident_blocks(reinterpret_cast<const void*>(L.cfg.kernel), smem) *
      kWarpsPerBlock;
  int64_t warps = resident / L.cfg.tiles;
  if (warps < 1) warps = 1;
  L.plan = plan_partitions(n_edges, n_nodes, warps, 16);
  const int64_t stride = (cells + 7) / 8 * 8;
  Carver carve(ws);
  float* slots = carve.take<float>(static_cast<size_t>(L.plan.parts) * 2 * stride);
  int* tickets = carve.take<int>(static_cast<size_t>(L.plan.parts) * L.cfg.tiles);
  L.bytes = carve.need;
  L.ss = SplitSlots{slots, tickets, stride, static_cast<int>(L.cfg.tiles)};
  return L;
}


using GieDegreeKernel = void (*)(GieArgs, int64_t);

template <int L>
GieDegreeKernel gie_degree_pick(int64_t lpe, bool backward) {
  if (backward) {
    switch (lpe) {
      case 1: return gie_bwd_degree_kernel<1, L>;
      case 2: return gie_bwd_degree_kernel<2, L>;
      case 4: return gie_bwd_degree_kernel<4, L>;
      case 8: return gie_bwd_degree_kernel<8, L>;
      case 16: return gie_bwd_degree_kernel<16, L>;
      default: return nullptr;
    }
  }
  switch (lpe) {
    case 1: return gie_fwd_degree_kernel<1, L>;
    case 2: return gie_fwd_degree_kernel<2, L>;
    case 4: return gie_fwd_degree_kernel<4, L>;
    case 8: return gie_fwd_degree_kernel<8, L>;
    case 16: return gie_fwd_degree_kernel<16, L>;
    case 32: return gie_fwd_degree_kernel<32, L>;
    default: return nullptr;
  }
}

GieDegreeKernel gie_degree_kernel(int64_t degrees, int64_t channels, bool backward) {
  if (channels % 4 != 0) return nullptr;
  const int64_t lpe = channels / 4;
  switch (degrees) {
    case 1: return gie_degree_pick<1>(lpe, backward);
    case 2: return gie_degree_pick<2>(lpe, backward);
    case 3: return gie_degree_pick<3>(lpe, backward);
    default: return nullptr;
  }
}

struct GieDegreeLayout {
  GieDegreeKernel kernel = nullptr;
  PartitionPlan plan;
  size_t bytes = 0;
  size_t smem = 0;  // dynamic shared memory per CTA
  int smem_status = BYSJ_OK;
  SplitSlots ss{};
};

template <int L>
size_t gie_bwd_smem_bytes(int64_t lpe) {
  switch (lpe) {
    case 1: return kWarpsPerBlock * GieBwdSmem<1, L>::kWarpBytes;
    case 2: return kWarpsPerBlock * GieBwdSmem<2, L>::kWarpBytes;
    case 4: return kWarpsPerBlock * GieBwdSmem<4, L>::kWarpBytes;
    case 8: return kWarpsPerBlock * GieBwdSmem<8, L>::kWarpBytes;
    default: return kWarpsPerBlock * GieBwdSmem<16, L>::kWarpBytes;
  }
}

size_t gie_bwd_smem_size(int64_t degrees, int64_t channels) {
  const int64_t lpe = channels / 4;
  if (degrees == 1) return gie_bwd_smem_bytes<1>(lpe);
  if (degrees == 2) return gie_bwd_smem_bytes<2>(lpe);
  return gie_bwd_smem_bytes<3>(lpe);
}

size_t gie_fwd_smem_size(int64_t degrees) {
  switch (degrees) {
    case 1: return gie_fwd_smem_bytes<1>();
    case 2: return gie_fwd_smem_bytes<2>();
    default: return gie_fwd_smem_bytes<3>();
  }
}

GieDegreeLayout gie_degree_layout(int64_t n_edges, int64_t n_nodes, int64_t degrees,
                                  int64_t channels, void* ws, bool backward = false) {
  GieDegreeLayout L;
  L.kernel = gie_degree_kernel(degrees, channels, backward);
  if (L.kernel == nullptr) return L;
  const int64_t rows = (degrees + 1) * (degrees + 1) - 1;
  L.smem = backward ? gie_bwd_smem_size(degrees, channels) : gie_fwd_smem_size(degrees);
  L.smem_status = allow_dynamic_smem(reinterpret_cast<const void*>(L.kernel), L.smem);
  const DeviceInfo& dev = current_device_info();
  const int64_t resident = static_cast<int64_t>(dev.sm_count) *
                           resident_blocks(reinterpret_cast<const void*>(L.kernel), L.smem) *
                           kWarpsPerBlock;
  L.plan = plan_partitions(n_edges, n_nodes, resident, 16);
  const int64_t stride = (rows * channels + 7) / 8 * 8;
  // Tickets first: they then follow the generic layout's tickets (which end
  // that layout) across at most 255 bytes of padding, so one memset clears both.
  Carver carve(ws);
  int* tickets = carve.take<int>(static_cast<size_t>(L.plan.parts));
  float* slots = carve.take<float>(static_cast<size_t>(L.plan.parts) * 2 * stride);
  L.bytes = carve.need;
  L.ss = SplitSlots{slots, tickets, stride, 1};
  return L;
}

int gie_check(int64_t n_edges, int64_t n_nodes, int64_t rows, int64_t n_radial,
              int64_t channels) {
  if (n_edges < 0 || n_nodes < 0 || rows < 0 || n_radial < 0 || channels < 0)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "zonal scatter: invalid sizes");
  if (rows > 0 && n_radial == 0)
    return fail(BYSJ_ERR_INVALID_ARGUMENT,
                "zonal scatter: radial slots are required for non-scalar rows");
  if (n_edges > 0 && n_nodes == 0)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "zonal scatter: edges require nodes");
  return BYSJ_OK;
}

// Degrees L when a generic call has the shape of the degree-grouped layout
// (R = (L+1)^2 - 1 rows, channels = 4 * 2^k <= max_channels, 16-byte aligned
// rows), else 0.  Such a call launches the degree kernel with the slot table
// left on the device (it returns unless the table is the degree table) and
// then the generic kernel (it returns if the table is): no read back.
int64_t degree_candidate(int64_t rows, int64_t channels, int64_t max_channels, bool aligned) {
  if (!aligned || channels % 4 != 0 || channels > max_channels ||
      ((channels / 4) & (channels / 4 - 1)) != 0)
    return 0;
  for (int64_t l = 1; l <= 3; ++l)
    if ((l + 1) * (l + 1) - 1 == rows) return l;
  return 0;
}

size_t after256(size_t bytes) { return (bytes + 255) & ~size_t(255); }

}  // namespace
}  // namespace bysj

using namespace bysj;

extern "C" {

size_t bysj_gie_zonal_scatter_workspace_size(int64_t n_edges, int64_t n_nodes,
                                             int64_t n_rows, int64_t channels) {
  if (n_edges < 0 || n_nodes <= 0 || n_rows <= 0 || channels <= 0) return 0;
  const size_t a = gie_layout(true, n_edges, n_nodes, n_rows, channels, false, nullptr).bytes;
  const size_t b = gie_layout(false, n_edges, n_nodes, n_rows, channels, false, nullptr).bytes;
  const size_t generic = a > b ? a : b;
  const int64_t degrees = degree_candidate(n_rows, channels, 128, true);
  if (degrees == 0) return generic;
  return after256(generic) +
         gie_degree_layout(n_edges, n_nodes, degrees, channels, nullptr).bytes;
}

}  // extern "C"

namespace {

int gie_forward_impl(const float* zonal, const float* radial, const int64_t* offsets,
                     const int64_t* order, const int64_t* radial_slot,
                     const float* inv_sqrt_deg, int64_t n_edges, int64_t n_nodes,
                     int64_t n_rows, int64_t n_radial, int64_t channels, float* out,
                     void* workspace, size_t workspace_bytes, void* stream,
                     const uint32_t* gate) {
  clear_error();
  int st = gie_check(n_edges, n_nodes, n_rows, n_radial, channels);
  if (st) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t block = (n_rows + 1) * channels;
  if (n_nodes == 0 || block == 0) return BYSJ_OK;
  if (out == nullptr || inv_sqrt_deg == nullptr)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "zonal scatter: NULL out/inv_sqrt_deg");
  if (n_rows == 0 || channels == 0)
    return cuda_check(cudaMemsetAsync(out, 0, sizeof(float) * n_nodes * block, s),
                      "zonal scatter: zero output");
  if (offsets == nullptr || radial_slot == nullptr ||
      (n_edges > 0 && (zonal == nullptr || radial == nullptr)))
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "zonal scatter: NULL pointer");
  const bool vec_ok = aligned16(radial) && aligned16(out);
  GieLayout L = gie_layout(vec_ok, n_edges, n_nodes, n_rows, channels, false, workspace);
  const int64_t degrees = degree_candidate(n_rows, channels, 128, vec_ok);
  GieDegreeLayout D;
  size_t need = L.bytes;
  if (degrees > 0) {
    D = gie_degree_layout(n_edges, n_nodes, degrees, channels,
                          workspace ? static_cast<char*>(workspace) + after256(L.bytes) : nullptr);
    need = after256(L.bytes) + D.bytes;
    if (D.smem_status != BYSJ_OK) return D.smem_status;
  }
  if (workspace == nullptr || workspace_bytes < need)
    return fail(BYSJ_ERR_WORKSPACE,
                "zonal scatter: workspace of %zu bytes needed, %zu given",
                need, workspace_bytes);
  // One memset for both kernels' tickets (the degree layout's tickets follow
  // the generic layout's, across the alignment padding).
  const size_t ticket_bytes =
      degrees > 0 ? static_cast<size_t>(reinterpret_cast<char*>(D.ss.tickets + D.plan.parts) -
                                        reinterpret_cast<char*>(L.ss.tickets))
                  : sizeof(int) * L.plan.parts * L.cfg.tiles;
  st = cuda_check(cudaMemsetAsync(L.ss.tickets, 0, ticket_bytes, s),
                  "zonal scatter: ticket reset");
  if (st) return st;
  GieArgs a{};
  a.gate = gate;
  a.zonal = zonal;
  a.radial = radial;
  a.order = order;
  a.slot = radial_slot;
  a.inv = inv_sqrt_deg;
  a.out = out;
  a.rows = n_rows;
  a.n_radial = n_radial;
  a.channels = channels;
  a.lv = L.cfg.lv;
  a.mp = MergePath{offsets, n_nodes, n_edges, L.plan.ipc, L.plan.parts};
  a.ss = L.ss;
  if (degrees > 0) {
    GieArgs d = a;
    d.lv = 0;
    d.mp = MergePath{offsets, n_nodes, n_edges, D.plan.ipc, D.plan.parts};
    d.ss = D.ss;
    D.kernel<<<D.plan.blocks, kBlock, D.smem, s>>>(d, kSlotBaseOnDevice);
    st = launch_check("gie_fwd_degree_kernel");
    if (st) return st;
    a.skip_degrees = degrees;
  }
  dim3 grid(L.plan.blocks, static_cast<unsigned>(L.cfg.tiles));
  L.cfg.kernel<<<grid, kBlock, 0, s>>>(a);
  return launch_check("gie_fwd_kernel");
}

}  // namespace

extern "C" {

int bysj_gie_zonal_scatter_forward(const float* zonal, const float* radial,
                                   const int64_t* offsets, const int64_t* order,
                                   const int64_t* radial_slot, const float* inv_sqrt_deg,
                                   int64_t n_edges, int64_t n_nodes, int64_t n_rows,
                                   int64_t n_radial, int64_t channels, float* out,
                                   void* workspace, size_t workspace_bytes, void* stream) {
  return gie_forward_impl(zonal, radial, offsets, order, radial_slot, inv_sqrt_deg, n_edges,
                          n_nodes, n_rows, n_radial, channels, out, workspace, workspace_bytes,
                          stream, nullptr);
}

int bysj_gie_zonal_scatter_forward_gated(const float* zonal, const float* radial,
                                         const int64_t* offsets, const int64_t* order,
                                         const int64_t* radial_slot, const float* inv_sqrt_deg,
                                         int64_t n_edges, int64_t n_nodes, int64_t n_rows,
                                         int64_t n_radial, int64_t channels, float* out,
                                         void* workspace, size_t workspace_bytes, void* stream,
                                         const uint32_t* gate) {
  return gie_forward_impl(zonal, radial, offsets, order, radial_slot, inv_sqrt_deg, n_edges,
                          n_nodes, n_rows, n_radial, channels, out, workspace, workspace_bytes,
                          stream, gate);
}

size_t bysj_gie_zonal_scatter_degree_workspace_size(int64_t n_edges, int64_t n_nodes,
                                                    int64_t degrees, int64_t channels) {
  if (n_edges < 0 || n_nodes <= 0 || channels <= 0) return 0;
  return gie_degree_layout(n_edges, n_nodes, degrees, channels, nullptr).bytes;
}

int bysj_gie_zonal_scatter_forward_degree(const float* zonal, const float* radial,
                                          const int64_t* offsets, const int64_t* order,
                                          int64_t slot_base, const float* inv_sqrt_deg,
                                          int64_t n_edges, int64_t n_nodes, int64_t degrees,
                                          int64_t n_radial, int64_t channels, float* out,
                                          void* workspace, size_t workspace_bytes,
                                          void* stream) {
  clear_error();
  const int64_t rows = (degrees + 1) * (degrees + 1) - 1;
  int st = gie_check(n_edges, n_nodes, rows, n_radial, channels);
  if (st) return st;
  if (degrees < 1 || degrees > 3 || channels % 4 != 0 || channels > 128 ||
      (channels / 4 & (channels / 4 - 1)) != 0)
    return fail(BYSJ_ERR_UNSUPPORTED,
                "zonal scatter (degree rows): needs 1..3 degrees and channels = 4 * 2^k <= 128");
  // Degree l reads slot slot_base + l, l = 1..degrees.
  if (slot_base < -1 || slot_base + degrees > n_radial - 1)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "zonal scatter (degree rows): slots out of range");
  if (n_nodes == 0) return BYSJ_OK;
  if (out == nullptr || inv_sqrt_deg == nullptr || offsets == nullptr ||
      (n_edges > 0 && (zonal == nullptr || radial == nullptr)))
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "zonal scatter (degree rows): NULL pointer");
  if (!aligned16(radial) || !aligned16(out))
    return fail(BYSJ_ERR_INVALID_ARGUMENT,
                "zonal scatter (degree rows): radial and out must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  GieDegreeLayout L = gie_degree_layout(n_edges, n_nodes, degrees, channels, workspace);
  if (workspace == nullptr || workspace_bytes < L.bytes)
    return fail(BYSJ_ERR_WORKSPACE,
                "zonal scatter (degree rows): workspace of %zu bytes needed, %zu given",
                L.bytes, workspace_bytes);
  st = cuda_check(cudaMemsetAsync(L.ss.tickets, 0, sizeof(int) * L.plan.parts, s),
                  "zonal scatter (degree rows): ticket reset");
  if (st) return st;
  GieArgs a{};
  a.zonal = zonal;
  a.radial = radial;
  a.order = order;
  a.inv = inv_sqrt_deg;
  a.out = out;
  a.rows = rows;
  a.n_radial = n_radial;
  a.channels = channels;
  a.mp = MergePath{offsets, n_nodes, n_edges, L.plan.ipc, L.plan.parts};
  a.ss = L.ss;
  if (L.smem_status != BYSJ_OK) return L.smem_status;
  L.kernel<<<L.plan.blocks, kBlock, L.smem, s>>>(a, slot_base);
  return launch_check("gie_fwd_degree_kernel");
}

size_t bysj_gie_zonal_scatter_backward_workspace_size(int64_t n_edges,
                                                      int64_t n_nodes,
                                                      int64_t n_rows,
                                                      int64_t channels) {
  if (n_edges < 0 || n_nodes <= 0 || n_rows <= 0 || channels <= 0) return 0;
  const size_t a = gie_layout(true, n_edges, n_nodes, n_rows, channels, true, nullptr).bytes;
  const size_t b = gie_layout(false, n_edges, n_nodes, n_rows, channels, true, nullptr).bytes;
  const size_t generic = a > b ? a : b;
  const int64_t degrees = degree_candidate(n_rows, channels, 64, true);
  if (degrees == 0) return generic;
  return after256(generic) +
         gie_degree_layout(n_edges, n_nodes, degrees, channels, nullptr, true).bytes;
}

}  // extern "C"

namespace {

int gie_backward_impl(const float* grad_out, const float* zonal, const float* radial,
                      const int64_t* dst, const int64_t* offsets, const int64_t* order,
                      const int64_t* radial_slot, const float* inv_sqrt_deg, int64_t n_edges,
                      int64_t n_nodes, int64_t n_rows, int64_t n_radial, int64_t channels,
                      float* grad_zonal, float* grad_radial, float* grad_inv, void* workspace,
                      size_t workspace_bytes, void* stream, const uint32_t* gate) {
  clear_error();
  (void)dst;
  int st = gie_check(n_edges, n_nodes, n_rows, n_radial, channels);
  if (st) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n_nodes == 0) return BYSJ_OK;
  if (grad_inv == nullptr || inv_sqrt_deg == nullptr)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "zonal scatter backward: NULL grad_inv");
  if (n_rows == 0 || channels == 0 || n_edges == 0) {
    st = cuda_check(cudaMemsetAsync(grad_inv, 0, sizeof(float) * n_nodes, s),
                    "zonal scatter backward: zero grad_inv");
    if (st) return st;
    if (n_edges > 0 && grad_zonal && n_rows > 0)
      st = cuda_check(cudaMemsetAsync(grad_zonal, 0, sizeof(float) * n_edges * n_rows, s),
                      "zonal scatter backward: zero grad_zonal");
    if (!st && n_edges > 0 && grad_radial && n_radial > 0 && channels > 0)
      st = cuda_check(cudaMemsetAsync(grad_radial, 0,
                                      sizeof(float) * n_edges * n_radial * channels, s),
                      "zonal scatter backward: zero grad_radial");
    return st;
  }
  if (offsets == nullptr || radial_slot == nullptr || zonal == nullptr ||
      radial == nullptr || grad_out == nullptr || grad_zonal == nullptr ||
      grad_radial == nullptr)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "zonal scatter backward: NULL pointer");
  const bool vec_ok = aligned16(radial) && aligned16(grad_out) &&
                      aligned16(grad_radial) && channels % 4 == 0;
  GieLayout L = gie_layout(vec_ok, n_edges, n_nodes, n_rows, channels, true, workspace);
  if (L.cfg.tiles != 1)
    return fail(BYSJ_ERR_UNSUPPORTED,
                "zonal scatter backward: rows*channels = %lld exceeds %d",
                (long long)(n_rows * channels), kWarp * 8 * L.cfg.vec);
  const int64_t degrees = degree_candidate(n_rows, channels, 64, vec_ok);
  GieDegreeLayout D;
  size_t need = L.bytes;
  if (degrees > 0) {
    D = gie_degree_layout(n_edges, n_nodes, degrees, channels,
                          workspace ? static_cast<char*>(workspace) + after256(L.bytes) : nullptr,
                          true);
    need = after256(L.bytes) + D.bytes;
    if (D.smem_status != BYSJ_OK) return D.smem_status;
  }
  if (workspace == nullptr || workspace_bytes < need)
    return fail(BYSJ_ERR_WORKSPACE,
                "zonal scatter backward: workspace of %zu bytes needed, %zu given",
                need, workspace_bytes);
  const size_t ticket_bytes =
      degrees > 0 ? static_cast<size_t>(reinterpret_cast<char*>(D.ss.tickets + D.plan.parts) -
                                        reinterpret_cast<char*>(L.ss.tickets))
                  : sizeof(int) * L.plan.parts;
  st = cuda_check(cudaMemsetAsync(L.ss.tickets, 0, ticket_bytes, s),
                  "zonal scatter backward: ticket reset");
  if (st) return st;
  GieArgs a{};
  a.gate = gate;
  a.zonal = zonal;
  a.radial = radial;
  a.order = order;
  a.slot = radial_slot;
  a.inv = inv_sqrt_deg;
  a.grad = grad_out;
  a.out = grad_inv;
  a.grad_zonal = grad_zonal;
  a.grad_radial = grad_radial;
  a.rows = n_rows;
  a.n_radial = n_radial;
  a.channels = channels;
  a.lv = L.cfg.lv;
  a.mp = MergePath{offsets, n_nodes, n_edges, L.plan.ipc, L.plan.parts};
  a.ss = L.ss;
  if (degrees > 0) {
    GieArgs d = a;
    d.lv = 0;
    d.mp = MergePath{offsets, n_nodes, n_edges, D.plan.ipc, D.plan.parts};
    d.ss = D.ss;
    D.kernel<<<D.plan.blocks, kBlock, D.smem, s>>>(d, kSlotBaseOnDevice);
    st = launch_check("gie_bwd_degree_kernel");
    if (st) return st;
    a.skip_degrees = degrees;
  }
  const size_t smem = sizeof(float) * kBlock * L.cfg.nv;
  L.cfg.kernel<<<L.plan.blocks, kBlock, smem, s>>>(a);
  return launch_check("gie_bwd_kernel");
}

}  // namespace

extern "C" {

int bysj_gie_zonal_scatter_backward(
    const float* grad_out, const float* zonal, const float* radial, const int64_t* dst,
    const int64_t* offsets, const int64_t* order, const int64_t* radial_slot,
    const float* inv_sqrt_deg, int64_t n_edges, int64_t n_nodes, int64_t n_rows,
    int64_t n_radial, int64_t channels, float* grad_zonal, float* grad_radial,
    float* grad_inv, void* workspace, size_t workspace_bytes, void* stream) {
  return gie_backward_impl(grad_out, zonal, radial, dst, offsets, order, radial_slot,
                           inv_sqrt_deg, n_edges, n_nodes, n_rows, n_radial, channels,
                           grad_zonal, grad_radial, grad_inv, workspace, workspace_bytes,
                           stream, nullptr);
}

int bysj_gie_zonal_scatter_backward_gated(
    const float* grad_out, const float* zonal, const float* radial, const int64_t* dst,
    const int64_t* offsets, const int64_t* order, const int64_t* radial_slot,
    const float* inv_sqrt_deg, int64_t n_edges, int64_t n_nodes, int64_t n_rows,
    int64_t n_radial, int64_t channels, float* grad_zonal, float* grad_radial,
    float* grad_inv, void* workspace, size_t workspace_bytes, void* stream,
    const uint32_t* gate) {
  return gie_backward_impl(grad_out, zonal, radial, dst, offsets, order, radial_slot,
                           inv_sqrt_deg, n_edges, n_nodes, n_rows, n_radial, channels,
                           grad_zonal, grad_radial, grad_inv, workspace, workspace_bytes,
                           stream, gate);
}

size_t bysj_gie_zonal_scatter_backward_degree_workspace_size(int64_t n_edges, int64_t n_nodes,
                                                             int64_t degrees, int64_t channels) {
  if (n_edges < 0 || n_nodes <= 0 || channels <= 0) return 0;
  return gie_degree_layout(n_edges, n_nodes, degrees, channels, nullptr, true).bytes;
}

int bysj_gie_zonal_scatter_backward_degree(
    const float* grad_out, const float* zonal, const float* radial, const int64_t* offsets,
    const int64_t* order, int64_t slot_base, const float* inv_sqrt_deg, int64_t n_edges,
    int64_t n_nodes, int64_t degrees, int64_t n_radial, int64_t channels, float* grad_zonal,
    float* grad_radial, float* grad_inv, void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  const int64_t rows = (degrees + 1) * (degrees + 1) - 1;
  int st = gie_check(n_edges, n_nodes, rows, n_radial, channels);
  if (st) return st;
  if (degrees < 1 || degrees > 3 || channels % 4 != 0 || channels > 64 ||
      (channels / 4 & (channels / 4 - 1)) != 0)
    return fail(BYSJ_ERR_UNSUPPORTED,
                "zonal scatter backward (degree rows): needs 1..3 degrees and channels = "
                "4 * 2^k <= 64");
  if (slot_base < -1 || slot_base + degrees > n_radial - 1)
    return fail(BYSJ_ERR_INVALID_ARGUMENT,
                "zonal scatter backward (degree rows): slots out of range");
  if (n_nodes == 0) return BYSJ_OK;
  if (grad_inv == nullptr || inv_sqrt_deg == nullptr || offsets == nullptr || grad_out == nullptr ||
      (n_edges > 0 && (zonal == nullptr || radial == nullptr || grad_zonal == nullptr ||
                       grad_radial == nullptr)))
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "zonal scatter backward (degree rows): NULL pointer");
  if (!aligned16(radial) || !aligned16(grad_out) || !aligned16(grad_radial))
    return fail(BYSJ_ERR_INVALID_ARGUMENT,
                "zonal scatter backward (degree rows): radial, grad_out and grad_radial must be "
                "16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  GieDegreeLayout L = gie_degree_layout(n_edges, n_nodes, degrees, channels, workspace, true);
  if (workspace == nullptr || workspace_bytes < L.bytes)
    return fail(BYSJ_ERR_WORKSPACE,
                "zonal scatter backward (degree rows): workspace of %zu bytes needed, %zu given",
                L.bytes, workspace_bytes);
  st = cuda_check(cudaMemsetAsync(L.ss.tickets, 0, sizeof(int) * L.plan.parts, s),
                  "zonal scatter backward (degree rows): ticket reset");
  if (st) return st;
  GieArgs a{};
  a.zonal = zonal;
  a.radial = radial;
  a.order = order;
  a.inv = inv_sqrt_deg;
  a.grad = grad_out;
  a.out = grad_inv;
  a.grad_zonal = grad_zonal;
  a.grad_radial = grad_radial;
  a.rows = rows;
  a.n_radial = n_radial;
  a.channels = channels;
  a.mp = MergePath{offsets, n_nodes, n_edges, L.plan.ipc, L.plan.parts};
  a.ss = L.ss;
  if (L.smem_status != BYSJ_OK) return L.smem_status;
  L.kernel<<<L.plan.blocks, kBlock, L.smem, s>>>(a, slot_base);
  return launch_check("gie_bwd_degree_kernel");
}

}  // extern "C"
