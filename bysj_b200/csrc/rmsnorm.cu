// Last-axis RMSNorm for sm_100a, fp32 or bf16 rows, fp32 math.
//
//   inv[r] = rsqrt(mean_c x[r,c]^2 + eps);  y[r,c] = x[r,c] * inv[r] * w[c]
//
// Contract of the reference's csrc/rmsnorm.cpp:24-77, plus a per-degree
// weight table: with scale_rows = L + 1 > 1, row r is irreps component
// i = r mod (L+1)^2 and uses weight row l = floor(sqrt(i)).
//
// Each row is read once into registers (16-byte loads; a narrow row packs
// several rows into one warp), reduced with a butterfly and written once, so
// HBM traffic is one read and one write of x.  Several rows are in flight per
// lane.  The backward's scale gradient is reduced in two deterministic stages
// (per row-chunk partial sums, then a fixed-order sum over chunks) instead of
// the reference's float atomicAdd.
#include "launch.cuh"

namespace bysj {
namespace {

// Degree l = floor(sqrt(i)) of irreps component i = r mod comps.  Row
// counts below 2^32 use 32-bit arithmetic (64-bit division is slow).
__device__ __forceinline__ int64_t degree_of_row(int64_t r, int64_t comps) {
  uint32_t i;
  if (r < (int64_t(1) << 32)) {
    i = static_cast<uint32_t>(r) % static_cast<uint32_t>(comps);
  } else {
    i = static_cast<uint32_t>(r % comps);
  }
  uint32_t l = 0;
  while ((l + 1) * (l + 1) <= i) ++l;
  return l;
}

struct NormArgs {
  const void* x;
  void* y;
  float* inv_rms;
  const float* scale;
  int64_t scale_rows;  // 0: none, 1: per channel, L+1: per degree
  int64_t comps;       // (L+1)^2 when scale_rows > 1
  int64_t rows, width, lv;
  float eps;
};

template <typename T>
__device__ __forceinline__ void store_row(T* dst, const float* v, int n);

template <>
__device__ __forceinline__ void store_row<float>(float* dst, const float* v, int n) {
  if (n == 4) *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
  else for (int i = 0; i < n; ++i) dst[i] = v[i];
}

template <>
__device__ __forceinline__ void store_row<__nv_bfloat16>(__nv_bfloat16* dst,
                                                         const float* v, int n) {
  if (n == 8) {
    uint4 w;
    __nv_bfloat162 p0 = __floats2bfloat162_rn(v[0], v[1]);
    __nv_bfloat162 p1 = __floats2bfloat162_rn(v[2], v[3]);
    __nv_bfloat162 p2 = __floats2bfloat162_rn(v[4], v[5]);
    __nv_bfloat162 p3 = __floats2bfloat162_rn(v[6], v[7]);
    w.x = *reinterpret_cast<uint32_t*>(&p0);
    w.y = *reinterpret_cast<uint32_t*>(&p1);
    w.z = *reinterpret_cast<uint32_t*>(&p2);
    w.w = *reinterpret_cast<uint32_t*>(&p3);
    *reinterpret_cast<uint4*>(dst) = w;
  } else {
    for (int i = 0; i < n; ++i) dst[i] = __float2bfloat16_rn(v[i]);
  }
}

// G rows per warp (LPG = 32/G lanes each), NV vectors per lane, R row-blocks
// loaded before any is reduced.  WMODE: 0 no weight, 1 one weight row,
// 2 per-degree weight table.  Weights are staged once per CTA in shared
// memory (at most kMaxSmemWeights floats), so the per-row cost is one
// shared-memory vector load per vector.
constexpr int kMaxSmemWeights = 8192;

template <typename T, int VEC, int NV, int G, int R, int WMODE>
__global__ void __launch_bounds__(kBlock) rmsnorm_fwd_kernel(NormArgs a) {
  constexpr int LPG = kWarp / G;
  extern __shared__ __align__(16) float s_w[];  // weights, dynamic size
  if constexpr (WMODE != 0) {
    const int64_t count = (WMODE == 2 ? a.scale_rows : 1) * a.width;
    for (int64_t i = threadIdx.x; i < count; i += blockDim.x) s_w[i] = __ldg(a.scale + i);
    __syncthreads();
  }
  const int lane = lane_id();
  const int g = lane / LPG;
  const int jl0 = lane % LPG;
  const T* x = static_cast<const T*>(a.x);
  T* y = static_cast<T*>(a.y);
  const int64_t warps = static_cast<int64_t>(gridDim.x) * kWarpsPerBlock;
  const int64_t step = warps * G * R;
  int64_t jl[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int64_t j = jl0 + k * LPG;
    jl[k] = j < a.lv ? j : a.lv - 1;
  }
  const bool pow2_comps = (a.comps & (a.comps - 1)) == 0;
  const float inv_width = 1.0f / static_cast<float>(a.width);
  for (int64_t base = global_warp() * G * R; base < a.rows; base += step) {
    // bf16 rows: the warp's block of rows two steps ahead (contiguous) is
    // requested into L2 by one bulk prefetch (C2 bf16: 34.8 -> 32.8 us);
    // fp32 rows gained nothing from it.
    if constexpr (sizeof(T) == 2 && VEC * sizeof(T) == 16) {
      const int64_t nb = base + 2 * step;
      if (lane == 0 && nb < a.rows) {
        const int64_t cnt = a.rows - nb < G * R ? a.rows - nb : G * R;
        prefetch_l2_bulk(x + nb * a.width, static_cast<uint32_t>(cnt * a.width * sizeof(T)));
      }
    }
    RowVec<T, VEC> buf[R][NV];
#pragma unroll
    for (int rr = 0; rr < R; ++rr) {
      int64_t r = base + rr * G + g;
      if (r >= a.rows) r = a.rows - 1;  // duplicate read, never stored
#pragma unroll
      for (int k = 0; k < NV; ++k) buf[rr][k].load(x + r * a.width, jl[k]);
    }
#pragma unroll
    for (int rr = 0; rr < R; ++rr) {
      const int64_t r = base + rr * G + g;
      float ss = 0.0f;
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        if (jl0 + k * LPG < a.lv) {  // partial tiles: clamped lanes hold duplicates
#pragma unroll
          for (int i = 0; i < VEC; ++i) {
            const float v = buf[rr][k].get(i);
            ss = fmaf(v, v, ss);
          }
        }
      }
      ss = group_sum(ss, LPG);
      const float inv = rsqrtf(ss * inv_width + a.eps);
      if (r >= a.rows) continue;
      if (jl0 == 0) a.inv_rms[r] = inv;
      int wrow = 0;
      if constexpr (WMODE == 2) {
        const uint32_t i = pow2_comps ? static_cast<uint32_t>(r) & static_cast<uint32_t>(a.comps - 1)
                                      : static_cast<uint32_t>(r % a.comps);
        wrow = (i >= 1) + (i >= 4) + (i >= 9) + (i >= 16) + (i >= 25) + (i >= 36) + (i >= 49);
      }
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const int64_t j = jl0 + k * LPG;
        if (j < a.lv) {
          float v[VEC];
          if constexpr (WMODE == 0) {
#pragma unroll
            for (int i = 0; i < VEC; ++i) v[i] = buf[rr][k].get(i) * inv;
          } else {
            const float* w = s_w + wrow * a.width + j * VEC;
#pragma unroll
            for (int i = 0; i < VEC; i += (VEC % 4 == 0 ? 4 : 1)) {
              if constexpr (VEC % 4 == 0) {
                const float4 t = *reinterpret_cast<const float4*>(w + i);
                v[i] = buf[rr][k].get(i) * inv * t.x;
                v[i + 1] = buf[rr][k].get(i + 1) * inv * t.y;
                v[i + 2] = buf[rr][k].get(i + 2) * inv * t.z;
                v[i + 3] = buf[rr][k].get(i + 3) * inv * t.w;
              } else {
                v[i] = buf[rr][k].get(i) * inv * w[i];
              }
            }
          }
          store_row<T>(y + r * a.width + j * VEC, v, VEC);
        }
      }
    }
  }
}

// Rows wider than one warp tile: two passes over the row (the second hits L2).
template <typename T>
__global__ void __launch_bounds__(kBlock) rmsnorm_fwd_wide_kernel(NormArgs a) {
  const int lane = lane_id();
  const T* x = static_cast<const T*>(a.x);
  T* y = static_cast<T*>(a.y);
  const int64_t warps = static_cast<int64_t>(gridDim.x) * kWarpsPerBlock;
  for (int64_t r = global_warp(); r < a.rows; r += warps) {
    const T* row = x + r * a.width;
    float ss = 0.0f;
    for (int64_t c = lane; c < a.width; c += kWarp) {
      RowVec<T, 1> v;
      v.load(row, c);
      ss = fmaf(v.get(0), v.get(0), ss);
    }
    ss = xor_sum(ss, 1);
    const float inv = rsqrtf(ss / static_cast<float>(a.width) + a.eps);
    if (lane == 0) a.inv_rms[r] = inv;
    const float* w = nullptr;
    if (a.scale) {
      const int64_t l = a.scale_rows > 1 ? degree_of_row(r, a.comps) : 0;
      w = a.scale + l * a.width;
    }
    for (int64_t c = lane; c < a.width; c += kWarp) {
      RowVec<T, 1> v;
      v.load(row, c);
      float o = v.get(0) * inv;
      if (w) o *= __ldg(w + c);
      store_row<T>(y + r * a.width + c, &o, 1);
    }
  }
}

// ---- backward -------------------------------------------------------------
// gx = inv*gw - x*inv^3*mean(x*gw), gw = g*w   (one warp per row, fp32)
__global__ void __launch_bounds__(kBlock)
    rmsnorm_bwd_kernel(const float* __restrict__ grad, const float* __restrict__ x,
                       const float* __restrict__ scale, int64_t scale_rows,
                       int64_t comps, const float* __restrict__ inv_rms,
                       int64_t rows, int64_t width, float* __restrict__ grad_x) {
  const int lane = lane_id();
  const int64_t warps = static_cast<int64_t>(gridDim.x) * kWarpsPerBlock;
  for (int64_t r = global_warp(); r < rows; r += warps) {
    const float* gr = grad + r * width;
    const float* xr = x + r * width;
    const float* w = nullptr;
    if (scale) {
      const int64_t l = scale_rows > 1 ? degree_of_row(r, comps) : 0;
      w = scale + l * width;
    }
    float dot = 0.0f;
    for (int64_t c = lane; c < width; c += kWarp) {
      const float up = __ldg(gr + c) * (w ? __ldg(w + c) : 1.0f);
      dot = fmaf(__ldg(xr + c), up, dot);
    }
    dot = xor_sum(dot, 1);
    const float mean_dot = dot / static_cast<float>(width);
    const float inv = __ldg(inv_rms + r);
    const float inv3 = inv * inv * inv;
    for (int64_t c = lane; c < width; c += kWarp) {
      const float up = __ldg(gr + c) * (w ? __ldg(w + c) : 1.0f);
      grad_x[r * width + c] = inv * up - __ldg(xr + c) * inv3 * mean_dot;
    }
  }
}

// Vectorised backward for rows of 4 K floats (K = 32 NV lanes x 4), at most
// kBwdMaxDegrees weight rows: one pass over g and x.  A warp takes R rows at a
// time (16-byte loads for all of them issued first), writes gx, and keeps
// its share of grad_scale per weight row in registers; the warps' partials
// land in partial[warp][l][c] and are summed in warp order afterwards.
constexpr int kBwdMaxDegrees = 4;

template <int NV, int R>
__global__ void __launch_bounds__(kBlock)
    rmsnorm_bwd_vec_kernel(const float* __restrict__ grad, const float* __restrict__ x,
                           const float* __restrict__ scale, int64_t scale_rows, int64_t comps,
                           const float* __restrict__ inv_rms, int64_t rows, int64_t width,
                           float* __restrict__ grad_x, float* __restrict__ partial) {
  const int lane = lane_id();
  const int64_t warps = static_cast<int64_t>(gridDim.x) * kWarpsPerBlock;
  const int64_t w = global_warp();
  const float inv_width = 1.0f / static_cast<float>(width);
  float acc[kBwdMaxDegrees][NV][4];
#pragma unroll
  for (int l = 0; l < kBwdMaxDegrees; ++l)
#pragma unroll
    for (int k = 0; k < NV; ++k)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[l][k][i] = 0.0f;
  for (int64_t r0 = w * R; r0 < rows; r0 += warps * R) {
    float4 gv[R][NV], xv[R][NV];
    float invr[R];
#pragma unroll
    for (int rr = 0; rr < R; ++rr) {
      const int64_t r = r0 + rr < rows ? r0 + rr : rows - 1;
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const int64_t c = 4 * (lane + kWarp * k);
        gv[rr][k] = ld_stream_f4(grad + r * width + c);
        xv[rr][k] = ld_stream_f4(x + r * width + c);
      }
      invr[rr] = __ldg(inv_rms + r);  // with the rows, not after their dot product
    }
#pragma unroll
    for (int rr = 0; rr < R; ++rr) {
      const int64_t r = r0 + rr;
      if (r >= rows) break;  // warp-uniform
      const int l = scale_rows > 1 ? static_cast<int>(degree_of_row(r, comps)) : 0;
      float4 wv[NV];
#pragma unroll
      for (int k = 0; k < NV; ++k)
        wv[k] = scale ? __ldg(reinterpret_cast<const float4*>(scale + l * width) + lane + kWarp * k)
                      : make_float4(1.0f, 1.0f, 1.0f, 1.0f);
      float dot = 0.0f;
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        dot = fmaf(xv[rr][k].x, gv[rr][k].x * wv[k].x, dot);
        dot = fmaf(xv[rr][k].y, gv[rr][k].y * wv[k].y, dot);
        dot = fmaf(xv[rr][k].z, gv[rr][k].z * wv[k].z, dot);
        dot = fmaf(xv[rr][k].w, gv[rr][k].w * wv[k].w, dot);
      }
      dot = xor_sum(dot, 1);
      const float inv = invr[rr];
      const float coef = inv * inv * inv * (dot * inv_width);
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const int64_t c = 4 * (lane + kWarp * k);
        const float4 g4 = gv[rr][k], x4 = xv[rr][k], w4 = wv[k];
        *reinterpret_cast<float4*>(grad_x + r * width + c) =
            make_float4(inv * (g4.x * w4.x) - x4.x * coef, inv * (g4.y * w4.y) - x4.y * coef,
                        inv * (g4.z * w4.z) - x4.z * coef, inv * (g4.w * w4.w) - x4.w * coef);
        if (partial) {
#pragma unroll
          for (int ll = 0; ll < kBwdMaxDegrees; ++ll) {
            if (ll != l) continue;
            acc[ll][k][0] = fmaf(g4.x * x4.x, inv, acc[ll][k][0]);
            acc[ll][k][1] = fmaf(g4.y * x4.y, inv, acc[ll][k][1]);
            acc[ll][k][2] = fmaf(g4.z * x4.z, inv, acc[ll][k][2]);
            acc[ll][k][3] = fmaf(g4.w * x4.w, inv, acc[ll][k][3]);
          }
        }
      }
    }
  }
  if (partial) {
    // Fold the CTA's warps in warp order through shared memory; one partial
    // per CTA: partial[block][l][c].
    __shared__ float4 fold[kWarpsPerBlock][kBwdMaxDegrees][2 * kWarp];
    const int64_t srows = scale_rows > 0 ? scale_rows : 1;
    const int warp = threadIdx.x >> 5;
#pragma unroll
    for (int l = 0; l < kBwdMaxDegrees; ++l)
#pragma unroll
      for (int k = 0; k < NV; ++k)
        fold[warp][l][lane + kWarp * k] =
            make_float4(acc[l][k][0], acc[l][k][1], acc[l][k][2], acc[l][k][3]);
    __syncthreads();
    const int cols4 = static_cast<int>(width / 4);
    for (int i = threadIdx.x; i < srows * cols4; i += blockDim.x) {
      const int l = i / cols4;
      const int c4 = i - l * cols4;
      float4 sum = fold[0][l][c4];
      for (int ww = 1; ww < kWarpsPerBlock; ++ww) {
        const float4 v = fold[ww][l][c4];
        sum.x += v.x;
        sum.y += v.y;
        sum.z += v.z;
        sum.w += v.w;
      }
      *reinterpret_cast<float4*>(partial + (blockIdx.x * srows + l) * width + 4 * c4) = sum;
    }
  }
}

// Stage 1 of grad_scale: partial[chunk, l, c] = sum over the chunk's rows of
// weight row l of g*x*inv.  Threads own columns; rows are visited in order.
__global__ void __launch_bounds__(kBlock)
    rmsnorm_scale_partial_kernel(const float* __restrict__ grad,
                                 const float* __restrict__ x,
                                 const float* __restrict__ inv_rms,
                                 int64_t rows, int64_t width, int64_t scale_rows,
                                 int64_t comps, int64_t chunk_rows,
                                 float* __restrict__ partial) {
  const int64_t chunk = blockIdx.x;
  const int64_t r0 = chunk * chunk_rows;
  int64_t r1 = r0 + chunk_rows;
  if (r1 > rows) r1 = rows;
  for (int64_t c = threadIdx.x + static_cast<int64_t>(blockIdx.y) * blockDim.x;
       c < width; c += static_cast<int64_t>(gridDim.y) * blockDim.x) {
    for (int64_t l = 0; l < scale_rows; ++l) {
      float acc = 0.0f;
      for (int64_t r = r0; r < r1; ++r) {
        if (scale_rows > 1 && degree_of_row(r, comps) != l) continue;
        acc = fmaf(__ldg(grad + r * width + c) * __ldg(x + r * width + c),
                   __ldg(inv_rms + r), acc);
      }
      partial[(chunk * scale_rows + l) * width + c] = acc;
    }
  }
}

// Stage 2: grad_scale[cell] = sum over k of partial[k, cell], in a fixed
// order: a CTA takes 32 cells; thread group g (8 groups) sums k = g, g+8, ...
// into four interleaved accumulators (k / 8 mod 4), which are added in
// order, and the 8 group sums are added in group order.
__global__ void __launch_bounds__(kBlock)
    rmsnorm_scale_reduce_kernel(const float* __restrict__ partial,
                                int64_t chunks, int64_t cells,
                                float* __restrict__ grad_scale) {
  __shared__ float groups[kWarpsPerBlock][kWarp];
  const int g = threadIdx.x >> 5;
  const int64_t cell = static_cast<int64_t>(blockIdx.x) * kWarp + lane_id();
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  if (cell < cells) {
    int64_t k = g;
    for (; k + 3 * kWarpsPerBlock < chunks; k += 4 * kWarpsPerBlock) {
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[j] += __ldcg(partial + (k + j * kWarpsPerBlock) * cells + cell);
    }
    for (int j = 0; k < chunks; k += kWarpsPerBlock, ++j)
      acc[j & 3] += __ldcg(partial + k * cells + cell);
  }
  groups[g][lane_id()] = (acc[0] + acc[1]) + (acc[2] + acc[3]);
  __syncthreads();
  if (g == 0 && cell < cells) {
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < kWarpsPerBlock; ++j) sum += groups[j][lane_id()];
    grad_scale[cell] = sum;
  }
}

unsigned reduce_blocks(int64_t cells) {
  return static_cast<unsigned>((cells + kWarp - 1) / kWarp);
}

using NormKernel = void (*)(NormArgs);

template <typename T, int VEC, int WM>
NormKernel norm_pick_w(int64_t lv, int* g_out) {
  *g_out = 1;
  if (lv > 256) return nullptr;
  if (lv > 128) return rmsnorm_fwd_kernel<T, VEC, 8, 1, 1, WM>;
  if (lv > 64) return rmsnorm_fwd_kernel<T, VEC, 4, 1, 2, WM>;
  if (lv > 32) return rmsnorm_fwd_kernel<T, VEC, 2, 1, 4, WM>;
  switch (next_pow2(lv)) {
    case 32: return rmsnorm_fwd_kernel<T, VEC, 1, 1, 4, WM>;
    case 16: *g_out = 4; return rmsnorm_fwd_kernel<T, VEC, 2, 4, 2, WM>;
    case 8: *g_out = 4; return rmsnorm_fwd_kernel<T, VEC, 1, 4, 4, WM>;
    case 4: *g_out = 8; return rmsnorm_fwd_kernel<T, VEC, 1, 8, 4, WM>;
    case 2: *g_out = 16; return rmsnorm_fwd_kernel<T, VEC, 1, 16, 4, WM>;
    default: *g_out = 32; return rmsnorm_fwd_kernel<T, VEC, 1, 32, 4, WM>;
  }
}

template <typename T, int VEC>
NormKernel norm_pick(int64_t lv, int wmode, int* g_out) {
  if (wmode == 0) return norm_pick_w<T, VEC, 0>(lv, g_out);
  if (wmode == 1) return norm_pick_w<T, VEC, 1>(lv, g_out);
  return norm_pick_w<T, VEC, 2>(lv, g_out);
}

int64_t scale_comps(int64_t scale_rows) { return scale_rows * scale_rows; }

int64_t scale_chunks(int64_t rows) {
  const int64_t target = static_cast<int64_t>(current_device_info().sm_count) * 4;
  int64_t chunk_rows = (rows + target - 1) / target;
  if (chunk_rows < 1) chunk_rows = 1;
  return chunk_rows;
}

}  // namespace
}  // namespace bysj

using namespace bysj;

extern "C" {

int bysj_rmsnorm_forward(const void* x, int dtype, int64_t rows, int64_t width,
                         const float* scale, int64_t scale_rows, float eps,
                         void* y, float* inv_rms, void* stream) {
  clear_error();
  if (rows < 0 || width <= 0)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "rmsnorm: invalid sizes");
  if (!(eps > 0.0f) || !isfinite(eps))
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "rmsnorm: eps must be finite and positive");
  if (dtype != BYSJ_F32 && dtype != BYSJ_BF16)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "rmsnorm: unknown dtype");
  if (scale == nullptr) scale_rows = 0;
  if (scale != nullptr && scale_rows < 1)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "rmsnorm: scale_rows must be >= 1");
  if (rows == 0) return BYSJ_OK;
  if (x == nullptr || y == nullptr || inv_rms == nullptr)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "rmsnorm: NULL pointer");
  const int64_t comps = scale_rows > 1 ? scale_comps(scale_rows) : 1;
  if (scale_rows > 1 && rows % comps != 0)
    return fail(BYSJ_ERR_INVALID_ARGUMENT,
                "rmsnorm: per-degree weights need rows to be a multiple of %lld",
                (long long)comps);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  NormArgs a;
  a.x = x;
  a.y = y;
  a.inv_rms = inv_rms;
  a.scale = scale;
  a.scale_rows = scale_rows;
  a.comps = comps;
  a.rows = rows;
  a.width = width;
  a.eps = eps;
  const bool bf16 = dtype == BYSJ_BF16;
  const int vec = bf16 ? 8 : 4;
  const bool vec_ok = width % vec == 0 && aligned16(x) && aligned16(y) &&
                      (scale == nullptr || aligned16(scale));
  int g = 1;
  NormKernel k = nullptr;
  // Weights staged in shared memory when they fit; otherwise the two-pass
  // wide kernel reads them from global memory.
  const int wmode = scale == nullptr ? 0 : (scale_rows > 1 ? 2 : 1);
  const bool smem_ok = scale == nullptr || scale_rows * width <= kMaxSmemWeights;
  const bool table_ok = scale_rows <= 8;  // degree test covers components < 64
  if (smem_ok && table_ok) {
    if (vec_ok) {
      a.lv = width / vec;
      k = bf16 ? norm_pick<__nv_bfloat16, 8>(a.lv, wmode, &g)
               : norm_pick<float, 4>(a.lv, wmode, &g);
    } else {
      a.lv = width;
      k = bf16 ? norm_pick<__nv_bfloat16, 1>(a.lv, wmode, &g)
               : norm_pick<float, 1>(a.lv, wmode, &g);
    }
  }
  const DeviceInfo& dev = current_device_info();
  const bool wide = k == nullptr;
  if (wide) {
    k = bf16 ? rmsnorm_fwd_wide_kernel<__nv_bfloat16> : rmsnorm_fwd_wide_kernel<float>;
    g = 1;
  }
  const size_t smem = (wide || wmode == 0)
                          ? 0
                          : sizeof(float) * static_cast<size_t>(wmode == 2 ? scale_rows : 1) * width;
  const int64_t resident = static_cast<int64_t>(dev.sm_count) *
                           resident_blocks(reinterpret_cast<const void*>(k), smem);
  int64_t blocks = (rows + static_cast<int64_t>(kWarpsPerBlock) * g - 1) /
                   (static_cast<int64_t>(kWarpsPerBlock) * g);
  if (blocks > resident) blocks = resident;
  if (blocks < 1) blocks = 1;
  k<<<static_cast<unsigned>(blocks), kBlock, smem, s>>>(a);
  return launch_check("rmsnorm_fwd_kernel");
}

// Warps of the vectorised backward: one wave of resident warps.
// Two rows per warp step and at most four CTAs per SM measured fastest at
// C2 (0.89 of the copy bandwidth, against 0.71 at four rows and eight CTAs):
// fewer CTAs also leave fewer grad_scale partials to reduce.
int64_t bwd_vec_warps(int64_t rows) {
  const int64_t per_block = static_cast<int64_t>(kWarpsPerBlock) * 2;
  int64_t blocks = (rows + per_block - 1) / per_block;
  const int64_t cap = static_cast<int64_t>(current_device_info().sm_count) * 4;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return blocks * kWarpsPerBlock;
}

bool bwd_vec_shape(int64_t width, int64_t scale_rows) {
  return width % 128 == 0 && width <= 256 && scale_rows <= kBwdMaxDegrees;
}

size_t bysj_rmsnorm_backward_workspace_size(int64_t rows, int64_t width,
                                            int64_t scale_rows) {
  if (rows <= 0 || width <= 0 || scale_rows < 1) return 0;
  const int64_t chunk_rows = scale_chunks(rows);
  const int64_t chunks = (rows + chunk_rows - 1) / chunk_rows;
  Carver carve(nullptr);
  carve.take<float>(static_cast<size_t>(chunks) * scale_rows * width);
  size_t need = carve.need;
  if (bwd_vec_shape(width, scale_rows)) {
    Carver vec(nullptr);
    vec.take<float>(static_cast<size_t>(bwd_vec_warps(rows) / kWarpsPerBlock) * scale_rows *
                    width);
    if (vec.need > need) need = vec.need;
  }
  return need;
}

int bysj_rmsnorm_backward(const float* grad_out, const float* x,
                          const float* scale, int64_t scale_rows,
                          const float* inv_rms, int64_t rows, int64_t width,
                          float* grad_x, float* grad_scale, void* workspace,
                          size_t workspace_bytes, void* stream) {
  clear_error();
  if (rows < 0 || width <= 0)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "rmsnorm backward: invalid sizes");
  if (scale == nullptr) scale_rows = 0;
  if (grad_scale != nullptr && scale == nullptr)
    return fail(BYSJ_ERR_INVALID_ARGUMENT,
                "rmsnorm backward: cannot compute a scale gradient without a scale");
  if (scale != nullptr && scale_rows < 1)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "rmsnorm backward: scale_rows must be >= 1");
  const int64_t comps = scale_rows > 1 ? scale_comps(scale_rows) : 1;
  if (scale_rows > 1 && rows % comps != 0)
    return fail(BYSJ_ERR_INVALID_ARGUMENT,
                "rmsnorm backward: rows must be a multiple of %lld", (long long)comps);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (rows == 0) {
    if (grad_scale)
      return cuda_check(cudaMemsetAsync(grad_scale, 0,
                                        sizeof(float) * scale_rows * width, s),
                        "rmsnorm backward: zero grad_scale");
    return BYSJ_OK;
  }
  if (grad_out == nullptr || x == nullptr || inv_rms == nullptr || grad_x == nullptr)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "rmsnorm backward: NULL pointer");
  const bool vec = bwd_vec_shape(width, scale_rows) && aligned16(grad_out) && aligned16(x) &&
                   aligned16(grad_x) && (scale == nullptr || aligned16(scale));
  if (vec) {
    const int64_t warps = bwd_vec_warps(rows);
    const int64_t vec_blocks = warps / kWarpsPerBlock;
    float* partial = nullptr;
    if (grad_scale != nullptr) {
      Carver carve(workspace);
      partial = carve.take<float>(static_cast<size_t>(vec_blocks) * scale_rows * width);
      if (workspace == nullptr || workspace_bytes < carve.need)
        return fail(BYSJ_ERR_WORKSPACE,
                    "rmsnorm backward: workspace of %zu bytes needed, %zu given", carve.need,
                    workspace_bytes);
    }
    const unsigned blocks = static_cast<unsigned>(warps / kWarpsPerBlock);
    if (width == 128)
      rmsnorm_bwd_vec_kernel<1, 2><<<blocks, kBlock, 0, s>>>(
          grad_out, x, scale, scale_rows, comps, inv_rms, rows, width, grad_x, partial);
    else
      rmsnorm_bwd_vec_kernel<2, 2><<<blocks, kBlock, 0, s>>>(
          grad_out, x, scale, scale_rows, comps, inv_rms, rows, width, grad_x, partial);
    int st = launch_check("rmsnorm_bwd_vec_kernel");
    if (st || grad_scale == nullptr) return st;
    const int64_t cells = scale_rows * width;
    rmsnorm_scale_reduce_kernel<<<reduce_blocks(cells), kBlock, 0, s>>>(partial, vec_blocks,
                                                                       cells, grad_scale);
    return launch_check("rmsnorm_scale_reduce_kernel");
  }
  const DeviceInfo& dev = current_device_info();
  int64_t blocks = (rows + kWarpsPerBlock - 1) / kWarpsPerBlock;
  const int64_t cap = static_cast<int64_t>(dev.sm_count) * 8;
  if (blocks > cap) blocks = cap;
  rmsnorm_bwd_kernel<<<static_cast<unsigned>(blocks), kBlock, 0, s>>>(
      grad_out, x, scale, scale_rows, comps, inv_rms, rows, width, grad_x);
  int st = launch_check("rmsnorm_bwd_kernel");
  if (st || grad_scale == nullptr) return st;
  const int64_t chunk_rows = scale_chunks(rows);
  const int64_t chunks = (rows + chunk_rows - 1) / chunk_rows;
  Carver carve(workspace);
  float* partial = carve.take<float>(static_cast<size_t>(chunks) * scale_rows * width);
  if (workspace == nullptr || workspace_bytes < carve.need)
    return fail(BYSJ_ERR_WORKSPACE,
                "rmsnorm backward: workspace of %zu bytes needed, %zu given",
                carve.need, workspace_bytes);
  int64_t col_blocks = (width + kBlock - 1) / kBlock;
  if (col_blocks > 65535) col_blocks = 65535;
  rmsnorm_scale_partial_kernel<<<dim3(static_cast<unsigned>(chunks),
                                      static_cast<unsigned>(col_blocks)),
                                 kBlock, 0, s>>>(grad_out, x, inv_rms, rows, width,
                                                 scale_rows, comps, chunk_rows,
                                                 partial);
  st = launch_check("rmsnorm_scale_partial_kernel");
  if (st) return st;
  const int64_t cells = scale_rows * width;
  rmsnorm_scale_reduce_kernel<<<reduce_blocks(cells), kBlock, 0, s>>>(partial, chunks, cells,
                                                                     grad_scale);
  return launch_check("rmsnorm_scale_reduce_kernel");
}

}  // extern "C"
