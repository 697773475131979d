// Edge-stream elementwise chain in one pass (sm_100a).
//
//   out[e, s, c] = act( sum_t coef_t * a_t[e, s, c] * b_t[e, s, c] )
//
// over an [E, S, C] edge stream, each factor a strided view that may
// broadcast along any of the three axes (stride 0), b_t optional.  This is
// the "term table -> one pass" kernel the reference plans for the largest
// remaining time pool of its DeepMD profile (docs/task2-hip-fusion-plan.md
// :280-302: residual adds, gates and attention-weighted broadcast
// multiply-adds over [E, 9/10, 64] rows, each a separate ATen pass today).
// Its gain is the pass count: k eager passes read and write the stream k
// times, this kernel reads each operand once and writes the result once, so
// it is HBM-bound at (sum of operand bytes + output bytes).
//
// Layout: the flat output index runs over rows r = e * S + s and columns c;
// a thread takes VEC = 4 consecutive columns when every operand whose column
// stride is 1 allows 16-byte loads (aligned base, row strides multiple of 4)
// and C % 4 == 0, else 1.  The kernel is instantiated per term count; a
// thread takes two elements per step and loads every operand of both before
// the first multiply-add, so all of them are in flight at once.  Index
// arithmetic divides by multiply-and-shift (32-bit flat indices).  Terms are summed in table order,
// acc = fma(coef * a, b, acc) with b = 1 for one-factor terms, so results are
// bit-identical run to run.
#include "launch.cuh"

namespace bysj {
namespace {

// Division of a 32-bit index by a fixed divisor d as a multiply and shifts
// (the round-up method of Granlund and Montgomery, "Division by invariant
// integers using multiplication", 1994): with l = ceil(log2 d) and
// m = floor(2^32 (2^l - d) / d) + 1, n / d = (t + ((n - t) >> 1)) >> (l - 1)
// where t = umulhi(n, m), for every n < 2^32 (d = 1: the identity).
struct FastDiv {
  uint32_t d = 1, m = 0, l = 0;
  FastDiv() = default;
  explicit FastDiv(uint32_t divisor) : d(divisor) {
    while ((uint64_t{1} << l) < d) ++l;
    m = static_cast<uint32_t>(((uint64_t{1} << 32) * ((uint64_t{1} << l) - d)) / d + 1);
  }
  __device__ __forceinline__ uint32_t div(uint32_t n) const {
    if (l == 0) return n;
    const uint32_t t = __umulhi(n, m);
    return (t + ((n - t) >> 1)) >> (l - 1);
  }
};

struct ChainArgs {
  bysj_chain_term terms[BYSJ_CHAIN_MAX_TERMS];
  int activation;
  int64_t comps, channels;
  int64_t vecs_per_row;  // channels / VEC
  int64_t total;         // rows * vecs_per_row
  FastDiv by_vecs, by_comps;  // valid when total < 2^32
  bool fast;
  float* out;
};

template <int VEC>
__device__ __forceinline__ void load_operand(const bysj_chain_operand& op, int64_t e, int64_t s,
                                             int64_t c, float (&v)[VEC]) {
  const float* p = op.data + e * op.stride[0] + s * op.stride[1] + c * op.stride[2];
  if (VEC == 4 && op.stride[2] == 1) {
    const float4 t = __ldg(reinterpret_cast<const float4*>(p));
    v[0] = t.x;
    v[1] = t.y;
    v[2] = t.z;
    v[3] = t.w;
  } else if (op.stride[2] == 0) {
    const float x = __ldg(p);
#pragma unroll
    for (int i = 0; i < VEC; ++i) v[i] = x;
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) v[i] = __ldg(p + i * op.stride[2]);
  }
}

__device__ __forceinline__ float activate(float z, int act) {
  if (act == BYSJ_ACT_SILU) return z / (1.0f + expf(-z));
  if (act == BYSJ_ACT_SIGMOID) return 1.0f / (1.0f + expf(-z));
  return z;
}

// Element i of the flat vector index: its edge, component and first column.
__device__ __forceinline__ void chain_coords(const ChainArgs& a, int64_t i, int64_t& e,
                                             int64_t& s, int64_t& c) {
  int64_t row;
  if (a.fast) {
    const uint32_t r = a.by_vecs.div(static_cast<uint32_t>(i));
    const uint32_t ee = a.by_comps.div(r);
    row = r;
    e = ee;
    s = static_cast<int64_t>(r) - static_cast<int64_t>(ee) * a.comps;
  } else {
    row = i / a.vecs_per_row;
    e = row / a.comps;
    s = row - e * a.comps;
  }
  c = i - row * a.vecs_per_row;
}

// NT terms (compile time); each thread takes two elements per step, loading
// every operand of both before the first multiply-add.
template <int VEC, int NT>
__global__ void __launch_bounds__(kBlock) edge_chain_kernel(ChainArgs a) {
  constexpr int U = 2;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i0 < a.total;
       i0 += U * stride) {
    int64_t e[U], s[U], c[U];
    bool ok[U];
    float x[U][NT][VEC], y[U][NT][VEC];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t i = i0 + u * stride;
      ok[u] = i < a.total;
      chain_coords(a, ok[u] ? i : i0, e[u], s[u], c[u]);
      c[u] *= VEC;
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        if (!ok[u]) continue;
        load_operand<VEC>(a.terms[t].a, e[u], s[u], c[u], x[u][t]);
        if (a.terms[t].b.data != nullptr) {
          load_operand<VEC>(a.terms[t].b, e[u], s[u], c[u], y[u][t]);
        } else {
#pragma unroll
          for (int k = 0; k < VEC; ++k) y[u][t][k] = 1.0f;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (!ok[u]) continue;
      float acc[VEC];
#pragma unroll
      for (int k = 0; k < VEC; ++k) acc[k] = 0.0f;
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const float coef = a.terms[t].coef;
#pragma unroll
        for (int k = 0; k < VEC; ++k) acc[k] = fmaf(coef * x[u][t][k], y[u][t][k], acc[k]);
      }
#pragma unroll
      for (int k = 0; k < VEC; ++k) acc[k] = activate(acc[k], a.activation);
      float* o = a.out + (e[u] * a.comps + s[u]) * a.channels + c[u];
      if constexpr (VEC == 4) {
        __stcs(reinterpret_cast<float4*>(o), make_float4(acc[0], acc[1], acc[2], acc[3]));
      } else {
        __stcs(o, acc[0]);
      }
    }
  }
}

using ChainKernel = void (*)(ChainArgs);

template <int VEC>
ChainKernel chain_kernel_for(int n_terms) {
  switch (n_terms) {
    case 1: return edge_chain_kernel<VEC, 1>;
    case 2: return edge_chain_kernel<VEC, 2>;
    case 3: return edge_chain_kernel<VEC, 3>;
    case 4: return edge_chain_kernel<VEC, 4>;
    case 5: return edge_chain_kernel<VEC, 5>;
    case 6: return edge_chain_kernel<VEC, 6>;
    case 7: return edge_chain_kernel<VEC, 7>;
    default: return edge_chain_kernel<VEC, 8>;
  }
}

bool operand_vec4_ok(const bysj_chain_operand& op) {
  if (op.data == nullptr) return true;
  if (op.stride[2] == 0) return true;  // broadcast along the columns: one scalar
  if (op.stride[2] != 1) return false;
  return aligned16(op.data) && op.stride[0] % 4 == 0 && op.stride[1] % 4 == 0;
}

}  // namespace
}  // namespace bysj

using namespace bysj;

extern "C" int bysj_edge_chain(const bysj_chain_term* terms, int n_terms, int64_t n_edges,
                               int64_t comps, int64_t channels, int activation, float* out,
                               void* stream) {
  clear_error();
  if (n_edges < 0 || comps <= 0 || channels <= 0)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "edge chain: invalid sizes");
  if (n_terms < 1 || n_terms > BYSJ_CHAIN_MAX_TERMS)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "edge chain: 1 to %d terms", BYSJ_CHAIN_MAX_TERMS);
  if (activation != BYSJ_ACT_NONE && activation != BYSJ_ACT_SILU &&
      activation != BYSJ_ACT_SIGMOID)
    return fail(BYSJ_ERR_INVALID_ARGUMENT, "edge chain: unknown activation %d", activation);
  if (terms == nullptr) return fail(BYSJ_ERR_INVALID_ARGUMENT, "edge chain: NULL term table");
  if (n_edges == 0) return BYSJ_OK;
  if (out == nullptr) return fail(BYSJ_ERR_INVALID_ARGUMENT, "edge chain: NULL output");
  ChainArgs a{};
  bool vec4 = channels % 4 == 0 && aligned16(out);
  for (int t = 0; t < n_terms; ++t) {
    if (terms[t].a.data == nullptr)
      return fail(BYSJ_ERR_INVALID_ARGUMENT, "edge chain: term %d has no first factor", t);
    a.terms[t] = terms[t];
    vec4 = vec4 && operand_vec4_ok(terms[t].a) && operand_vec4_ok(terms[t].b);
  }
  a.activation = activation;
  a.comps = comps;
  a.channels = channels;
  const int vec = vec4 ? 4 : 1;
  a.vecs_per_row = channels / vec;
  a.total = n_edges * comps * a.vecs_per_row;
  a.fast = a.total < (int64_t{1} << 32);
  if (a.fast) {
    a.by_vecs = FastDiv(static_cast<uint32_t>(a.vecs_per_row));
    a.by_comps = FastDiv(static_cast<uint32_t>(comps));
  }
  a.out = out;
  // A grid-stride loop over at most a few waves of resident CTAs.
  int64_t blocks = (a.total + kBlock - 1) / kBlock;
  const int64_t cap = static_cast<int64_t>(current_device_info().sm_count) * 16;
  if (blocks > cap) blocks = cap;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const ChainKernel kernel = vec4 ? chain_kernel_for<4>(n_terms) : chain_kernel_for<1>(n_terms);
  kernel<<<static_cast<unsigned>(blocks), kBlock, 0, s>>>(a);
  return launch_check("edge_chain_kernel");
}
