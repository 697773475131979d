// Torch extension `bysj_b200._C`: a thin shim over the C ABI in
// include/bysj_b200.h.  It keeps the Python-visible names and keyword
// defaults of the reference's kernels._C module (csrc/bindings.cpp:6-29),
// allocates outputs and workspace through the torch caching allocator and
// launches on the current torch stream of the inputs' device.  No arithmetic
// happens here.
#include <ATen/cuda/CUDAContext.h>
#include <ATen/cuda/CUDAEvent.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <optional>
#include <tuple>

#include "../../include/bysj_b200.h"

namespace {

using Tensor = torch::Tensor;
using OptTensor = std::optional<Tensor>;

void check(int status, const char* op) {
  TORCH_CHECK(status == BYSJ_OK, op, " failed (", bysj_status_string(status),
              "): ", bysj_last_error());
}

void cuda_tensor(const Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

void f32(const Tensor& t, const char* name) {
  cuda_tensor(t, name);
  TORCH_CHECK(t.scalar_type() == torch::kFloat32, name, " must be float32");
}

void i64(const Tensor& t, const char* name) {
  cuda_tensor(t, name);
  TORCH_CHECK(t.scalar_type() == torch::kInt64, name, " must be int64");
}

int value_dtype(const Tensor& t, const char* name) {
  cuda_tensor(t, name);
  if (t.scalar_type() == torch::kFloat32) return BYSJ_F32;
  if (t.scalar_type() == torch::kBFloat16) return BYSJ_BF16;
  TORCH_CHECK(false, name, " must be float32 or bfloat16");
  return -1;
}

void same_device(const Tensor& ref, const OptTensor& t, const char* name) {
  if (t.has_value())
    TORCH_CHECK(t->device() == ref.device(), name, " must be on ", ref.device());
}

void* stream_of(const Tensor& t) {
  return at::cuda::getCurrentCUDAStream(t.device().index()).stream();
}

// A zeroed int32 flags word on the device of `like`, cleared by a memset on
// the current stream (cheaper to issue than a fill kernel).
Tensor zero_word(const Tensor& like) {
  Tensor w = torch::empty({1}, like.options().dtype(torch::kInt32));
  C10_CUDA_CHECK(cudaMemsetAsync(w.data_ptr(), 0, sizeof(int32_t),
                                 static_cast<cudaStream_t>(stream_of(like))));
  return w;
}

Tensor workspace(const Tensor& like, size_t bytes) {
  return torch::empty({static_cast<int64_t>(bytes > 0 ? bytes : 1)},
                      like.options().dtype(torch::kUInt8));
}

template <typename T>
const T* opt_ptr(const OptTensor& t) {
  return t.has_value() ? t->data_ptr<T>() : nullptr;
}

// ---- segment_offsets / CSR view -------------------------------------------

// Returns (offsets, flags) where flags is the BYSJ_FLAG_* word (read back on
// the host, like the reference's min/max range check).  Sorted input takes
// the boundary path; anything else falls back to the histogram path.
std::tuple<Tensor, int64_t> segment_offsets(Tensor dst, int64_t n_nodes) {
  i64(dst, "dst");
  TORCH_CHECK(dst.dim() == 1, "dst must be one-dimensional");
  TORCH_CHECK(n_nodes >= 0, "n_nodes must be non-negative");
  c10::cuda::CUDAGuard guard(dst.device());
  const int64_t edges = dst.size(0);
  Tensor offsets = torch::empty({n_nodes + 1}, dst.options());
  Tensor flags = zero_word(dst);
  void* s = stream_of(dst);
  auto* fp = reinterpret_cast<uint32_t*>(flags.data_ptr<int32_t>());
  check(bysj_segment_offsets_sorted(dst.data_ptr<int64_t>(), edges, n_nodes,
                                    offsets.data_ptr<int64_t>(), fp, s),
        "segment_offsets");
  int64_t word = flags.item<int32_t>();
  if (word & BYSJ_FLAG_OUT_OF_RANGE) return {offsets, word};
  if (word & BYSJ_FLAG_UNSORTED) {
    flags.zero_();
    Tensor ws = workspace(dst, bysj_segment_offsets_workspace_size(n_nodes));
    check(bysj_segment_offsets_histogram(
              dst.data_ptr<int64_t>(), edges, n_nodes, offsets.data_ptr<int64_t>(), fp,
              ws.data_ptr(), static_cast<size_t>(ws.numel()), s),
          "segment_offsets");
    word = flags.item<int32_t>() | BYSJ_FLAG_UNSORTED;
  }
  return {offsets, word};
}

// Launch-only form of the sorted path for pipelines that must not
// synchronise: ORs the BYSJ_FLAG_* word into the caller's device tensor
// `flags` (int32 [1]) and returns the offsets without reading it back.
Tensor segment_offsets_device(Tensor dst, int64_t n_nodes, Tensor flags) {
  i64(dst, "dst");
  cuda_tensor(flags, "flags");
  TORCH_CHECK(flags.scalar_type() == torch::kInt32 && flags.numel() >= 1,
              "flags must be an int32 tensor");
  c10::cuda::CUDAGuard guard(dst.device());
  Tensor offsets = torch::empty({n_nodes + 1}, dst.options());
  check(bysj_segment_offsets_sorted(dst.data_ptr<int64_t>(), dst.numel(), n_nodes,
                                    offsets.data_ptr<int64_t>(),
                                    reinterpret_cast<uint32_t*>(flags.data_ptr<int32_t>()),
                                    stream_of(dst)),
        "segment_offsets_device");
  return offsets;
}

// Stable grouping of edges by key on the device: (order, offsets, flags word).
// The flags word is read back (one synchronisation), as the reference's
// range check does.
std::tuple<Tensor, Tensor, int64_t> group_by_key(Tensor keys, int64_t n_keys) {
  i64(keys, "keys");
  TORCH_CHECK(n_keys >= 0, "n_keys must be non-negative");
  c10::cuda::CUDAGuard guard(keys.device());
  const int64_t edges = keys.numel();
  Tensor order = torch::empty({edges}, keys.options());
  Tensor offsets = torch::empty({n_keys + 1}, keys.options());
  Tensor flags = zero_word(keys);
  Tensor ws = workspace(keys, bysj_group_by_key_workspace_size(edges, n_keys));
  check(bysj_group_by_key(keys.data_ptr<int64_t>(), edges, n_keys, order.data_ptr<int64_t>(),
                          offsets.data_ptr<int64_t>(),
                          reinterpret_cast<uint32_t*>(flags.data_ptr<int32_t>()), ws.data_ptr(),
                          static_cast<size_t>(ws.numel()), stream_of(keys)),
        "group_by_key");
  return {order, offsets, static_cast<int64_t>(flags.item<int32_t>())};
}

// CSR view (offsets, order) of an arbitrary-order dst, for operators whose
// reference API takes only dst (GIE).  order is undefined for sorted input.
std::tuple<Tensor, OptTensor> csr_view(const Tensor& dst, int64_t n_nodes) {
  auto [offsets, word] = segment_offsets(dst, n_nodes);
  TORCH_CHECK(!(word & BYSJ_FLAG_OUT_OF_RANGE),
              "destination values must be within the node range");
  OptTensor order;
  if (word & BYSJ_FLAG_UNSORTED) {
    auto [grouped, grouped_offsets, gword] = group_by_key(dst, n_nodes);
    order = grouped;
  }
  return {offsets, order};
}

// Launch-only CSR view for a destination-sorted dst: the boundary offsets and
// the device flags word, not read back (the GIE entry points take the word as
// their gate and read it once their kernels are queued).
std::tuple<Tensor, Tensor> csr_view_launch(const Tensor& dst, int64_t n_nodes) {
  Tensor offsets = torch::empty({n_nodes + 1}, dst.options());
  Tensor flags = zero_word(dst);
  check(bysj_segment_offsets_sorted(dst.data_ptr<int64_t>(), dst.numel(), n_nodes,
                                    offsets.data_ptr<int64_t>(),
                                    reinterpret_cast<uint32_t*>(flags.data_ptr<int32_t>()),
                                    stream_of(dst)),
        "segment_offsets");
  return {offsets, flags};
}

// An early read of a device flags word: the 4-byte copy into pinned memory
// runs on a side stream, ordered after the work queued so far on the current
// stream (the kernel that writes the word) but not after what is queued next.
// A caller that launches its gated operator between start() and word() keeps
// the GPU busy while the host waits only for the small kernel.
class EarlyFlags {
 public:
  explicit EarlyFlags(const Tensor& flags)
      : flags_(flags),
        host_(at::empty({1}, flags.options().device(at::kCPU).pinned_memory(true))) {
    const auto dev = flags.device().index();
    at::cuda::CUDAStream main = at::cuda::getCurrentCUDAStream(dev);
    at::cuda::CUDAStream side = at::cuda::getStreamFromPool(false, dev);
    ready_.record(main);
    ready_.block(side);
    C10_CUDA_CHECK(cudaMemcpyAsync(host_.data_ptr(), flags_.data_ptr(), sizeof(int32_t),
                                   cudaMemcpyDeviceToHost, side.stream()));
    done_.record(side);
  }
  EarlyFlags(const EarlyFlags&) = delete;
  EarlyFlags& operator=(const EarlyFlags&) = delete;
  // An exception between start and word() must not free the buffers under
  // the pending copy.
  ~EarlyFlags() {
    if (!read_ && done_.isCreated()) (void)cudaEventSynchronize(done_.event());
  }
  int64_t word() {
    done_.synchronize();
    read_ = true;
    return host_.data_ptr<int32_t>()[0];
  }

 private:
  Tensor flags_, host_;
  at::cuda::CUDAEvent ready_, done_;
  bool read_ = false;
};

// Index guard: the BYSJ_INDEX_* word (read back).
int64_t check_indices(OptTensor offsets, int64_t n_edges, OptTensor order, OptTensor values,
                      int64_t value_limit) {
  const Tensor& ref = offsets ? *offsets : (order ? *order : *values);
  TORCH_CHECK(offsets || order || values, "check_indices needs something to check");
  TORCH_CHECK(n_edges >= 0, "check_indices: n_edges must be non-negative");
  if (offsets) {
    i64(*offsets, "offsets");
    TORCH_CHECK(offsets->dim() == 1 && offsets->numel() >= 1,
                "check_indices: offsets must be one-dimensional with at least one entry");
  }
  if (order) {
    i64(*order, "order");
    TORCH_CHECK(order->numel() == n_edges, "check_indices: order must have n_edges entries");
  }
  if (values) i64(*values, "values");
  same_device(ref, offsets, "offsets");
  same_device(ref, order, "order");
  same_device(ref, values, "values");
  c10::cuda::CUDAGuard guard(ref.device());
  Tensor error = zero_word(ref);
  Tensor ws = workspace(ref, bysj_check_indices_workspace_size(order ? n_edges : 0));
  const int64_t nodes = offsets ? offsets->numel() - 1 : 0;
  check(bysj_check_indices(opt_ptr<int64_t>(offsets), nodes, n_edges, opt_ptr<int64_t>(order),
                           opt_ptr<int64_t>(values), values ? values->numel() : 0, value_limit,
                           reinterpret_cast<uint32_t*>(error.data_ptr<int32_t>()), ws.data_ptr(),
                           static_cast<size_t>(ws.numel()), stream_of(ref)),
        "check_indices");
  return error.item<int32_t>();
}

// ---- segment_sum ------------------------------------------------------------

Tensor segment_sum_forward(Tensor src, Tensor offsets, OptTensor edge_scale,
                           OptTensor node_scale, OptTensor order) {
  const int dt = value_dtype(src, "segment sum src");
  TORCH_CHECK(src.dim() == 2, "segment sum src must have shape (n_edges, channels)");
  i64(offsets, "segment sum offsets");
  TORCH_CHECK(offsets.dim() == 1 && offsets.size(0) >= 1,
              "segment sum offsets must be a one-dimensional exclusive prefix sum");
  const int64_t edges = src.size(0), channels = src.size(1);
  const int64_t nodes = offsets.size(0) - 1;
  TORCH_CHECK(channels > 0, "segment sum requires at least one channel");
  if (edge_scale) {
    f32(*edge_scale, "segment sum edge_scale");
    TORCH_CHECK(edge_scale->numel() == edges, "segment sum edge_scale must have shape (n_edges,)");
  }
  if (node_scale) {
    f32(*node_scale, "segment sum node_scale");
    TORCH_CHECK(node_scale->numel() == nodes, "segment sum node_scale must have one value per segment");
  }
  if (order) {
    i64(*order, "segment sum order");
    TORCH_CHECK(order->numel() == edges, "segment sum order must have shape (n_edges,)");
  }
  same_device(src, offsets, "offsets");
  same_device(src, edge_scale, "edge_scale");
  same_device(src, node_scale, "node_scale");
  same_device(src, order, "order");
  c10::cuda::CUDAGuard guard(src.device());
  Tensor out = torch::empty({nodes, channels}, src.options().dtype(torch::kFloat32));
  if (nodes == 0) return out;
  Tensor ws = workspace(src, bysj_segment_sum_workspace_size(edges, nodes, channels, dt));
  check(bysj_segment_sum_forward(src.data_ptr(), dt, edges, channels,
                                 offsets.data_ptr<int64_t>(), nodes,
                                 opt_ptr<float>(edge_scale), opt_ptr<float>(node_scale),
                                 opt_ptr<int64_t>(order), out.data_ptr<float>(),
                                 ws.data_ptr(), static_cast<size_t>(ws.numel()),
                                 stream_of(src)),
        "segment_sum_forward");
  return out;
}

std::tuple<Tensor, Tensor> segment_sum_backward(Tensor grad_out, Tensor src, Tensor dst,
                                                Tensor offsets, OptTensor edge_scale,
                                                OptTensor node_scale,
                                                bool want_node_scale_grad,
                                                OptTensor order) {
  const int dt = value_dtype(src, "segment sum src");
  f32(grad_out, "segment sum grad_out");
  i64(dst, "segment sum dst");
  i64(offsets, "segment sum offsets");
  const int64_t edges = src.size(0), channels = src.size(1);
  const int64_t nodes = offsets.size(0) - 1;
  TORCH_CHECK(grad_out.dim() == 2 && grad_out.size(0) == nodes && grad_out.size(1) == channels,
              "segment sum grad_out must have shape (n_nodes, channels)");
  TORCH_CHECK(dst.numel() == edges, "segment sum dst must have shape (n_edges,)");
  if (edge_scale) f32(*edge_scale, "segment sum edge_scale");
  if (node_scale) f32(*node_scale, "segment sum node_scale");
  if (order) i64(*order, "segment sum order");
  c10::cuda::CUDAGuard guard(src.device());
  Tensor grad_src = torch::empty({edges, channels}, grad_out.options());
  const bool want = want_node_scale_grad && node_scale.has_value();
  Tensor grad_scale = want ? torch::empty_like(*node_scale) : Tensor();
  if (nodes == 0) return {grad_src, grad_scale};
  Tensor ws = workspace(src, want ? bysj_segment_sum_backward_workspace_size(
                                        edges, nodes, channels, dt)
                                  : 0);
  check(bysj_segment_sum_backward(
            grad_out.data_ptr<float>(), src.data_ptr(), dt, dst.data_ptr<int64_t>(),
            offsets.data_ptr<int64_t>(), edges, nodes, channels,
            opt_ptr<float>(edge_scale), opt_ptr<float>(node_scale), opt_ptr<int64_t>(order),
            grad_src.data_ptr<float>(), want ? grad_scale.data_ptr<float>() : nullptr,
            ws.data_ptr(), static_cast<size_t>(ws.numel()), stream_of(src)),
        "segment_sum_backward");
  return {grad_src, grad_scale};
}

// ---- segment_softmax --------------------------------------------------------

std::tuple<Tensor, Tensor> segment_softmax_forward(Tensor logit, Tensor env, Tensor offsets,
                                                   OptTensor null_logit, OptTensor order) {
  f32(logit, "segment softmax logit");
  f32(env, "segment softmax env");
  i64(offsets, "segment softmax offsets");
  TORCH_CHECK(logit.dim() == 2, "segment softmax logit must have shape (n_edges, channels)");
  const int64_t edges = logit.size(0), channels = logit.size(1);
  const int64_t nodes = offsets.size(0) - 1;
  TORCH_CHECK(channels > 0, "segment softmax requires at least one channel");
  TORCH_CHECK(env.dim() == 1 && env.size(0) == edges, "segment softmax env must have shape (n_edges,)");
  if (null_logit) {
    f32(*null_logit, "segment softmax null_logit");
    TORCH_CHECK(null_logit->numel() == nodes * channels,
                "segment softmax null_logit must have shape (n_nodes, channels)");
  }
  if (order) i64(*order, "segment softmax order");
  same_device(logit, env, "env");
  same_device(logit, offsets, "offsets");
  same_device(logit, null_logit, "null_logit");
  same_device(logit, order, "order");
  c10::cuda::CUDAGuard guard(logit.device());
  Tensor alpha = torch::empty({edges, channels}, logit.options());
  Tensor null_alpha = null_logit ? torch::empty({nodes, channels}, logit.options()) : Tensor();
  if (nodes == 0) return {alpha, null_alpha};
  Tensor ws = workspace(logit, bysj_segment_softmax_workspace_size(edges, nodes, channels));
  check(bysj_segment_softmax_forward(
            logit.data_ptr<float>(), env.data_ptr<float>(), offsets.data_ptr<int64_t>(),
            edges, nodes, channels, opt_ptr<float>(null_logit), opt_ptr<int64_t>(order),
            alpha.data_ptr<float>(), null_logit ? null_alpha.data_ptr<float>() : nullptr,
            ws.data_ptr(), static_cast<size_t>(ws.numel()), stream_of(logit)),
        "segment_softmax_forward");
  return {alpha, null_alpha};
}

std::tuple<Tensor, Tensor, Tensor> segment_softmax_backward(
    Tensor alpha, Tensor grad_alpha, Tensor env, Tensor offsets, OptTensor null_alpha,
    OptTensor grad_null_alpha, OptTensor order) {
  f32(alpha, "segment softmax alpha");
  f32(grad_alpha, "segment softmax grad_alpha");
  f32(env, "segment softmax env");
  i64(offsets, "segment softmax offsets");
  TORCH_CHECK(grad_alpha.sizes() == alpha.sizes(), "segment softmax grad_alpha must match alpha");
  TORCH_CHECK(null_alpha.has_value() == grad_null_alpha.has_value(),
              "segment softmax requires null_alpha and grad_null_alpha together");
  const int64_t edges = alpha.size(0), channels = alpha.size(1);
  const int64_t nodes = offsets.size(0) - 1;
  if (null_alpha) {
    f32(*null_alpha, "segment softmax null_alpha");
    f32(*grad_null_alpha, "segment softmax grad_null_alpha");
  }
  if (order) i64(*order, "segment softmax order");
  c10::cuda::CUDAGuard guard(alpha.device());
  Tensor grad_logit = torch::empty_like(alpha);
  Tensor grad_null = null_alpha ? torch::empty({nodes, channels}, alpha.options()) : Tensor();
  Tensor grad_env = torch::empty({edges}, alpha.options());
  if (nodes == 0) return {grad_logit, grad_null, grad_env};
  Tensor ws = workspace(alpha, bysj_segment_softmax_backward_workspace_size(edges, nodes, channels));
  check(bysj_segment_softmax_backward(
            alpha.data_ptr<float>(), grad_alpha.data_ptr<float>(), env.data_ptr<float>(),
            offsets.data_ptr<int64_t>(), edges, nodes, channels, opt_ptr<float>(null_alpha),
            opt_ptr<float>(grad_null_alpha), opt_ptr<int64_t>(order),
            grad_logit.data_ptr<float>(), null_alpha ? grad_null.data_ptr<float>() : nullptr,
            grad_env.data_ptr<float>(), ws.data_ptr(), static_cast<size_t>(ws.numel()),
            stream_of(alpha)),
        "segment_softmax_backward");
  return {grad_logit, grad_null, grad_env};
}

// ---- segment_attention (fused softmax + weighted sum) ----------------------

Tensor segment_attention_forward(Tensor logit, Tensor value, Tensor offsets, OptTensor env,
                                 OptTensor null_logit, OptTensor order) {
  f32(logit, "segment attention logit");
  const int dt = value_dtype(value, "segment attention value");
  i64(offsets, "segment attention offsets");
  TORCH_CHECK(logit.dim() == 2, "segment attention logit must have shape (n_edges, heads)");
  TORCH_CHECK(value.dim() == 3 && value.size(0) == logit.size(0),
              "segment attention value must have shape (n_edges, components, channels)");
  const int64_t edges = logit.size(0), heads = logit.size(1);
  const int64_t comps = value.size(1), channels = value.size(2);
  const int64_t nodes = offsets.size(0) - 1;
  TORCH_CHECK(heads > 0 && channels % heads == 0,
              "segment attention heads must divide the channel count");
  if (env) {
    f32(*env, "segment attention env");
    TORCH_CHECK(env->numel() == edges, "segment attention env must have shape (n_edges,)");
  }
  if (null_logit) {
    f32(*null_logit, "segment attention null_logit");
    TORCH_CHECK(null_logit->numel() == nodes * heads,
                "segment attention null_logit must have shape (n_nodes, heads)");
  }
  if (order) i64(*order, "segment attention order");
  same_device(logit, value, "value");
  same_device(logit, offsets, "offsets");
  same_device(logit, env, "env");
  same_device(logit, null_logit, "null_logit");
  same_device(logit, order, "order");
  c10::cuda::CUDAGuard guard(logit.device());
  Tensor out = torch::empty({nodes, heads, comps, channels / heads}, logit.options());
  if (nodes == 0) return out;
  Tensor ws = workspace(logit, bysj_segment_attention_workspace_size(edges, nodes, heads, comps,
                                                                     channels, dt));
  check(bysj_segment_attention_forward(
            logit.data_ptr<float>(), value.data_ptr(), dt, opt_ptr<float>(env),
            opt_ptr<float>(null_logit), offsets.data_ptr<int64_t>(), opt_ptr<int64_t>(order),
            edges, nodes, heads, comps, channels, out.data_ptr<float>(), ws.data_ptr(),
            static_cast<size_t>(ws.numel()), stream_of(logit)),
        "segment_attention_forward");
  return out;
}

// ---- rotate-back aggregation --------------------------------------------------

Tensor rotate_back_aggregate_forward(Tensor x_local, Tensor rotation, OptTensor rescale,
                                     Tensor alpha, Tensor offsets, OptTensor order,
                                     int64_t lmax, int64_t heads) {
  f32(x_local, "rotate-back x_local");
  f32(rotation, "rotate-back rotation");
  f32(alpha, "rotate-back attn_alpha");
  i64(offsets, "rotate-back row_ptr");
  TORCH_CHECK(x_local.dim() == 3, "rotate-back x_local must have shape (n_edges, S, channels)");
  const int64_t edges = x_local.size(0), comps = x_local.size(1), channels = x_local.size(2);
  TORCH_CHECK(lmax >= 0 && comps == (lmax + 1) * (lmax + 1),
              "rotate-back x_local must have (lmax + 1)^2 components");
  const int64_t packed = (lmax + 1) * (2 * lmax + 1) * (2 * lmax + 3) / 3;
  TORCH_CHECK(rotation.dim() == 2 && rotation.size(0) == edges && rotation.size(1) == packed,
              "rotate-back rotation must have shape (n_edges, sum_l (2l+1)^2)");
  TORCH_CHECK(heads > 0 && channels % heads == 0, "rotate-back heads must divide the channels");
  TORCH_CHECK(alpha.dim() == 2 && alpha.size(0) == edges && alpha.size(1) == heads,
              "rotate-back attn_alpha must have shape (n_edges, heads)");
  if (rescale) {
    f32(*rescale, "rotate-back rotate_inv_rescale");
    TORCH_CHECK(rescale->numel() == edges, "rotate-back rotate_inv_rescale must have n_edges");
  }
  if (order) i64(*order, "rotate-back order");
  same_device(x_local, rotation, "rotation");
  same_device(x_local, alpha, "attn_alpha");
  same_device(x_local, offsets, "row_ptr");
  same_device(x_local, rescale, "rotate_inv_rescale");
  same_device(x_local, order, "order");
  const int64_t nodes = offsets.size(0) - 1;
  c10::cuda::CUDAGuard guard(x_local.device());
  Tensor out = torch::empty({nodes, comps, channels}, x_local.options());
  if (nodes == 0) return out;
  Tensor ws = workspace(x_local, bysj_rotate_back_aggregate_workspace_size(edges, nodes, lmax,
                                                                           heads, channels));
  check(bysj_rotate_back_aggregate(
            x_local.data_ptr<float>(), rotation.data_ptr<float>(), opt_ptr<float>(rescale),
            alpha.data_ptr<float>(), offsets.data_ptr<int64_t>(), opt_ptr<int64_t>(order),
            edges, nodes, lmax, heads, channels, out.data_ptr<float>(), ws.data_ptr(),
            static_cast<size_t>(ws.numel()), stream_of(x_local)),
        "rotate_back_aggregate_forward");
  return out;
}

// ---- edge-stream elementwise chain ----------------------------------------------

bysj_chain_operand chain_operand(const Tensor& t, int64_t e, int64_t s, int64_t c) {
  // A broadcast view of the factor over [E, S, C]: stride 0 on broadcast axes.
  Tensor v = t.expand({e, s, c});
  bysj_chain_operand op{};
  op.data = v.data_ptr<float>();
  for (int i = 0; i < 3; ++i) op.stride[i] = v.size(i) == 1 ? 0 : v.stride(i);
  return op;
}

Tensor edge_chain(std::vector<Tensor> first, std::vector<OptTensor> second,
                  std::vector<double> coefs, int64_t n_edges, int64_t comps, int64_t channels,
                  int64_t activation) {
  const size_t n = first.size();
  TORCH_CHECK(n >= 1 && n <= BYSJ_CHAIN_MAX_TERMS && second.size() == n && coefs.size() == n,
              "edge chain: 1 to ", BYSJ_CHAIN_MAX_TERMS, " terms with matching lists");
  // Factors are strided views (any strides, broadcasts included): float32
  // on one CUDA device, no contiguity required.
  auto factor = [&](const Tensor& f) {
    TORCH_CHECK(f.is_cuda(), "edge chain factor must be a CUDA tensor");
    TORCH_CHECK(f.scalar_type() == torch::kFloat32, "edge chain factor must be float32");
    TORCH_CHECK(f.device() == first[0].device(), "edge chain factors must share a device");
  };
  for (size_t t = 0; t < n; ++t) {
    factor(first[t]);
    if (second[t]) factor(*second[t]);
  }
  c10::cuda::CUDAGuard guard(first[0].device());
  Tensor out = torch::empty({n_edges, comps, channels}, first[0].options());
  if (n_edges == 0) return out;
  std::vector<bysj_chain_term> terms(n);
  for (size_t t = 0; t < n; ++t) {
    terms[t].coef = static_cast<float>(coefs[t]);
    terms[t].a = chain_operand(first[t], n_edges, comps, channels);
    if (second[t]) terms[t].b = chain_operand(*second[t], n_edges, comps, channels);
  }
  check(bysj_edge_chain(terms.data(), static_cast<int>(n), n_edges, comps, channels,
                        static_cast<int>(activation), out.data_ptr<float>(),
                        stream_of(first[0])),
        "edge_chain");
  return out;
}

// ---- force_assembly ---------------------------------------------------------

std::tuple<Tensor, Tensor> force_assembly(Tensor grad_edge, Tensor edge_vec, Tensor dst_offsets,
                                          Tensor src_offsets, Tensor src_order) {
  f32(grad_edge, "force assembly grad_edge");
  f32(edge_vec, "force assembly edge_vec");
  i64(dst_offsets, "force assembly dst_offsets");
  i64(src_offsets, "force assembly src_offsets");
  i64(src_order, "force assembly src_order");
  TORCH_CHECK(grad_edge.dim() == 2 && grad_edge.size(1) == 3,
              "force assembly grad_edge must have shape (n_edges, 3)");
  TORCH_CHECK(edge_vec.sizes() == grad_edge.sizes(), "force assembly edge_vec must match grad_edge");
  TORCH_CHECK(dst_offsets.size(0) == src_offsets.size(0),
              "force assembly offsets must describe the same atom count");
  const int64_t edges = grad_edge.size(0);
  const int64_t nodes = dst_offsets.size(0) - 1;
  TORCH_CHECK(nodes > 0, "force assembly requires at least one atom");
  TORCH_CHECK(src_order.numel() == edges, "force assembly src_order must have shape (n_edges,)");
  c10::cuda::CUDAGuard guard(grad_edge.device());
  Tensor force = torch::empty({nodes, 3}, grad_edge.options());
  Tensor virial = torch::empty({nodes, 9}, grad_edge.options());
  check(bysj_force_assembly(grad_edge.data_ptr<float>(), edge_vec.data_ptr<float>(),
                            dst_offsets.data_ptr<int64_t>(), src_offsets.data_ptr<int64_t>(),
                            src_order.data_ptr<int64_t>(), edges, nodes,
                            force.data_ptr<float>(), virial.data_ptr<float>(),
                            stream_of(grad_edge)),
        "force_assembly");
  return {force, virial};
}

Tensor force_assembly_src_partial(Tensor grad_edge, Tensor edge_vec, Tensor src_offsets,
                                  Tensor src_order) {
  f32(grad_edge, "grad_edge");
  f32(edge_vec, "edge_vec");
  i64(src_offsets, "src_offsets");
  i64(src_order, "src_order");
  const int64_t nodes = src_offsets.size(0) - 1;
  c10::cuda::CUDAGuard guard(grad_edge.device());
  Tensor partial = torch::empty({nodes, 12}, grad_edge.options().dtype(torch::kFloat64));
  check(bysj_force_assembly_src_partial(grad_edge.data_ptr<float>(), edge_vec.data_ptr<float>(),
                                        src_offsets.data_ptr<int64_t>(),
                                        src_order.data_ptr<int64_t>(), grad_edge.size(0), nodes,
                                        partial.data_ptr<double>(), stream_of(grad_edge)),
        "force_assembly_src_partial");
  return partial;
}

std::tuple<Tensor, Tensor> force_assembly_dst_add(Tensor grad_edge, Tensor dst_offsets,
                                                  Tensor summed_partial) {
  f32(grad_edge, "grad_edge");
  i64(dst_offsets, "dst_offsets");
  TORCH_CHECK(summed_partial.scalar_type() == torch::kFloat64 && summed_partial.is_contiguous(),
              "summed_partial must be a contiguous float64 tensor");
  const int64_t local = dst_offsets.size(0) - 1;
  TORCH_CHECK(summed_partial.numel() == local * 12, "summed_partial must have shape (n_local, 12)");
  c10::cuda::CUDAGuard guard(grad_edge.device());
  Tensor force = torch::empty({local, 3}, grad_edge.options());
  Tensor virial = torch::empty({local, 9}, grad_edge.options());
  check(bysj_force_assembly_dst_add(grad_edge.data_ptr<float>(), dst_offsets.data_ptr<int64_t>(),
                                    local, summed_partial.data_ptr<double>(),
                                    force.data_ptr<float>(), virial.data_ptr<float>(),
                                    stream_of(grad_edge)),
        "force_assembly_dst_add");
  return {force, virial};
}

// ---- rmsnorm ---------------------------------------------------------------

int64_t scale_rows_of(const Tensor& x, const Tensor& scale) {
  if (scale.numel() == 0) return 0;
  if (scale.dim() == 1) {
    TORCH_CHECK(scale.size(0) == x.size(-1), "RMSNorm scale must have shape (feature_dim,)");
    return 1;
  }
  TORCH_CHECK(scale.dim() == 2 && scale.size(1) == x.size(-1) && x.dim() >= 2 &&
                  x.size(-2) == scale.size(0) * scale.size(0),
              "RMSNorm per-degree scale must have shape (L+1, feature_dim) with "
              "x.shape[-2] == (L+1)^2");
  return scale.size(0);
}

std::tuple<Tensor, Tensor> rmsnorm_forward(Tensor x, Tensor scale, double eps) {
  const int dt = value_dtype(x, "RMSNorm input");
  TORCH_CHECK(x.dim() >= 1, "RMSNorm input must have at least one dimension");
  TORCH_CHECK(x.size(-1) > 0, "RMSNorm feature dimension must be positive");
  TORCH_CHECK(std::isfinite(eps) && eps > 0.0, "RMSNorm eps must be a finite positive number");
  if (scale.numel()) f32(scale, "RMSNorm scale");
  const int64_t srows = scale_rows_of(x, scale);
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t width = x.size(-1);
  const int64_t rows = x.numel() / width;
  Tensor y = torch::empty_like(x);
  Tensor inv = torch::empty({rows}, x.options().dtype(torch::kFloat32));
  if (rows == 0) return {y, inv};
  check(bysj_rmsnorm_forward(x.data_ptr(), dt, rows, width,
                             srows ? scale.data_ptr<float>() : nullptr, srows,
                             static_cast<float>(eps), y.data_ptr(), inv.data_ptr<float>(),
                             stream_of(x)),
        "rmsnorm_forward");
  return {y, inv};
}

std::tuple<Tensor, Tensor> rmsnorm_backward(Tensor grad_output, Tensor x, Tensor scale,
                                            Tensor inverse_rms, bool compute_scale_grad) {
  f32(grad_output, "RMSNorm grad_output");
  f32(x, "RMSNorm input");
  f32(inverse_rms, "RMSNorm inverse_rms");
  TORCH_CHECK(grad_output.sizes() == x.sizes(), "RMSNorm grad_output must have the input shape");
  if (scale.numel()) f32(scale, "RMSNorm scale");
  const int64_t srows = scale_rows_of(x, scale);
  TORCH_CHECK(!compute_scale_grad || srows > 0,
              "cannot compute a scale gradient when scale is omitted");
  const int64_t width = x.size(-1);
  const int64_t rows = x.numel() / width;
  TORCH_CHECK(inverse_rms.numel() == rows, "RMSNorm saved inverse_rms has an invalid shape");
  c10::cuda::CUDAGuard guard(x.device());
  Tensor gx = torch::empty_like(x);
  Tensor gs = compute_scale_grad ? torch::empty_like(scale) : torch::empty({0}, x.options());
  Tensor ws = workspace(x, compute_scale_grad
                               ? bysj_rmsnorm_backward_workspace_size(rows, width, srows)
                               : 0);
  check(bysj_rmsnorm_backward(grad_output.data_ptr<float>(), x.data_ptr<float>(),
                              srows ? scale.data_ptr<float>() : nullptr, srows,
                              inverse_rms.data_ptr<float>(), rows, width,
                              gx.data_ptr<float>(),
                              compute_scale_grad ? gs.data_ptr<float>() : nullptr,
                              ws.data_ptr(), static_cast<size_t>(ws.numel()), stream_of(x)),
        "rmsnorm_backward");
  return {gx, gs};
}

// ---- GIE zonal scatter ------------------------------------------------------

void check_gie(const Tensor& zonal, const Tensor& radial, const Tensor& dst,
               const Tensor& slot, const Tensor& inv) {
  f32(zonal, "GIE zonal");
  f32(radial, "GIE radial");
  f32(inv, "GIE inv_sqrt_deg");
  i64(dst, "GIE dst");
  i64(slot, "GIE radial_slot");
  TORCH_CHECK(zonal.dim() == 2, "GIE zonal must have shape (n_edges, n_rows)");
  TORCH_CHECK(radial.dim() == 3 && radial.size(0) == zonal.size(0),
              "GIE radial must have shape (n_edges, n_radial, channels)");
  TORCH_CHECK(dst.numel() == zonal.size(0), "GIE dst must have shape (n_edges,)");
  TORCH_CHECK(slot.numel() == zonal.size(1), "GIE radial_slot must have shape (n_rows,)");
  TORCH_CHECK(inv.dim() == 1 || (inv.dim() == 3 && inv.size(1) == 1 && inv.size(2) == 1),
              "GIE inv_sqrt_deg must have shape (n_nodes,) or (n_nodes, 1, 1)");
}

// dst_offsets: the caller's CSR of an already grouped dst (offsets[n] =
// number of edges with dst < n), taken as given: no derivation kernel and no
// flags read back, so the host does not wait for the device.
void check_dst_offsets(const Tensor& zonal, const Tensor& dst_offsets, int64_t nodes) {
  i64(dst_offsets, "GIE dst_offsets");
  same_device(zonal, dst_offsets, "GIE dst_offsets");
  TORCH_CHECK(dst_offsets.dim() == 1 && dst_offsets.size(0) == nodes + 1,
              "GIE dst_offsets must have shape (n_nodes + 1,)");
}

Tensor gie_zonal_scatter_forward(Tensor zonal, Tensor radial, Tensor dst, Tensor radial_slot,
                                 Tensor inv_sqrt_deg, OptTensor dst_offsets) {
  check_gie(zonal, radial, dst, radial_slot, inv_sqrt_deg);
  c10::cuda::CUDAGuard guard(zonal.device());
  const int64_t edges = zonal.size(0), rows = zonal.size(1);
  const int64_t n_radial = radial.size(1), channels = radial.size(2);
  const int64_t nodes = inv_sqrt_deg.size(0);
  if (dst_offsets) check_dst_offsets(zonal, *dst_offsets, nodes);
  if (nodes == 0) return torch::empty({nodes, rows + 1, channels}, zonal.options());
  if (dst_offsets) {
    Tensor out = torch::empty({nodes, rows + 1, channels}, zonal.options());
    Tensor ws =
        workspace(zonal, bysj_gie_zonal_scatter_workspace_size(edges, nodes, rows, channels));
    check(bysj_gie_zonal_scatter_forward(
              zonal.data_ptr<float>(), radial.data_ptr<float>(),
              dst_offsets->data_ptr<int64_t>(), nullptr, radial_slot.data_ptr<int64_t>(),
              inv_sqrt_deg.data_ptr<float>(), edges, nodes, rows, n_radial, channels,
              out.data_ptr<float>(), ws.data_ptr(), static_cast<size_t>(ws.numel()),
              stream_of(zonal)),
          "gie_zonal_scatter_forward");
    return out;
  }
  // The slot table stays on the device: for the degree-grouped shape the
  // library launches the degree kernel and the generic one, and each checks
  // the table itself (no read back here).
  // The sorted-path CSR and the operator are queued together, the operator
  // gated on the CSR flags; the flags are read as soon as the CSR kernel is
  // done, while the operator runs (the host does not wait for it).  An
  // unsorted dst (flag set, operator skipped) is then grouped on the device
  // and the operator runs again; a destination out of range is an error.
  // The CSR kernel is queued first, so that the output and workspace are
  // allocated while it runs.
  auto [offsets, flags] = csr_view_launch(dst, nodes);
  EarlyFlags early(flags);
  Tensor out = torch::empty({nodes, rows + 1, channels}, zonal.options());
  Tensor ws = workspace(zonal, bysj_gie_zonal_scatter_workspace_size(edges, nodes, rows, channels));
  check(bysj_gie_zonal_scatter_forward_gated(
            zonal.data_ptr<float>(), radial.data_ptr<float>(), offsets.data_ptr<int64_t>(),
            nullptr, radial_slot.data_ptr<int64_t>(), inv_sqrt_deg.data_ptr<float>(), edges,
            nodes, rows, n_radial, channels, out.data_ptr<float>(), ws.data_ptr(),
            static_cast<size_t>(ws.numel()), stream_of(zonal),
            reinterpret_cast<const uint32_t*>(flags.data_ptr<int32_t>())),
        "gie_zonal_scatter_forward");
  const int64_t word = early.word();
  if (word == 0) return out;
  TORCH_CHECK(!(word & BYSJ_FLAG_OUT_OF_RANGE),
              "destination values must be within the node range");
  auto [grouped_offsets, order] = csr_view(dst, nodes);
  check(bysj_gie_zonal_scatter_forward(
            zonal.data_ptr<float>(), radial.data_ptr<float>(),
            grouped_offsets.data_ptr<int64_t>(), opt_ptr<int64_t>(order),
            radial_slot.data_ptr<int64_t>(), inv_sqrt_deg.data_ptr<float>(), edges, nodes, rows,
            n_radial, channels, out.data_ptr<float>(), ws.data_ptr(),
            static_cast<size_t>(ws.numel()), stream_of(zonal)),
        "gie_zonal_scatter_forward");
  return out;
}

std::tuple<Tensor, Tensor, Tensor> gie_zonal_scatter_backward(Tensor grad_output, Tensor zonal,
                                                              Tensor radial, Tensor dst,
                                                              Tensor radial_slot,
                                                              Tensor inv_sqrt_deg,
                                                              OptTensor dst_offsets) {
  check_gie(zonal, radial, dst, radial_slot, inv_sqrt_deg);
  f32(grad_output, "GIE grad_output");
  const int64_t edges = zonal.size(0), rows = zonal.size(1);
  const int64_t n_radial = radial.size(1), channels = radial.size(2);
  const int64_t nodes = inv_sqrt_deg.size(0);
  TORCH_CHECK(grad_output.dim() == 3 && grad_output.size(0) == nodes &&
                  grad_output.size(1) == rows + 1 && grad_output.size(2) == channels,
              "GIE grad_output must have shape (n_nodes, n_rows + 1, channels)");
  c10::cuda::CUDAGuard guard(zonal.device());
  if (dst_offsets) check_dst_offsets(zonal, *dst_offsets, nodes);
  if (nodes == 0)
    return {torch::empty_like(zonal), torch::empty_like(radial), torch::empty_like(inv_sqrt_deg)};
  if (dst_offsets) {
    Tensor gz = torch::empty_like(zonal);
    Tensor gr = torch::empty_like(radial);
    Tensor gi = torch::empty_like(inv_sqrt_deg);
    Tensor ws = workspace(
        zonal, bysj_gie_zonal_scatter_backward_workspace_size(edges, nodes, rows, channels));
    check(bysj_gie_zonal_scatter_backward(
              grad_output.data_ptr<float>(), zonal.data_ptr<float>(), radial.data_ptr<float>(),
              dst.data_ptr<int64_t>(), dst_offsets->data_ptr<int64_t>(), nullptr,
              radial_slot.data_ptr<int64_t>(), inv_sqrt_deg.data_ptr<float>(), edges, nodes,
              rows, n_radial, channels, gz.data_ptr<float>(), gr.data_ptr<float>(),
              gi.data_ptr<float>(), ws.data_ptr(), static_cast<size_t>(ws.numel()),
              stream_of(zonal)),
          "gie_zonal_scatter_backward");
    return {gz, gr, gi};
  }
  // As the forward: gated on the sorted-path flags, read early; the CSR
  // kernel is queued before the outputs and the workspace are allocated.
  auto [offsets, flags] = csr_view_launch(dst, nodes);
  EarlyFlags early(flags);
  Tensor gz = torch::empty_like(zonal);
  Tensor gr = torch::empty_like(radial);
  Tensor gi = torch::empty_like(inv_sqrt_deg);
  Tensor ws = workspace(zonal, bysj_gie_zonal_scatter_backward_workspace_size(edges, nodes, rows,
                                                                              channels));
  check(bysj_gie_zonal_scatter_backward_gated(
            grad_output.data_ptr<float>(), zonal.data_ptr<float>(), radial.data_ptr<float>(),
            dst.data_ptr<int64_t>(), offsets.data_ptr<int64_t>(), nullptr,
            radial_slot.data_ptr<int64_t>(), inv_sqrt_deg.data_ptr<float>(), edges, nodes, rows,
            n_radial, channels, gz.data_ptr<float>(), gr.data_ptr<float>(),
            gi.data_ptr<float>(), ws.data_ptr(), static_cast<size_t>(ws.numel()),
            stream_of(zonal), reinterpret_cast<const uint32_t*>(flags.data_ptr<int32_t>())),
        "gie_zonal_scatter_backward");
  const int64_t word = early.word();
  if (word == 0) return {gz, gr, gi};
  TORCH_CHECK(!(word & BYSJ_FLAG_OUT_OF_RANGE),
              "destination values must be within the node range");
  auto [grouped_offsets, order] = csr_view(dst, nodes);
  check(bysj_gie_zonal_scatter_backward(
            grad_output.data_ptr<float>(), zonal.data_ptr<float>(), radial.data_ptr<float>(),
            dst.data_ptr<int64_t>(), grouped_offsets.data_ptr<int64_t>(),
            opt_ptr<int64_t>(order), radial_slot.data_ptr<int64_t>(),
            inv_sqrt_deg.data_ptr<float>(), edges, nodes, rows, n_radial, channels,
            gz.data_ptr<float>(), gr.data_ptr<float>(), gi.data_ptr<float>(), ws.data_ptr(),
            static_cast<size_t>(ws.numel()), stream_of(zonal)),
        "gie_zonal_scatter_backward");
  return {gz, gr, gi};
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  namespace py = pybind11;
  m.doc() = "B200 (sm_100a) segmented operators: thin shim over libbysj_b200";
  m.def("rmsnorm_forward", &rmsnorm_forward);
  m.def("rmsnorm_backward", &rmsnorm_backward);
  m.def("gie_zonal_scatter_forward", &gie_zonal_scatter_forward, py::arg("zonal"),
        py::arg("radial"), py::arg("dst"), py::arg("radial_slot"), py::arg("inv_sqrt_deg"),
        py::arg("dst_offsets") = py::none());
  m.def("gie_zonal_scatter_backward", &gie_zonal_scatter_backward, py::arg("grad_output"),
        py::arg("zonal"), py::arg("radial"), py::arg("dst"), py::arg("radial_slot"),
        py::arg("inv_sqrt_deg"), py::arg("dst_offsets") = py::none());
  m.def("segment_sum_forward", &segment_sum_forward, py::arg("src"), py::arg("offsets"),
        py::arg("edge_scale") = py::none(), py::arg("node_scale") = py::none(),
        py::arg("order") = py::none());
  m.def("segment_sum_backward", &segment_sum_backward, py::arg("grad_out"), py::arg("src"),
        py::arg("dst"), py::arg("offsets"), py::arg("edge_scale") = py::none(),
        py::arg("node_scale") = py::none(), py::arg("want_node_scale_grad") = false,
        py::arg("order") = py::none());
  m.def("segment_softmax_forward", &segment_softmax_forward, py::arg("logit"), py::arg("env"),
        py::arg("offsets"), py::arg("null_logit") = py::none(), py::arg("order") = py::none());
  m.def("segment_softmax_backward", &segment_softmax_backward, py::arg("alpha"),
        py::arg("grad_alpha"), py::arg("env"), py::arg("offsets"),
        py::arg("null_alpha") = py::none(), py::arg("grad_null_alpha") = py::none(),
        py::arg("order") = py::none());
  m.def("force_assembly", &force_assembly, py::arg("grad_edge"), py::arg("edge_vec"),
        py::arg("dst_offsets"), py::arg("src_offsets"), py::arg("src_order"));
  // Additions beyond the reference module.
  m.def("segment_offsets", &segment_offsets, py::arg("dst"), py::arg("n_nodes"));
  m.def("segment_offsets_device", &segment_offsets_device, py::arg("dst"), py::arg("n_nodes"),
        py::arg("flags"));
  m.def("segment_attention_forward", &segment_attention_forward, py::arg("logit"),
        py::arg("value"), py::arg("offsets"), py::arg("env") = py::none(),
        py::arg("null_logit") = py::none(), py::arg("order") = py::none());
  m.def("check_indices", &check_indices, py::arg("offsets"), py::arg("n_edges"),
        py::arg("order") = py::none(), py::arg("values") = py::none(),
        py::arg("value_limit") = 0);
  m.def("edge_chain", &edge_chain, py::arg("first"), py::arg("second"), py::arg("coefs"),
        py::arg("n_edges"), py::arg("comps"), py::arg("channels"), py::arg("activation"));
  m.def("rotate_back_aggregate_forward", &rotate_back_aggregate_forward, py::arg("x_local"),
        py::arg("rotation"), py::arg("rotate_inv_rescale"), py::arg("attn_alpha"),
        py::arg("row_ptr"), py::arg("order"), py::arg("lmax"), py::arg("heads"));
  m.def("force_assembly_src_partial", &force_assembly_src_partial, py::arg("grad_edge"),
        py::arg("edge_vec"), py::arg("src_offsets"), py::arg("src_order"));
  m.def("force_assembly_dst_add", &force_assembly_dst_add, py::arg("grad_edge"),
        py::arg("dst_offsets"), py::arg("summed_partial"));
  m.def("group_by_key", &group_by_key, py::arg("keys"), py::arg("n_keys"));
  m.def("library_version", []() { return bysj_version(); });
}
