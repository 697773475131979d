/*
 * bysj_b200.h -- C ABI of the B200 (sm_100a) segmented-operator library.
 *
 * Every entry point takes plain device pointers, element counts and a CUDA
 * stream (passed as `void*`, i.e. a `cudaStream_t`; NULL is the legacy default
 * stream), launches its kernels asynchronously on that stream and returns a
 * `bysj_status`.  Nothing here allocates device memory: outputs and scratch
 * ("workspace") are owned by the caller.  Each operator that needs scratch has
 * a `*_workspace_size` query; pass a buffer of at least that many bytes,
 * 256-byte aligned.  Inputs are borrowed and never written.
 *
 * Layout contract shared by the segmented operators: the edge list is grouped
 * by destination node ("segment").  `offsets[n_nodes + 1]` is the exclusive
 * prefix sum of the per-node edge counts; the edges of node n are the slots
 * offsets[n] .. offsets[n+1]-1.  When `order` is non-NULL, slot s refers to
 * edge order[s]; otherwise slot s is edge s.  Index values are trusted to be in
 * range (the Python layer validates shapes and dtypes before calling).
 *
 * All reductions are deterministic: for fixed inputs, sizes and device, two
 * calls produce bit-identical outputs (no floating-point atomics; partial
 * results of a segment split across warps are combined in a fixed order).
 *
 * Reference interfaces replaced (lipengfei1409/bysj):
 *   csrc/ops.h:8-45        (declarations of the HIP operators)
 *   csrc/bindings.cpp:6-29 (the nine Python-visible entry points)
 *   python/kernels/segment.py:46-71 (segment_offsets / group_by_source)
 */
#ifndef BYSJ_B200_H
#define BYSJ_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define BYSJ_API __attribute__((visibility("default")))
#else
#define BYSJ_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum bysj_status {
  BYSJ_OK = 0,
  BYSJ_ERR_INVALID_ARGUMENT = 1, /* bad size, NULL pointer, misalignment    */
  BYSJ_ERR_WORKSPACE = 2,        /* workspace missing or too small           */
  BYSJ_ERR_UNSUPPORTED = 3,      /* shape outside what the kernels support   */
  BYSJ_ERR_CUDA = 4,             /* a CUDA runtime call failed               */
  BYSJ_ERR_LAUNCH = 5,           /* a kernel launch failed                   */
  BYSJ_ERR_TOO_LARGE = 6         /* size beyond a fixed capacity             */
} bysj_status;

typedef enum bysj_dtype {
  BYSJ_F32 = 0,
  BYSJ_BF16 = 1
} bysj_dtype;

/* Flags written to the device word `flags` by the segment_offsets kernels. */
#define BYSJ_FLAG_OUT_OF_RANGE 1u /* some dst < 0 or dst >= n_nodes       */
#define BYSJ_FLAG_UNSORTED 2u     /* dst is not non-decreasing           */

/* Library version (major * 10000 + minor * 100 + patch). */
BYSJ_API int bysj_version(void);
/* Static description of a status code. */
BYSJ_API const char* bysj_status_string(int status);
/* Detail of the last failure on the calling host thread ("" if none). */
BYSJ_API const char* bysj_last_error(void);

/* ------------------------------------------------------------------------
 * Index guard (opt-in).  The operators trust their index inputs, as the
 * reference's native paths do (python/kernels/gie.py:80-81); this pass checks
 * what they trust and ORs one bit per violated invariant into *error (a device
 * word the caller zeroes and reads back):
 *   BYSJ_INDEX_OFFSETS  offsets[0] != 0, offsets[n_nodes] != n_edges, or a
 *                       decreasing / out-of-range entry   (offsets may be NULL)
 *   BYSJ_INDEX_ORDER    order[] not a permutation of [0, n_edges)  (NULL: skip)
 *   BYSJ_INDEX_VALUES   values[0..n_values) outside [0, value_limit) (NULL: skip)
 * The order check needs bysj_check_indices_workspace_size(n_edges) bytes of
 * workspace.  No reference counterpart: the stand-in for a bounds-checked
 * debug build (the reference's opt-in check is the grouping comparison of
 * python/kernels/segment.py:38-43,182-193).
 * ------------------------------------------------------------------------ */
#define BYSJ_INDEX_OFFSETS 1u
#define BYSJ_INDEX_ORDER 2u
#define BYSJ_INDEX_VALUES 4u
BYSJ_API size_t bysj_check_indices_workspace_size(int64_t n_edges);
BYSJ_API int bysj_check_indices(const int64_t* offsets, int64_t n_nodes, int64_t n_edges,
                                const int64_t* order, const int64_t* values, int64_t n_values,
                                int64_t value_limit, uint32_t* error, void* workspace,
                                size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * segment_offsets
 * Replaces python/kernels/segment.py:46-57 (bincount + cumsum over dst).
 * ------------------------------------------------------------------------ */

/* Fast path for a destination-sorted edge list: one pass, no atomics.
 * Writes offsets[0..n_nodes] and ORs BYSJ_FLAG_* into *flags (a device
 * uint32 that the caller zeroes).  If the flags come back non-zero the
 * offsets are meaningless: use bysj_segment_offsets_histogram instead
 * (unsorted input) or report the range error. */
BYSJ_API int bysj_segment_offsets_sorted(const int64_t* dst, int64_t n_edges,
                                int64_t n_nodes, int64_t* offsets,
                                uint32_t* flags, void* stream);

/* General path (any order): histogram with integer atomics, then an
 * exclusive scan.  Integer results are exact; out-of-range dst values are
 * skipped and flagged. */
BYSJ_API size_t bysj_segment_offsets_workspace_size(int64_t n_nodes);
BYSJ_API int bysj_segment_offsets_histogram(const int64_t* dst, int64_t n_edges,
                                   int64_t n_nodes, int64_t* offsets,
                                   uint32_t* flags, void* workspace,
                                   size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * group_by_key (group_by_source / CSR view of an unsorted dst)
 * Replaces python/kernels/segment.py:60-71 (stable argsort of the keys plus
 * bincount + cumsum) and the argsort in python/model/fused_deepmd.py:111-124.
 *   offsets[k] = number of edges with key < k          (int64 [n_keys + 1])
 *   order[offsets[k] .. offsets[k+1]) = the edges with key k, ascending
 * keys: int64 [n_edges]; out-of-range keys are skipped and flagged with
 * BYSJ_FLAG_OUT_OF_RANGE in *flags (device uint32 the caller zeroes); the
 * outputs are then incomplete.  Bit-exact and run-to-run identical.
 * n_keys must be below 2^31 - 1.
 * ------------------------------------------------------------------------ */
BYSJ_API size_t bysj_group_by_key_workspace_size(int64_t n_edges, int64_t n_keys);
BYSJ_API int bysj_group_by_key(const int64_t* keys, int64_t n_edges, int64_t n_keys,
                               int64_t* order, int64_t* offsets, uint32_t* flags,
                               void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * segment_sum
 * Replaces csrc/segment_sum.cpp:214-317 (segment_sum_forward_hip /
 * segment_sum_backward_hip).
 *   out[n, c] = node_scale[n] * sum_{slot in seg(n)} edge_scale[e] * src[e, c]
 * src is [n_edges, channels] in `src_dtype`; out is float32 [n_nodes, channels].
 * edge_scale [n_edges], node_scale [n_nodes] and order [n_edges] may be NULL.
 * ------------------------------------------------------------------------ */
BYSJ_API size_t bysj_segment_sum_workspace_size(int64_t n_edges, int64_t n_nodes,
                                       int64_t channels, int src_dtype);
BYSJ_API int bysj_segment_sum_forward(const void* src, int src_dtype, int64_t n_edges,
                             int64_t channels, const int64_t* offsets,
                             int64_t n_nodes, const float* edge_scale,
                             const float* node_scale, const int64_t* order,
                             float* out, void* workspace,
                             size_t workspace_bytes, void* stream);

/* grad_src[e, c] = grad_out[dst[e], c] * edge_scale[e] * node_scale[dst[e]]
 * grad_node_scale[n] = sum_c grad_out[n, c] * sum_{e in n} edge_scale[e] src[e, c]
 * grad_node_scale may be NULL (not wanted); it requires node_scale != NULL. */
BYSJ_API size_t bysj_segment_sum_backward_workspace_size(int64_t n_edges,
                                                int64_t n_nodes,
                                                int64_t channels,
                                                int src_dtype);
BYSJ_API int bysj_segment_sum_backward(const float* grad_out, const void* src,
                              int src_dtype, const int64_t* dst,
                              const int64_t* offsets, int64_t n_edges,
                              int64_t n_nodes, int64_t channels,
                              const float* edge_scale, const float* node_scale,
                              const int64_t* order, float* grad_src,
                              float* grad_node_scale, void* workspace,
                              size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * segment_softmax
 * Replaces csrc/segment_softmax.cpp:235-343.  Per segment and channel:
 *   l_e = logit[e,c] + 2 ln env[e] for env[e] > 0 (other edges carry no mass)
 *   m = max(null_logit[n,c], max_e l_e);  D = exp(null - m) + sum_e exp(l_e - m)
 *   alpha[e,c] = exp(l_e - m) / D;  null_alpha[n,c] = exp(null - m) / D
 * A segment whose maximum is -inf gets all-zero weights.
 * null_logit / null_alpha may both be NULL.
 * ------------------------------------------------------------------------ */
BYSJ_API size_t bysj_segment_softmax_workspace_size(int64_t n_edges, int64_t n_nodes,
                                           int64_t channels);
BYSJ_API int bysj_segment_softmax_forward(const float* logit, const float* env,
                                 const int64_t* offsets, int64_t n_edges,
                                 int64_t n_nodes, int64_t channels,
                                 const float* null_logit,
                                 const int64_t* order, float* alpha,
                                 float* null_alpha, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* S = sum_e alpha*grad_alpha + null_alpha*grad_null_alpha
 * grad_logit = alpha (grad_alpha - S);  grad_null_logit = null_alpha (grad_null_alpha - S)
 * grad_env[e] = 2 / env[e] * sum_c grad_logit[e, c]  (0 where env[e] <= 0)
 * null_alpha, grad_null_alpha and grad_null_logit are all NULL or all set. */
BYSJ_API size_t bysj_segment_softmax_backward_workspace_size(int64_t n_edges,
                                                    int64_t n_nodes,
                                                    int64_t channels);
BYSJ_API int bysj_segment_softmax_backward(const float* alpha, const float* grad_alpha,
                                  const float* env, const int64_t* offsets,
                                  int64_t n_edges, int64_t n_nodes,
                                  int64_t channels, const float* null_alpha,
                                  const float* grad_null_alpha,
                                  const int64_t* order, float* grad_logit,
                                  float* grad_null_logit, float* grad_env,
                                  void* workspace, size_t workspace_bytes,
                                  void* stream);

/* ------------------------------------------------------------------------
 * segment_attention: fused gated segment softmax + weighted segment sum.
 * No single counterpart in the reference; it is the composition
 * python/reference/segment.py:63-118 (softmax) followed by :39-60 (sum).
 *   alpha[e,h] as in segment_softmax over logit [n_edges, heads]
 *   out[n, h, s, k] = sum_e alpha[e,h] * value[e, s, h*(channels/heads) + k]
 * value is [n_edges, components, channels] in `value_dtype`; out is float32
 * [n_nodes, heads, components, channels/heads].  env [n_edges] and
 * null_logit [n_nodes, heads] may be NULL.  heads must divide channels.
 * ------------------------------------------------------------------------ */
BYSJ_API size_t bysj_segment_attention_workspace_size(int64_t n_edges, int64_t n_nodes,
                                             int64_t heads,
                                             int64_t components,
                                             int64_t channels,
                                             int value_dtype);
BYSJ_API int bysj_segment_attention_forward(const float* logit, const void* value,
                                   int value_dtype, const float* env,
                                   const float* null_logit,
                                   const int64_t* offsets,
                                   const int64_t* order, int64_t n_edges,
                                   int64_t n_nodes, int64_t heads,
                                   int64_t components, int64_t channels,
                                   float* out, void* workspace,
                                   size_t workspace_bytes, void* stream);

/* Allocation-free form of bysj_segment_attention_forward.  It has no
 * counterpart in the reference.  It is for callers that cannot allocate device
 * memory or hand over a workspace: a plugin hook that only sees its inputs,
 * outputs and a stream, a serving runtime whose memory footprint is frozen
 * after warm-up, or a hot path where cudaMalloc would synchronise the device.
 * Same arguments and results (within fp32 rounding: segments may be split at
 * different points) as the workspace form, minus the workspace.
 *
 * Scratch: one file-scope device array of BYSJ_ATTENTION_NOALLOC_SCRATCH_BYTES
 * per GPU, held from library load until process exit.  The partition count is
 * capped so the split-segment slots fit; a value row (components * channels)
 * too wide for even one partition is rejected with BYSJ_ERR_TOO_LARGE.
 * The first call on a device looks up the array's device address (with that
 * device current) and keeps it for the device's CUDA context.  All calls
 * on a device share the array and it keeps the last call's contents (each
 * call zeroes, on its own stream, the counters that must start at zero):
 * calls that overlap on the GPU, e.g. on two streams at once, race and must
 * be serialised by the caller. */
#define BYSJ_ATTENTION_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)
BYSJ_API int bysj_segment_attention_forward_noalloc(
    const float* logit, const void* value, int value_dtype, const float* env,
    const float* null_logit, const int64_t* offsets, const int64_t* order,
    int64_t n_edges, int64_t n_nodes, int64_t heads, int64_t components,
    int64_t channels, float* out, void* stream);

/* ------------------------------------------------------------------------
 * rotate-back aggregation (the flash aggregation seam of DeepMD's SO(2)
 * block).  No single counterpart in the reference's kernels: the reference
 * records the seam SO2Convolution._flash_atten_fn(x_local, rotation,
 * rotate_inv_rescale, attn_alpha, order, row_ptr, dst, lmax, heads) as not yet
 * wired (docs/deepmd-fused-dispatch.md:127-128); its eager form is a rotate,
 * a weighting and an index_add_.  With the edges grouped by destination
 * (offsets / order as above):
 *   out[n, l*l + b, c] = sum_{e in n} alpha[e, c / dh] * rescale[e] *
 *                        sum_a D_{e,l}[a, b] * x_local[e, l*l + a, c]
 * x_local [n_edges, (lmax+1)^2, channels]; rotation [n_edges, sum_l (2l+1)^2]
 * packs each edge's block-diagonal rotation per degree (block l row-major,
 * x_local = D x_global, so this is the transpose); rescale [n_edges] may be
 * NULL (1); alpha [n_edges, heads]; out float32 [n_nodes, (lmax+1)^2,
 * channels]; dh = channels / heads; 0 <= lmax <= 3.  Deterministic.
 * ------------------------------------------------------------------------ */
BYSJ_API size_t bysj_rotate_back_aggregate_workspace_size(int64_t n_edges, int64_t n_nodes,
                                                          int64_t lmax, int64_t heads,
                                                          int64_t channels);
BYSJ_API int bysj_rotate_back_aggregate(const float* x_local, const float* rotation,
                                        const float* rescale, const float* alpha,
                                        const int64_t* offsets, const int64_t* order,
                                        int64_t n_edges, int64_t n_nodes, int64_t lmax,
                                        int64_t heads, int64_t channels, float* out,
                                        void* workspace, size_t workspace_bytes,
                                        void* stream);

/* ------------------------------------------------------------------------
 * Edge-stream elementwise chain in one pass.  No counterpart in the
 * reference's kernels: the reference plans it for the elementwise pool of its
 * DeepMD profile (docs/task2-hip-fusion-plan.md:280-302: "a descriptor-driven
 * kernel that reads k inputs once and sums a term table of pointer + strides
 * + coefficient + broadcast axes into one output, with an optional
 * activation"), where each term is a separate ATen pass today.
 *   out[e, s, c] = act( sum_t coef_t * a_t[e, s, c] * b_t[e, s, c] )
 * out is a contiguous float32 [n_edges, comps, channels]; each factor is a
 * float32 strided view: element (e, s, c) is data[e*stride[0] + s*stride[1]
 * + c*stride[2]], a stride of 0 broadcasts along that axis; b.data == NULL
 * means the term has one factor.  Terms are summed in table order with fused
 * multiply-adds (deterministic).  act: BYSJ_ACT_NONE, _SILU (z sigmoid(z)) or
 * _SIGMOID.
 * ------------------------------------------------------------------------ */
#define BYSJ_CHAIN_MAX_TERMS 8
enum { BYSJ_ACT_NONE = 0, BYSJ_ACT_SILU = 1, BYSJ_ACT_SIGMOID = 2 };
typedef struct bysj_chain_operand {
  const float* data;
  int64_t stride[3];
} bysj_chain_operand;
typedef struct bysj_chain_term {
  float coef;
  bysj_chain_operand a;
  bysj_chain_operand b;
} bysj_chain_term;
BYSJ_API int bysj_edge_chain(const bysj_chain_term* terms, int n_terms, int64_t n_edges,
                             int64_t comps, int64_t channels, int activation, float* out,
                             void* stream);

/* ------------------------------------------------------------------------
 * force_assembly
 * Replaces csrc/force_assembly.cpp:106-146.
 *   force[k]  = sum_{dst(e)=k} g_e - sum_{src(e)=k} g_e        (fp64 accumulate)
 *   virial[k] = - sum_{src(e)=k} g_e (x) v_e  (row-major 3x3)
 * grad_edge, edge_vec: float32 [n_edges, 3]; dst_offsets / src_offsets
 * [n_nodes + 1]; src_order [n_edges] groups the edges by source atom.
 * force [n_nodes, 3], virial [n_nodes, 9] (virial may be NULL).
 * ------------------------------------------------------------------------ */
BYSJ_API int bysj_force_assembly(const float* grad_edge, const float* edge_vec,
                        const int64_t* dst_offsets, const int64_t* src_offsets,
                        const int64_t* src_order, int64_t n_edges,
                        int64_t n_nodes, float* force, float* virial,
                        void* stream);

/* Source-side half of force_assembly for a destination-range partition of a
 * larger graph: partial[k, 0:3] = -sum_{src(e)=k} g_e and
 * partial[k, 3:12] = -sum_{src(e)=k} g_e (x) v_e for every k in [0, n_nodes),
 * where the edges given here are only this partition's; the destination side
 * force[k] += sum_{dst(e)=k} g_e is added by bysj_force_assembly_dst_add for
 * the local atoms [node_begin, node_begin + n_local) after the partials of all
 * partitions have been summed (reduce-scattered).  The partials are float64
 * (the per-partition fp64 sums, unrounded), so the exchanged sums are rounded
 * to float32 once, as on one device.  No reference counterpart: this is the
 * multi-GPU decomposition of csrc/force_assembly.cpp:64-96. */
BYSJ_API int bysj_force_assembly_src_partial(const float* grad_edge,
                                    const float* edge_vec,
                                    const int64_t* src_offsets,
                                    const int64_t* src_order, int64_t n_edges,
                                    int64_t n_nodes, double* partial,
                                    void* stream);
BYSJ_API int bysj_force_assembly_dst_add(const float* grad_edge,
                                const int64_t* dst_offsets, int64_t n_local,
                                const double* summed_partial, float* force,
                                float* virial, void* stream);

/* ------------------------------------------------------------------------
 * rmsnorm (last axis)
 * Replaces csrc/rmsnorm.cpp:99-157.
 *   inv_rms[r] = rsqrt(mean_c x[r,c]^2 + eps);  y[r,c] = x[r,c] inv_rms[r] w[c]
 * x / y: [rows, width] in `dtype` (y has the dtype of x); inv_rms float32.
 * scale: NULL (no scale), float32 [width] (scale_rows == 1) or the
 * per-degree form float32 [scale_rows, width] with scale_rows = L + 1, where
 * row r of x is component i = r mod (L+1)^2 and uses weight row floor(sqrt(i)).
 * ------------------------------------------------------------------------ */
BYSJ_API int bysj_rmsnorm_forward(const void* x, int dtype, int64_t rows, int64_t width,
                         const float* scale, int64_t scale_rows, float eps,
                         void* y, float* inv_rms, void* stream);

/* gx = inv*gw - x*inv^3*mean(x*gw), gw = grad_out*w;
 * grad_scale[l, c] = sum over rows r using weight row l of grad_out*x*inv.
 * grad_scale may be NULL.  Deterministic two-stage reduction (no atomics). */
BYSJ_API size_t bysj_rmsnorm_backward_workspace_size(int64_t rows, int64_t width,
                                            int64_t scale_rows);
BYSJ_API int bysj_rmsnorm_backward(const float* grad_out, const float* x,
                          const float* scale, int64_t scale_rows,
                          const float* inv_rms, int64_t rows, int64_t width,
                          float* grad_x, float* grad_scale, void* workspace,
                          size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * GIE zonal scatter (CSR form)
 * Replaces csrc/gie.cpp:148-228.  With the edges grouped by destination
 * (offsets / order as above):
 *   out[n, 0, :] = 0
 *   out[n, r+1, c] = inv_sqrt_deg[n] * sum_{e in n} zonal[e, r] *
 *                    radial[e, radial_slot[r], c]      (normalise after sum)
 * zonal [n_edges, n_rows], radial [n_edges, n_radial, channels],
 * radial_slot int64 [n_rows], inv_sqrt_deg [n_nodes], out [n_nodes, n_rows+1,
 * channels].  When the shape allows DPA4's degree-grouped layout (3, 8 or 15
 * rows, channels = 4 * 2^k, 16-byte aligned rows) the forward and backward
 * also launch the degree kernel; each kernel checks radial_slot on the device
 * and only the matching one computes (radial_slot is not read back).
 * ------------------------------------------------------------------------ */
BYSJ_API size_t bysj_gie_zonal_scatter_workspace_size(int64_t n_edges, int64_t n_nodes,
                                             int64_t n_rows, int64_t channels);
BYSJ_API int bysj_gie_zonal_scatter_forward(const float* zonal, const float* radial,
                                   const int64_t* offsets,
                                   const int64_t* order,
                                   const int64_t* radial_slot,
                                   const float* inv_sqrt_deg, int64_t n_edges,
                                   int64_t n_nodes, int64_t n_rows,
                                   int64_t n_radial, int64_t channels,
                                   float* out, void* workspace,
                                   size_t workspace_bytes, void* stream);

/* The same operator with a device gate: when *gate != 0 at kernel time every
 * kernel returns at once (outputs untouched).  A caller that derives the
 * destination CSR on the device (bysj_segment_offsets_sorted, whose flags word
 * is the gate) can launch both without reading the flags back first, and read
 * them afterwards to recompute through the unsorted path or report a range
 * error.  No reference counterpart: the pipelining form of
 * csrc/gie.cpp:148-228's entry. */
BYSJ_API int bysj_gie_zonal_scatter_forward_gated(const float* zonal, const float* radial,
                                         const int64_t* offsets, const int64_t* order,
                                         const int64_t* radial_slot,
                                         const float* inv_sqrt_deg, int64_t n_edges,
                                         int64_t n_nodes, int64_t n_rows, int64_t n_radial,
                                         int64_t channels, float* out, void* workspace,
                                         size_t workspace_bytes, void* stream,
                                         const uint32_t* gate);

/* Same operator for the degree-grouped row layout the DPA4 GIE uses: rows
 * r = 0 .. (degrees+1)^2 - 2, row r has degree l = floor(sqrt(r + 1)) and
 * reads radial slot l + slot_base (slot_base = 0 for slots 1..L, -1 for
 * slots 0..L-1), i.e. radial_slot[r] == floor(sqrt(r+1)) + slot_base.  It
 * needs 1 <= degrees <= 3, channels = 4 * 2^k <= 128 and 16-byte-aligned
 * radial and out; each lane then loads every degree's radial row once per
 * edge instead of once per output row. */
BYSJ_API size_t bysj_gie_zonal_scatter_degree_workspace_size(int64_t n_edges,
                                                             int64_t n_nodes,
                                                             int64_t degrees,
                                                             int64_t channels);
BYSJ_API int bysj_gie_zonal_scatter_forward_degree(
    const float* zonal, const float* radial, const int64_t* offsets,
    const int64_t* order, int64_t slot_base, const float* inv_sqrt_deg,
    int64_t n_edges, int64_t n_nodes, int64_t degrees, int64_t n_radial,
    int64_t channels, float* out, void* workspace, size_t workspace_bytes,
    void* stream);

/* Backward of bysj_gie_zonal_scatter_forward_degree (same row layout; see
 * bysj_gie_zonal_scatter_backward for the gradients).  channels = 4 * 2^k
 * <= 64; radial, grad_out and grad_radial 16-byte aligned; grad_radial's
 * slots that no row reads are written as zeros.  No reference counterpart:
 * the degree-specialised form of csrc/gie.cpp:170-228. */
BYSJ_API size_t bysj_gie_zonal_scatter_backward_degree_workspace_size(int64_t n_edges,
                                                                      int64_t n_nodes,
                                                                      int64_t degrees,
                                                                      int64_t channels);
BYSJ_API int bysj_gie_zonal_scatter_backward_degree(
    const float* grad_out, const float* zonal, const float* radial, const int64_t* offsets,
    const int64_t* order, int64_t slot_base, const float* inv_sqrt_deg, int64_t n_edges,
    int64_t n_nodes, int64_t degrees, int64_t n_radial, int64_t channels, float* grad_zonal,
    float* grad_radial, float* grad_inv, void* workspace, size_t workspace_bytes, void* stream);

/* grad_zonal[e, r]     = inv[dst e] * sum_c g[dst e, r+1, c] radial[e, slot r, c]
 * grad_radial[e, s, c] = inv[dst e] * sum_{r: slot r = s} g[dst e, r+1, c] zonal[e, r]
 * grad_inv[n]          = sum_{r,c} g[n, r+1, c] * sum_{e in n} zonal[e,r] radial[e, slot r, c]
 * dst [n_edges] is the destination of each edge (natural order). */
BYSJ_API size_t bysj_gie_zonal_scatter_backward_workspace_size(int64_t n_edges,
                                                      int64_t n_nodes,
                                                      int64_t n_rows,
                                                      int64_t channels);
BYSJ_API int bysj_gie_zonal_scatter_backward(
    const float* grad_out, const float* zonal, const float* radial,
    const int64_t* dst, const int64_t* offsets, const int64_t* order,
    const int64_t* radial_slot, const float* inv_sqrt_deg, int64_t n_edges,
    int64_t n_nodes, int64_t n_rows, int64_t n_radial, int64_t channels,
    float* grad_zonal, float* grad_radial, float* grad_inv, void* workspace,
    size_t workspace_bytes, void* stream);

/* Backward with the same device gate as bysj_gie_zonal_scatter_forward_gated. */
BYSJ_API int bysj_gie_zonal_scatter_backward_gated(
    const float* grad_out, const float* zonal, const float* radial,
    const int64_t* dst, const int64_t* offsets, const int64_t* order,
    const int64_t* radial_slot, const float* inv_sqrt_deg, int64_t n_edges,
    int64_t n_nodes, int64_t n_rows, int64_t n_radial, int64_t channels,
    float* grad_zonal, float* grad_radial, float* grad_inv, void* workspace,
    size_t workspace_bytes, void* stream, const uint32_t* gate);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* BYSJ_B200_H */
