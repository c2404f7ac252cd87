/*
 * cign_sm100.h -- C ABI of libcign_sm100.so, the B200 (sm_100a) kernels of
 * CIGN's sparse message-passing hot path.
 *
 * Conventions
 *   - Every pointer argument is a DEVICE pointer unless stated otherwise;
 *     pointer arrays (float* const* ...) are HOST arrays of device pointers.
 *   - Dense matrices are row-major, fp32, contiguous, rows of the stated width.
 *   - CSR indices are int32 (the reference converts to int32 before any
 *     kernel: multihop_csr_pipeline.py:38-48, collapsed_gat.cpp:32-43).
 *   - `stream` is a cudaStream_t passed as void*; 0 = legacy default stream.
 *   - Every function returns CIGN_OK (0) or one of the CIGN_ERR_* codes; the
 *     message of the last failure on the calling thread is returned by
 *     cign_last_error().  Arguments are checked before anything is launched,
 *     so an error return means nothing was enqueued.
 *   - Kernels never allocate.  Scratch ("ws") is passed in by the caller,
 *     sized by the matching *_workspace_bytes() query.
 *   - Reductions are deterministic: repeated calls on the same inputs give
 *     bitwise identical outputs (no floating-point atomics).
 *   - Dropout entry points take `uint64_t seed, const uint64_t* seed_ptr`:
 *     with seed_ptr == NULL the seed is `seed`; otherwise it is the value at
 *     the device address seed_ptr when the kernel runs (so a captured CUDA
 *     graph can draw a fresh seed on every replay).
 *
 * Each entry point names the reference interface it replaces
 * (rabbit-art/CIGN, path within that project:line).
 */
#ifndef CIGN_SM100_H
#define CIGN_SM100_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define CIGN_API __attribute__((visibility("default")))
#else
#define CIGN_API
#endif

typedef void* cign_stream_t;

enum {
  CIGN_OK = 0,
  CIGN_ERR_INVALID_ARGUMENT = 1, /* bad size / shape / mode value          */
  CIGN_ERR_NULL_POINTER = 2,     /* required pointer is NULL               */
  CIGN_ERR_ALIGNMENT = 3,        /* pointer not aligned as documented      */
  CIGN_ERR_LAUNCH = 4,           /* kernel launch failed                   */
  CIGN_ERR_TIMEOUT = 5,          /* a bounded device-side wait expired     */
  CIGN_ERR_UNSUPPORTED = 6,      /* shape outside the supported range      */
  CIGN_ERR_CUDA = 7              /* other CUDA runtime error               */
};

/* ------------------------------------------------------------------ misc */
CIGN_API int cign_version(void);
CIGN_API const char* cign_last_error(void);
/* Number of kernels this library has launched in the process so far
 * (all threads, all devices); for launch accounting in benchmarks. */
CIGN_API uint64_t cign_kernel_launches(void);

/* ------------------------------------------------------------------ CSR
 * A fixed sparse graph operator in CSR form (device arrays).
 * Replaces the CSR parts held by FixedCSRGraphOperator (model.py:109-146)
 * and cloned to int32 by _csr_parts_int32 (multihop_csr_pipeline.py:38-48). */
typedef struct cign_csr_f32 {
  int64_t rows;
  int64_t cols;
  int64_t nnz;
  const int32_t* crow; /* [rows+1], crow[0] = 0, non-decreasing */
  const int32_t* col;  /* [nnz], 0 <= col < cols                */
  const float* val;    /* [nnz]                                 */
} cign_csr_f32;

/* SpMM plan over P (and P^T).  Validates the CSR on the device and cuts rows
 * with more than 128 non-zeros ("hub" rows of power-law graphs) into
 * 128-edge segments processed in parallel and combined in a fixed order.  The CSR
 * arrays stay owned by the caller and must outlive the plan.  Immutable
 * after creation: one plan may be used from several streams at once.
 * Replaces MultiHopCsrPlan (multihop_csr_ext/multihop_csr_pipeline_cuda.cu:
 * 113-322) and its Python owner MultiHopCSR3GraphOperator
 * (multihop_csr_pipeline.py:89-140).  `pt` may be NULL when P is symmetric
 * (or the caller only runs forward); the transposed entry points then use P.
 * Synchronises the device once (reads crow to the host). */
typedef struct cign_spmm_plan cign_spmm_plan;

typedef struct cign_spmm_plan_info {
  int64_t rows;
  int64_t nnz;
  int64_t heavy_rows;     /* hub rows of P (split into segments)           */
  int64_t heavy_rows_t;   /* same for P^T                                  */
  int64_t segments;       /* segments of P's hub rows                      */
  int64_t segments_t;
  int32_t max_degree;
  int32_t max_degree_t;
  int32_t segment_length; /* edges per segment                             */
  int32_t transpose_is_forward; /* 1 when P^T calls reuse P              */
} cign_spmm_plan_info;

CIGN_API int cign_spmm_plan_create(const cign_csr_f32* p, const cign_csr_f32* pt,
                          cign_spmm_plan** out);
CIGN_API int cign_spmm_plan_destroy(cign_spmm_plan* plan);
CIGN_API int cign_spmm_plan_get_info(const cign_spmm_plan* plan,
                            cign_spmm_plan_info* info /* host */);

/* Workspace of one cign_spmm call with F feature columns (hub-row partials). */
CIGN_API size_t cign_spmm_workspace_bytes(const cign_spmm_plan* plan, int64_t F);

/* Y = op(P) @ X (+ addend).  op = P (transpose=0) or P^T (transpose=1).
 * X: [cols of op(P), F]; Y, addend: [rows of op(P), F].  P may be
 * rectangular (a row block of a partitioned operator); its transposed
 * product then needs `pt` at plan creation.  addend may be NULL.  Y must not
 * alias X.
 * Replaces FixedCSRSpMMFunction.forward/backward (model.py:57-106). */
CIGN_API int cign_spmm(const cign_spmm_plan* plan, int transpose, const float* X,
              int64_t F, const float* addend, float* Y, void* ws,
              size_t ws_bytes, cign_stream_t stream);

/* Workspace of cign_multihop_fwd/bwd: the backward's [rows, F] recurrence
 * state (max_power >= 2) plus the hub-row partials. */
CIGN_API size_t cign_multihop_workspace_bytes(const cign_spmm_plan* plan,
                                     int max_power, int64_t F);

/* k-hop forward recurrence Y[p-1] = P^p X for p = 1..max_power.
 * Y: host array of max_power device pointers, each [rows, F]; entries for
 * powers the caller does not need still need a buffer (they are the
 * recurrence state).
 * Replaces MultiHopCsrPlan::forward3 (multihop_csr_pipeline_cuda.cu:287-297),
 * GenericMultiHopCSRFunction.forward (multihop_csr_pipeline.py:233-246) and
 * the hybrid native3 + tail path (multihop_csr_pipeline.py:214-230). */
CIGN_API int cign_multihop_fwd(const cign_spmm_plan* plan, int max_power,
                      const float* X, int64_t F, float* const* Y, void* ws,
                      size_t ws_bytes, cign_stream_t stream);

/* cign_multihop_fwd with hop 1's input given as its two column blocks
 * X = [X0 | X1], each [rows, d] row-major (the block's H_norm and C_norm), so
 * the [rows, 2d] concatenation is never written; Y[p] as cign_multihop_fwd
 * (F = 2d).  d % 256 == 0, 16-byte aligned tensors. */
CIGN_API int cign_multihop_fwd_split(const cign_spmm_plan* plan, int max_power,
                                     const float* X0, const float* X1, int64_t d,
                                     float* const* Y, void* ws, size_t ws_bytes,
                                     cign_stream_t stream);

/* k-hop transposed backward: acc = 0; for p = max_power..1:
 *   acc = P^T (acc + G[p-1]);   GX = acc.
 * G: host array of max_power device pointers ([rows, F]) or NULL entries
 * for powers that received no gradient.  The "+ G" is fused into the SpMM
 * epilogue (one pass per hop).
 * Replaces MultiHopCsrPlan::backward3 (multihop_csr_pipeline_cuda.cu:299-321)
 * and GenericMultiHopCSRFunction.backward (multihop_csr_pipeline.py:248-265).*/
CIGN_API int cign_multihop_bwd(const cign_spmm_plan* plan, int max_power,
                      const float* const* G, int64_t F, float* GX, void* ws,
                      size_t ws_bytes, cign_stream_t stream);

/* bf16 feature storage (the large-graph configuration stores node features
 * as bf16 with fp32 accumulation; the reference's sparse path is fp32 only,
 * multihop_csr_pipeline_cuda.cu:63).  X is bf16 [rows, F] (F % 8 == 0, 16-byte
 * aligned); products accumulate in fp32 in the edge order of cign_spmm, so a
 * float32 Y (y_bf16 == 0) equals cign_spmm on the widened X; with y_bf16 != 0
 * Y is bf16, rounded to nearest even.  Workspace: cign_spmm_workspace_bytes. */
CIGN_API int cign_spmm_bf16(const cign_spmm_plan* plan, int transpose, const void* X, int64_t F,
                   void* Y, int y_bf16, void* ws, size_t ws_bytes, cign_stream_t stream);
/* Y[p-1] = P^p X for p = 1..max_power, every hop stored as bf16. */
CIGN_API int cign_multihop_fwd_bf16(const cign_spmm_plan* plan, int max_power, const void* X,
                           int64_t F, void* const* Y, void* ws, size_t ws_bytes,
                           cign_stream_t stream);

/* ------------------------------------------------------------------ GAT
 * Collapsed multi-head GAT (concat=False) over a fixed graph.
 *
 * Graph plan: destination-major CSR (rowptr [n+1], col [nnz]) and its CSC
 * (colptr [n+1], row [nnz]) with perm[csc position] = CSR edge id -- the
 * triple PyG's FusedGATConv.to_graph_format yields and the reference keeps
 * in GraphCliffordNet.prepare_fused_gat_graph (generic_engine/model_cign.py:
 * 1069-1158).  The plan validates the triple on the device, cuts rows and
 * columns with more than 32 edges into 32-edge segments (processed in
 * parallel, combined in a fixed order) and keeps pointers to the caller's
 * arrays, which must outlive it.  Synchronises the device once. */
typedef struct cign_gat_plan cign_gat_plan;

CIGN_API int cign_gat_plan_create(int64_t n, int64_t nnz, const int32_t* rowptr,
                         const int32_t* col, const int32_t* colptr,
                         const int32_t* row, const int32_t* perm,
                         cign_gat_plan** out);
/* Rectangular form: destination rows 0..n_rows-1 (rowptr [n_rows+1]) and
 * source columns 0..n_cols-1 (colptr [n_cols+1]) -- e.g. the row block of a
 * partitioned graph whose columns index local rows plus halo rows.  Only the
 * cign_gat_agg_* entry points accept n_rows != n_cols. */
CIGN_API int cign_gat_plan_create_rect(int64_t n_rows, int64_t n_cols, int64_t nnz,
                                       const int32_t* rowptr, const int32_t* col,
                                       const int32_t* colptr, const int32_t* row,
                                       const int32_t* perm, cign_gat_plan** out);
CIGN_API int cign_gat_plan_destroy(cign_gat_plan* plan);
/* info (host, 8 entries): n, nnz, hub rows, hub columns, max row length,
 * max column length, row segments, column segments. */
CIGN_API int cign_gat_plan_get_info(const cign_gat_plan* plan, int64_t* info);

CIGN_API size_t cign_gat_fwd_workspace_bytes(const cign_gat_plan* plan, int32_t heads,
                                    int32_t channels);

/* Forward, for destination row i and head h:
 *   e_ij = LeakyReLU(attn_row[i,h] + attn_col[j,h]),
 *   w_ij = keep(e*H+h) * exp(e_ij - max_j e) / sum_j exp(e_ij - max_j e) / (1-p),
 *   pre[i,:] = (1/H) sum_h sum_j w_ij in_feat[j,h,:] + bias,  out = SiLU(pre),
 *   edge_max/edge_sum [N,H] = the row's max and exp-sum (saved for backward).
 * keep(idx) is the splitmix64 Bernoulli of make_dropout_mask_kernel
 * (collapsed_gat_cuda.cu:34-47), recomputed from (seed, idx), never stored.
 * in_feat [N,H,C]; out, pre [N,C].  attn_drop in [0,1); 1 <= H <= 64.
 * Replaces collapsed_gat_forward_cuda (collapsed_gat_ext/collapsed_gat_cuda.cu:
 * 434-478) behind collapsed_gat_mean_bias_silu (collapsed_gat.py:164-225),
 * without its H=6,C=256 restriction (collapsed_gat.cpp:67-68). */
CIGN_API int cign_gat_fwd(const cign_gat_plan* plan, int32_t heads, int32_t channels,
                 const float* attn_row, const float* attn_col,
                 const float* in_feat, const float* bias, float negative_slope,
                 float attn_drop, uint64_t seed,
                              const uint64_t* seed_ptr, float* out, float* pre,
                 float* edge_max, float* edge_sum, void* ws, size_t ws_bytes,
                 cign_stream_t stream);

CIGN_API size_t cign_gat_bwd_workspace_bytes(const cign_gat_plan* plan, int32_t heads,
                                    int32_t channels);

/* Backward of cign_gat_fwd: grad_feat [N,H,C], grad_attn_row/col [N,H],
 * grad_bias [C].  Deterministic: grad_attn_col is gathered over the CSC
 * instead of the reference's atomicAdd scatter.
 * Replaces collapsed_gat_backward_cuda (collapsed_gat_cuda.cu:480-545). */
CIGN_API int cign_gat_bwd(const cign_gat_plan* plan, int32_t heads, int32_t channels,
                 const float* attn_row, const float* attn_col,
                 const float* in_feat, const float* pre, const float* edge_max,
                 const float* edge_sum, const float* grad_y,
                 float negative_slope, float attn_drop, uint64_t seed,
                              const uint64_t* seed_ptr,
                 float* grad_feat, float* grad_attn_row, float* grad_attn_col,
                 float* grad_bias, void* ws, size_t ws_bytes,
                 cign_stream_t stream);

/* Materialise the GAT dropout keep-mask (uint8 [nnz*H], 1 = kept) exactly
 * as make_dropout_mask_kernel (collapsed_gat_cuda.cu:34-47) does.  The
 * forward/backward never need it; it exists for parity checks. */
CIGN_API int cign_gat_dropout_mask(int64_t nnz, int32_t heads, float attn_drop,
                          uint64_t seed,
                              const uint64_t* seed_ptr, uint8_t* mask, cign_stream_t stream);

/* Aggregate-first form of the same layer.  GATConv's lin is linear, so with
 * in_feat[j,h,:] = W_h x[j,:] (W = lin.weight viewed [H, C, D]):
 *   sum_j w_ij in_feat[j,h,:] = W_h z[i,h,:],  z[i,h,:] = sum_j w_ij x[j,:].
 * cign_gat_agg_fwd computes z [N,H,D] (and edge_max/edge_sum [N,H]) from the
 * layer input x [N,D] with exactly the weights of cign_gat_fwd; the caller
 * applies pre = z.view(N, H*D) @ M + bias with M[(h,d), c] = W_h[c,d] / H.
 * Each edge then gathers one D-float row instead of H*C floats.
 * cign_gat_agg_bwd: given grad_z = dL/dz [N,H,D] (= g_pre @ M^T) and
 * grad_pre = dL/dpre [N,C], writes grad_attn_row/col [N,H] and
 * grad_feat [N,H,C] = sum_i w_ij g_pre[i,:] / H (so dL/dx through the
 * aggregation is grad_feat.view(N, H*C) @ lin.weight).
 * x, z, grad_z, grad_pre, grad_feat and ws 16-byte aligned; D, C multiples
 * of 4.  Same results as collapsed_gat_forward_cuda / _backward_cuda
 * (collapsed_gat_cuda.cu:434-545) applied to lin(x), up to the order of
 * the floating-point sums; it is the form the CIGN block calls
 * (generic_engine/model_cign.py:551-567). */
CIGN_API size_t cign_gat_agg_workspace_bytes(const cign_gat_plan* plan, int32_t heads,
                                             int64_t dim, int64_t channels);
CIGN_API int cign_gat_agg_fwd(const cign_gat_plan* plan, int32_t heads, int64_t dim,
                              const float* attn_row, const float* attn_col, const float* x,
                              float negative_slope, float attn_drop, uint64_t seed,
                              const uint64_t* seed_ptr, float* z,
                              float* edge_max, float* edge_sum, void* ws, size_t ws_bytes,
                              cign_stream_t stream);
/* cign_gat_agg_fwd over a bf16 layer input x [n_cols, dim] (dim % 8 == 0):
 * z [n, H, dim] fp32, equal to cign_gat_agg_fwd on the widened x (same
 * weights, edge order and fp32 FMA order); workspace as cign_gat_agg_fwd. */
CIGN_API int cign_gat_agg_fwd_bf16(const cign_gat_plan* plan, int32_t heads, int64_t dim,
                          const float* attn_row, const float* attn_col, const void* x,
                          float negative_slope, float attn_drop, uint64_t seed_value,
                          const uint64_t* seed_ptr, float* z, float* edge_max, float* edge_sum,
                          void* ws, size_t ws_bytes, cign_stream_t stream);

CIGN_API int cign_gat_agg_bwd(const cign_gat_plan* plan, int32_t heads, int64_t dim,
                              int64_t channels, const float* attn_row, const float* attn_col,
                              const float* x, const float* edge_max, const float* edge_sum,
                              const float* grad_z, const float* grad_pre, float negative_slope,
                              float attn_drop, uint64_t seed,
                              const uint64_t* seed_ptr, float* grad_feat,
                              float* grad_attn_row, float* grad_attn_col, void* ws,
                              size_t ws_bytes, cign_stream_t stream);

/* cign_gat_agg_fwd / cign_gat_agg_bwd with the edge weights [nnz, H] (CSR
 * edge order) kept between them: the forward writes them to `wts` and the
 * backward reads them there instead of forming them again from
 * edge_max / edge_sum (the same values, bit for bit).  The caller keeps
 * `wts` (16-byte aligned, nnz * H floats) alive from the forward to the
 * backward of the same call; workspace as cign_gat_agg_fwd / _bwd. */
CIGN_API int cign_gat_agg_fwd_w(const cign_gat_plan* plan, int32_t heads, int64_t dim,
                                const float* attn_row, const float* attn_col, const float* x,
                                float negative_slope, float attn_drop, uint64_t seed,
                                const uint64_t* seed_ptr, float* z, float* edge_max,
                                float* edge_sum, float* wts, void* ws, size_t ws_bytes,
                                cign_stream_t stream);
CIGN_API int cign_gat_agg_bwd_w(const cign_gat_plan* plan, int32_t heads, int64_t dim,
                                int64_t channels, const float* attn_row, const float* attn_col,
                                const float* x, const float* edge_max, const float* edge_sum,
                                const float* grad_z, const float* grad_pre, const float* wts,
                                float negative_slope, float attn_drop, uint64_t seed,
                                const uint64_t* seed_ptr, float* grad_feat,
                                float* grad_attn_row, float* grad_attn_col, void* ws,
                                size_t ws_bytes, cign_stream_t stream);

/* ------------------------------------------------------------ side ops
 * alpha_src[n,h] = sum_c x[n,h,c] att_src[h,c];  same for dst.
 * Replaces attention_forward_cuda (fused_gat_sideops_cuda.cu:243-260). */
CIGN_API int cign_attn_logits_fwd(int64_t n, int32_t heads, int32_t channels,
                         const float* x, const float* att_src,
                         const float* att_dst, float* alpha_src,
                         float* alpha_dst, cign_stream_t stream);

CIGN_API size_t cign_attn_logits_bwd_workspace_bytes(int64_t n, int32_t heads,
                                            int32_t channels);

/* grad_x = g_src (x) att_src + g_dst (x) att_dst;  grad_att_* = sum_n g x.
 * accumulate != 0 adds into grad_x instead of overwriting it.
 * Replaces attention_backward_cuda (fused_gat_sideops_cuda.cu:262-299). */
CIGN_API int cign_attn_logits_bwd(int64_t n, int32_t heads, int32_t channels,
                         const float* grad_src, const float* grad_dst,
                         const float* x, const float* att_src,
                         const float* att_dst, float* grad_x,
                         float* grad_att_src, float* grad_att_dst,
                         int32_t accumulate, void* ws, size_t ws_bytes,
                         cign_stream_t stream);

/* Attention logits of lin(x) without forming lin(x) (the side op of
 * fused_gat_sideops.py:50-71 applied to lin(x).view(N, H, C),
 * generic_engine/model_cign.py:551-567): out[n, j] = <x[n, :], V[j, :]>
 * for K <= 16 vectors V [K, D] (V = [W_h^T att_src[h] ; W_h^T att_dst[h]]
 * gives the 2H logits).  fp32, fixed summation order.  D % 4 == 0, x and V
 * 16-byte aligned.  One read of x. */
CIGN_API int cign_row_dots_fwd(int64_t n, int64_t d, int32_t k, const float* x,
                      const float* V, float* out, cign_stream_t stream);

CIGN_API size_t cign_row_dots_bwd_workspace_bytes(int64_t n, int64_t d, int32_t k);

/* grad_x = (accumulate ? grad_x : 0) + grad_out V;  grad_V = grad_out^T x
 * (chunk partials summed in a fixed order).  grad_out [n, K]. */
CIGN_API int cign_row_dots_bwd(int64_t n, int64_t d, int32_t k, const float* x,
                      const float* V, const float* grad_out, float* grad_x,
                      int32_t accumulate, float* grad_V, void* ws, size_t ws_bytes,
                      cign_stream_t stream);

/* y = SiLU(mean_h out[n,h,:] + bias).  Replaces head_silu_forward_cuda
 * (fused_gat_sideops_cuda.cu:301-316). */
CIGN_API int cign_head_mean_bias_silu_fwd(int64_t n, int32_t heads, int32_t channels,
                                 const float* out, const float* bias,
                                 float* y, float* pre, cign_stream_t stream);

CIGN_API size_t cign_head_mean_bias_silu_bwd_workspace_bytes(int64_t n,
                                                    int32_t channels);

/* Replaces head_silu_backward_cuda (fused_gat_sideops_cuda.cu:318-337). */
CIGN_API int cign_head_mean_bias_silu_bwd(int64_t n, int32_t heads, int32_t channels,
                                 const float* grad_y, const float* pre,
                                 float* grad_out, float* grad_bias, void* ws,
                                 size_t ws_bytes, cign_stream_t stream);

/* ------------------------------------------------------------------ pack
 * Clifford interaction pack.  For hop k with T_H = P_k[:, :D], T_C = P_k[:, D:]:
 *   b_hr = H*T_C, b_rh = C*T_H
 *   interaction 0 ("old"): D_k = SiLU(b_hr),           W_k = b_hr - b_rh
 *   interaction 1 ("new"): D_k = SiLU((b_hr+b_rh)/2),  W_k = o((b_hr-b_rh)/2)
 *     with outer o = identity (outer 0, "none") or tanh (outer 1)
 *   weighting 0 ("old"): out[n, k*2D + d] = a_k W_k, out[n, k*2D + D + d] = a_k D_k
 *   weighting 1 ("new"): out[n, d] = sum_k a_k D_k,  out[n, D + d] = sum_k a_k W_k
 * P: host array of K device pointers, each [N, 2D] with row stride ldp floats.
 * alpha: [N, K] or NULL (all ones).
 * Replaces fused_pack_forward_kernel (fused_clifford_pack_ext/
 * fused_clifford_pack_cuda.cu:22-56), the generic-K kernels
 * (fused_clifford_pack.py:88-117, generic_engine/fused_clifford_cign_generic.py:
 * 58-87) and the switch/CIGN packs (generic_engine/fused_clifford_switch_pack_ext/
 * fused_clifford_switch_pack_cuda.cu:65-179). */
CIGN_API int cign_pack_fwd(int64_t n, int64_t d, int32_t k, int32_t interaction,
                  int32_t outer, int32_t weighting, const float* H,
                  const float* C, const float* const* P, int64_t ldp,
                  const float* alpha, float* out, cign_stream_t stream);

/* The block's hop gate evaluated inside the pack forward
 * (generic_engine/model_cign.py:721-749 followed by :817-925): alpha =
 * softmax_k(gate_input @ gate_w^T + gate_b) with gate_input = [H + C | |H - C|]
 * (gate_mode 1, score mode "new") or [H | C] (0), gate_w [K, 2D], gate_b [K];
 * alpha [n, K] is written and the pack (modes as cign_pack_fwd) uses it.
 * H and C are read once for both.  alpha and out equal cign_hop_gate_fwd
 * followed by cign_pack_fwd bit for bit.  1 <= K <= 8, D % 4 == 0,
 * D <= 1024, 16-byte aligned tensors. */
CIGN_API int cign_gate_pack_fwd(int64_t n, int64_t d, int32_t k, int32_t gate_mode,
                       int32_t interaction, int32_t outer, int32_t weighting, const float* H,
                       const float* C, const float* const* P, int64_t ldp,
                       const float* gate_w, const float* gate_b, float* alpha, float* out,
                       cign_stream_t stream);
/* Backward: grad_H, grad_C [N,D]; grad_P: host array of K device pointers
 * ([N,2D], stride ldgp); grad_alpha [N,K] or NULL.
 * accumulate_p != 0 adds into grad_P instead of overwriting it.
 * Replaces fused_pack_backward_main/alpha_kernel (fused_clifford_pack_cuda.cu:
 * 58-152), the generic-K backward (fused_clifford_cign_generic.py:70-87) and
 * backward_main/alpha_kernel (fused_clifford_switch_pack_cuda.cu:186-368). */
CIGN_API int cign_pack_bwd(int64_t n, int64_t d, int32_t k, int32_t interaction,
                  int32_t outer, int32_t weighting, const float* grad_out,
                  const float* H, const float* C, const float* const* P,
                  int64_t ldp, const float* alpha, float* grad_H,
                  float* grad_C, float* const* grad_P, int64_t ldgp,
                  int32_t accumulate_p, float* grad_alpha,
                  cign_stream_t stream);

/* ---------------------------------------------------- JK output LayerNorm
 * y = LayerNorm([seg_0 | seg_1 | ... | seg_{S-1}]) over rows of
 * D = S * seg_width <= 2048 floats (biased variance), reading the S segment
 * tensors [n, seg_width] directly instead of their concatenation; mean and
 * rstd [n] are saved for the backward.  Replaces
 * output_norm(torch.cat(states, dim=-1)) of GraphCliffordNet
 * (generic_engine/model_cign.py:1195-1201).  segs / grad_segs: host arrays
 * of S device pointers; seg_width % 4 == 0, 16-byte aligned rows.  The
 * backward writes the per-segment input gradients and the LayerNorm weight
 * and bias gradients (fixed-order sums over rows). */
CIGN_API size_t cign_jk_ln_workspace_bytes(int64_t n, int64_t d);
CIGN_API int cign_jk_ln_fwd(int64_t n, int32_t n_seg, int64_t seg_width,
                   const float* const* segs, const float* w, const float* b, float eps,
                   float* y, float* mean, float* rstd, cign_stream_t stream);
CIGN_API int cign_jk_ln_bwd(int64_t n, int32_t n_seg, int64_t seg_width, const float* grad_y,
                   const float* const* segs, const float* w, const float* mean,
                   const float* rstd, float* const* grad_segs, float* grad_w,
                   float* grad_b, void* ws, size_t ws_bytes, cign_stream_t stream);

/* ------------------------------------------------------- pack + proj GEMM
 * out[n,:] = G[n,:] @ W^T + bias with G = pack(H, C, P_1..P_K, alpha) in the
 * production switches (interaction "new", outer none, weighting "old"),
 * on tcgen05 tensor cores in TF32 with fp32 accumulation.  Replaces the
 * pack call (fused_clifford_switch_pack(..., "new", "old"),
 * generic_engine/model_cign.py:869-876) followed by the proj linear layer
 * (model_cign.py:927-929).  W is [dout, 2*K*d] row-major, bias [dout]; P as in
 * cign_pack_fwd (ldp >= 2d, 16-byte aligned rows).  G is never stored unless
 * g_out is non-NULL ([n, 2*K*d], written exactly as cign_pack_fwd writes it).
 * Requires d % 32 == 0, 1 <= K <= 8, dout % 32 == 0 and dout <= 512.
 * The workspace holds W re-laid out for the MMA plus a status word that
 * cign_pack_proj_status reads (CIGN_ERR_TIMEOUT if a bounded device-side
 * wait expired; it synchronises `stream`). */
CIGN_API size_t cign_pack_proj_workspace_bytes(int64_t d, int32_t k, int64_t dout);
CIGN_API int cign_pack_proj_gemm_tf32(int64_t n, int64_t d, int32_t k, int64_t dout,
                             const float* H, const float* C, const float* const* P,
                             int64_t ldp, const float* alpha, const float* W,
                             const float* bias, float* out, float* g_out, void* ws,
                             size_t ws_bytes, cign_stream_t stream);
CIGN_API int cign_pack_proj_status(const void* ws, int64_t d, int32_t k, int64_t dout,
                          cign_stream_t stream);

/* ------------------------------------------------------------ input projection
 * The net's dual input projection after one GEMM has formed both halves
 * z = [x W0^T + b0 | x W1^T + b1] ([n, 2d]) (generic_engine/model_cign.py:
 * 1162-1170, H = SiLU(z0) + eta * SiLU(z1)).  eta is a device scalar.
 * cign_silu_mix_fwd: out [n, d].  cign_silu_mix_bwd: grad_z [n, 2d] and
 * grad_eta (a device scalar, summed in a fixed order).  d % 4 == 0,
 * 16-byte aligned tensors. */
CIGN_API int cign_silu_mix_fwd(int64_t n, int64_t d, const float* z, const float* eta,
                               float* out, cign_stream_t stream);
CIGN_API size_t cign_silu_mix_bwd_workspace_bytes(int64_t n, int64_t d);
CIGN_API int cign_silu_mix_bwd(int64_t n, int64_t d, const float* grad_out, const float* z,
                               const float* eta, float* grad_z, float* grad_eta, void* ws,
                               size_t ws_bytes, cign_stream_t stream);

/* ------------------------------------------------------------ peer memory
 * Halo exchange of the row-partitioned path over NVLink peer memory
 * (the reference trains on one GPU: these entry points have no reference
 * counterpart).
 * cign_device_alloc/free: plain cudaMalloc'd buffers whose CUDA IPC handles
 * (CIGN_IPC_HANDLE_BYTES bytes, cign_ipc_handle) other processes map with
 * cign_ipc_open (peer access enabled lazily) and unmap with cign_ipc_close.
 * cign_halo_push: for flat row k < total of the send list (peer p owns rows
 * peer_begin[p] .. peer_begin[p+1]-1; peer_begin is a device array of
 * n_peers+1 entries), copy row idx[k] of src (row k when idx is NULL) to
 * peer_dst[p] + (k - peer_begin[p]) * F -- peer_dst is a device array of
 * n_peers (usually IPC-mapped) pointers.  F % 4 == 0, 16-byte aligned rows.
 * order (device, optional): the rows are copied in the sequence order[0..total)
 * -- a sequence that interleaves the peers spreads the stores over every
 * peer's links at once. 
 * The copies are ordinary stores; order them against the readers with a
 * collective (or event) after the launch. */
#define CIGN_IPC_HANDLE_BYTES 64
CIGN_API int cign_device_alloc(size_t bytes, void** ptr);
CIGN_API int cign_device_free(void* ptr);
CIGN_API int cign_ipc_handle(const void* ptr, void* handle);
CIGN_API int cign_ipc_open(const void* handle, void** ptr);
CIGN_API int cign_ipc_close(void* ptr);
CIGN_API int cign_halo_push(int32_t n_peers, const float* src, int64_t F, const int64_t* idx,
                            const int64_t* peer_begin, float* const* peer_dst, int64_t total,
                            const int64_t* order, cign_stream_t stream);
/* The same copies by the copy engines: with idx, the send rows are first
 * gathered into `staging` (this GPU's memory, total * F floats); then each
 * peer's contiguous block goes to peer_dst_host[p] as one cudaMemcpyAsync
 * on `stream`, peers in turn from first_peer.  peer_begin_host / peer_dst_host
 * are HOST arrays here.  No SM time is spent on the transfer itself. */
CIGN_API int cign_halo_push_copy(int32_t n_peers, const float* src, int64_t F,
                                 const int64_t* idx, const int64_t* peer_begin_host,
                                 float* const* peer_dst_host, int64_t total, float* staging,
                                 int32_t first_peer, cign_stream_t stream);

/* ------------------------------------------------------------ column sum
 * out[j] = sum_i a[i, j] for a row-major [n, c] matrix, in a fixed order
 * (two stages: fixed 128-row chunks, then the chunk partials) -- the bias
 * gradient of a linear layer, which the reference leaves to autograd's
 * grad.sum(0) (e.g. the proj and input linears, generic_engine/
 * model_cign.py:700-704).  ws: cign_colsum_workspace_bytes(n, c) bytes. */
CIGN_API size_t cign_colsum_workspace_bytes(int64_t n, int64_t c);
CIGN_API int cign_colsum_f32(int64_t n, int64_t c, const float* a, float* out, void* ws,
                             size_t ws_bytes, cign_stream_t stream);

/* ------------------------------------------------------------ seed table
 * Device-side dropout seed streams for CUDA-graph training steps.  For slot
 * i < n_slots with layout[3i..3i+2] = (kind, tag, offset):
 *   kind 0 (GAT):   table[i] = (base + 0x9E3779B97F4A7C15 * (counters[0] + offset + 1)) mod 2^63
 *   kind 1 (block): table[i] = (base + 0x9E3779B97F4A7C15 * (counters[1] + offset + 1)
 *                               + 0xD2B74407B1CE6E93 * tag) mod 2^63
 * then counters[0] += n_gat, counters[1] += n_block -- the per-call seeds of
 * collapsed_gat.py:201-211 and fused_block_ops.py:46-50 with the call
 * counters kept on the device.  layout, counters (int64 [2]) and table
 * (uint64 [n_slots]) are device arrays; n_slots <= 4096. */
CIGN_API int cign_seed_table_step(uint64_t base, int32_t n_slots, const int32_t* layout,
                                  int64_t* counters, int32_t n_gat, int32_t n_block,
                                  uint64_t* table, cign_stream_t stream);

/* ------------------------------------------------------------ hop gate
 * alpha [N,K] = softmax_k(g @ W^T + b) with g = [H + C | |H - C|] (mode 1,
 * alpha_score_mode "new") or [H | C] (mode 0, "old"); H, C [N,D], W [K,2D],
 * b [K], 1 <= K <= 8, D a multiple of 4, H/C/W 16-byte aligned.  The gate
 * input is never materialised and the linear runs in fp32.
 * Replaces GraphCliffordBlock.compute_hop_gate (generic_engine/
 * model_cign.py:721-749: torch.cat + abs + nn.Linear + softmax). */
CIGN_API int cign_hop_gate_fwd(int64_t n, int64_t d, int32_t k, int32_t mode, const float* h,
                               const float* c, const float* w, const float* b, float* alpha,
                               cign_stream_t stream);
CIGN_API size_t cign_hop_gate_bwd_workspace_bytes(int64_t n, int64_t d, int32_t k);
/* Backward: grad_h, grad_c [N,D], grad_w [K,2D], grad_b [K] (fixed-order
 * sums: deterministic); sign(0) = 0 for |H - C|.  grad_h/grad_c receive
 * (accumulate ? their current value : 0) + add_h/add_c rows (row stride
 * add_ld floats; either may be NULL) + this op's gradient, so callers can
 * merge the other consumers' gradients of H and C into the same pass. */
CIGN_API int cign_hop_gate_bwd(int64_t n, int64_t d, int32_t k, int32_t mode, const float* h,
                               const float* c, const float* w, const float* alpha,
                               const float* grad_alpha, float* grad_h, float* grad_c,
                               float* grad_w, float* grad_b, int32_t accumulate,
                               const float* add_h, const float* add_c, int64_t add_ld, void* ws,
                               size_t ws_bytes, cign_stream_t stream);

/* ------------------------------------------------------------ block ops
 * Row LayerNorm over D with biased variance and rsqrt(var + eps); optional
 * dropout (keep iff (splitmix64(seed ^ idx*0xD2B74407B1CE6E93) >> 11) * 2^-53
 * >= p, idx = n*D + d) applied to x before the norm.  Masks are recomputed
 * in backward from (seed, idx), never stored.
 * Replaces the kernels of fused_block_ops.py:15 and fused_block_ops_ext/
 * fused_block_ops_cuda.cu:45-322 without their D<=256 limit. */
CIGN_API int cign_dropout_ln_fwd(int64_t n, int64_t d, const float* x, const float* w,
                        const float* b, float p, float eps, uint64_t seed,
                              const uint64_t* seed_ptr,
                        float* y, float* mean, float* rstd,
                        cign_stream_t stream);

CIGN_API size_t cign_ln_bwd_workspace_bytes(int64_t n, int64_t d);

CIGN_API int cign_dropout_ln_bwd(int64_t n, int64_t d, const float* grad_y,
                        const float* x, const float* w, const float* mean,
                        const float* rstd, float p, uint64_t seed,
                              const uint64_t* seed_ptr,
                        float* grad_x, float* grad_w, float* grad_b, void* ws,
                        size_t ws_bytes, cign_stream_t stream);

/* cign_dropout_ln_bwd with the gradient of a second consumer of x added:
 * grad_x = d LN(dropout(x)) / dx + addend (addend [n, d], not aliasing
 * grad_x).  A CIGN block's input H feeds both its dropout-LayerNorm and its
 * residual (model_cign.py:781 and :929); this writes H's whole gradient in
 * the LayerNorm backward's own pass instead of a separate add. */
CIGN_API int cign_dropout_ln_bwd_add(int64_t n, int64_t d, const float* grad_y,
                        const float* x, const float* w, const float* mean,
                        const float* rstd, float p, uint64_t seed,
                              const uint64_t* seed_ptr, const float* addend,
                        float* grad_x, float* grad_w, float* grad_b, void* ws,
                        size_t ws_bytes, cign_stream_t stream);

/* Allocation-free variant of cign_dropout_ln_bwd (this entry point has no
 * counterpart in the reference).  For callers that cannot allocate device
 * memory -- e.g. a plugin inside a host framework that owns all device memory
 * through its own pool and passes kernels only their inputs and outputs --
 * the reduction scratch is a fixed 3.5 MiB array inside the library (444 row
 * chunks x 1024 columns x 2 floats), held on every GPU that loads the
 * library until the process exits.  Limit: D <= 1024 (the same as the
 * workspace version); larger shapes return CIGN_ERR_UNSUPPORTED.  No
 * cudaMalloc/cudaFree is called.  All calls share the array: calls that
 * overlap on the GPU (other streams or threads) race; order them on one
 * stream.  The first call on each device looks up the array's device
 * address with that device current; make that first call before any stream
 * capture.  The dropout seed is a host value only (there is no device seed
 * slot): a captured graph replaying this call applies the same mask on every
 * replay. */
CIGN_API int cign_dropout_ln_bwd_static(int64_t n, int64_t d, const float* grad_y,
                               const float* x, const float* w,
                               const float* mean, const float* rstd, float p,
                               uint64_t seed, float* grad_x, float* grad_w,
                               float* grad_b, cign_stream_t stream);

/* y = LayerNorm(a + b). */
CIGN_API int cign_add_ln_fwd(int64_t n, int64_t d, const float* a, const float* b,
                    const float* w, const float* bias, float eps, float* y,
                    float* mean, float* rstd, cign_stream_t stream);

/* grad_z = d LN / d(a+b); the caller uses it for both a and b. */
CIGN_API int cign_add_ln_bwd(int64_t n, int64_t d, const float* grad_y, const float* a,
                    const float* b, const float* w, const float* mean,
                    const float* rstd, float* grad_z, float* grad_w,
                    float* grad_b, void* ws, size_t ws_bytes,
                    cign_stream_t stream);

/* GAT side ops and the block's add-LayerNorm in one pass (replaces the
 * head-mean + bias + SiLU epilogue of collapsed_gat_cuda.cu:167-173 followed by
 * fused_add_layernorm, fused_block_ops.py:112 / model_cign.py:767-787):
 *   pre = lin + bias;  y = LayerNorm(SiLU(pre) + h) * w + b.
 * lin [n,d] is the head-mean GAT output before its bias; writes pre, y and
 * the row mean / rstd; SiLU(pre) itself is not stored. */
CIGN_API int cign_silu_add_ln_fwd(int64_t n, int64_t d, const float* lin, const float* bias,
                         const float* h, const float* w, const float* b, float eps,
                         float* pre, float* y, float* mean, float* rstd,
                         cign_stream_t stream);
CIGN_API size_t cign_silu_add_ln_bwd_workspace_bytes(int64_t n, int64_t d);
/* Backward of cign_silu_add_ln_fwd: grad_z = d LN / d(SiLU(pre) + h) (the
 * gradient of h), grad_pre = grad_z * SiLU'(pre) (the gradient of lin), and
 * the LN weight / bias and GAT bias gradients (fixed-order sums).  With
 * accumulate_z != 0, grad_z is added to what grad_z holds (h's gradient from
 * its other consumers) instead of overwriting it. */
CIGN_API int cign_silu_add_ln_bwd(int64_t n, int64_t d, const float* grad_y, const float* pre,
                         const float* h, const float* w, const float* mean,
                         const float* rstd, int accumulate_z, float* grad_z, float* grad_pre,
                         float* grad_w, float* grad_b, float* grad_bias, void* ws,
                         size_t ws_bytes, cign_stream_t stream);

/* y = h + gamma * dropout(g). */
CIGN_API int cign_gamma_residual_fwd(int64_t n, int64_t d, const float* h,
                            const float* g, const float* gamma, float p,
                            uint64_t seed,
                              const uint64_t* seed_ptr, float* y, cign_stream_t stream);

CIGN_API size_t cign_gamma_residual_bwd_workspace_bytes(int64_t n, int64_t d);

/* grad_g = grad_y * gamma * mask/(1-p);  grad_gamma = sum_n grad_y * g * mask/(1-p).
 * (grad_h = grad_y is returned by the caller without a kernel.) */
CIGN_API int cign_gamma_residual_bwd(int64_t n, int64_t d, const float* grad_y,
                            const float* g, const float* gamma, float p,
                            uint64_t seed,
                              const uint64_t* seed_ptr, float* grad_g, float* grad_gamma,
                            void* ws, size_t ws_bytes, cign_stream_t stream);

/* Materialise the block-op dropout keep-mask (uint8 [count]) for indices
 * 0..count-1, for parity checks only. */
CIGN_API int cign_block_dropout_mask(int64_t count, float p, uint64_t seed,
                              const uint64_t* seed_ptr,
                            uint8_t* mask, cign_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* CIGN_SM100_H */
