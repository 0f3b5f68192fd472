/*
 * hrm_moe.h -- C ABI of the B200-native routed MoE-FFN forward.
 *
 * Drop-in for the grouped expert path of XiaoYee/HRM-MoE
 * (models/layers.py SparseMoESwiGLU / SparseMoEGroupedExperts and
 * models/moe_triton_grouped_gemm.py triton_grouped_linear).  Every entry
 * point takes plain device pointers and sizes, runs stream-ordered on the
 * given cudaStream_t (passed as void*; NULL = legacy default stream) and
 * never synchronises the host.  Buffers are owned by the caller.  Scratch
 * memory comes from a caller-owned workspace whose size the matching
 * *_workspace_bytes() function returns; one call may be in flight per
 * workspace at a time.
 *
 * Layouts (row-major, contiguous):
 *   x           [T, d]       hidden states, layer dtype
 *   w_router    [E, d]       gate.weight            (layers.py:548)
 *   router_bias [E]          gate.bias or NULL, layer dtype
 *   w_gate_up   [E, 2I, d]   experts.gate_up_weight (layers.py:272-277);
 *                            rows 0..I-1 gate, I..2I-1 up (layers.py:328)
 *   w_down      [E, d, I]    experts.down_weight    (layers.py:278-283)
 *   topk_idx    [T, k]       int32 expert ids
 *   topk_weight [T, k]       layer dtype
 *   counts      [E]          int32 tokens_per_expert
 *   sort_idx    [T*k]        int32; position p holds the flat index t*k+j of
 *                            the p-th assignment in stable expert order
 *                            (torch.sort(flat, stable=True), layers.py:317)
 *
 * Status codes are errno values; hmoe_last_error() describes the last
 * failure on the calling thread.  A call with tokens == 0 launches nothing;
 * where it has a counts output, it writes E zeros there (the reference's
 * bincount(..., minlength=E)).
 */
#ifndef HRM_MOE_H
#define HRM_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HMOE_OK 0
#define HMOE_EIO 5          /* CUDA runtime error */
#define HMOE_EINVAL 22      /* bad shape, dtype or pointer */
#define HMOE_ENOSPC 28      /* workspace too small */
#define HMOE_ENOSYS 38      /* device is not an sm_100 GPU */
#define HMOE_ETIMEDOUT 110  /* a bounded device-side wait gave up */

#define HMOE_DTYPE_BF16 0
#define HMOE_DTYPE_F32 1

typedef struct hmoe_shape {
  int64_t tokens;          /* T */
  int32_t hidden;          /* d, multiple of 8 */
  int32_t experts;         /* E, 1..128 */
  int32_t intermediate;    /* I, multiple of 8 */
  int32_t top_k;           /* k, 1..min(E, 32) */
  int32_t dtype;           /* HMOE_DTYPE_* : hidden / weight / output dtype */
  int32_t norm_topk_prob;  /* renormalise the top-k probabilities */
} hmoe_shape;

/* Library identification, and the message of the last failing call. */
const char* hmoe_version(void);
const char* hmoe_last_error(void);

/*
 * Whole layer: SparseMoESwiGLU.forward (models/layers.py:596-634) without
 * the training-only aux-loss block (layers.py:619-632).
 *   y = [y +] sum_j w[t,j] * SwiGLU_{idx[t,j]}(x[t])
 * accumulate = 0 writes y; 1 adds into it (the reference adds into a zeros
 * accumulator, layers.py:612-617).  topk_idx / topk_weight / counts /
 * sort_idx are optional outputs (NULL = not written).
 */
size_t hmoe_ffn_workspace_bytes(const hmoe_shape* shape);
int hmoe_ffn_forward(const hmoe_shape* shape, const void* x, const void* w_router,
                     const void* router_bias, const void* w_gate_up, const void* w_down,
                     void* y, int accumulate, int32_t* topk_idx, void* topk_weight,
                     int32_t* counts, int32_t* sort_idx, void* workspace,
                     size_t workspace_bytes, void* stream);

/*
 * hmoe_ffn_forward on HOST buffers: x_host [T, d] in, y_host [T, d] out
 * (pinned host memory lets the copies overlap), weights on the device.  The
 * tokens go through in chunks of chunk_tokens: the copy of chunk c+1 in, the
 * layer on chunk c and the copy of chunk c-1 out run at the same time on two
 * internal copy streams and `stream`, ordered by events; the call is
 * complete when `stream` reaches its end.  Calls on one device must not
 * overlap (the copy streams and events are per device).  Workspace:
 * hmoe_ffn_host_workspace_bytes(shape, chunk_tokens).
 */
size_t hmoe_ffn_host_workspace_bytes(const hmoe_shape* shape, int64_t chunk_tokens);
int hmoe_ffn_forward_host(const hmoe_shape* shape, const void* x_host, const void* w_router,
                          const void* router_bias, const void* w_gate_up, const void* w_down,
                          void* y_host, int64_t chunk_tokens, void* workspace,
                          size_t workspace_bytes, void* stream);

/*
 * hmoe_ffn_forward with timing marks: phase_events points to 6 cudaEvent_t
 * (NULL entries skipped) recorded on the stream before the router, after
 * the router, after dispatch, after the gate_up GEMM, after the down GEMM
 * and after the combine.  Same kernels, same results.  Under stream
 * capture the marks become event-record nodes of the graph, recorded by
 * every replay.
 */
int hmoe_ffn_forward_marked(const hmoe_shape* shape, const void* x, const void* w_router,
                            const void* router_bias, const void* w_gate_up, const void* w_down,
                            void* y, int accumulate, void* workspace, size_t workspace_bytes,
                            void* stream, void* const* phase_events);

/*
 * Router: self.gate + fp32 softmax + top-k + renormalise + cast
 * (models/layers.py:604-610).  The routing is that of logits accumulated in
 * fp32 in a fixed order (one fma per k, ascending, from +0) plus the bias and
 * rounded to the layer dtype, as the reference's F.linear output is;
 * selection takes the k largest logits, equal logits going to the lower
 * expert index.  bf16 layers compute the logits on the tensor cores and
 * recompute, in the fixed order, every token whose top-k the tensor-core
 * sums cannot certify, so the result is the same.  logits (optional, [T, E],
 * layer dtype) returns the rounded logits the routing used.
 */
size_t hmoe_router_workspace_bytes(const hmoe_shape* shape);
int hmoe_router_topk(const hmoe_shape* shape, const void* x, const void* w_router,
                     const void* router_bias, int32_t* topk_idx, void* topk_weight,
                     void* logits, void* workspace, size_t workspace_bytes, void* stream);

/*
 * hmoe_router_topk (bf16 layers) that also writes `sums` [T, E] fp32: the
 * tensor-core sums of x . w_router^T (before the bias) from which the router
 * certifies its top-k against the fixed-order definition.  No counterpart in
 * the reference: a diagnostic that lets a test measure how far those sums
 * are from the fixed-order sums, next to the certification margin.  Same
 * routing and workspace as hmoe_router_topk.
 */
int hmoe_router_topk_sums(const hmoe_shape* shape, const void* x, const void* w_router,
                          const void* router_bias, int32_t* topk_idx, void* topk_weight,
                          void* logits, float* sums, void* workspace, size_t workspace_bytes,
                          void* stream);

/*
 * Dispatch: flatten, stable sort by expert, gather rows, count
 * (models/layers.py:311-322).  Writes sort_idx [T*k], counts [E] and, when
 * non-NULL, sorted_token [T*k] (int32), sorted_weight [T*k] (layer dtype)
 * and x_sorted [T*k, d].  Deterministic, no atomics on positions.
 */
size_t hmoe_dispatch_workspace_bytes(const hmoe_shape* shape);
int hmoe_dispatch(const hmoe_shape* shape, const int32_t* topk_idx,
                  const void* topk_weight, const void* x, int32_t* sort_idx,
                  int32_t* counts, int32_t* sorted_token, void* sorted_weight,
                  void* x_sorted, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Experts: SparseMoEGroupedExperts.forward (models/layers.py:285-335) --
 * dispatch, gate_up GEMM + SiLU(gate)*up, down GEMM, weighted combine into
 * final_hidden_states (accumulated in place, like the reference's
 * index_add_).  topk_idx is int32 here; ids outside [0, E) are dropped.
 */
size_t hmoe_experts_workspace_bytes(const hmoe_shape* shape);
int hmoe_experts_forward(const hmoe_shape* shape, const void* hidden,
                         const int32_t* topk_idx, const void* topk_weight,
                         const void* w_gate_up, const void* w_down,
                         void* final_hidden_states, int32_t* counts, int32_t* sort_idx,
                         void* workspace, size_t workspace_bytes, void* stream);

/*
 * Grouped GEMM: triton_grouped_linear(input, weight, tokens_per_expert)
 * (models/moe_triton_grouped_gemm.py:478-485, kernel :113-184):
 *   output[rows of group g] = input[rows of group g] @ weight[g]^T
 * input [M, K], weight [G, N, K], output [M, N], tokens_per_expert [G]
 * int32 on the device, groups contiguous in row order.  bf16 runs on the
 * tcgen05 tensor cores, fp32 on CUDA cores.  K and N multiples of 8.
 */
size_t hmoe_grouped_linear_workspace_bytes(int32_t groups);
int hmoe_grouped_linear(const void* input, const void* weight,
                        const int32_t* tokens_per_expert, int64_t M, int32_t N,
                        int32_t K, int32_t groups, int32_t dtype, void* output,
                        void* workspace, size_t workspace_bytes, void* stream);

/*
 * Fused gate_up GEMM + activation (models/layers.py:326-329):
 *   gate_up = grouped_linear(input, w_gate_up, tokens_per_expert)  [M, 2I]
 *   output  = silu(gate_up[:, :I]) * gate_up[:, I:]                 [M, I]
 * with the bf16 roundings of the reference's intermediate tensors applied
 * in the epilogue.  w_gate_up [G, 2I, K].
 */
int hmoe_grouped_swiglu(const void* input, const void* w_gate_up,
                        const int32_t* tokens_per_expert, int64_t M, int32_t I,
                        int32_t K, int32_t groups, int32_t dtype, void* output,
                        void* workspace, size_t workspace_bytes, void* stream);

/*
 * Backward of hmoe_grouped_linear: _TritonGroupedLinear.backward
 * (models/moe_triton_grouped_gemm.py:427-456), for output = input @ W[g]^T
 * with weight [G, N, K] and grad_out [M, N]:
 *   grad_input  [M, K]    = grad_out[rows of g] @ W[g]
 *                           (_m_grouped_gemm(trans_b=False), :358-417, kernel :187-260)
 *   grad_weight [G, N, K] = grad_out[rows of g]^T @ input[rows of g]
 *                           (_k_grouped_gemm, :350-..., kernel :277-347)
 * fp32 accumulation on the tcgen05 tensor cores, one rounding to bf16; a
 * group without rows gets a zero weight gradient.  bf16 only: fp32 is
 * refused with HMOE_EINVAL, as the reference's Triton path raises TypeError
 * for it (:350-355).  Either output may be NULL (not computed).  K and N
 * multiples of 8.  Workspace: hmoe_grouped_linear_workspace_bytes (the
 * device error word).
 */
int hmoe_grouped_linear_backward(const void* grad_out, const void* input, const void* weight,
                                 const int32_t* tokens_per_expert, int64_t M, int32_t N,
                                 int32_t K, int32_t groups, int32_t dtype, void* grad_input,
                                 void* grad_weight, void* workspace, size_t workspace_bytes,
                                 void* stream);

/*
 * Backward through the down projection and SiLU(gate) * up
 * (models/layers.py:327-331) in one GEMM: with h = silu(gate) * up and
 * expert_out = h @ w_down[g]^T, given grad_out = d(expert_out) [M, d],
 *   dh     = grad_out @ w_down[g]                    (rounded to bf16)
 *   d_up   = dh * bf16(silu(gate)),  d_sg = dh * up  (each rounded)
 *   d_gate = d_sg * s * (1 + gate * (1 - s)),  s = sigmoid(gate)
 * written as d_gate_up [M, 2I] (gate half, then up half), from the saved
 * gate_up [M, 2I] of the forward.  w_down [G, d, I].  bf16 only.
 */
int hmoe_grouped_swiglu_backward(const void* grad_out, const void* w_down,
                                 const void* gate_up, const int32_t* tokens_per_expert,
                                 int64_t M, int32_t d, int32_t I, int32_t groups,
                                 void* d_gate_up, void* workspace, size_t workspace_bytes,
                                 void* stream);

/*
 * Grouped GEMM over groups that reuse weights: group g (group_rows[g] rows,
 * contiguous in order) is multiplied by weight[group_weight[g]] (of
 * num_weights).  swiglu = 0: output [M, N] = rows @ W^T with W [N, K];
 * swiglu = 1: the fused gate_up + SiLU*up with W [2N, K], output [M, N].
 * This is the local expert computation of the expert-parallel backend
 * (models/layers.py:462-468), where the received rows arrive grouped by
 * (source rank, local expert) (layers.py:456-460).
 */
int hmoe_grouped_gemm_mapped(const void* input, const void* weight, const int32_t* group_rows,
                             const int32_t* group_weight, int64_t M, int32_t N, int32_t K,
                             int32_t groups, int32_t num_weights, int32_t dtype, int32_t swiglu,
                             void* output, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Combine (models/layers.py:332-334): for every token t,
 *   final[t] += sum_j topk_weight[t, j] * expert_out[pos(t, j)]
 * where pos is the inverse of sort_idx (sort_idx[pos(t,j)] = t*k + j).
 * Accumulates in fp32 and rounds once per output element.
 */
size_t hmoe_combine_workspace_bytes(const hmoe_shape* shape);
int hmoe_combine(const hmoe_shape* shape, const void* expert_out, const int32_t* sort_idx,
                 const void* topk_weight, void* final_hidden_states, void* workspace,
                 size_t workspace_bytes, void* stream);

/*
 * hmoe_dispatch without a workspace.  No counterpart in the reference: it
 * exists for hosts that cannot give this library device memory for scratch
 * (a plugin host with no CUDA allocator binding, a process whose device
 * memory another framework has reserved up front, a serving loop that must
 * not allocate after start-up).  Same inputs and outputs as hmoe_dispatch,
 * and the same results while every expert id is in [0, E); the scratch
 * lives in one fixed __device__ array of about 2.3 MiB that every GPU
 * loading the library keeps until exit.  At most
 * HMOE_DISPATCH_NOALLOC_MAX_ASSIGNMENTS assignments (tokens * top_k) per
 * call; larger calls fail with HMOE_EINVAL.  The first call in each CUDA
 * context looks up the array's device address there and caches it per
 * context (make that call before any stream capture).  Calls share the
 * array: two calls that overlap on the GPU race.  Expert ids outside [0, E)
 * are dropped without an error report (there is no error word): counts
 * leave them out, and only the first sum(counts) entries of sort_idx,
 * sorted_token, sorted_weight and x_sorted are written.  Allocates nothing.
 */
#define HMOE_DISPATCH_NOALLOC_MAX_ASSIGNMENTS 262144
int hmoe_dispatch_noalloc(const hmoe_shape* shape, const int32_t* topk_idx,
                          const void* topk_weight, const void* x, int32_t* sort_idx,
                          int32_t* counts, int32_t* sorted_token, void* sorted_weight,
                          void* x_sorted, void* stream);

/*
 * Expert parallelism over peer memory: SparseMoEExpertParallel.forward
 * (models/layers.py:427-478) without host-driven all_to_all.  Every rank of
 * a job holds one symmetric region (same size on all ranks) that all ranks
 * map by CUDA IPC; rank r owns experts [r*E/R, (r+1)*E/R) and passes only its
 * own experts' weights (w_gate_up_local [E/R, 2I, d], w_down_local
 * [E/R, d, I]).  The kernels exchange per-expert counts through the regions,
 * store each routed row straight into its owner's region over NVLink, run the
 * owner's grouped GEMMs there, copy the results back to their sources and
 * combine in token order; the result equals one GPU running all experts.
 * All ranks call hmoe_ep_forward in lockstep with the same, strictly
 * increasing epoch; every cross-GPU wait is bounded (HMOE_ETIMEDOUT in the
 * workspace error word).  max_tokens bounds any rank's token count.
 *
 * Set-up: hmoe_ep_symmetric_alloc (cudaMalloc + zero; writes a handle of
 * HMOE_EP_HANDLE_BYTES: the CUDA IPC handle and the owning GPU's UUID),
 * exchange the handles (any transport), hmoe_ep_symmetric_open each peer's.
 * Every rank needs its own GPU: open refuses a region of the calling GPU.
 */
#define HMOE_EP_HANDLE_BYTES 80
size_t hmoe_ep_symmetric_bytes(const hmoe_shape* shape, int64_t max_tokens, int32_t world);
size_t hmoe_ep_workspace_bytes(const hmoe_shape* shape, int64_t max_tokens, int32_t world);
int hmoe_ep_symmetric_alloc(size_t bytes, void** ptr, void* handle);
int hmoe_ep_symmetric_open(const void* handle, void** peer_ptr);
int hmoe_ep_symmetric_close(void* peer_ptr);
int hmoe_ep_symmetric_free(void* ptr);
int hmoe_ep_forward(const hmoe_shape* shape, int64_t max_tokens, int32_t rank, int32_t world,
                    void* const* peer_bases, uint32_t epoch, const void* x, const void* w_router,
                    const void* router_bias, const void* w_gate_up_local,
                    const void* w_down_local, void* y, void* workspace, size_t workspace_bytes,
                    void* stream);
/*
 * hmoe_ep_forward that also records six caller-owned cudaEvent_t on the
 * stream.  bf16: before the router, after the router and the index-only
 * dispatch, after the count exchange, after the gate_up GEMM (whose sender
 * warps push the rows to their owners while it runs), after the down GEMM
 * has stored every result back at its source, and after the combine.  fp32:
 * before the router, after the count exchange, after every peer's rows have
 * landed, after the gate_up GEMM, after the results are back, and after the
 * combine.  Same kernels, same results.
 */
int hmoe_ep_forward_marked(const hmoe_shape* shape, int64_t max_tokens, int32_t rank,
                           int32_t world, void* const* peer_bases, uint32_t epoch, const void* x,
                           const void* w_router, const void* router_bias,
                           const void* w_gate_up_local, const void* w_down_local, void* y,
                           void* workspace, size_t workspace_bytes, void* stream,
                           void* const* phase_events);

/*
 * Training: the layer forward that keeps what its backward needs, and the
 * backward of SparseMoESwiGLU.forward (models/layers.py:596-634) with the
 * aux load-balancing loss (layers.py:163-170, 619-632): the gradients
 * autograd computes through the reference with the grouped expert backend
 * (the grouped GEMMs' backward is _TritonGroupedLinear.backward,
 * models/moe_triton_grouped_gemm.py:420-456).  bf16 only, experts a
 * multiple of 8.
 *
 * hmoe_ffn_forward_train computes y as hmoe_ffn_forward does (same kernels,
 * same bits) and fills `saved` (hmoe_ffn_train_saved_bytes: router logits,
 * routing, positions, counts, the gathered rows, the gate_up, SiLU*up and
 * expert outputs) for hmoe_ffn_backward.  aux_tokens >= 0 also computes, over
 * the first aux_tokens tokens (the reference's total_seqlen, layers.py:
 * 620-626), the aux loss (aux_loss, device fp32 scalar, may be NULL) and the
 * expert selection counts (expert_counts, device fp32 [E], may be NULL):
 * the values the reference appends to moe_context.  Negative: no aux.
 *
 * hmoe_ffn_backward: given grad_y [T, d] and, when the aux loss was part of
 * the loss, aux_grad (device fp32 scalar, its gradient; NULL = none) with the
 * same aux_tokens, writes grad_x [T, d], grad_w_router [E, d],
 * grad_router_bias [E] (only with a router_bias), grad_w_gate_up [E, 2I, d]
 * and grad_w_down [E, d, I], each in bf16, each optional (NULL = not
 * computed).  `saved` must come from the matching forward call, with the same
 * inputs.  Workspace: hmoe_ffn_train_workspace_bytes (also the forward's).
 * Rounding follows the reference's bf16 tensors: every GEMM accumulates in
 * fp32 and rounds once; the SiLU and combine products are rounded as the
 * reference rounds them; a token's d_x sums its rows' gradients in fp32.
 */
size_t hmoe_ffn_train_saved_bytes(const hmoe_shape* shape);
size_t hmoe_ffn_train_workspace_bytes(const hmoe_shape* shape);
int hmoe_ffn_forward_train(const hmoe_shape* shape, const void* x, const void* w_router,
                           const void* router_bias, const void* w_gate_up, const void* w_down,
                           void* y, int64_t aux_tokens, float* aux_loss, float* expert_counts,
                           void* saved, size_t saved_bytes, void* workspace,
                           size_t workspace_bytes, void* stream);
int hmoe_ffn_backward(const hmoe_shape* shape, const void* grad_y, const float* aux_grad,
                      int64_t aux_tokens, const void* x, const void* w_router,
                      const void* router_bias, const void* w_gate_up, const void* w_down,
                      const void* saved, size_t saved_bytes, void* grad_x, void* grad_w_router,
                      void* grad_router_bias, void* grad_w_gate_up, void* grad_w_down,
                      void* workspace, size_t workspace_bytes, void* stream);

/*
 * hmoe_ffn_backward that also records 8 caller-owned cudaEvent_t (NULL
 * entries skipped) on the stream: at the start, after the combine/router
 * backward, after the down projection's dgrad (with the SiLU backward), after
 * its wgrad, after the gate_up dgrad, after its wgrad, after the router dgrad
 * and the d_x gather, and at the end (router wgrad and bias).  Same kernels,
 * same results.
 */
int hmoe_ffn_backward_marked(const hmoe_shape* shape, const void* grad_y, const float* aux_grad,
                             int64_t aux_tokens, const void* x, const void* w_router,
                             const void* router_bias, const void* w_gate_up, const void* w_down,
                             const void* saved, size_t saved_bytes, void* grad_x,
                             void* grad_w_router, void* grad_router_bias, void* grad_w_gate_up,
                             void* grad_w_down, void* workspace, size_t workspace_bytes,
                             void* stream, void* const* phase_events);

/*
 * Read (and synchronise the stream for) the error word kernels leave at the
 * start of a workspace used by hmoe_ffn_forward, hmoe_experts_forward,
 * hmoe_dispatch, hmoe_grouped_* or hmoe_ep_forward: HMOE_OK, HMOE_EINVAL (an
 * expert id was outside [0, E) and was dropped), HMOE_ETIMEDOUT, or HMOE_EIO
 * (expert-parallel counts beyond the symmetric buffers).  Not for hot loops.
 */
int hmoe_workspace_status(const void* workspace, void* stream);

/*
 * Programmatic dependent launch: the classes of the layer's forward kernels
 * (1 router pass, 2 dispatch, 4 grouped GEMMs, 8 combine) launched so that
 * their launch and on-chip setup overlap the tail of the kernel before them
 * (each still waits for that kernel's results before touching memory).
 * The environment variable HMOE_PDL gives the initial mask (default 7:
 * every class but the combine).
 * Affects launches made after the call; a captured CUDA graph keeps the
 * launches it was captured with.  Returns the previous mask.
 */
unsigned hmoe_set_pdl_mask(unsigned mask);

#ifdef __cplusplus
}
#endif

#endif /* HRM_MOE_H */
