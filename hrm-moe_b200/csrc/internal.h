// Host-side launchers shared between the kernel files and the C ABI.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <utility>

struct hmoe_shape;  // include/hrm_moe.h

namespace hmoe {

// Programmatic dependent launch for the layer's forward kernels (router pair
// pass, hist_rank, scan, permute_gather, the grouped GEMMs, combine): the
// grid may be scheduled while the kernel before it in the stream is still
// running.  Every kernel launched this way calls grid_dependency_wait()
// before its first global-memory access and grid_launch_dependents() only
// after it, so at most two grids are in flight and only the launch and the
// on-chip setup (barriers, TMEM, descriptor prefetch) overlap the previous
// kernel.  HMOE_PDL (read once per process; hmoe_set_pdl_mask changes it) is
// a mask of the kernel classes launched this way, default router, dispatch
// and GEMMs.  Measured on B200 (XL layer, one CUDA graph, replays
// interleaved in one process): 93.8 -> 91.3 us at T=64, neutral at
// T=16384.  The combine is left out by default: its CTAs, resident early
// next to the down GEMM, made T=16384 15 us slower.
enum PdlClass : unsigned { kPdlRouter = 1, kPdlDispatch = 2, kPdlGemm = 4, kPdlCombine = 8 };
bool pdl_enabled(unsigned cls);
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(unsigned cls, void (*kernel)(KArgs...), dim3 grid, dim3 block,
                       size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled(cls) ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  return e != cudaSuccess ? e : cudaGetLastError();
}

// router.cu -------------------------------------------------------------
// topk_w_f32: fp32 copy of the routing weights (rounded to the layer dtype).
cudaError_t launch_router_topk(const void* x, const void* w_router, const void* bias,
                               int64_t T, int d, int E, int k, int dtype, int norm,
                               int32_t* topk_idx, float* topk_w_f32, void* topk_w_dtype,
                               void* logits_out, cudaStream_t stream);

// router_tc.cu (bf16 only) -----------------------------------------------
// Relative margin (of the token's largest |logit|) inside which a tensor-core
// sum is treated as possibly rounding differently from the exact-order sum.
// Measured on B200 over nine shapes and value scales, the largest
// |tensor-core sum - exact-order sum| was 0.13 of this margin (0.033 of a
// four times wider one); tests/test_gpu_10_certification.py keeps it below
// a quarter.
constexpr float kRouterCertRel = 1.0f / 65536.0f;
size_t router_tc_scratch_bytes(int64_t T);
// sums_out (optional, diagnostic): the fp32 tensor-core sums [T, E] before
// the bias, as the certification sees them.  reset_err: clear *err first
// (the pair pass does it in the kernel, saving the memset in front of it).
cudaError_t launch_router_topk_tc(const void* x, const void* w_router, const void* bias,
                                  int64_t T, int d, int E, int k, int norm, int32_t* topk_idx,
                                  float* topk_w_f32, void* topk_w_dtype, void* logits_out,
                                  void* scratch, int* err, cudaStream_t stream,
                                  float* sums_out = nullptr, bool reset_err = false);

// dispatch.cu -----------------------------------------------------------
// Tokens per histogram block for a given top_k.
int dispatch_block_tokens(int k);
int64_t dispatch_num_blocks(int64_t T, int k);

// local_rank[T*k], block_counts[nblk*E] (turned into block offsets by scan).
cudaError_t launch_hist_rank(const int32_t* topk_idx, int64_t T, int k, int E,
                             int32_t* local_rank, int32_t* block_counts, int* err,
                             cudaStream_t stream);
// In place: block_counts -> row offsets inside each expert; counts[E].
// (expert_offsets is unused and may be null.)
cudaError_t launch_scan(int32_t* block_counts, int64_t nblk, int E, int32_t* counts,
                        int32_t* expert_offsets, cudaStream_t stream);
// hist_rank then scan (the scan is folded into hist_rank when T fits one
// histogram block): local_rank, block offsets and counts[E].
cudaError_t launch_hist_scan(const int32_t* topk_idx, int64_t T, int k, int E,
                             int32_t* local_rank, int32_t* block_counts, int32_t* counts, int* err,
                             cudaStream_t stream);
// True when the T*k assignments fit one histogram block: then
// launch_dispatch_small does all of dispatch in one kernel (counts, pos and
// the optional outputs; no local_rank / block_counts scratch).
bool dispatch_fits_one_block(int64_t T, int k);
cudaError_t launch_dispatch_small(const int32_t* topk_idx, const void* topk_w, int topk_w_is_f32,
                                  const void* x, int64_t T, int d, int k, int E, int dtype,
                                  int32_t* counts, int32_t* pos, int32_t* sort_idx,
                                  int32_t* sorted_token, void* sorted_w, void* x_sorted, int* err,
                                  cudaStream_t stream);
// pos[T*k] and (optionally) sort_idx, sorted_token, sorted weights, x_sorted.
cudaError_t launch_permute_gather(const int32_t* topk_idx, const int32_t* local_rank,
                                  const int32_t* block_offsets, const int32_t* counts,
                                  const void* topk_w,
                                  int topk_w_is_f32, const void* x, int64_t T, int d, int k,
                                  int E, int dtype, int32_t* pos, int32_t* sort_idx,
                                  int32_t* sorted_token, void* sorted_w, void* x_sorted,
                                  cudaStream_t stream);
// pos[sort_idx[p]] = p for p < n.
cudaError_t launch_invert_perm(const int32_t* sort_idx, int64_t n, int32_t* pos,
                               cudaStream_t stream);

// combine.cu ------------------------------------------------------------
cudaError_t launch_combine(const void* expert_out, const int32_t* pos, const void* topk_w,
                           int topk_w_is_f32, const int32_t* topk_idx, int E, int64_t T,
                           int d, int k, int dtype, const void* final_in, void* out,
                           cudaStream_t stream);

// gemm_sm100.cu (bf16, tcgen05) and gemm_simt.cu (fp32) ------------------
struct GroupedGemmArgs {
  const void* a;             // [M, K]
  const void* b;             // [G, Nw, K]  (Nw = 2N for swiglu, N otherwise)
  const int32_t* counts;     // [G] rows per group, device
  const int32_t* group_weight = nullptr;  // [G] weight index per group (null = g)
  int num_weights = 0;       // weights in b (0 = G)
  void* out;                 // [M, N]
  int64_t M;
  int N;                     // output columns
  int K;
  int G;
  int swiglu;                // fused silu(gate) * up epilogue
  int dtype;
  int* err;                  // device error word (may be null)
  int sm_limit;              // persistent CTAs (0 = all SMs)
  // Training forward (CTA-pair SwiGLU kernel only): also store the rounded
  // gate and up values, [M, 2N] (gate columns [0, N), up [N, 2N)).
  void* save_gate_up = nullptr;
  // Expert-parallel return (plain bf16 GEMM only; `out` unused): output row r
  // goes to scatter_base[src] + pos * N elements, where src and pos come from
  // scatter_src[r] = (src << kEpSrcShift) | pos; pos < scatter_cap.  Once every
  // CTA has fenced its stores, the last one to finish sets *flag[i] = epoch
  // for i < scatter_world (unless the error word is set); `done` is a zeroed
  // counter.
  const int32_t* scatter_src = nullptr;
  char* scatter_base[8] = {};
  int scatter_world = 0;
  int64_t scatter_cap = 0;
  unsigned* done = nullptr;
  uint32_t* flag[8] = {};
  uint32_t epoch = 0;
  // Expert-parallel dispatch fused into the (bf16 SwiGLU) GEMM: extra warps
  // copy this rank's routed rows into their owners' receive buffers, in
  // expert-sorted order (push_sorted_token[pos] = token of sorted position
  // pos, push_counts[e] rows of expert e, push_send_base[e] their first row
  // at the owner; -1 = send nothing), each row's origin into push_src, and
  // add each finished run to the owner's push_arrived[local expert].  The
  // GEMM loads a group's tiles only once arrived[g] reaches counts[g].  Set
  // `arrived` to select this mode (push_x may be null when push_A is 0).
  const void* push_x = nullptr;
  const int32_t* push_sorted_token = nullptr;
  const int32_t* push_counts = nullptr;
  const int32_t* push_send_base = nullptr;
  char* push_rows[8] = {};
  int32_t* push_src[8] = {};
  uint32_t* push_arrived[8] = {};
  const uint32_t* arrived = nullptr;
  int64_t push_A = 0;
  int64_t push_cap = 0;
  int push_E = 0, push_El = 0, push_world = 0, push_me = 0;
};
constexpr uint32_t kEpSrcShift = 28;  // row origin = (source rank << 28) | source position
cudaError_t launch_grouped_gemm_sm100(const GroupedGemmArgs& args, cudaStream_t stream);
cudaError_t launch_grouped_gemm_simt(const GroupedGemmArgs& args, cudaStream_t stream);
// bf16, local output only (no scatter / push): CTA pairs, 256-row tiles
cudaError_t launch_grouped_gemm_pair(const GroupedGemmArgs& args, cudaStream_t stream);

// gemm_sm100_bwd.cu (bf16, tcgen05): backward of the grouped linear ---------
// dgrad: out[r, :] = grad_out[r, :Kc] @ weight[g] with weight [G][Kc][Nout]
// (the grouped linear's own [G, N, K] weight, contracted over N).  With
// gate_up set, the epilogue is the SiLU(gate) * up backward instead: the
// product is d(h) for h [M, Nout = I], gate_up [M, 2I] holds the saved gate
// and up values, and d_gate_up [M, 2I] receives their gradients.
struct GroupedDgradArgs {
  const void* grad_out;   // [M, Kc]
  const void* weight;     // [G, Kc, Nout]
  const int32_t* counts;  // [G]
  void* out;              // [M, Nout] (plain)
  const void* gate_up = nullptr;  // [M, 2 * Nout] (SwiGLU backward)
  void* d_gate_up = nullptr;      // [M, 2 * Nout]
  int64_t M;
  int Kc;
  int Nout;
  int G;
  int* err;
  int sm_limit;
};
cudaError_t launch_grouped_dgrad(const GroupedDgradArgs& args, cudaStream_t stream);
// wgrad: out[g] = grad_out[rows of g]^T @ input[rows of g], out [G, Mw, Nw].
// With ksplit > 1 and `partial` set (fp32, ksplit * G * Mw * Nw floats) each
// group's rows are cut into ksplit slices whose fp32 products are summed in
// slice order and rounded once (split-K, for few output tiles over many rows).
struct GroupedWgradArgs {
  const void* grad_out;   // [M, Mw]
  const void* input;      // [M, Nw]
  const int32_t* counts;  // [G]
  void* out;              // [G, Mw, Nw]
  int64_t M;
  int Mw;
  int Nw;
  int G;
  int* err;
  int sm_limit;
  int ksplit = 1;
  float* partial = nullptr;
};
// Slices for a split-K wgrad of G groups over M rows (fills the SMs).
int wgrad_ksplit(int64_t M, int Mw, int Nw, int G);
cudaError_t launch_grouped_wgrad(const GroupedWgradArgs& args, cudaStream_t stream);

// train.cu (bf16): the backward's non-GEMM kernels and the aux statistics ----
// Blocks of the deterministic partial sums below (partials: blocks * E).
int train_partial_blocks(int64_t T);
// Per token: d_expert_out rows (at pos), d_logits [T, E]; writes T to
// *count_out (if set) for the router's single-group GEMMs.
cudaError_t launch_combine_router_bwd(const void* grad_y, const void* expert_out,
                                      const int32_t* pos, const int32_t* topk_idx,
                                      const float* topk_w, const void* logits, int64_t T, int d,
                                      int k, int E, int norm, const float* aux_grad,
                                      const float* expert_counts, int64_t n_valid,
                                      void* d_expert_out, void* d_logits, int32_t* count_out,
                                      cudaStream_t stream);
// dx[t] = bf16(dx_router[t] + bf16(sum over the token's rows of d_x_sorted)).
cudaError_t launch_dx(const void* d_x_sorted, const int32_t* pos, const void* dx_router, int64_t T,
                      int d, int k, void* dx, cudaStream_t stream);
// aux loss and expert counts over the first n tokens (partials: nblocks * E each).
cudaError_t launch_aux_stats(const void* logits, const int32_t* topk_idx, int64_t n, int E, int k,
                             float* partial_p, int* partial_c, int nblocks, float* aux_out,
                             float* counts_out, cudaStream_t stream);
// out[e] = bf16(sum_t m[t, e]) for a bf16 [T, E] matrix.
cudaError_t launch_colsum_bf16(const void* m, int64_t T, int E, float* partial, int nblocks,
                               void* out, cudaStream_t stream);

// ep_p2p.cu -------------------------------------------------------------
size_t ep_symmetric_bytes(const ::hmoe_shape& s, int64_t max_tokens, int world);
size_t ep_workspace_bytes(const ::hmoe_shape& s, int64_t max_tokens, int world);
cudaError_t ep_forward_launch(const ::hmoe_shape& s, int64_t max_tokens, int rank, int world,
                              void* const* peer_bases, uint32_t epoch, const void* x,
                              const void* w_router, const void* bias, const void* w_gate_up,
                              const void* w_down, void* y, void* workspace, cudaStream_t st,
                              const cudaEvent_t* marks);  // 6 events or nullptr

// capi.cu ---------------------------------------------------------------
int num_sms_for_current_device();
// Entry-point plumbing for files other than capi.cu: set hmoe_last_error()
// and return `code`; make the device owning `ptr` current (sm_100 only);
// validate a shape.
int report_error(int code, const char* fmt, ...);
int make_device_current(const void* ptr);
int validate_shape_public(const ::hmoe_shape* shape);

}  // namespace hmoe
