// extern "C" entry points declared in include/hrm_moe.h.
//
// Each call validates its arguments, selects the device that owns the first
// data pointer, carves its scratch buffers out of the caller's workspace and
// enqueues the kernels on the caller's stream.  Nothing here synchronises
// the host except hmoe_workspace_status().
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <mutex>
#include <cstdlib>
#include <cstring>
#include <string>

#include "common.cuh"
#include "hrm_moe.h"
#include "internal.h"

using namespace hmoe;

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* where) {
  return fail(HMOE_EIO, "%s: %s", where, cudaGetErrorString(e));
}

#define HMOE_CUDA(call, where)                  \
  do {                                          \
    cudaError_t e_ = (call);                    \
    if (e_ != cudaSuccess) return cuda_fail(e_, where); \
  } while (0)

constexpr size_t kAlign = 1024;
size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

size_t elem_size(int dtype) { return dtype == kDtypeBF16 ? 2 : 4; }

int validate_shape(const hmoe_shape* s) {
  if (!s) return fail(HMOE_EINVAL, "shape is NULL");
  if (s->tokens < 0) return fail(HMOE_EINVAL, "tokens must be >= 0, got %lld", (long long)s->tokens);
  if (s->dtype != HMOE_DTYPE_BF16 && s->dtype != HMOE_DTYPE_F32)
    return fail(HMOE_EINVAL, "unsupported dtype %d (bf16 = 0, f32 = 1)", s->dtype);
  if (s->hidden <= 0 || s->hidden % 8 != 0)
    return fail(HMOE_EINVAL, "hidden must be a positive multiple of 8, got %d", s->hidden);
  if (s->intermediate <= 0 || s->intermediate % 8 != 0)
    return fail(HMOE_EINVAL, "intermediate must be a positive multiple of 8, got %d", s->intermediate);
  if (s->experts <= 0 || s->experts > 128)
    return fail(HMOE_EINVAL, "experts must be in [1, 128], got %d", s->experts);
  if (s->top_k <= 0 || s->top_k > s->experts || s->top_k > 32)
    return fail(HMOE_EINVAL, "top_k must be in [1, min(experts, 32)], got %d", s->top_k);
  if (s->tokens * (int64_t)s->top_k > 0x7fffffffll)
    return fail(HMOE_EINVAL, "tokens * top_k must fit in int32");
  return HMOE_OK;
}

int aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Make the device that owns `ptr` current; refuse non-sm_100 devices.
int select_device(const void* ptr) {
  cudaPointerAttributes attr;
  cudaError_t e = cudaPointerGetAttributes(&attr, ptr);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return cuda_fail(e, "cudaPointerGetAttributes");
  }
  if (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged)
    return fail(HMOE_EINVAL, "expected a device pointer (got host memory)");
  int cur = -1;
  HMOE_CUDA(cudaGetDevice(&cur), "cudaGetDevice");
  if (cur != attr.device) HMOE_CUDA(cudaSetDevice(attr.device), "cudaSetDevice");
  static int major[64];
  static std::once_flag once[64];
  const int dev = attr.device;
  if (dev < 0 || dev >= 64) return fail(HMOE_EINVAL, "device ordinal %d out of range", dev);
  std::call_once(once[dev], [dev] {
    int m = 0;
    cudaDeviceGetAttribute(&m, cudaDevAttrComputeCapabilityMajor, dev);
    major[dev] = m;
  });
  if (major[dev] != 10)
    return fail(HMOE_ENOSYS, "device %d is sm_%d0, this library is built for sm_100a", dev,
                major[dev]);
  return HMOE_OK;
}

// ------------------------------------------------------- workspace plans ----
struct Carve {
  char* base;
  size_t off = 0;
  template <class T>
  T* take(size_t bytes) {
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off = align_up(off + bytes);
    return p;
  }
};

struct DispatchBufs {
  int* err;
  int32_t* local_rank;
  int32_t* block_counts;
  int32_t* counts;
  int32_t* offsets;
};

DispatchBufs carve_dispatch(Carve& c, const hmoe_shape& s) {
  DispatchBufs b;
  const int64_t A = s.tokens * s.top_k;
  const int64_t nblk = dispatch_num_blocks(s.tokens, s.top_k);
  b.err = c.take<int>(sizeof(int));
  b.local_rank = c.take<int32_t>(sizeof(int32_t) * A);
  b.block_counts = c.take<int32_t>(sizeof(int32_t) * nblk * s.experts);
  b.counts = c.take<int32_t>(sizeof(int32_t) * s.experts);
  b.offsets = c.take<int32_t>(sizeof(int32_t) * (s.experts + 1));
  return b;
}

struct ExpertBufs {
  DispatchBufs d;
  int32_t* pos;
  void* xs;   // [A, d]: gathered rows, then (aliased) the down-projection output
  void* h;    // [A, I]
};

ExpertBufs carve_experts(Carve& c, const hmoe_shape& s) {
  ExpertBufs b;
  const int64_t A = s.tokens * s.top_k;
  const size_t es = elem_size(s.dtype);
  b.d = carve_dispatch(c, s);
  b.pos = c.take<int32_t>(sizeof(int32_t) * A);
  b.xs = c.take<void>(es * A * s.hidden);
  b.h = c.take<void>(es * A * s.intermediate);
  return b;
}

struct FfnBufs {
  ExpertBufs x;
  int32_t* topk_idx;
  float* topk_w;
  void* router_scratch;  // fix-up list of the tensor-core router
};

FfnBufs carve_ffn(Carve& c, const hmoe_shape& s) {
  FfnBufs b;
  const int64_t A = s.tokens * s.top_k;
  b.x = carve_experts(c, s);
  b.topk_idx = c.take<int32_t>(sizeof(int32_t) * A);
  b.topk_w = c.take<float>(sizeof(float) * A);
  b.router_scratch = c.take<void>(router_tc_scratch_bytes(s.tokens));
  return b;
}

// Router stage: tensor cores with exact-order fix-up for bf16, CUDA cores for fp32.
// reset_err: the error word is cleared first (in the default pass's kernel).
cudaError_t run_router(const hmoe_shape& s, const void* x, const void* w_router, const void* bias,
                       int32_t* idx, float* w_f32, void* w_dtype, void* logits, void* scratch,
                       int* err, cudaStream_t st, bool reset_err = false) {
  if (s.dtype == kDtypeBF16)
    return launch_router_topk_tc(x, w_router, bias, s.tokens, s.hidden, s.experts, s.top_k,
                                 s.norm_topk_prob, idx, w_f32, w_dtype, logits, scratch, err, st,
                                 nullptr, reset_err);
  if (reset_err) {
    const cudaError_t e = cudaMemsetAsync(err, 0, sizeof(int), st);
    if (e != cudaSuccess) return e;
  }
  return launch_router_topk(x, w_router, bias, s.tokens, s.hidden, s.experts, s.top_k, s.dtype,
                            s.norm_topk_prob, idx, w_f32, w_dtype, logits, st);
}

template <class F>
size_t plan_bytes(const hmoe_shape* s, F carve) {
  if (validate_shape(s) != HMOE_OK) return 0;
  Carve c{nullptr};
  carve(c, *s);
  return c.off;
}

int check_ws(void* ws, size_t have, size_t need) {
  if (need > have) return fail(HMOE_ENOSPC, "workspace too small: need %zu bytes, got %zu", need, have);
  if (need > 0 && !ws) return fail(HMOE_EINVAL, "workspace is NULL");
  if (reinterpret_cast<uintptr_t>(ws) % 256 != 0) return fail(HMOE_EINVAL, "workspace must be 256-byte aligned");
  return HMOE_OK;
}

// A call with no tokens still defines tokens_per_expert: E zeros (the
// reference's bincount(..., minlength=E), models/layers.py:322).
int zero_counts_if_empty(int32_t* counts, int E, void* stream) {
  if (!counts) return HMOE_OK;
  int rc = select_device(counts);
  if (rc) return rc;
  HMOE_CUDA(cudaMemsetAsync(counts, 0, sizeof(int32_t) * E, static_cast<cudaStream_t>(stream)),
            "clear counts");
  return HMOE_OK;
}

int sm_margin() {
  static int margin = [] {
    const char* v = getenv("HRM_MOE_B200_SM_MARGIN");
    return v ? atoi(v) : 0;
  }();
  return margin;
}

// Dispatch stages shared by the layer, the experts module and hmoe_dispatch.
int run_dispatch(const hmoe_shape& s, const int32_t* idx, const void* w, int w_is_f32,
                 const void* x, const DispatchBufs& b, int32_t* pos, int32_t* sort_idx,
                 int32_t* sorted_token, void* sorted_w, void* x_sorted, cudaStream_t st) {
  if (dispatch_fits_one_block(s.tokens, s.top_k)) {
    HMOE_CUDA(launch_dispatch_small(idx, w, w_is_f32, x, s.tokens, s.hidden, s.top_k, s.experts,
                                    s.dtype, b.counts, pos, sort_idx, sorted_token, sorted_w,
                                    x_sorted, b.err, st),
              "dispatch_small");
    return HMOE_OK;
  }
  HMOE_CUDA(launch_hist_scan(idx, s.tokens, s.top_k, s.experts, b.local_rank, b.block_counts,
                             b.counts, b.err, st), "hist_rank/scan");
  HMOE_CUDA(launch_permute_gather(idx, b.local_rank, b.block_counts, b.counts, w, w_is_f32, x, s.tokens,
                                  s.hidden, s.top_k, s.experts, s.dtype, pos, sort_idx,
                                  sorted_token, sorted_w, x_sorted, st), "permute_gather");
  return HMOE_OK;
}

// Which tcgen05 kernel runs a local grouped GEMM.  Both give the same bits.
// The CTA-pair kernel (256-row tiles over two SMs, half the operand traffic
// per SM) is faster once the groups average more than 192 rows; below that
// its tiles are mostly padding and the single-CTA kernel's 128-row tiles do
// half the wasted MMA work (XL layer: single-CTA faster up to T=1024 tokens,
// pair from T=2048).  HMOE_GEMM_KERNEL=pair or =single (read once per
// process) forces one kernel.
bool use_cta_pair_gemm(int64_t M, int G) {
  static const int forced = [] {
    const char* v = std::getenv("HMOE_GEMM_KERNEL");
    if (v && std::strcmp(v, "pair") == 0) return 1;
    if (v && std::strcmp(v, "single") == 0) return 0;
    return -1;
  }();
  if (forced >= 0) return forced == 1;
  return M > 192 * static_cast<int64_t>(G);
}

int run_grouped(const void* a, const void* b, const int32_t* counts, int64_t M, int N, int K,
                int G, int dtype, int swiglu, void* out, int* err, cudaStream_t st,
                const int32_t* group_weight = nullptr, int num_weights = 0) {
  GroupedGemmArgs g;
  g.group_weight = group_weight;
  g.num_weights = num_weights;
  g.a = a;
  g.b = b;
  g.counts = counts;
  g.out = out;
  g.M = M;
  g.N = N;
  g.K = K;
  g.G = G;
  g.swiglu = swiglu;
  g.dtype = dtype;
  g.err = err;
  g.sm_limit = 0;
  const cudaError_t e = dtype != kDtypeBF16 ? launch_grouped_gemm_simt(g, st)
                        : use_cta_pair_gemm(M, G) ? launch_grouped_gemm_pair(g, st)
                                              : launch_grouped_gemm_sm100(g, st);
  if (e != cudaSuccess) return cuda_fail(e, swiglu ? "grouped_swiglu" : "grouped_linear");
  return HMOE_OK;
}

// Experts on routed tokens: dispatch, two grouped GEMMs, combine.
// Optional timing marks between stages (events[i] recorded after stage i).
// Under stream capture a mark becomes an event-record node of the graph
// (cudaEventRecordExternal), so each replay records it and the caller can
// time the stages of a replay.
struct PhaseMarks {
  void* const* ev = nullptr;
  int mark(int i, cudaStream_t st) const {
    if (ev && ev[i]) {
      cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
      cudaError_t e = cudaStreamIsCapturing(st, &cs);
      if (e == cudaSuccess)
        e = cs == cudaStreamCaptureStatusActive
                ? cudaEventRecordWithFlags(static_cast<cudaEvent_t>(ev[i]), st, cudaEventRecordExternal)
                : cudaEventRecord(static_cast<cudaEvent_t>(ev[i]), st);
      if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord");
    }
    return HMOE_OK;
  }
};

int run_experts(const hmoe_shape& s, const void* x, const int32_t* idx, const void* w,
                int w_is_f32, const void* w_gate_up, const void* w_down, const void* final_in,
                void* out, int32_t* counts_out, int32_t* sort_idx, const ExpertBufs& b,
                cudaStream_t st, const PhaseMarks& pm = PhaseMarks()) {
  const int64_t A = s.tokens * s.top_k;
  int rc = run_dispatch(s, idx, w, w_is_f32, x, b.d, b.pos, sort_idx, nullptr, nullptr, b.xs, st);
  if (rc) return rc;
  if (counts_out)
    HMOE_CUDA(cudaMemcpyAsync(counts_out, b.d.counts, sizeof(int32_t) * s.experts,
                              cudaMemcpyDeviceToDevice, st), "copy counts");
  if ((rc = pm.mark(2, st))) return rc;
  rc = run_grouped(b.xs, w_gate_up, b.d.counts, A, s.intermediate, s.hidden, s.experts, s.dtype,
                   1, b.h, b.d.err, st);
  if (rc) return rc;
  if ((rc = pm.mark(3, st))) return rc;
  rc = run_grouped(b.h, w_down, b.d.counts, A, s.hidden, s.intermediate, s.experts, s.dtype, 0,
                   b.xs, b.d.err, st);
  if (rc) return rc;
  if ((rc = pm.mark(4, st))) return rc;
  HMOE_CUDA(launch_combine(b.xs, b.pos, w, w_is_f32, idx, s.experts, s.tokens, s.hidden, s.top_k,
                           s.dtype, final_in, out, st), "combine");
  return pm.mark(5, st);
}

int ffn_forward_impl(const hmoe_shape* shape, const void* x, const void* w_router,
                     const void* router_bias, const void* w_gate_up, const void* w_down, void* y,
                     int accumulate, int32_t* topk_idx, void* topk_weight, int32_t* counts,
                     int32_t* sort_idx, void* workspace, size_t workspace_bytes, void* stream,
                     const PhaseMarks& pm);

}  // namespace

namespace hmoe {
int report_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return fail(code, "%s", buf);
}

int make_device_current(const void* ptr) { return select_device(ptr); }

std::atomic<unsigned>& pdl_mask() {
  static std::atomic<unsigned> mask{[] {
    const char* v = std::getenv("HMOE_PDL");
    return v ? static_cast<unsigned>(std::strtoul(v, nullptr, 0))
             : static_cast<unsigned>(kPdlRouter | kPdlDispatch | kPdlGemm);
  }()};
  return mask;
}

bool pdl_enabled(unsigned cls) { return (pdl_mask().load(std::memory_order_relaxed) & cls) != 0; }

int validate_shape_public(const hmoe_shape* shape) { return validate_shape(shape); }

int num_sms_for_current_device() {
  static int sms[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!sms[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    sms[dev] = n > 0 ? n : 148;
  }
  const int n = sms[dev] - sm_margin();
  return n > 0 ? n : 1;
}
}  // namespace hmoe

extern "C" {

const char* hmoe_version(void) { return "hrm-moe-b200 0.1 (sm_100a)"; }

const char* hmoe_last_error(void) { return g_last_error.c_str(); }

size_t hmoe_ffn_workspace_bytes(const hmoe_shape* shape) {
  return plan_bytes(shape, [](Carve& c, const hmoe_shape& s) { carve_ffn(c, s); });
}

int hmoe_ffn_forward(const hmoe_shape* shape, const void* x, const void* w_router,
                     const void* router_bias, const void* w_gate_up, const void* w_down, void* y,
                     int accumulate, int32_t* topk_idx, void* topk_weight, int32_t* counts,
                     int32_t* sort_idx, void* workspace, size_t workspace_bytes, void* stream) {
  return ffn_forward_impl(shape, x, w_router, router_bias, w_gate_up, w_down, y, accumulate,
                          topk_idx, topk_weight, counts, sort_idx, workspace, workspace_bytes,
                          stream, PhaseMarks());
}

int hmoe_ffn_forward_marked(const hmoe_shape* shape, const void* x, const void* w_router,
                            const void* router_bias, const void* w_gate_up, const void* w_down,
                            void* y, int accumulate, void* workspace, size_t workspace_bytes,
                            void* stream, void* const* phase_events) {
  PhaseMarks pm;
  pm.ev = phase_events;
  return ffn_forward_impl(shape, x, w_router, router_bias, w_gate_up, w_down, y, accumulate,
                          nullptr, nullptr, nullptr, nullptr, workspace, workspace_bytes, stream,
                          pm);
}

}  // extern "C"

namespace {
int ffn_forward_impl(const hmoe_shape* shape, const void* x, const void* w_router,
                     const void* router_bias, const void* w_gate_up, const void* w_down, void* y,
                     int accumulate, int32_t* topk_idx, void* topk_weight, int32_t* counts,
                     int32_t* sort_idx, void* workspace, size_t workspace_bytes, void* stream,
                     const PhaseMarks& pm) {
  int rc = validate_shape(shape);
  if (rc) return rc;
  const hmoe_shape& s = *shape;
  if (s.tokens == 0) return zero_counts_if_empty(counts, s.experts, stream);
  if (!x || !w_router || !w_gate_up || !w_down || !y)
    return fail(HMOE_EINVAL, "x, w_router, w_gate_up, w_down and y are required");
  if (!aligned16(x) || !aligned16(w_gate_up) || !aligned16(w_down) || !aligned16(y) ||
      !aligned16(w_router))
    return fail(HMOE_EINVAL, "x, weights and y must be 16-byte aligned");
  if ((rc = select_device(x))) return rc;
  const size_t need = hmoe_ffn_workspace_bytes(shape);
  if ((rc = check_ws(workspace, workspace_bytes, need))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carve c{static_cast<char*>(workspace)};
  FfnBufs b = carve_ffn(c, s);
  int32_t* idx = topk_idx ? topk_idx : b.topk_idx;
  if ((rc = pm.mark(0, st))) return rc;
  HMOE_CUDA(run_router(s, x, w_router, router_bias, idx, b.topk_w, topk_weight, nullptr,
                       b.router_scratch, b.x.d.err, st, true),
            "router_topk");
  if ((rc = pm.mark(1, st))) return rc;
  return run_experts(s, x, idx, b.topk_w, 1, w_gate_up, w_down, accumulate ? y : nullptr, y,
                     counts, sort_idx, b.x, st, pm);
}
}  // namespace

extern "C" {

// ------------------------------------------------- host-buffer pipeline ----
namespace {
struct HostPipe {
  cudaStream_t in = nullptr, out = nullptr;
  cudaEvent_t x_ready[2], x_free[2], y_ready[2], y_free[2], done;
  bool ok = false;
};

int host_pipe(int dev, HostPipe** out) {
  static HostPipe pipes[64];
  static std::mutex mu;
  if (dev < 0 || dev >= 64) return fail(HMOE_EINVAL, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(mu);
  HostPipe& p = pipes[dev];
  if (!p.ok) {
    HMOE_CUDA(cudaStreamCreateWithFlags(&p.in, cudaStreamNonBlocking), "cudaStreamCreate");
    HMOE_CUDA(cudaStreamCreateWithFlags(&p.out, cudaStreamNonBlocking), "cudaStreamCreate");
    for (int i = 0; i < 2; ++i) {
      HMOE_CUDA(cudaEventCreateWithFlags(&p.x_ready[i], cudaEventDisableTiming), "cudaEventCreate");
      HMOE_CUDA(cudaEventCreateWithFlags(&p.x_free[i], cudaEventDisableTiming), "cudaEventCreate");
      HMOE_CUDA(cudaEventCreateWithFlags(&p.y_ready[i], cudaEventDisableTiming), "cudaEventCreate");
      HMOE_CUDA(cudaEventCreateWithFlags(&p.y_free[i], cudaEventDisableTiming), "cudaEventCreate");
    }
    HMOE_CUDA(cudaEventCreateWithFlags(&p.done, cudaEventDisableTiming), "cudaEventCreate");
    p.ok = true;
  }
  *out = &p;
  return HMOE_OK;
}

hmoe_shape chunk_shape(const hmoe_shape& s, int64_t tokens) {
  hmoe_shape c = s;
  c.tokens = tokens;
  return c;
}
}  // namespace

size_t hmoe_ffn_host_workspace_bytes(const hmoe_shape* shape, int64_t chunk_tokens) {
  if (validate_shape(shape) != HMOE_OK || chunk_tokens <= 0) return 0;
  const hmoe_shape c = chunk_shape(*shape, chunk_tokens);
  const size_t row = elem_size(shape->dtype) * shape->hidden;
  return 4 * align_up(row * chunk_tokens) + hmoe_ffn_workspace_bytes(&c);
}

int hmoe_ffn_forward_host(const hmoe_shape* shape, const void* x_host, const void* w_router,
                          const void* router_bias, const void* w_gate_up, const void* w_down,
                          void* y_host, int64_t chunk_tokens, void* workspace,
                          size_t workspace_bytes, void* stream) {
  int rc = validate_shape(shape);
  if (rc) return rc;
  const hmoe_shape& s = *shape;
  if (s.tokens == 0) return HMOE_OK;
  if (chunk_tokens <= 0) return fail(HMOE_EINVAL, "chunk_tokens must be positive");
  if (!x_host || !y_host || !w_router || !w_gate_up || !w_down)
    return fail(HMOE_EINVAL, "x_host, y_host and the weights are required");
  if ((rc = select_device(w_gate_up))) return rc;
  const size_t need = hmoe_ffn_host_workspace_bytes(shape, chunk_tokens);
  if ((rc = check_ws(workspace, workspace_bytes, need))) return rc;
  int dev = 0;
  HMOE_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  HostPipe* hp = nullptr;
  if ((rc = host_pipe(dev, &hp))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t row = elem_size(s.dtype) * s.hidden;
  const size_t buf = align_up(row * chunk_tokens);
  char* base = static_cast<char*>(workspace);
  char* xb[2] = {base, base + buf};
  char* yb[2] = {base + 2 * buf, base + 3 * buf};
  void* ffn_ws = base + 4 * buf;
  const size_t ffn_bytes = workspace_bytes - 4 * buf;
  // the buffers start free once the caller's earlier work on `stream` is done
  for (int i = 0; i < 2; ++i) {
    HMOE_CUDA(cudaEventRecord(hp->x_free[i], st), "cudaEventRecord");
    HMOE_CUDA(cudaEventRecord(hp->y_free[i], st), "cudaEventRecord");
  }
  const int64_t nchunks = cdiv64(s.tokens, chunk_tokens);
  for (int64_t c = 0; c < nchunks; ++c) {
    const int i = static_cast<int>(c & 1);
    const int64_t t0 = c * chunk_tokens;
    const int64_t tc = (t0 + chunk_tokens <= s.tokens) ? chunk_tokens : s.tokens - t0;
    // H2D of this chunk once the compute of chunk c-2 stopped reading the buffer
    HMOE_CUDA(cudaStreamWaitEvent(hp->in, hp->x_free[i], 0), "cudaStreamWaitEvent");
    HMOE_CUDA(cudaMemcpyAsync(xb[i], static_cast<const char*>(x_host) + t0 * row, tc * row,
                              cudaMemcpyHostToDevice, hp->in), "H2D chunk");
    HMOE_CUDA(cudaEventRecord(hp->x_ready[i], hp->in), "cudaEventRecord");
    // compute once the rows are in and the D2H of chunk c-2 freed the output
    HMOE_CUDA(cudaStreamWaitEvent(st, hp->x_ready[i], 0), "cudaStreamWaitEvent");
    HMOE_CUDA(cudaStreamWaitEvent(st, hp->y_free[i], 0), "cudaStreamWaitEvent");
    const hmoe_shape cs = chunk_shape(s, tc);
    rc = hmoe_ffn_forward(&cs, xb[i], w_router, router_bias, w_gate_up, w_down, yb[i], 0, nullptr,
                          nullptr, nullptr, nullptr, ffn_ws, ffn_bytes, st);
    if (rc) return rc;
    HMOE_CUDA(cudaEventRecord(hp->x_free[i], st), "cudaEventRecord");
    HMOE_CUDA(cudaEventRecord(hp->y_ready[i], st), "cudaEventRecord");
    // D2H of the result
    HMOE_CUDA(cudaStreamWaitEvent(hp->out, hp->y_ready[i], 0), "cudaStreamWaitEvent");
    HMOE_CUDA(cudaMemcpyAsync(static_cast<char*>(y_host) + t0 * row, yb[i], tc * row,
                              cudaMemcpyDeviceToHost, hp->out), "D2H chunk");
    HMOE_CUDA(cudaEventRecord(hp->y_free[i], hp->out), "cudaEventRecord");
  }
  // the call completes, in stream order, on the caller's stream
  HMOE_CUDA(cudaEventRecord(hp->done, hp->out), "cudaEventRecord");
  HMOE_CUDA(cudaStreamWaitEvent(st, hp->done, 0), "cudaStreamWaitEvent");
  return HMOE_OK;
}

// ------------------------------------------------- expert parallel (P2P) ----
size_t hmoe_ep_symmetric_bytes(const hmoe_shape* shape, int64_t max_tokens, int32_t world) {
  if (validate_shape(shape) != HMOE_OK || max_tokens < 0 || world < 1 || world > 8) return 0;
  return ep_symmetric_bytes(*shape, max_tokens, world);
}

size_t hmoe_ep_workspace_bytes(const hmoe_shape* shape, int64_t max_tokens, int32_t world) {
  if (validate_shape(shape) != HMOE_OK || max_tokens < 0 || world < 1 || world > 8) return 0;
  return ep_workspace_bytes(*shape, max_tokens, world);
}

// The exchanged handle: the region's cudaIpcMemHandle_t, then the UUID of
// the GPU that owns it (so that open can refuse a region of its own GPU).
static_assert(sizeof(cudaIpcMemHandle_t) + sizeof(cudaUUID_t) == HMOE_EP_HANDLE_BYTES,
              "handle layout");

static int current_uuid(cudaUUID_t* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  cudaDeviceProp prop;
  if (e == cudaSuccess) e = cudaGetDeviceProperties(&prop, dev);
  if (e != cudaSuccess) return cuda_fail(e, "device UUID");
  *out = prop.uuid;
  return HMOE_OK;
}

int hmoe_ep_symmetric_alloc(size_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return fail(HMOE_EINVAL, "bad arguments");
  cudaUUID_t uuid;
  int rc = current_uuid(&uuid);
  if (rc) return rc;
  void* p = nullptr;
  HMOE_CUDA(cudaMalloc(&p, bytes), "cudaMalloc(symmetric region)");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "symmetric region");
  }
  memcpy(handle, &h, sizeof(h));
  memcpy(static_cast<char*>(handle) + sizeof(h), &uuid, sizeof(uuid));
  *ptr = p;
  return HMOE_OK;
}

int hmoe_ep_symmetric_open(const void* handle, void** peer_ptr) {
  if (!handle || !peer_ptr) return fail(HMOE_EINVAL, "bad arguments");
  // The exchange kernels of different ranks wait on one another, so each
  // rank needs its own GPU: two of them sharing one could wait forever.
  cudaUUID_t mine;
  int rc = current_uuid(&mine);
  if (rc) return rc;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  if (memcmp(static_cast<const char*>(handle) + sizeof(h), &mine, sizeof(mine)) == 0)
    return fail(HMOE_EINVAL, "peer region lives on this GPU: every rank needs its own GPU");
  HMOE_CUDA(cudaIpcOpenMemHandle(peer_ptr, h, cudaIpcMemLazyEnablePeerAccess),
            "cudaIpcOpenMemHandle");
  return HMOE_OK;
}

int hmoe_ep_symmetric_close(void* peer_ptr) {
  HMOE_CUDA(cudaIpcCloseMemHandle(peer_ptr), "cudaIpcCloseMemHandle");
  return HMOE_OK;
}

int hmoe_ep_symmetric_free(void* ptr) {
  HMOE_CUDA(cudaFree(ptr), "cudaFree(symmetric region)");
  return HMOE_OK;
}

int hmoe_ep_forward_marked(const hmoe_shape* shape, int64_t max_tokens, int32_t rank,
                           int32_t world, void* const* peer_bases, uint32_t epoch, const void* x,
                           const void* w_router, const void* router_bias,
                           const void* w_gate_up_local, const void* w_down_local, void* y,
                           void* workspace, size_t workspace_bytes, void* stream,
                           void* const* phase_events) {
  int rc = validate_shape(shape);
  if (rc) return rc;
  const hmoe_shape& s = *shape;
  if (world < 1 || world > 8 || rank < 0 || rank >= world)
    return fail(HMOE_EINVAL, "rank %d of world %d (1..8 ranks)", rank, world);
  if (s.experts % world) return fail(HMOE_EINVAL, "experts %d not divisible by world %d", s.experts, world);
  if (s.tokens > max_tokens) return fail(HMOE_EINVAL, "tokens %lld exceed max_tokens %lld",
                                         (long long)s.tokens, (long long)max_tokens);
  if (static_cast<int64_t>(world) * max_tokens * s.top_k >= (1ll << 28))
    return fail(HMOE_EINVAL, "world * max_tokens * top_k must stay below 2^28");
  if (!peer_bases || !w_router || !w_gate_up_local || !w_down_local || (s.tokens > 0 && (!x || !y)))
    return fail(HMOE_EINVAL, "NULL argument");
  for (int p = 0; p < world; ++p)
    if (!peer_bases[p]) return fail(HMOE_EINVAL, "peer base %d is NULL", p);
  if (s.tokens > 0 && (!aligned16(x) || !aligned16(y)))
    return fail(HMOE_EINVAL, "x and y must be 16-byte aligned");
  cudaEvent_t marks[6];
  if (phase_events) {
    for (int i = 0; i < 6; ++i) {
      if (!phase_events[i]) return fail(HMOE_EINVAL, "phase event %d is NULL", i);
      marks[i] = static_cast<cudaEvent_t>(phase_events[i]);
    }
  }
  if ((rc = select_device(w_gate_up_local))) return rc;
  if ((rc = check_ws(workspace, workspace_bytes, ep_workspace_bytes(s, max_tokens, world)))) return rc;
  HMOE_CUDA(ep_forward_launch(s, max_tokens, rank, world, peer_bases, epoch, x, w_router,
                              router_bias, w_gate_up_local, w_down_local, y, workspace,
                              static_cast<cudaStream_t>(stream), phase_events ? marks : nullptr),
            "ep_forward");
  return HMOE_OK;
}

int hmoe_ep_forward(const hmoe_shape* shape, int64_t max_tokens, int32_t rank, int32_t world,
                    void* const* peer_bases, uint32_t epoch, const void* x, const void* w_router,
                    const void* router_bias, const void* w_gate_up_local,
                    const void* w_down_local, void* y, void* workspace, size_t workspace_bytes,
                    void* stream) {
  return hmoe_ep_forward_marked(shape, max_tokens, rank, world, peer_bases, epoch, x, w_router,
                                router_bias, w_gate_up_local, w_down_local, y, workspace,
                                workspace_bytes, stream, nullptr);
}

size_t hmoe_router_workspace_bytes(const hmoe_shape* shape) {
  return plan_bytes(shape, [](Carve& c, const hmoe_shape& s) {
    c.take<int>(sizeof(int));  // error word
    c.take<void>(router_tc_scratch_bytes(s.tokens));
  });
}

int hmoe_router_topk(const hmoe_shape* shape, const void* x, const void* w_router,
                     const void* router_bias, int32_t* topk_idx, void* topk_weight, void* logits,
                     void* workspace, size_t workspace_bytes, void* stream) {
  int rc = validate_shape(shape);
  if (rc) return rc;
  const hmoe_shape& s = *shape;
  if (s.tokens == 0) return HMOE_OK;
  if (!x || !w_router || !topk_idx) return fail(HMOE_EINVAL, "x, w_router and topk_idx are required");
  if (!aligned16(x) || !aligned16(w_router)) return fail(HMOE_EINVAL, "x and w_router must be 16-byte aligned");
  if ((rc = select_device(x))) return rc;
  if ((rc = check_ws(workspace, workspace_bytes, hmoe_router_workspace_bytes(shape)))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carve c{static_cast<char*>(workspace)};
  int* err = c.take<int>(sizeof(int));
  void* scratch = c.take<void>(router_tc_scratch_bytes(s.tokens));
  HMOE_CUDA(cudaMemsetAsync(err, 0, sizeof(int), st), "reset error word");
  HMOE_CUDA(run_router(s, x, w_router, router_bias, topk_idx, nullptr, topk_weight, logits, scratch,
                       err, st),
            "router_topk");
  return HMOE_OK;
}

int hmoe_router_topk_sums(const hmoe_shape* shape, const void* x, const void* w_router,
                          const void* router_bias, int32_t* topk_idx, void* topk_weight,
                          void* logits, float* sums, void* workspace, size_t workspace_bytes,
                          void* stream) {
  int rc = validate_shape(shape);
  if (rc) return rc;
  const hmoe_shape& s = *shape;
  if (s.dtype != HMOE_DTYPE_BF16)
    return fail(HMOE_EINVAL, "tensor-core sums exist for bf16 layers only");
  if (s.tokens == 0) return HMOE_OK;
  if (!x || !w_router || !topk_idx || !sums)
    return fail(HMOE_EINVAL, "x, w_router, topk_idx and sums are required");
  if (!aligned16(x) || !aligned16(w_router)) return fail(HMOE_EINVAL, "x and w_router must be 16-byte aligned");
  if ((rc = select_device(x))) return rc;
  if ((rc = check_ws(workspace, workspace_bytes, hmoe_router_workspace_bytes(shape)))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carve c{static_cast<char*>(workspace)};
  int* err = c.take<int>(sizeof(int));
  void* scratch = c.take<void>(router_tc_scratch_bytes(s.tokens));
  HMOE_CUDA(cudaMemsetAsync(err, 0, sizeof(int), st), "reset error word");
  HMOE_CUDA(launch_router_topk_tc(x, w_router, router_bias, s.tokens, s.hidden, s.experts,
                                  s.top_k, s.norm_topk_prob, topk_idx, nullptr, topk_weight,
                                  logits, scratch, err, st, sums),
            "router_topk");
  return HMOE_OK;
}

size_t hmoe_dispatch_workspace_bytes(const hmoe_shape* shape) {
  return plan_bytes(shape, [](Carve& c, const hmoe_shape& s) {
    carve_dispatch(c, s);
    c.take<int32_t>(sizeof(int32_t) * s.tokens * s.top_k);  // pos
  });
}

int hmoe_dispatch(const hmoe_shape* shape, const int32_t* topk_idx, const void* topk_weight,
                  const void* x, int32_t* sort_idx, int32_t* counts, int32_t* sorted_token,
                  void* sorted_weight, void* x_sorted, void* workspace, size_t workspace_bytes,
                  void* stream) {
  int rc = validate_shape(shape);
  if (rc) return rc;
  const hmoe_shape& s = *shape;
  if (s.tokens == 0) return zero_counts_if_empty(counts, s.experts, stream);
  if (!topk_idx) return fail(HMOE_EINVAL, "topk_idx is required");
  if (sorted_weight && !topk_weight) return fail(HMOE_EINVAL, "sorted_weight needs topk_weight");
  if (x_sorted && (!x || !aligned16(x) || !aligned16(x_sorted)))
    return fail(HMOE_EINVAL, "x_sorted needs a 16-byte aligned x");
  if ((rc = select_device(topk_idx))) return rc;
  if ((rc = check_ws(workspace, workspace_bytes, hmoe_dispatch_workspace_bytes(shape)))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carve c{static_cast<char*>(workspace)};
  DispatchBufs b = carve_dispatch(c, s);
  int32_t* pos = c.take<int32_t>(sizeof(int32_t) * s.tokens * s.top_k);
  HMOE_CUDA(cudaMemsetAsync(b.err, 0, sizeof(int), st), "reset error word");
  rc = run_dispatch(s, topk_idx, topk_weight, 0, x, b, pos, sort_idx, sorted_token, sorted_weight,
                    x_sorted, st);
  if (rc) return rc;
  if (counts)
    HMOE_CUDA(cudaMemcpyAsync(counts, b.counts, sizeof(int32_t) * s.experts,
                              cudaMemcpyDeviceToDevice, st), "copy counts");
  return HMOE_OK;
}

size_t hmoe_experts_workspace_bytes(const hmoe_shape* shape) {
  return plan_bytes(shape, [](Carve& c, const hmoe_shape& s) { carve_experts(c, s); });
}

int hmoe_experts_forward(const hmoe_shape* shape, const void* hidden, const int32_t* topk_idx,
                         const void* topk_weight, const void* w_gate_up, const void* w_down,
                         void* final_hidden_states, int32_t* counts, int32_t* sort_idx,
                         void* workspace, size_t workspace_bytes, void* stream) {
  int rc = validate_shape(shape);
  if (rc) return rc;
  const hmoe_shape& s = *shape;
  if (s.tokens == 0) return zero_counts_if_empty(counts, s.experts, stream);
  if (!hidden || !topk_idx || !topk_weight || !w_gate_up || !w_down || !final_hidden_states)
    return fail(HMOE_EINVAL, "all tensor arguments are required");
  if (!aligned16(hidden) || !aligned16(w_gate_up) || !aligned16(w_down) ||
      !aligned16(final_hidden_states))
    return fail(HMOE_EINVAL, "hidden, weights and final_hidden_states must be 16-byte aligned");
  if ((rc = select_device(hidden))) return rc;
  if ((rc = check_ws(workspace, workspace_bytes, hmoe_experts_workspace_bytes(shape)))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carve c{static_cast<char*>(workspace)};
  ExpertBufs b = carve_experts(c, s);
  HMOE_CUDA(cudaMemsetAsync(b.d.err, 0, sizeof(int), st), "reset error word");
  return run_experts(s, hidden, topk_idx, topk_weight, 0, w_gate_up, w_down, final_hidden_states,
                     final_hidden_states, counts, sort_idx, b, st);
}

size_t hmoe_grouped_linear_workspace_bytes(int32_t groups) {
  (void)groups;
  return kAlign;  // the device error word
}

static int grouped_common(const void* input, const void* weight, const int32_t* tpe, int64_t M,
                          int32_t N, int32_t K, int32_t G, int32_t dtype, void* output,
                          void* workspace, size_t workspace_bytes, void* stream, int swiglu,
                          const int32_t* group_weight = nullptr, int32_t num_weights = 0) {
  if (M < 0 || N <= 0 || K <= 0 || G <= 0)
    return fail(HMOE_EINVAL, "bad grouped GEMM shape M=%lld N=%d K=%d G=%d", (long long)M, N, K, G);
  if (dtype != HMOE_DTYPE_BF16 && dtype != HMOE_DTYPE_F32)
    return fail(HMOE_EINVAL, "unsupported dtype %d", dtype);
  if (N % 8 != 0 || K % 8 != 0) return fail(HMOE_EINVAL, "N and K must be multiples of 8");
  if (G > 1024) return fail(HMOE_EINVAL, "at most 1024 groups");
  if (M == 0) return HMOE_OK;
  if (!input || !weight || !tpe || !output) return fail(HMOE_EINVAL, "NULL tensor argument");
  if (!aligned16(input) || !aligned16(weight) || !aligned16(output))
    return fail(HMOE_EINVAL, "input, weight and output must be 16-byte aligned");
  int rc = select_device(input);
  if (rc) return rc;
  int* err = nullptr;
  if (workspace && workspace_bytes >= sizeof(int)) {
    err = static_cast<int*>(workspace);
    HMOE_CUDA(cudaMemsetAsync(err, 0, sizeof(int), static_cast<cudaStream_t>(stream)),
              "reset error word");
  }
  if (group_weight && num_weights <= 0)
    return fail(HMOE_EINVAL, "a group->weight map needs the number of weights");
  return run_grouped(input, weight, tpe, M, N, K, G, dtype, swiglu, output, err,
                     static_cast<cudaStream_t>(stream), group_weight, num_weights);
}

int hmoe_grouped_linear(const void* input, const void* weight, const int32_t* tokens_per_expert,
                        int64_t M, int32_t N, int32_t K, int32_t groups, int32_t dtype,
                        void* output, void* workspace, size_t workspace_bytes, void* stream) {
  return grouped_common(input, weight, tokens_per_expert, M, N, K, groups, dtype, output,
                        workspace, workspace_bytes, stream, 0);
}

int hmoe_grouped_swiglu(const void* input, const void* w_gate_up,
                        const int32_t* tokens_per_expert, int64_t M, int32_t I, int32_t K,
                        int32_t groups, int32_t dtype, void* output, void* workspace,
                        size_t workspace_bytes, void* stream) {
  return grouped_common(input, w_gate_up, tokens_per_expert, M, I, K, groups, dtype, output,
                        workspace, workspace_bytes, stream, 1);
}

int hmoe_grouped_gemm_mapped(const void* input, const void* weight, const int32_t* group_rows,
                             const int32_t* group_weight, int64_t M, int32_t N, int32_t K,
                             int32_t groups, int32_t num_weights, int32_t dtype, int32_t swiglu,
                             void* output, void* workspace, size_t workspace_bytes, void* stream) {
  return grouped_common(input, weight, group_rows, M, N, K, groups, dtype, output, workspace,
                        workspace_bytes, stream, swiglu ? 1 : 0, group_weight, num_weights);
}

int hmoe_grouped_linear_backward(const void* grad_out, const void* input, const void* weight,
                                 const int32_t* tpe, int64_t M, int32_t N, int32_t K, int32_t G,
                                 int32_t dtype, void* grad_input, void* grad_weight,
                                 void* workspace, size_t workspace_bytes, void* stream) {
  if (M < 0 || N <= 0 || K <= 0 || G <= 0)
    return fail(HMOE_EINVAL, "bad grouped GEMM shape M=%lld N=%d K=%d G=%d", (long long)M, N, K, G);
  if (dtype != HMOE_DTYPE_BF16)
    return fail(HMOE_EINVAL, "the grouped GEMM backward supports bf16 only (dtype %d)", dtype);
  if (N % 8 != 0 || K % 8 != 0) return fail(HMOE_EINVAL, "N and K must be multiples of 8");
  if (G > 1024) return fail(HMOE_EINVAL, "at most 1024 groups");
  if (!tpe) return fail(HMOE_EINVAL, "tokens_per_expert is required");
  if (grad_input && (!grad_out || !weight || !aligned16(grad_out) || !aligned16(weight) ||
                     !aligned16(grad_input)))
    return fail(HMOE_EINVAL, "grad_input needs 16-byte aligned grad_out, weight, grad_input");
  if (grad_weight && (!aligned16(grad_weight) ||
                      (M > 0 && (!grad_out || !input || !aligned16(grad_out) || !aligned16(input)))))
    return fail(HMOE_EINVAL, "grad_weight needs 16-byte aligned grad_out, input, grad_weight");
  if (!grad_input && !grad_weight) return HMOE_OK;
  int rc = select_device(tpe);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int* err = nullptr;
  if (workspace && workspace_bytes >= sizeof(int)) {
    err = static_cast<int*>(workspace);
    HMOE_CUDA(cudaMemsetAsync(err, 0, sizeof(int), st), "reset error word");
  }
  if (grad_input && M > 0) {
    GroupedDgradArgs a;
    a.grad_out = grad_out;
    a.weight = weight;
    a.counts = tpe;
    a.out = grad_input;
    a.M = M;
    a.Kc = N;
    a.Nout = K;
    a.G = G;
    a.err = err;
    a.sm_limit = 0;
    HMOE_CUDA(launch_grouped_dgrad(a, st), "grouped dgrad");
  }
  if (grad_weight) {
    GroupedWgradArgs a;
    a.grad_out = grad_out;
    a.input = input;
    a.counts = tpe;
    a.out = grad_weight;
    a.M = M;
    a.Mw = N;
    a.Nw = K;
    a.G = G;
    a.err = err;
    a.sm_limit = 0;
    HMOE_CUDA(launch_grouped_wgrad(a, st), "grouped wgrad");
  }
  return HMOE_OK;
}

int hmoe_grouped_swiglu_backward(const void* grad_out, const void* w_down, const void* gate_up,
                                 const int32_t* tpe, int64_t M, int32_t d, int32_t I, int32_t G,
                                 void* d_gate_up, void* workspace, size_t workspace_bytes,
                                 void* stream) {
  if (M < 0 || d <= 0 || I <= 0 || G <= 0)
    return fail(HMOE_EINVAL, "bad shape M=%lld d=%d I=%d G=%d", (long long)M, d, I, G);
  if (d % 8 != 0 || I % 8 != 0) return fail(HMOE_EINVAL, "d and I must be multiples of 8");
  if (G > 1024) return fail(HMOE_EINVAL, "at most 1024 groups");
  if (M == 0) return HMOE_OK;
  if (!grad_out || !w_down || !gate_up || !tpe || !d_gate_up)
    return fail(HMOE_EINVAL, "NULL tensor argument");
  if (!aligned16(grad_out) || !aligned16(w_down) || !aligned16(gate_up) || !aligned16(d_gate_up))
    return fail(HMOE_EINVAL, "tensors must be 16-byte aligned");
  int rc = select_device(grad_out);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int* err = nullptr;
  if (workspace && workspace_bytes >= sizeof(int)) {
    err = static_cast<int*>(workspace);
    HMOE_CUDA(cudaMemsetAsync(err, 0, sizeof(int), st), "reset error word");
  }
  GroupedDgradArgs a;
  a.grad_out = grad_out;
  a.weight = w_down;
  a.counts = tpe;
  a.out = nullptr;
  a.gate_up = gate_up;
  a.d_gate_up = d_gate_up;
  a.M = M;
  a.Kc = d;
  a.Nout = I;
  a.G = G;
  a.err = err;
  a.sm_limit = 0;
  HMOE_CUDA(launch_grouped_dgrad(a, st), "grouped swiglu dgrad");
  return HMOE_OK;
}

size_t hmoe_combine_workspace_bytes(const hmoe_shape* shape) {
  return plan_bytes(shape, [](Carve& c, const hmoe_shape& s) {
    c.take<int32_t>(sizeof(int32_t) * s.tokens * s.top_k);
  });
}

int hmoe_combine(const hmoe_shape* shape, const void* expert_out, const int32_t* sort_idx,
                 const void* topk_weight, void* final_hidden_states, void* workspace,
                 size_t workspace_bytes, void* stream) {
  int rc = validate_shape(shape);
  if (rc) return rc;
  const hmoe_shape& s = *shape;
  if (s.tokens == 0) return HMOE_OK;
  if (!expert_out || !sort_idx || !topk_weight || !final_hidden_states)
    return fail(HMOE_EINVAL, "all tensor arguments are required");
  if (!aligned16(expert_out) || !aligned16(final_hidden_states))
    return fail(HMOE_EINVAL, "expert_out and final_hidden_states must be 16-byte aligned");
  if ((rc = select_device(expert_out))) return rc;
  if ((rc = check_ws(workspace, workspace_bytes, hmoe_combine_workspace_bytes(shape)))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t* pos = static_cast<int32_t*>(workspace);
  const int64_t A = s.tokens * s.top_k;
  HMOE_CUDA(cudaMemsetAsync(pos, 0xff, sizeof(int32_t) * A, st), "clear positions");
  HMOE_CUDA(launch_invert_perm(sort_idx, A, pos, st), "invert_perm");
  HMOE_CUDA(launch_combine(expert_out, pos, topk_weight, 0, nullptr, s.experts, s.tokens, s.hidden,
                           s.top_k, s.dtype, final_hidden_states, final_hidden_states, st),
            "combine");
  return HMOE_OK;
}

// ------------------------------------------------------------ training ----
}  // extern "C"

namespace {

// Activations the backward needs, kept by the training forward.
struct TrainSaved {
  uint16_t* logits;     // [T, E]
  int32_t* topk_idx;    // [A]
  float* topk_w;        // [A] (rounded to bf16)
  int32_t* counts;      // [E] rows per expert
  int32_t* pos;         // [A] sorted position of assignment t*k+j
  float* aux_counts;    // [E] selections among the aux tokens
  void* x_sorted;       // [A, d]
  void* gate_up;        // [A, 2I]
  void* h;              // [A, I]
  void* expert_out;     // [A, d] before the routing weight
};

TrainSaved carve_saved(Carve& c, const hmoe_shape& s) {
  TrainSaved b;
  const int64_t A = s.tokens * s.top_k;
  b.logits = c.take<uint16_t>(sizeof(uint16_t) * s.tokens * s.experts);
  b.topk_idx = c.take<int32_t>(sizeof(int32_t) * A);
  b.topk_w = c.take<float>(sizeof(float) * A);
  b.counts = c.take<int32_t>(sizeof(int32_t) * s.experts);
  b.pos = c.take<int32_t>(sizeof(int32_t) * A);
  b.aux_counts = c.take<float>(sizeof(float) * s.experts);
  b.x_sorted = c.take<void>(2 * A * s.hidden);
  b.gate_up = c.take<void>(2 * A * 2 * s.intermediate);
  b.h = c.take<void>(2 * A * s.intermediate);
  b.expert_out = c.take<void>(2 * A * s.hidden);
  return b;
}

// Scratch of the training forward and of the backward (one size for both).
struct TrainWs {
  int* err;
  DispatchBufs d;        // forward
  void* router_scratch;  // forward
  float* part_p;         // aux / bias partial sums
  int* part_c;
  float* aux_tmp;        // forward: aux loss when the caller wants none
  int32_t* count_T;      // backward: T, the router GEMMs' one group
  uint16_t* d_logits;    // backward [T, E]
  void* d_eo;            // backward [A, d], later d_x_sorted
  void* d_gu;            // backward [A, 2I]
  void* dx_router;       // backward [T, d]
  float* wr_partial;     // backward: split-K partials of the router wgrad [<= 64, E, d]
};

TrainWs carve_train_ws(Carve& c, const hmoe_shape& s) {
  TrainWs b;
  const int64_t A = s.tokens * s.top_k;
  const int nb = train_partial_blocks(s.tokens);
  b.d = carve_dispatch(c, s);
  b.err = b.d.err;
  b.router_scratch = c.take<void>(router_tc_scratch_bytes(s.tokens));
  b.part_p = c.take<float>(sizeof(float) * nb * s.experts);
  b.part_c = c.take<int>(sizeof(int) * nb * s.experts);
  b.aux_tmp = c.take<float>(sizeof(float));
  b.count_T = c.take<int32_t>(sizeof(int32_t));
  b.d_logits = c.take<uint16_t>(sizeof(uint16_t) * s.tokens * s.experts);
  b.d_eo = c.take<void>(2 * A * s.hidden);
  b.d_gu = c.take<void>(2 * A * 2 * s.intermediate);
  b.dx_router = c.take<void>(2 * s.tokens * s.hidden);
  b.wr_partial = c.take<float>(sizeof(float) * 64 * s.experts * s.hidden);
  return b;
}

int check_train_shape(const hmoe_shape* shape) {
  int rc = validate_shape(shape);
  if (rc) return rc;
  if (shape->dtype != HMOE_DTYPE_BF16)
    return fail(HMOE_EINVAL, "the training path supports bf16 only (the reference's Triton "
                             "backward raises TypeError for other dtypes)");
  if (shape->experts % 8 != 0)
    return fail(HMOE_EINVAL, "the training path needs experts to be a multiple of 8 (got %d)",
                shape->experts);
  return HMOE_OK;
}

}  // namespace

extern "C" {

size_t hmoe_ffn_train_saved_bytes(const hmoe_shape* shape) {
  return plan_bytes(shape, [](Carve& c, const hmoe_shape& s) { carve_saved(c, s); });
}

size_t hmoe_ffn_train_workspace_bytes(const hmoe_shape* shape) {
  return plan_bytes(shape, [](Carve& c, const hmoe_shape& s) { carve_train_ws(c, s); });
}

int hmoe_ffn_forward_train(const hmoe_shape* shape, const void* x, const void* w_router,
                           const void* router_bias, const void* w_gate_up, const void* w_down,
                           void* y, int64_t aux_tokens, float* aux_loss, float* expert_counts,
                           void* saved, size_t saved_bytes, void* workspace,
                           size_t workspace_bytes, void* stream) {
  int rc = check_train_shape(shape);
  if (rc) return rc;
  const hmoe_shape& s = *shape;
  if (aux_tokens > s.tokens) return fail(HMOE_EINVAL, "aux_tokens exceeds tokens");
  if (s.tokens == 0) {
    if (aux_loss && (rc = select_device(aux_loss)) == HMOE_OK)
      HMOE_CUDA(cudaMemsetAsync(aux_loss, 0, sizeof(float), static_cast<cudaStream_t>(stream)),
                "clear aux");
    if (rc) return rc;
    if (expert_counts && (rc = select_device(expert_counts)) == HMOE_OK)
      HMOE_CUDA(cudaMemsetAsync(expert_counts, 0, sizeof(float) * s.experts,
                                static_cast<cudaStream_t>(stream)), "clear counts");
    return rc;
  }
  if (!x || !w_router || !w_gate_up || !w_down || !y)
    return fail(HMOE_EINVAL, "x, w_router, w_gate_up, w_down and y are required");
  if (!aligned16(x) || !aligned16(w_gate_up) || !aligned16(w_down) || !aligned16(y) ||
      !aligned16(w_router))
    return fail(HMOE_EINVAL, "x, weights and y must be 16-byte aligned");
  if ((rc = select_device(x))) return rc;
  if ((rc = check_ws(saved, saved_bytes, hmoe_ffn_train_saved_bytes(shape)))) return rc;
  if ((rc = check_ws(workspace, workspace_bytes, hmoe_ffn_train_workspace_bytes(shape)))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carve cs{static_cast<char*>(saved)};
  const TrainSaved sv = carve_saved(cs, s);
  Carve cw{static_cast<char*>(workspace)};
  const TrainWs w = carve_train_ws(cw, s);
  const int64_t A = s.tokens * s.top_k;
  HMOE_CUDA(cudaMemsetAsync(w.err, 0, sizeof(int), st), "reset error word");
  HMOE_CUDA(run_router(s, x, w_router, router_bias, sv.topk_idx, sv.topk_w, nullptr, sv.logits,
                       w.router_scratch, w.err, st),
            "router_topk");
  rc = run_dispatch(s, sv.topk_idx, sv.topk_w, 1, x, w.d, sv.pos, nullptr, nullptr, nullptr,
                    sv.x_sorted, st);
  if (rc) return rc;
  HMOE_CUDA(cudaMemcpyAsync(sv.counts, w.d.counts, sizeof(int32_t) * s.experts,
                            cudaMemcpyDeviceToDevice, st), "copy counts");
  {
    GroupedGemmArgs g;
    g.a = sv.x_sorted;
    g.b = w_gate_up;
    g.counts = sv.counts;
    g.out = sv.h;
    g.M = A;
    g.N = s.intermediate;
    g.K = s.hidden;
    g.G = s.experts;
    g.swiglu = 1;
    g.dtype = s.dtype;
    g.err = w.err;
    g.sm_limit = 0;
    g.save_gate_up = sv.gate_up;
    HMOE_CUDA(launch_grouped_gemm_pair(g, st), "grouped swiglu (training)");
  }
  rc = run_grouped(sv.h, w_down, sv.counts, A, s.hidden, s.intermediate, s.experts, s.dtype, 0,
                   sv.expert_out, w.err, st);
  if (rc) return rc;
  HMOE_CUDA(launch_combine(sv.expert_out, sv.pos, sv.topk_w, 1, sv.topk_idx, s.experts, s.tokens,
                           s.hidden, s.top_k, s.dtype, nullptr, y, st), "combine");
  // aux statistics over the first aux_tokens tokens (none when negative)
  const int64_t n_aux = aux_tokens < 0 ? 0 : aux_tokens;
  const int nb = train_partial_blocks(s.tokens);
  HMOE_CUDA(launch_aux_stats(sv.logits, sv.topk_idx, n_aux, s.experts, s.top_k, w.part_p,
                             w.part_c, nb, aux_loss ? aux_loss : w.aux_tmp, sv.aux_counts, st),
            "aux statistics");
  if (expert_counts)
    HMOE_CUDA(cudaMemcpyAsync(expert_counts, sv.aux_counts, sizeof(float) * s.experts,
                              cudaMemcpyDeviceToDevice, st), "copy expert counts");
  return HMOE_OK;
}

int hmoe_ffn_backward_marked(const hmoe_shape* shape, const void* grad_y, const float* aux_grad,
                             int64_t aux_tokens, const void* x, const void* w_router,
                             const void* router_bias, const void* w_gate_up, const void* w_down,
                             const void* saved, size_t saved_bytes, void* grad_x,
                             void* grad_w_router, void* grad_router_bias, void* grad_w_gate_up,
                             void* grad_w_down, void* workspace, size_t workspace_bytes,
                             void* stream, void* const* phase_events) {
  PhaseMarks pm;
  pm.ev = phase_events;
  int rc = check_train_shape(shape);
  if (rc) return rc;
  const hmoe_shape& s = *shape;
  if (aux_tokens > s.tokens) return fail(HMOE_EINVAL, "aux_tokens exceeds tokens");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (s.tokens == 0) {
    // no tokens: every parameter gradient is zero
    const void* any = grad_w_gate_up ? grad_w_gate_up : grad_w_down ? grad_w_down : grad_w_router;
    if (!any) return HMOE_OK;
    if ((rc = select_device(any))) return rc;
    const size_t E = s.experts, d = s.hidden, I = s.intermediate;
    if (grad_w_router) HMOE_CUDA(cudaMemsetAsync(grad_w_router, 0, 2 * E * d, st), "zero grad");
    if (grad_router_bias) HMOE_CUDA(cudaMemsetAsync(grad_router_bias, 0, 2 * E, st), "zero grad");
    if (grad_w_gate_up) HMOE_CUDA(cudaMemsetAsync(grad_w_gate_up, 0, 2 * E * 2 * I * d, st), "zero grad");
    if (grad_w_down) HMOE_CUDA(cudaMemsetAsync(grad_w_down, 0, 2 * E * d * I, st), "zero grad");
    return HMOE_OK;
  }
  if (!grad_y || !x || !w_router || !w_gate_up || !w_down || !saved)
    return fail(HMOE_EINVAL, "grad_y, x, the weights and saved are required");
  if (!aligned16(grad_y) || !aligned16(x) || !aligned16(w_router) || !aligned16(w_gate_up) ||
      !aligned16(w_down) || (grad_x && !aligned16(grad_x)) ||
      (grad_w_router && !aligned16(grad_w_router)) ||
      (grad_w_gate_up && !aligned16(grad_w_gate_up)) || (grad_w_down && !aligned16(grad_w_down)))
    return fail(HMOE_EINVAL, "tensors must be 16-byte aligned");
  if (grad_router_bias && !router_bias)
    return fail(HMOE_EINVAL, "grad_router_bias needs the layer's router_bias");
  if ((rc = select_device(grad_y))) return rc;
  if ((rc = check_ws(const_cast<void*>(saved), saved_bytes, hmoe_ffn_train_saved_bytes(shape))))
    return rc;
  if ((rc = check_ws(workspace, workspace_bytes, hmoe_ffn_train_workspace_bytes(shape)))) return rc;
  Carve cs{static_cast<char*>(const_cast<void*>(saved))};
  const TrainSaved sv = carve_saved(cs, s);
  Carve cw{static_cast<char*>(workspace)};
  const TrainWs w = carve_train_ws(cw, s);
  const int64_t A = s.tokens * s.top_k;
  const int E = s.experts, d = s.hidden, I = s.intermediate;
  HMOE_CUDA(cudaMemsetAsync(w.err, 0, sizeof(int), st), "reset error word");
  if ((rc = pm.mark(0, st))) return rc;
  // 1. combine and router backward: d_expert_out rows, d_logits
  HMOE_CUDA(launch_combine_router_bwd(grad_y, sv.expert_out, sv.pos, sv.topk_idx, sv.topk_w,
                                      sv.logits, s.tokens, d, s.top_k, E, s.norm_topk_prob,
                                      aux_grad, sv.aux_counts, aux_tokens < 0 ? 0 : aux_tokens,
                                      w.d_eo, w.d_logits, w.count_T, st),
            "combine/router backward");
  if ((rc = pm.mark(1, st))) return rc;
  // 2. down projection dgrad fused with the SiLU(gate) * up backward -> d_gate_up
  {
    GroupedDgradArgs a;
    a.grad_out = w.d_eo;
    a.weight = w_down;  // [E, d, I]: contraction over d
    a.counts = sv.counts;
    a.out = nullptr;
    a.gate_up = sv.gate_up;
    a.d_gate_up = w.d_gu;
    a.M = A;
    a.Kc = d;
    a.Nout = I;
    a.G = E;
    a.err = w.err;
    a.sm_limit = 0;
    HMOE_CUDA(launch_grouped_dgrad(a, st), "down dgrad + SwiGLU backward");
  }
  if ((rc = pm.mark(2, st))) return rc;
  // 3. down projection wgrad: d_w_down[e] = d_eo[e]^T @ h[e]
  if (grad_w_down) {
    GroupedWgradArgs a;
    a.grad_out = w.d_eo;
    a.input = sv.h;
    a.counts = sv.counts;
    a.out = grad_w_down;
    a.M = A;
    a.Mw = d;
    a.Nw = I;
    a.G = E;
    a.err = w.err;
    a.sm_limit = 0;
    HMOE_CUDA(launch_grouped_wgrad(a, st), "down wgrad");
  }
  if ((rc = pm.mark(3, st))) return rc;
  // 4. gate_up dgrad: d_x_sorted = d_gate_up @ w_gate_up[e] (into d_eo's buffer)
  void* d_xs = w.d_eo;
  if (grad_x) {
    GroupedDgradArgs a;
    a.grad_out = w.d_gu;
    a.weight = w_gate_up;  // [E, 2I, d]: contraction over 2I
    a.counts = sv.counts;
    a.out = d_xs;
    a.M = A;
    a.Kc = 2 * I;
    a.Nout = d;
    a.G = E;
    a.err = w.err;
    a.sm_limit = 0;
    HMOE_CUDA(launch_grouped_dgrad(a, st), "gate_up dgrad");
  }
  if ((rc = pm.mark(4, st))) return rc;
  // 5. gate_up wgrad: d_w_gate_up[e] = d_gate_up[e]^T @ x_sorted[e]
  if (grad_w_gate_up) {
    GroupedWgradArgs a;
    a.grad_out = w.d_gu;
    a.input = sv.x_sorted;
    a.counts = sv.counts;
    a.out = grad_w_gate_up;
    a.M = A;
    a.Mw = 2 * I;
    a.Nw = d;
    a.G = E;
    a.err = w.err;
    a.sm_limit = 0;
    HMOE_CUDA(launch_grouped_wgrad(a, st), "gate_up wgrad");
  }
  if ((rc = pm.mark(5, st))) return rc;
  // 6. router: dx_router = d_logits @ w_router, d_w_router = d_logits^T @ x, d_bias
  if (grad_x) {
    GroupedDgradArgs a;
    a.grad_out = w.d_logits;
    a.weight = w_router;  // [1, E, d]
    a.counts = w.count_T;
    a.out = w.dx_router;
    a.M = s.tokens;
    a.Kc = E;
    a.Nout = d;
    a.G = 1;
    a.err = w.err;
    a.sm_limit = 0;
    HMOE_CUDA(launch_grouped_dgrad(a, st), "router dgrad");
    HMOE_CUDA(launch_dx(d_xs, sv.pos, w.dx_router, s.tokens, d, s.top_k, grad_x, st), "dx");
  }
  if ((rc = pm.mark(6, st))) return rc;
  if (grad_w_router) {
    GroupedWgradArgs a;
    a.grad_out = w.d_logits;
    a.input = x;
    a.counts = w.count_T;
    a.out = grad_w_router;
    a.M = s.tokens;
    a.Mw = E;
    a.Nw = d;
    a.G = 1;
    a.err = w.err;
    a.sm_limit = 0;
    // E x d is only a few output tiles: split the tokens (fp32 partials,
    // summed in order, one rounding)
    a.ksplit = wgrad_ksplit(s.tokens, E, d, 1);
    a.partial = w.wr_partial;
    HMOE_CUDA(launch_grouped_wgrad(a, st), "router wgrad");
  }
  if (grad_router_bias)
    HMOE_CUDA(launch_colsum_bf16(w.d_logits, s.tokens, E, w.part_p,
                                 train_partial_blocks(s.tokens), grad_router_bias, st),
              "router bias grad");
  return pm.mark(7, st);
}

int hmoe_ffn_backward(const hmoe_shape* shape, const void* grad_y, const float* aux_grad,
                      int64_t aux_tokens, const void* x, const void* w_router,
                      const void* router_bias, const void* w_gate_up, const void* w_down,
                      const void* saved, size_t saved_bytes, void* grad_x, void* grad_w_router,
                      void* grad_router_bias, void* grad_w_gate_up, void* grad_w_down,
                      void* workspace, size_t workspace_bytes, void* stream) {
  return hmoe_ffn_backward_marked(shape, grad_y, aux_grad, aux_tokens, x, w_router, router_bias,
                                  w_gate_up, w_down, saved, saved_bytes, grad_x, grad_w_router,
                                  grad_router_bias, grad_w_gate_up, grad_w_down, workspace,
                                  workspace_bytes, stream, nullptr);
}

int hmoe_workspace_status(const void* workspace, void* stream) {
  if (!workspace) return fail(HMOE_EINVAL, "workspace is NULL");
  int rc = select_device(workspace);
  if (rc) return rc;
  int word = 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  HMOE_CUDA(cudaMemcpyAsync(&word, workspace, sizeof(int), cudaMemcpyDeviceToHost, st),
            "read error word");
  HMOE_CUDA(cudaStreamSynchronize(st), "cudaStreamSynchronize");
  if (word == kDevBadExpert) return fail(HMOE_EINVAL, "an expert id outside [0, experts) was dropped");
  if (word == kDevTimeout) return fail(HMOE_ETIMEDOUT, "a device-side wait gave up");
  if (word == kDevEpOverflow)
    return fail(HMOE_EIO, "expert-parallel counts exceeded the symmetric buffers");
  if (word != kDevOk) return fail(HMOE_EIO, "unknown device error word %d", word);
  return HMOE_OK;
}

unsigned hmoe_set_pdl_mask(unsigned mask) {
  return hmoe::pdl_mask().exchange(mask & (hmoe::kPdlRouter | hmoe::kPdlDispatch | hmoe::kPdlGemm |
                                           hmoe::kPdlCombine));
}

}  // extern "C"
