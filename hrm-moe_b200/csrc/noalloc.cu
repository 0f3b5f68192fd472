// hmoe_dispatch_noalloc: the dispatch stage (stable expert sort, counts,
// gather) with its scratch in a fixed device array instead of a caller
// workspace.
//
// Some hosts that embed this library cannot hand it device memory for
// scratch: a plugin whose host language has no CUDA allocator binding, a
// serving loop whose device memory is fully reserved up front by another
// framework's caching allocator (so a fresh cudaMalloc can fail even though
// that framework holds free blocks), or a real-time path with a
// no-allocation-after-start-up rule.  They still own the inputs and
// outputs; only the scratch moves here.
//
// The scratch is one file-scope __device__ array of kScratchBytes (about
// 2.3 MiB).  Every GPU that loads the library holds its own copy until the
// process exits.  In host code the array's name is only a host-side stand-in,
// never a device address, so the first call on each device (with that device
// current) looks the real address up with cudaGetSymbolAddress and caches
// it per CUDA context (a context of its own, or one made after
// cudaDeviceReset(), gets a fresh lookup); make the first call in each
// context before any stream capture.  All calls on a device
// share the array and it keeps the last call's contents; the kernels below
// write every scratch word they later read, so nothing needs clearing, but
// two calls that overlap on the GPU (different streams, no ordering between
// them) race on it.  Expert ids outside [0, E) are dropped; this variant has
// no error word to report them.
#include <mutex>

#include "common.cuh"
#include "hrm_moe.h"
#include "internal.h"

namespace {

constexpr int64_t kMaxAssign = HMOE_DISPATCH_NOALLOC_MAX_ASSIGNMENTS;
constexpr int64_t kMaxBlocks = 512;
constexpr int64_t kMaxExperts = 128;
constexpr size_t align256(size_t x) { return (x + 255) / 256 * 256; }
constexpr size_t kOffRank = 0;
constexpr size_t kOffPos = align256(kOffRank + sizeof(int32_t) * kMaxAssign);
constexpr size_t kOffBlocks = align256(kOffPos + sizeof(int32_t) * kMaxAssign);
constexpr size_t kOffCounts = align256(kOffBlocks + sizeof(int32_t) * kMaxBlocks * kMaxExperts);
constexpr size_t kOffOffsets = align256(kOffCounts + sizeof(int32_t) * kMaxExperts);
constexpr size_t kScratchBytes = align256(kOffOffsets + sizeof(int32_t) * (kMaxExperts + 1));

static __device__ __align__(256) unsigned char g_dispatch_scratch[kScratchBytes];

// Device address of the scratch array in the CUDA context current on the
// calling thread.  A __device__ symbol has one address per context (each
// context loads its own copy of the module), so the cache is keyed by the
// context's unique id (cuCtxGetId), not by the device ordinal: a host that
// makes its own context current, or a context created after
// cudaDeviceReset(), gets its own lookup instead of a stale address.
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

struct CtxFns {
  CtxGetCurrentFn get_current = nullptr;
  CtxGetIdFn get_id = nullptr;
};

const CtxFns& ctx_fns() {
  static CtxFns fns;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess && q == cudaDriverEntryPointSuccess)
      fns.get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess && q == cudaDriverEntryPointSuccess)
      fns.get_id = reinterpret_cast<CtxGetIdFn>(p);
  });
  return fns;
}

int scratch_address(char** out) {
  constexpr int kSlots = 64;
  struct Slot {
    unsigned long long ctx_id;
    char* addr;
  };
  static Slot slots[kSlots] = {};
  static int next = 0;
  static std::mutex mu;
  const CtxFns& f = ctx_fns();
  if (!f.get_current || !f.get_id)
    return hmoe::report_error(HMOE_EIO, "cuCtxGetCurrent / cuCtxGetId are not available");
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (f.get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr || f.get_id(ctx, &id) != CUDA_SUCCESS)
    return hmoe::report_error(HMOE_EIO, "no current CUDA context for the dispatch scratch");
  std::lock_guard<std::mutex> lock(mu);
  for (const Slot& s : slots)
    if (s.addr && s.ctx_id == id) {
      *out = s.addr;
      return HMOE_OK;
    }
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_dispatch_scratch);
  if (e != cudaSuccess || p == nullptr)
    return hmoe::report_error(HMOE_EIO, "cudaGetSymbolAddress(dispatch scratch): %s",
                              cudaGetErrorString(e));
  slots[next] = Slot{id, static_cast<char*>(p)};
  next = (next + 1) % kSlots;
  *out = static_cast<char*>(p);
  return HMOE_OK;
}

}  // namespace

extern "C" int hmoe_dispatch_noalloc(const hmoe_shape* shape, const int32_t* topk_idx,
                                     const void* topk_weight, const void* x, int32_t* sort_idx,
                                     int32_t* counts, int32_t* sorted_token, void* sorted_weight,
                                     void* x_sorted, void* stream) {
  using namespace hmoe;
  int rc = validate_shape_public(shape);
  if (rc) return rc;
  const hmoe_shape& s = *shape;
  const int64_t A = s.tokens * s.top_k;
  if (A > kMaxAssign)
    return report_error(HMOE_EINVAL,
                        "hmoe_dispatch_noalloc handles at most %lld assignments (tokens * top_k), "
                        "got %lld; use hmoe_dispatch with a workspace",
                        static_cast<long long>(kMaxAssign), static_cast<long long>(A));
  const int64_t nblk = dispatch_num_blocks(s.tokens, s.top_k);
  if (nblk > kMaxBlocks)
    return report_error(HMOE_EINVAL, "hmoe_dispatch_noalloc: %lld histogram blocks exceed %lld",
                        static_cast<long long>(nblk), static_cast<long long>(kMaxBlocks));
  if (s.tokens == 0) {
    // no assignments: tokens_per_expert is E zeros (bincount with minlength=E)
    if (!counts) return HMOE_OK;
    if ((rc = make_device_current(counts))) return rc;
    const cudaError_t e = cudaMemsetAsync(counts, 0, sizeof(int32_t) * s.experts,
                                          static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return report_error(HMOE_EIO, "clear counts: %s", cudaGetErrorString(e));
    return HMOE_OK;
  }
  if (!topk_idx || !sort_idx) return report_error(HMOE_EINVAL, "topk_idx and sort_idx are required");
  if (sorted_weight && !topk_weight)
    return report_error(HMOE_EINVAL, "sorted_weight needs topk_weight");
  if (x_sorted && (!x || (reinterpret_cast<uintptr_t>(x) & 15u) ||
                   (reinterpret_cast<uintptr_t>(x_sorted) & 15u)))
    return report_error(HMOE_EINVAL, "x_sorted needs 16-byte aligned x and x_sorted");
  if ((rc = make_device_current(topk_idx))) return rc;
  char* base = nullptr;
  if ((rc = scratch_address(&base))) return rc;
  cudaError_t e;
  int32_t* local_rank = reinterpret_cast<int32_t*>(base + kOffRank);
  int32_t* pos = reinterpret_cast<int32_t*>(base + kOffPos);
  int32_t* blocks = reinterpret_cast<int32_t*>(base + kOffBlocks);
  int32_t* cnt = reinterpret_cast<int32_t*>(base + kOffCounts);
  int32_t* offs = reinterpret_cast<int32_t*>(base + kOffOffsets);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((e = launch_hist_rank(topk_idx, s.tokens, s.top_k, s.experts, local_rank, blocks, nullptr,
                            st)) != cudaSuccess ||
      (e = launch_scan(blocks, nblk, s.experts, cnt, offs, st)) != cudaSuccess ||
      (e = launch_permute_gather(topk_idx, local_rank, blocks, cnt, topk_weight, 0, x, s.tokens,
                                 s.hidden, s.top_k, s.experts, s.dtype, pos, sort_idx,
                                 sorted_token, sorted_weight, x_sorted, st)) != cudaSuccess)
    return report_error(HMOE_EIO, "dispatch_noalloc launch: %s", cudaGetErrorString(e));
  if (counts) {
    e = cudaMemcpyAsync(counts, cnt, sizeof(int32_t) * s.experts, cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return report_error(HMOE_EIO, "copy counts: %s", cudaGetErrorString(e));
  }
  return HMOE_OK;
}
