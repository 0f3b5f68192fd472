// Expert parallelism over peer memory (NVLink / NVSwitch), no host sync.
//
// Mirrors SparseMoEExpertParallel.forward (models/layers.py:427-478): rank r
// owns experts [r*El, (r+1)*El) (layers.py:403-405); each rank routes its own
// tokens, sends every routed row to the owner of its expert, the owner runs
// its experts, and the outputs come back to be combined in token order.
//
// Instead of host-driven all_to_all calls (layers.py:360-380, which read the
// split sizes on the host), every rank holds one "symmetric" region of the
// same layout, mapped into all ranks by CUDA IPC, and the kernels move the
// data with plain NVLink loads/stores:
//   ep_exchange  writes this rank's per-expert counts into every peer's
//                mailbox, raises its flag there, waits (bounded) for every
//                peer's counts, then derives where its rows go in each
//                owner's receive buffer and how many rows it will receive.
//   ep_dispatch  one warp per token: the token's row is read once and stored
//                straight into the owners' receive buffers (expert-major:
//                local expert, then source rank, then the source's stable
//                order), with the row's origin alongside; the last CTA raises
//                the "dispatched" flag at every peer.
//   ep_wait      bounded wait for a flag from every peer.
//   (gate_up grouped GEMM on the receive buffer: El groups, plain counts)
//   down GEMM    bf16: the grouped GEMM's epilogue stores each result row
//                straight back into its source rank's region, at the position
//                the source's own dispatch gave it, so the return transfer
//                runs under the GEMM's math; its last CTA raises "returned"
//                at every peer.  fp32 layers run the GEMM into local memory
//                and ep_return copies the rows back.
//   (the single-GPU combine on the returned rows)
// A row thus meets exactly the kernels and the order it meets on one GPU, so
// the result is bit-identical to one GPU running all experts.
//
// Flags hold call epochs (strictly increasing per call, same on all ranks).
// Every wait gives up after kWaitLimitNs, recording kDevTimeout in the
// error word; no wait is unbounded.  Once the error word is set, the kernels
// store nothing into peer memory and raise no flag, so the peers' waits run
// out as well and every rank reports the failure; every index into a peer's
// region is also checked against its capacity.  No multicast or NVLS is used.
#include "common.cuh"
#include "hrm_moe.h"
#include "internal.h"

namespace hmoe {
namespace {

constexpr int kEpMaxRanks = 8;
constexpr uint32_t kSrcShift = kEpSrcShift;  // recv_src = (src << 28) | source position
constexpr uint32_t kPosMask = (1u << kSrcShift) - 1u;

enum FlagKind { kFlagCounts = 0, kFlagDispatched = 1, kFlagReturned = 2 };

struct Peers {
  char* base[kEpMaxRanks];
};

struct EpOffsets {
  size_t flags, mailbox, arrived, recv_src, recv_rows, y_back;
};

__device__ __forceinline__ int read_err(const int* err) {
  return *reinterpret_cast<const volatile int*>(err);
}

__host__ __device__ __forceinline__ uint32_t* flag_ptr(char* base, const EpOffsets& o, int kind,
                                                       int src) {
  return reinterpret_cast<uint32_t*>(base + o.flags) + kind * kEpMaxRanks + src;
}

// Bounded wait until every rank's flag of `kind` in my region reached epoch.
__device__ bool wait_flags(char* mine, const EpOffsets& o, int kind, int world, uint32_t epoch,
                           int* err) {
  bool ok = true;
  if (threadIdx.x < world) {
    const uint32_t* f = flag_ptr(mine, o, kind, threadIdx.x);
    const unsigned long long t0 = global_timer_ns();
    while (static_cast<int32_t>(ld_acquire_sys(f) - epoch) < 0) {
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        record_error(err, kDevTimeout);
        ok = false;
        break;
      }
    }
  }
  return __syncthreads_and(ok);
}

// Every CTA fences its stores; the last CTA to finish raises `kind` at all
// ranks, unless the call has failed.
__device__ void signal_when_all_done(const Peers& peers, const EpOffsets& o, int kind, int me,
                                     int world, uint32_t epoch, unsigned* done, const int* err) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(done, 1u);
    if (prev == gridDim.x - 1 && read_err(err) == kDevOk) {
      __threadfence_system();
      for (int p = 0; p < world; ++p) st_release_sys(flag_ptr(peers.base[p], o, kind, me), epoch);
    }
  }
}

// Tables this rank derives from the full count matrix cnt[src][expert].
struct EpTables {
  int32_t* send_base;   // [E]  first row in the owner's receive buffer for my rows of e
  int32_t* recv_count;  // [El] rows I receive per local expert (the GEMM groups)
  int32_t* recv_total;  // [1]
};

// One CTA.  Always leaves usable tables: on any failure send_base is -1 (no
// row is sent) and the receive counts are 0 (no GEMM rows, nothing returned).
__global__ void __launch_bounds__(256)
ep_exchange_kernel(const int32_t* __restrict__ counts, int E, int me, int world, Peers peers,
                   EpOffsets o, uint32_t epoch, int64_t max_recv, EpTables tab, int* err) {
  __shared__ int32_t cnt[kEpMaxRanks][128];
  const int El = E / world;
  char* mine = peers.base[me];
  // No peer sends rows of this call before it has seen this rank's counts
  // flag, and every row of the previous call has landed (the previous
  // gate_up GEMM waited for them): the arrival counters can restart here.
  for (int el = threadIdx.x; el < El; el += blockDim.x)
    reinterpret_cast<uint32_t*>(mine + o.arrived)[el] = 0;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    tab.send_base[e] = -1;
    if (e < El) tab.recv_count[e] = 0;
  }
  if (threadIdx.x == 0) *tab.recv_total = 0;
  if (read_err(err) != kDevOk) return;
  for (int i = threadIdx.x; i < world * E; i += blockDim.x) {
    const int p = i / E, e = i % E;
    reinterpret_cast<int32_t*>(peers.base[p] + o.mailbox)[me * E + e] = counts[e];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < world) st_release_sys(flag_ptr(peers.base[threadIdx.x], o, kFlagCounts, me), epoch);
  if (!wait_flags(mine, o, kFlagCounts, world, epoch, err)) return;
  int bad = 0;
  for (int i = threadIdx.x; i < world * E; i += blockDim.x) {
    const int32_t c = reinterpret_cast<volatile int32_t*>(mine + o.mailbox)[i];
    bad |= c < 0;
    cnt[i / E][i % E] = c;
  }
  __syncthreads();
  // every owner's receive buffer holds at most max_recv rows
  if (threadIdx.x < world) {
    int64_t tot = 0;
    for (int e = threadIdx.x * El; e < (threadIdx.x + 1) * El; ++e)
      for (int s = 0; s < world; ++s) tot += cnt[s][e];
    bad |= tot > max_recv;
  }
  if (__syncthreads_or(bad)) {
    record_error(err, kDevEpOverflow);
    return;
  }
  // rows per (owner, local expert) summed over sources, prefix inside each owner
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int owner = e / El, el = e % El;
    int base = 0;
    for (int e2 = owner * El; e2 < owner * El + el; ++e2)
      for (int s = 0; s < world; ++s) base += cnt[s][e2];
    for (int s = 0; s < me; ++s) base += cnt[s][e];
    tab.send_base[e] = base;
    if (owner == me) {
      int r = 0;
      for (int s = 0; s < world; ++s) r += cnt[s][e];
      tab.recv_count[el] = r;
    }
  }
  if (threadIdx.x == 0) {
    int tot = 0;
    for (int e = me * El; e < (me + 1) * El; ++e)
      for (int s = 0; s < world; ++s) tot += cnt[s][e];
    *tab.recv_total = tot;
  }
}

constexpr int kEpThreads = 256;
constexpr int kEpSeg = 8;

__global__ void __launch_bounds__(kEpThreads)
ep_dispatch_kernel(const int32_t* __restrict__ topk_idx, const int32_t* __restrict__ local_rank,
                   const int32_t* __restrict__ block_offsets, const int32_t* __restrict__ counts,
                   const int32_t* __restrict__ send_base, const uint4* __restrict__ x, int64_t T,
                   int row_chunks, int k, int E, int tblk, int me, int world, Peers peers,
                   EpOffsets o, uint32_t epoch, int64_t max_recv, int32_t* __restrict__ pos,
                   unsigned* done, int* err) {
  __shared__ int32_t base[129];
  const bool failed = read_err(err) != kDevOk;
  if (threadIdx.x < 32) {  // exclusive scan of my counts: my expert bases
    const int lane = threadIdx.x;
    int c[4], s = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = lane * 4 + i;
      c[i] = e < E ? counts[e] : 0;
      s += c[i];
    }
    int incl = s;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += v;
    }
    int run = incl - s;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (lane * 4 + i < 128) base[lane * 4 + i] = run;
      run += c[i];
    }
  }
  __syncthreads();
  const int El = E / world;
  const int lane = threadIdx.x & 31;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * (kEpThreads / 32) + (threadIdx.x >> 5);
  if (t < T) {
    const int64_t blk = t / tblk;
    int q = -1, dst = 0;
    if (lane < k) {
      const int64_t f = t * k + lane;
      const int e = topk_idx[f];
      const int r = local_rank[f];
      int p = -1;
      if (!failed && e >= 0 && e < E && r >= 0 && send_base[e] >= 0) {
        const int rel = block_offsets[blk * E + e] + r;  // rank among my rows of e
        const int64_t qq = static_cast<int64_t>(send_base[e]) + rel;
        if (qq < max_recv) {
          p = base[e] + rel;
          dst = e / El;
          q = static_cast<int>(qq);
          reinterpret_cast<int32_t*>(peers.base[dst] + o.recv_src)[q] = static_cast<int32_t>(
              (static_cast<uint32_t>(me) << kSrcShift) | static_cast<uint32_t>(p));
        } else {
          record_error(err, kDevEpOverflow);
        }
      }
      pos[f] = p;
    }
    const uint4* src = x + t * row_chunks;
    const bool any = __any_sync(0xffffffffu, q >= 0);
    for (int c0 = 0; any && c0 < row_chunks; c0 += 32 * kEpSeg) {
      uint4 buf[kEpSeg];
#pragma unroll
      for (int s = 0; s < kEpSeg; ++s) {
        const int c = c0 + s * 32 + lane;
        if (c < row_chunks) buf[s] = __ldg(src + c);
      }
      for (int j = 0; j < k; ++j) {
        const int qj = __shfl_sync(0xffffffffu, q, j);
        const int dj = __shfl_sync(0xffffffffu, dst, j);
        if (qj < 0) continue;
        uint4* out = reinterpret_cast<uint4*>(peers.base[dj] + o.recv_rows) +
                     static_cast<int64_t>(qj) * row_chunks;
#pragma unroll
        for (int s = 0; s < kEpSeg; ++s) {
          const int c = c0 + s * 32 + lane;
          if (c < row_chunks) out[c] = buf[s];
        }
      }
    }
  }
  signal_when_all_done(peers, o, kFlagDispatched, me, world, epoch, done, err);
}

__global__ void __launch_bounds__(32)
ep_wait_kernel(int kind, int me, int world, Peers peers, EpOffsets o, uint32_t epoch, int* err) {
  wait_flags(peers.base[me], o, kind, world, epoch, err);
}

__global__ void __launch_bounds__(kEpThreads)
ep_return_kernel(const uint4* __restrict__ y_recv, const int32_t* __restrict__ recv_total,
                 int row_chunks, int me, int world, Peers peers, EpOffsets o, uint32_t epoch,
                 int64_t max_recv, int64_t max_send, unsigned* done, int* err) {
  const int lane = threadIdx.x & 31;
  const int64_t total = *recv_total;
  const int n = read_err(err) == kDevOk ? static_cast<int>(total < max_recv ? total : max_recv) : 0;
  const int32_t* rsrc = reinterpret_cast<const int32_t*>(peers.base[me] + o.recv_src);
  const int warps = gridDim.x * (kEpThreads / 32);
  for (int q = blockIdx.x * (kEpThreads / 32) + (threadIdx.x >> 5); q < n; q += warps) {
    const uint32_t v = static_cast<uint32_t>(rsrc[q]);
    const int s = static_cast<int>(v >> kSrcShift);
    const int64_t p = v & kPosMask;
    if (s >= world || p >= max_send) {
      if (lane == 0) record_error(err, kDevEpOverflow);
      continue;
    }
    uint4* out = reinterpret_cast<uint4*>(peers.base[s] + o.y_back) + p * row_chunks;
    const uint4* in = y_recv + static_cast<int64_t>(q) * row_chunks;
    for (int c = lane; c < row_chunks; c += 32) out[c] = __ldg(in + c);
  }
  signal_when_all_done(peers, o, kFlagReturned, me, world, epoch, done, err);
}

size_t al(size_t x) { return (x + 1023) / 1024 * 1024; }

EpOffsets ep_offsets(int64_t max_tokens, int d, int E, int k, int world, int es) {
  EpOffsets o;
  const size_t max_recv = static_cast<size_t>(world) * max_tokens * k;
  const size_t max_send = static_cast<size_t>(max_tokens) * k;
  size_t off = 0;
  o.flags = off;
  off = al(off + sizeof(uint32_t) * 3 * kEpMaxRanks);
  o.mailbox = off;
  off = al(off + sizeof(int32_t) * kEpMaxRanks * E);
  o.arrived = off;  // rows landed per local expert (fused dispatch)
  off = al(off + sizeof(uint32_t) * 128);
  o.recv_src = off;
  off = al(off + sizeof(int32_t) * max_recv);
  o.recv_rows = off;
  off = al(off + static_cast<size_t>(es) * d * max_recv);
  o.y_back = off;
  off = al(off + static_cast<size_t>(es) * d * max_send);
  (void)off;
  return o;
}

size_t ep_sym_bytes(int64_t max_tokens, int d, int E, int k, int world, int es) {
  const EpOffsets o = ep_offsets(max_tokens, d, E, k, world, es);
  return al(o.y_back + static_cast<size_t>(es) * d * max_tokens * k);
}

}  // namespace

// ------------------------------------------------------------------- host --
struct EpWs {
  int* err;
  int32_t* topk_idx;
  float* topk_w;
  void* router_scratch;
  int32_t* local_rank;
  int32_t* sorted_token;  // [A] token of each expert-sorted row (fused dispatch)
  int32_t* block_counts;
  int32_t* counts;
  int32_t* pos;
  int32_t* send_base;
  int32_t* recv_count;
  int32_t* recv_total;
  unsigned* done;  // 2 counters
  void* h;         // [max_recv, I]
  void* y_recv;    // [max_recv, d], fp32 layers only (bf16 returns from the GEMM)
  size_t total;
};

static EpWs ep_ws(char* base, const hmoe_shape& s, int64_t max_tokens, int world) {
  EpWs w;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    char* p = base ? base + off : nullptr;
    off = al(off + bytes);
    return p;
  };
  const int64_t A = s.tokens * s.top_k;
  const int64_t max_recv = static_cast<int64_t>(world) * max_tokens * s.top_k;
  const size_t es = s.dtype == kDtypeBF16 ? 2 : 4;
  w.err = reinterpret_cast<int*>(take(sizeof(int)));
  w.topk_idx = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * A));
  w.topk_w = reinterpret_cast<float*>(take(sizeof(float) * A));
  w.router_scratch = take(router_tc_scratch_bytes(s.tokens));
  w.local_rank = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * A));
  w.sorted_token = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * A));
  w.block_counts = reinterpret_cast<int32_t*>(
      take(sizeof(int32_t) * dispatch_num_blocks(s.tokens, s.top_k) * s.experts));
  w.counts = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * s.experts));
  w.pos = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * A));
  w.send_base = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * s.experts));
  w.recv_count = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * s.experts));
  w.recv_total = reinterpret_cast<int32_t*>(take(sizeof(int32_t)));
  w.done = reinterpret_cast<unsigned*>(take(sizeof(unsigned) * 2));
  w.h = take(es * s.intermediate * max_recv);
  w.y_recv = take(s.dtype == kDtypeBF16 ? 0 : es * s.hidden * max_recv);
  w.total = off;
  return w;
}

size_t ep_symmetric_bytes(const hmoe_shape& s, int64_t max_tokens, int world) {
  return ep_sym_bytes(max_tokens, s.hidden, s.experts, s.top_k, world, s.dtype == kDtypeBF16 ? 2 : 4);
}

size_t ep_workspace_bytes(const hmoe_shape& s, int64_t max_tokens, int world) {
  return ep_ws(nullptr, s, max_tokens, world).total;
}

cudaError_t ep_forward_launch(const hmoe_shape& s, int64_t max_tokens, int rank, int world,
                              void* const* peer_bases, uint32_t epoch, const void* x,
                              const void* w_router, const void* bias, const void* w_gate_up,
                              const void* w_down, void* y, void* workspace, cudaStream_t st,
                              const cudaEvent_t* marks) {
  cudaError_t e;
  auto mark = [&](int i) { return marks ? cudaEventRecord(marks[i], st) : cudaSuccess; };
  if ((e = mark(0)) != cudaSuccess) return e;
  EpWs w = ep_ws(static_cast<char*>(workspace), s, max_tokens, world);
  Peers peers;
  for (int p = 0; p < kEpMaxRanks; ++p)
    peers.base[p] = p < world ? static_cast<char*>(peer_bases[p]) : nullptr;
  const int es = s.dtype == kDtypeBF16 ? 2 : 4;
  const EpOffsets o = ep_offsets(max_tokens, s.hidden, s.experts, s.top_k, world, es);
  const int El = s.experts / world;
  const int64_t max_recv = static_cast<int64_t>(world) * max_tokens * s.top_k;
  const int row_chunks = s.hidden * es / 16;
  if ((e = cudaMemsetAsync(w.err, 0, sizeof(int), st)) != cudaSuccess) return e;
  if ((e = cudaMemsetAsync(w.done, 0, 2 * sizeof(unsigned), st)) != cudaSuccess) return e;
  if (s.tokens > 0) {
    e = s.dtype == kDtypeBF16
            ? launch_router_topk_tc(x, w_router, bias, s.tokens, s.hidden, s.experts, s.top_k,
                                    s.norm_topk_prob, w.topk_idx, w.topk_w, nullptr, nullptr,
                                    w.router_scratch, w.err, st)
            : launch_router_topk(x, w_router, bias, s.tokens, s.hidden, s.experts, s.top_k,
                                 s.dtype, s.norm_topk_prob, w.topk_idx, w.topk_w, nullptr, nullptr,
                                 st);
    if (e != cudaSuccess) return e;
    if ((e = launch_hist_rank(w.topk_idx, s.tokens, s.top_k, s.experts, w.local_rank,
                              w.block_counts, w.err, st)) != cudaSuccess)
      return e;
    if ((e = launch_scan(w.block_counts, dispatch_num_blocks(s.tokens, s.top_k), s.experts,
                         w.counts, nullptr, st)) != cudaSuccess)
      return e;
  } else if ((e = cudaMemsetAsync(w.counts, 0, sizeof(int32_t) * s.experts, st)) != cudaSuccess) {
    return e;
  }
  const bool fused = s.dtype == kDtypeBF16;
  if (fused && s.tokens > 0) {
    // positions for the combine and the token of each sorted row for the senders
    if ((e = launch_permute_gather(w.topk_idx, w.local_rank, w.block_counts, w.counts, nullptr, 1,
                                   nullptr, s.tokens, s.hidden, s.top_k, s.experts, s.dtype, w.pos,
                                   nullptr, w.sorted_token, nullptr, nullptr, st)) != cudaSuccess)
      return e;
  }
  if (fused && (e = mark(1)) != cudaSuccess) return e;
  EpTables tab{w.send_base, w.recv_count, w.recv_total};
  ep_exchange_kernel<<<1, 256, 0, st>>>(w.counts, s.experts, rank, world, peers, o, epoch,
                                        max_recv, tab, w.err);
  if ((e = cudaGetLastError()) != cudaSuccess || (e = mark(fused ? 2 : 1)) != cudaSuccess) return e;
  GroupedGemmArgs g;
  g.a = peers.base[rank] + o.recv_rows;
  g.b = w_gate_up;
  g.counts = w.recv_count;
  g.out = w.h;
  g.M = max_recv;
  g.N = s.intermediate;
  g.K = s.hidden;
  g.G = El;
  g.swiglu = 1;
  g.dtype = s.dtype;
  g.err = w.err;
  g.sm_limit = 0;
  if (fused) {
    // one kernel: sender warps store every routed row into its owner's
    // receive buffer while the GEMM runs each group as soon as it is complete
    g.push_x = x;
    g.push_sorted_token = w.sorted_token;
    g.push_counts = w.counts;
    g.push_send_base = w.send_base;
    for (int p = 0; p < world; ++p) {
      g.push_rows[p] = peers.base[p] + o.recv_rows;
      g.push_src[p] = reinterpret_cast<int32_t*>(peers.base[p] + o.recv_src);
      g.push_arrived[p] = reinterpret_cast<uint32_t*>(peers.base[p] + o.arrived);
    }
    g.arrived = reinterpret_cast<const uint32_t*>(peers.base[rank] + o.arrived);
    g.push_A = s.tokens * s.top_k;
    g.push_cap = max_recv;
    g.push_E = s.experts;
    g.push_El = El;
    g.push_world = world;
    g.push_me = rank;
    if ((e = launch_grouped_gemm_sm100(g, st)) != cudaSuccess) return e;
    g.arrived = nullptr;  // the down GEMM below does not wait for rows
  } else {
    const unsigned disp_grid =
        static_cast<unsigned>(s.tokens > 0 ? cdiv64(s.tokens, kEpThreads / 32) : 1);
    ep_dispatch_kernel<<<disp_grid, kEpThreads, 0, st>>>(
        w.topk_idx, w.local_rank, w.block_counts, w.counts, w.send_base,
        static_cast<const uint4*>(x), s.tokens, row_chunks, s.top_k, s.experts,
        dispatch_block_tokens(s.top_k), rank, world, peers, o, epoch, max_recv, w.pos, &w.done[0],
        w.err);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    ep_wait_kernel<<<1, 32, 0, st>>>(kFlagDispatched, rank, world, peers, o, epoch, w.err);
    if ((e = cudaGetLastError()) != cudaSuccess || (e = mark(2)) != cudaSuccess) return e;
    if ((e = launch_grouped_gemm_simt(g, st)) != cudaSuccess) return e;
  }
  if ((e = mark(3)) != cudaSuccess) return e;
  g.a = w.h;
  g.b = w_down;
  g.N = s.hidden;
  g.K = s.intermediate;
  g.swiglu = 0;
  if (fused) {
    // down projection fused with the return: rows go straight to their source
    g.out = nullptr;
    g.scatter_src = reinterpret_cast<const int32_t*>(peers.base[rank] + o.recv_src);
    g.scatter_world = world;
    g.scatter_cap = static_cast<int64_t>(max_tokens) * s.top_k;
    g.done = &w.done[1];
    g.epoch = epoch;
    for (int p = 0; p < world; ++p) {
      g.scatter_base[p] = peers.base[p] + o.y_back;
      g.flag[p] = flag_ptr(peers.base[p], o, kFlagReturned, rank);
    }
    if ((e = launch_grouped_gemm_sm100(g, st)) != cudaSuccess) return e;
  } else {
    g.out = w.y_recv;
    if ((e = launch_grouped_gemm_simt(g, st)) != cudaSuccess) return e;
    ep_return_kernel<<<num_sms_for_current_device() * 4, kEpThreads, 0, st>>>(
        static_cast<const uint4*>(w.y_recv), w.recv_total, row_chunks, rank, world, peers, o,
        epoch, max_recv, static_cast<int64_t>(max_tokens) * s.top_k, &w.done[1], w.err);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  ep_wait_kernel<<<1, 32, 0, st>>>(kFlagReturned, rank, world, peers, o, epoch, w.err);
  if ((e = cudaGetLastError()) != cudaSuccess || (e = mark(4)) != cudaSuccess) return e;
  if (s.tokens > 0 &&
      (e = launch_combine(peers.base[rank] + o.y_back, w.pos, w.topk_w, 1, w.topk_idx, s.experts,
                          s.tokens, s.hidden, s.top_k, s.dtype, nullptr, y, st)) != cudaSuccess)
    return e;
  return mark(5);
}

}  // namespace hmoe
