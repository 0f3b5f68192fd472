// Dispatch: stable sort of the T*k assignments by expert, counts, gather.
//
// Mirrors models/layers.py:311-322 of HRM-MoE:
//   flat_experts = selected_experts.reshape(-1)
//   sorted_experts, sort_idx = torch.sort(flat_experts, stable=True)
//   sorted_hidden_states = hidden_states.index_select(0, sort_idx // k)
//   tokens_per_expert = bincount(sorted_experts)
//
// Positions are computed without atomics, so they equal the stable sort:
//  1. hist_rank: each block of tokens counts its assignments per expert and
//     gives every assignment its rank among same-expert assignments of the
//     block with a smaller flat index (warp __match_any_sync + chunk scan).
//  2. scan (one CTA per expert): block counts -> row offset of (expert,
//     block) inside the expert, plus tokens_per_expert.
//  3. permute_gather: position = base(expert) + offset(expert, block) + rank
//     (each CTA scans the E counts for the bases); one warp per token reads
//     its hidden row once and writes it to its k positions.
#include "common.cuh"
#include "internal.h"

namespace hmoe {
namespace {

constexpr int kHistThreads = 256;
constexpr int kHistFlat = 1024;          // assignments per histogram block
constexpr int kHistChunks = kHistFlat / 32;
constexpr int kMaxExperts = 128;

__global__ void __launch_bounds__(kHistThreads)
hist_rank_kernel(const int32_t* __restrict__ topk_idx, int64_t T, int k, int E, int tblk,
                 int32_t* __restrict__ local_rank, int32_t* __restrict__ block_counts,
                 int* __restrict__ err, int32_t* __restrict__ single_counts) {
  __shared__ int32_t cnt[kHistChunks][kMaxExperts];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t f0 = static_cast<int64_t>(blockIdx.x) * tblk * k;  // first flat index
  const int64_t fend = min(static_cast<int64_t>(T) * k, f0 + static_cast<int64_t>(tblk) * k);
  const int nflat = static_cast<int>(fend - f0);
  const int nchunks = cdiv(nflat, 32);

  for (int i = tid; i < kHistChunks * kMaxExperts; i += kHistThreads)
    (&cnt[0][0])[i] = 0;
  __syncthreads();
  grid_dependency_wait();  // launched early (launch_pdl): the routing is written before this
  grid_launch_dependents();

  constexpr int kRounds = kHistChunks / (kHistThreads / 32);  // 4
  int my_e[kRounds], my_rank[kRounds];
#pragma unroll
  for (int r = 0; r < kRounds; ++r) {
    const int c = r * (kHistThreads / 32) + warp;
    const int f = c * 32 + lane;
    int e = -1;
    if (f < nflat) {
      e = topk_idx[f0 + f];
      if (e < 0 || e >= E) {
        record_error(err, kDevBadExpert);
        e = -1;
      }
    }
    const unsigned m = __match_any_sync(0xffffffffu, e);
    my_e[r] = e;
    my_rank[r] = __popc(m & ((1u << lane) - 1u));
    if (e >= 0 && lane == __ffs(m) - 1) cnt[c][e] = __popc(m);
  }
  __syncthreads();
  // exclusive scan over chunks, per expert
  if (tid < E) {
    int run = 0;
    for (int c = 0; c < nchunks; ++c) {
      const int v = cnt[c][tid];
      cnt[c][tid] = run;
      run += v;
    }
    if (single_counts) {
      // the only block: what the scan would produce (offset 0, total)
      block_counts[tid] = 0;
      single_counts[tid] = run;
    } else {
      block_counts[static_cast<int64_t>(blockIdx.x) * E + tid] = run;
    }
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < kRounds; ++r) {
    const int c = r * (kHistThreads / 32) + warp;
    const int f = c * 32 + lane;
    if (f < nflat) local_rank[f0 + f] = my_e[r] >= 0 ? cnt[c][my_e[r]] + my_rank[r] : -1;
  }
}

// One CTA per expert: exclusive scan of the expert's block counts (in place,
// relative to the expert's first row) and its total -> counts[e].  The
// expert bases (a scan over E totals) are formed where they are used.
constexpr int kScanThreads = 256;
constexpr int kScanPer = 8;  // block counts per thread and pass

__global__ void __launch_bounds__(kScanThreads)
scan_kernel(int32_t* __restrict__ block_counts, int64_t nblk, int E, int32_t* __restrict__ counts) {
  __shared__ int32_t warp_tot[kScanThreads / 32];
  __shared__ int32_t carry_s;
  const int e = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) carry_s = 0;
  __syncthreads();
  grid_dependency_wait();  // launched early (launch_pdl)
  grid_launch_dependents();
  for (int64_t b0 = 0; b0 < nblk; b0 += kScanThreads * kScanPer) {
    int v[kScanPer];
    int sum = 0;
#pragma unroll
    for (int i = 0; i < kScanPer; ++i) {
      const int64_t b = b0 + static_cast<int64_t>(tid) * kScanPer + i;
      v[i] = b < nblk ? block_counts[b * E + e] : 0;
      sum += v[i];
    }
    int incl = sum;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += o;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    int before = carry_s;
    for (int w = 0; w < warp; ++w) before += warp_tot[w];
    int run = before + incl - sum;
#pragma unroll
    for (int i = 0; i < kScanPer; ++i) {
      const int64_t b = b0 + static_cast<int64_t>(tid) * kScanPer + i;
      if (b < nblk) block_counts[b * E + e] = run;
      run += v[i];
    }
    __syncthreads();
    if (tid == kScanThreads - 1) carry_s = run;
    __syncthreads();
  }
  if (tid == 0) counts[e] = carry_s;
}

// Exclusive scan of counts[0..E) into smem base[0..E] by warp 0 (E <= 128).
__device__ __forceinline__ void expert_bases(const int32_t* __restrict__ counts, int E,
                                             int32_t* base) {
  if (threadIdx.x < 32) {
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
      const int o = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += o;
    }
    int run = incl - s;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = lane * 4 + i;
      if (e <= E) base[e] = run;
      run += c[i];
    }
    if (lane == 31 && 128 <= E) base[E] = run;
  }
  __syncthreads();
}

// ncb warps per token (1: the whole row; small T: a 512-byte slice each, so
// that enough copies are in flight).  Row bytes must be a multiple of 16.
constexpr int kPermThreads = 256;
constexpr int kPermSeg = 8;  // 16-byte chunks per lane held in registers at a time

// Routing records of assignment f (token t) at sorted position p.
__device__ __forceinline__ void write_record(int p, int64_t f, int64_t t, const void* topk_w,
                                             int topk_w_is_f32, int dtype, int32_t* sort_idx,
                                             int32_t* sorted_token, void* sorted_w) {
  if (sort_idx) sort_idx[p] = static_cast<int32_t>(f);
  if (sorted_token) sorted_token[p] = static_cast<int32_t>(t);
  if (sorted_w) {
    const float w = topk_w_is_f32 ? static_cast<const float*>(topk_w)[f]
                                  : load_elem(topk_w, f, dtype);
    store_elem(sorted_w, p, w, dtype);
  }
}

// Slice cb (of ncb) of token t's row to its k positions; lane j < k holds
// position j (< 0: not placed).
__device__ __forceinline__ void copy_row_slice(const uint4* __restrict__ src,
                                               uint4* __restrict__ x_sorted, int row_chunks,
                                               int ncb, int cb, int k, int p, int lane) {
  const int span = ncb == 1 ? row_chunks : cdiv(row_chunks, 32 * ncb) * 32;
  const int cbeg = cb * span, cend = min(row_chunks, cbeg + span);
  for (int c0 = cbeg; c0 < cend; c0 += 32 * kPermSeg) {
    uint4 buf[kPermSeg];
#pragma unroll
    for (int s = 0; s < kPermSeg; ++s) {
      const int c = c0 + s * 32 + lane;
      if (c < cend) buf[s] = __ldg(src + c);
    }
    for (int j = 0; j < k; ++j) {
      const int pj = __shfl_sync(0xffffffffu, p, j);
      if (pj < 0) continue;
      uint4* dst = x_sorted + static_cast<int64_t>(pj) * row_chunks;
#pragma unroll
      for (int s = 0; s < kPermSeg; ++s) {
        const int c = c0 + s * 32 + lane;
        if (c < cend) dst[c] = buf[s];
      }
    }
  }
}

__global__ void __launch_bounds__(kPermThreads)
permute_gather_kernel(const int32_t* __restrict__ topk_idx, const int32_t* __restrict__ local_rank,
                      const int32_t* __restrict__ block_offsets, const int32_t* __restrict__ counts,
                      const void* __restrict__ topk_w,
                      int topk_w_is_f32, const void* __restrict__ x, int64_t T, int row_chunks,
                      int k, int E, int tblk, int dtype, int32_t* __restrict__ pos,
                      int32_t* __restrict__ sort_idx, int32_t* __restrict__ sorted_token,
                      void* __restrict__ sorted_w, uint4* __restrict__ x_sorted, int ncb) {
  __shared__ int32_t base[kMaxExperts + 1];
  grid_dependency_wait();  // launched early (launch_pdl)
  grid_launch_dependents();
  expert_bases(counts, E, base);
  const int lane = threadIdx.x & 31;
  const int64_t wid = static_cast<int64_t>(blockIdx.x) * (kPermThreads / 32) + (threadIdx.x >> 5);
  const int64_t t = wid / ncb;
  const int cb = static_cast<int>(wid - t * ncb);  // this warp's slice of the row
  if (t >= T) return;
  const int64_t blk = t / tblk;
  // lane j < k resolves assignment j of this token (the slice-0 warp writes
  // the routing records)
  int p = -1;
  if (lane < k) {
    const int64_t f = t * k + lane;
    const int e = topk_idx[f];
    const int r = local_rank[f];
    if (e >= 0 && e < E && r >= 0) {
      p = base[e] + block_offsets[blk * E + e] + r;
      if (cb == 0)
        write_record(p, f, t, topk_w, topk_w_is_f32, dtype, sort_idx, sorted_token, sorted_w);
    }
    if (cb == 0) pos[f] = p;
  }
  if (!x_sorted) return;
  copy_row_slice(static_cast<const uint4*>(x) + t * row_chunks, x_sorted, row_chunks, ncb, cb, k,
                 p, lane);
}

// All of dispatch in one kernel when the T*k assignments fit one histogram
// block (T*k <= kHistFlat): every CTA ranks all assignments in shared memory
// (the hist_rank computation, repeated per CTA), CTA 0 writes the counts,
// and each warp then places its slice of a token's row as permute_gather
// does.  Same positions, one launch instead of two.
__global__ void __launch_bounds__(kPermThreads)
dispatch_small_kernel(const int32_t* __restrict__ topk_idx, const void* __restrict__ topk_w,
                      int topk_w_is_f32, const void* __restrict__ x, int64_t T, int row_chunks,
                      int k, int E, int dtype, int32_t* __restrict__ counts,
                      int32_t* __restrict__ pos, int32_t* __restrict__ sort_idx,
                      int32_t* __restrict__ sorted_token, void* __restrict__ sorted_w,
                      uint4* __restrict__ x_sorted, int ncb, int* __restrict__ err) {
  static_assert(kPermThreads == kHistThreads, "one histogram pass per CTA");
  __shared__ int32_t cnt[kHistChunks][kMaxExperts];
  __shared__ int32_t rank_s[kHistFlat];
  __shared__ int32_t base[kMaxExperts + 1];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nflat = static_cast<int>(T * k);
  const int nchunks = cdiv(nflat, 32);
  for (int i = tid; i < kHistChunks * kMaxExperts; i += kHistThreads)
    (&cnt[0][0])[i] = 0;
  __syncthreads();
  grid_dependency_wait();  // launched early (launch_pdl): the routing is written before this
  grid_launch_dependents();

  constexpr int kRounds = kHistChunks / (kHistThreads / 32);
  int my_e[kRounds], my_rank[kRounds];
#pragma unroll
  for (int r = 0; r < kRounds; ++r) {
    const int c = r * (kHistThreads / 32) + warp;
    const int f = c * 32 + lane;
    int e = -1;
    if (f < nflat) {
      e = topk_idx[f];
      if (e < 0 || e >= E) {
        if (blockIdx.x == 0) record_error(err, kDevBadExpert);
        e = -1;
      }
    }
    const unsigned m = __match_any_sync(0xffffffffu, e);
    my_e[r] = e;
    my_rank[r] = __popc(m & ((1u << lane) - 1u));
    if (e >= 0 && lane == __ffs(m) - 1) cnt[c][e] = __popc(m);
  }
  __syncthreads();
  if (tid < E) {  // exclusive scan over chunks, per expert; the total is the count
    int run = 0;
    for (int c = 0; c < nchunks; ++c) {
      const int v = cnt[c][tid];
      cnt[c][tid] = run;
      run += v;
    }
    base[tid] = run;
    if (blockIdx.x == 0) counts[tid] = run;
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < kRounds; ++r) {
    const int c = r * (kHistThreads / 32) + warp;
    const int f = c * 32 + lane;
    if (f < nflat) rank_s[f] = my_e[r] >= 0 ? cnt[c][my_e[r]] + my_rank[r] : -1;
  }
  // counts -> expert bases, in place (warp 0; E <= 128)
  if (warp == 0) {
    int c4[4], sum = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = lane * 4 + i;
      c4[i] = e < E ? base[e] : 0;
      sum += c4[i];
    }
    int incl = sum;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += o;
    }
    int run = incl - sum;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = lane * 4 + i;
      if (e <= E) base[e] = run;
      run += c4[i];
    }
    if (lane == 31 && 128 <= E) base[E] = run;
  }
  __syncthreads();

  const int64_t wid = static_cast<int64_t>(blockIdx.x) * (kPermThreads / 32) + warp;
  const int64_t t = wid / ncb;
  const int cb = static_cast<int>(wid - t * ncb);
  if (t >= T) return;
  int p = -1;
  if (lane < k) {
    const int64_t f = t * k + lane;
    const int e = topk_idx[f];
    const int r = rank_s[f];
    if (e >= 0 && e < E && r >= 0) {
      p = base[e] + r;
      if (cb == 0)
        write_record(p, f, t, topk_w, topk_w_is_f32, dtype, sort_idx, sorted_token, sorted_w);
    }
    if (cb == 0) pos[f] = p;
  }
  if (!x_sorted) return;
  copy_row_slice(static_cast<const uint4*>(x) + t * row_chunks, x_sorted, row_chunks, ncb, cb, k,
                 p, lane);
}

__global__ void invert_perm_kernel(const int32_t* __restrict__ sort_idx, int64_t n,
                                   int32_t* __restrict__ pos) {
  const int64_t p = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (p < n) {
    const int32_t f = sort_idx[p];
    if (f >= 0 && f < n) pos[f] = static_cast<int32_t>(p);
  }
}

}  // namespace

int dispatch_block_tokens(int k) { return k > 0 ? (kHistFlat / k > 0 ? kHistFlat / k : 1) : 1; }

int64_t dispatch_num_blocks(int64_t T, int k) { return cdiv64(T, dispatch_block_tokens(k)); }

cudaError_t launch_hist_rank(const int32_t* topk_idx, int64_t T, int k, int E,
                             int32_t* local_rank, int32_t* block_counts, int* err,
                             cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  const int tblk = dispatch_block_tokens(k);
  const int64_t nblk = dispatch_num_blocks(T, k);
  return launch_pdl(kPdlDispatch, hist_rank_kernel, dim3(static_cast<unsigned>(nblk)),
                    dim3(kHistThreads), 0, stream, topk_idx, T, k, E, tblk, local_rank,
                    block_counts, err, nullptr);
}

cudaError_t launch_scan(int32_t* block_counts, int64_t nblk, int E, int32_t* counts,
                        int32_t* /*expert_offsets*/, cudaStream_t stream) {
  return launch_pdl(kPdlDispatch, scan_kernel, dim3(E), dim3(kScanThreads), 0, stream,
                    block_counts, nblk, E, counts);
}

cudaError_t launch_hist_scan(const int32_t* topk_idx, int64_t T, int k, int E,
                             int32_t* local_rank, int32_t* block_counts, int32_t* counts, int* err,
                             cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  const int tblk = dispatch_block_tokens(k);
  const int64_t nblk = dispatch_num_blocks(T, k);
  // one histogram block (small T): it writes the counts itself, no scan launch
  cudaError_t e = launch_pdl(kPdlDispatch, hist_rank_kernel, dim3(static_cast<unsigned>(nblk)),
                             dim3(kHistThreads), 0, stream, topk_idx, T, k, E, tblk, local_rank,
                             block_counts, err, nblk == 1 ? counts : nullptr);
  if (e != cudaSuccess || nblk == 1) return e;
  return launch_scan(block_counts, nblk, E, counts, nullptr, stream);
}

cudaError_t launch_permute_gather(const int32_t* topk_idx, const int32_t* local_rank,
                                  const int32_t* block_offsets, const int32_t* counts,
                                  const void* topk_w,
                                  int topk_w_is_f32, const void* x, int64_t T, int d, int k,
                                  int E, int dtype, int32_t* pos, int32_t* sort_idx,
                                  int32_t* sorted_token, void* sorted_w, void* x_sorted,
                                  cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  const int es = dtype == kDtypeBF16 ? 2 : 4;
  const int row_chunks = d * es / 16;
  // small T: a row over several warps (512 bytes each); measured on B200
  // (XL layer): 12.6 -> 11.6 us at T=64, slower at T=1024 (more CTAs, each
  // scanning the counts) and at T=16384 (2, 3 or 6 warps per row: 1-6 %
  // slower for the whole layer)
  const int ncb = T < 512 && x_sorted ? cdiv(row_chunks, 32) : 1;
  const int64_t blocks = cdiv64(T * ncb, kPermThreads / 32);
  return launch_pdl(kPdlDispatch, permute_gather_kernel, dim3(static_cast<unsigned>(blocks)),
                    dim3(kPermThreads), 0, stream, topk_idx, local_rank, block_offsets, counts,
                    topk_w, topk_w_is_f32, x, T, row_chunks, k, E, dispatch_block_tokens(k), dtype,
                    pos, sort_idx, sorted_token, sorted_w, static_cast<uint4*>(x_sorted), ncb);
}

bool dispatch_fits_one_block(int64_t T, int k) { return T > 0 && dispatch_num_blocks(T, k) == 1; }

cudaError_t launch_dispatch_small(const int32_t* topk_idx, const void* topk_w, int topk_w_is_f32,
                                  const void* x, int64_t T, int d, int k, int E, int dtype,
                                  int32_t* counts, int32_t* pos, int32_t* sort_idx,
                                  int32_t* sorted_token, void* sorted_w, void* x_sorted, int* err,
                                  cudaStream_t stream) {
  if (!dispatch_fits_one_block(T, k) || E > kMaxExperts) return cudaErrorInvalidValue;
  const int es = dtype == kDtypeBF16 ? 2 : 4;
  const int row_chunks = d * es / 16;
  const int ncb = x_sorted ? cdiv(row_chunks, 32) : 1;
  const int64_t blocks = cdiv64(T * ncb, kPermThreads / 32);
  return launch_pdl(kPdlDispatch, dispatch_small_kernel, dim3(static_cast<unsigned>(blocks)),
                    dim3(kPermThreads), 0, stream, topk_idx, topk_w, topk_w_is_f32, x, T,
                    row_chunks, k, E, dtype, counts, pos, sort_idx, sorted_token, sorted_w,
                    static_cast<uint4*>(x_sorted), ncb, err);
}

cudaError_t launch_invert_perm(const int32_t* sort_idx, int64_t n, int32_t* pos,
                               cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  invert_perm_kernel<<<static_cast<unsigned>(cdiv64(n, 256)), 256, 0, stream>>>(sort_idx, n, pos);
  return cudaGetLastError();
}

}  // namespace hmoe
