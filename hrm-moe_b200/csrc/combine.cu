// Combine: weighted sum of each token's k expert outputs, back in token order.
//
// Mirrors models/layers.py:332-334 of HRM-MoE:
//   expert_output = expert_output * sorted_weights[:, None]      # layer dtype
//   final_hidden_states.index_add_(0, sorted_token_idx, expert_output)
// as a gather instead of a scatter: one warp per token reads the k rows
// pos(t, 0..k-1) of the expert-sorted output (SPLIT: small T, where one warp
// per token leaves too few loads in flight, one warp per (token, block of 32
// 16-byte columns)).  The arithmetic follows the
// reference step by step: each product w * y is rounded to the layer dtype,
// and the products are added into the accumulator one at a time, each sum
// rounded, in ascending sorted position -- the order index_add_ visits a
// token's rows (ascending expert id, the stable sort order).  No atomics, so
// the result is deterministic (the reference's CUDA index_add_ is not).
#include "common.cuh"
#include "internal.h"

namespace hmoe {
namespace {

constexpr int kCombThreads = 256;
constexpr int kMaxK = 32;

// At most 64 registers, so that four CTAs (32 warps, 32 rows of loads in
// flight per warp batch) fit an SM: with 76 registers and three CTAs the
// XL combine took 130 instead of 88 us.
template <bool BF16, bool SPLIT>
__global__ void __launch_bounds__(kCombThreads, 4)
combine_kernel(const void* __restrict__ expert_out, const int32_t* __restrict__ pos,
               const void* __restrict__ topk_w, int topk_w_is_f32, int64_t T, int row_chunks,
               int k, const void* __restrict__ final_in, void* __restrict__ out) {
  grid_dependency_wait();  // launched early (launch_pdl): the expert rows are written before this
  grid_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t wid = static_cast<int64_t>(blockIdx.x) * (kCombThreads / 32) + (threadIdx.x >> 5);
  const int ncb = SPLIT ? (row_chunks + 31) / 32 : 1;  // warps per token
  const int64_t t = SPLIT ? wid / ncb : wid;
  const int cfirst = SPLIT ? static_cast<int>(wid - t * ncb) * 32 : 0;
  const int cend = SPLIT ? cfirst + 32 : row_chunks;
  if (t >= T) return;
  int p = -1;
  float w = 0.0f;
  if (lane < k) {
    p = pos[t * k + lane];
    if (topk_w_is_f32)
      w = static_cast<const float*>(topk_w)[t * k + lane];
    else
      w = BF16 ? bf16_bits_to_f32(static_cast<const uint16_t*>(topk_w)[t * k + lane])
               : static_cast<const float*>(topk_w)[t * k + lane];
  }
  // visit the token's assignments in ascending position: lane r ends up
  // holding the (position, weight) of the r-th assignment in that order
  const unsigned live_k = __ballot_sync(0xffffffffu, lane < k && p >= 0);
  int rank = 0;
  for (int j = 0; j < k; ++j) {
    const int pj = __shfl_sync(0xffffffffu, p, j);
    if (((live_k >> j) & 1u) && pj < p) ++rank;
  }
  const int nlive = __popc(live_k);
  int sp = -1;
  float sw = 0.0f;
  for (int r = 0; r < nlive; ++r) {
    const unsigned m = __ballot_sync(0xffffffffu, ((live_k >> lane) & 1u) && rank == r);
    const int src = __ffs(m) - 1;
    const int pr = __shfl_sync(0xffffffffu, p, src);
    const float wr = __shfl_sync(0xffffffffu, w, src);
    if (lane == r) { sp = pr; sw = wr; }
  }

  const uint4* src = static_cast<const uint4*>(expert_out);
  const uint4* fin = static_cast<const uint4*>(final_in);
  uint4* dst = static_cast<uint4*>(out);
  constexpr int EPC = BF16 ? 8 : 4;  // elements per 16-byte chunk
  constexpr int kBatch = 8;          // rows loaded before they are summed
  // every lane runs the same trip count so the shuffles below see all 32 lanes
  for (int c0 = cfirst; c0 < cend; c0 += 32) {
    const int c = c0 + lane;
    const bool live = c < row_chunks;
    float acc[EPC];
    if (fin && live) {
      const uint4 u = fin[t * row_chunks + c];
      if (BF16) {
        const uint32_t q[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) { acc[2 * i] = bf16_lo(q[i]); acc[2 * i + 1] = bf16_hi(q[i]); }
      } else {
        acc[0] = __uint_as_float(u.x); acc[1] = __uint_as_float(u.y);
        acc[2] = __uint_as_float(u.z); acc[3] = __uint_as_float(u.w);
      }
    } else {
#pragma unroll
      for (int i = 0; i < EPC; ++i) acc[i] = 0.0f;
    }
    for (int r0 = 0; r0 < nlive; r0 += kBatch) {
      uint4 rows[kBatch];
      float ws[kBatch];
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        const int pj = __shfl_sync(0xffffffffu, sp, (r0 + b) & 31);
        ws[b] = __shfl_sync(0xffffffffu, sw, (r0 + b) & 31);
        rows[b] = (live && r0 + b < nlive)
                      ? __ldg(src + static_cast<int64_t>(pj) * row_chunks + c)
                      : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        if (r0 + b >= nlive) break;
        const uint4 u = rows[b];
        if (BF16) {
          // product rounded to bf16 (paired, exact = round(fp32 product)),
          // then fp32 add and one rounding of the sum, as torch does
          const uint32_t w2 = cvt_bf16x2(ws[b], ws[b]);
          const uint32_t q[4] = {mul_bf16x2(u.x, w2), mul_bf16x2(u.y, w2), mul_bf16x2(u.z, w2),
                                 mul_bf16x2(u.w, w2)};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint32_t s2 = cvt_bf16x2(__fadd_rn(acc[2 * i], bf16_lo(q[i])),
                                           __fadd_rn(acc[2 * i + 1], bf16_hi(q[i])));
            acc[2 * i] = bf16_lo(s2);
            acc[2 * i + 1] = bf16_hi(s2);
          }
        } else {
          const float y[4] = {__uint_as_float(u.x), __uint_as_float(u.y), __uint_as_float(u.z),
                              __uint_as_float(u.w)};
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[i] = __fadd_rn(acc[i], __fmul_rn(y[i], ws[b]));
        }
      }
    }
    uint4 o;
    if (BF16) {
      o.x = cvt_bf16x2(acc[0], acc[1]);
      o.y = cvt_bf16x2(acc[2], acc[3]);
      o.z = cvt_bf16x2(acc[4], acc[5]);
      o.w = cvt_bf16x2(acc[6], acc[7]);
    } else {
      o.x = __float_as_uint(acc[0]); o.y = __float_as_uint(acc[1]);
      o.z = __float_as_uint(acc[2]); o.w = __float_as_uint(acc[3]);
    }
    if (live) dst[t * row_chunks + c] = o;
  }
}

}  // namespace

cudaError_t launch_combine(const void* expert_out, const int32_t* pos, const void* topk_w,
                           int topk_w_is_f32, const int32_t* /*topk_idx*/, int /*E*/, int64_t T,
                           int d, int k, int dtype, const void* final_in, void* out,
                           cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  if (k > kMaxK) return cudaErrorInvalidValue;
  const bool bf16 = dtype == kDtypeBF16;
  const int row_chunks = d * (bf16 ? 2 : 4) / 16;
  // small T: a row over several warps, so that enough loads are in flight
  const bool split = T < 4096;
  const unsigned blocks = static_cast<unsigned>(
      cdiv64(T * (split ? cdiv(row_chunks, 32) : 1), kCombThreads / 32));
  if (bf16 && split)
    return launch_pdl(kPdlCombine, combine_kernel<true, true>, dim3(blocks), dim3(kCombThreads), 0,
                      stream, expert_out, pos, topk_w, topk_w_is_f32, T, row_chunks, k, final_in,
                      out);
  else if (bf16)
    return launch_pdl(kPdlCombine, combine_kernel<true, false>, dim3(blocks), dim3(kCombThreads), 0,
                      stream, expert_out, pos, topk_w, topk_w_is_f32, T, row_chunks, k, final_in,
                      out);
  else if (split)
    return launch_pdl(kPdlCombine, combine_kernel<false, true>, dim3(blocks), dim3(kCombThreads), 0,
                      stream, expert_out, pos, topk_w, topk_w_is_f32, T, row_chunks, k, final_in,
                      out);
  else
    return launch_pdl(kPdlCombine, combine_kernel<false, false>, dim3(blocks), dim3(kCombThreads),
                      0, stream, expert_out, pos, topk_w, topk_w_is_f32, T, row_chunks, k,
                      final_in, out);
}

}  // namespace hmoe
