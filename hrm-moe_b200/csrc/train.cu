// Backward-pass kernels of the routed MoE layer that are not GEMMs, and the
// aux load-balancing statistics.  bf16 layers only.
//
// What autograd computes through models/layers.py:596-634 (the GEMMs'
// backward is gemm_sm100_bwd.cu):
//
//  combine_router_bwd_kernel  (one warp per token t)
//    combine (layers.py:332-334, index_add_ of bf16(expert_out * w)):
//      d_expert_out[pos(t,j)] = bf16(grad_y[t] * w[t,j])
//      d_w[t,j]               = bf16(sum_c bf16(grad_y[t,c] * expert_out[pos(t,j), c]))
//    renormalise / top-k / fp32 softmax (layers.py:606-610), from the saved
//    bf16 logits:  p = softmax(logits), s_j = p[idx_j], S = max(sum s_j, 1e-12)
//      d_s_j = d_w_j / S - sum_i d_w_i s_i / S^2   (d_s_j = d_w_j without renormalising)
//      d_p[e] = d_s_j at e = idx_j, plus the aux loss term
//               aux_grad * E * (count_e / n) / n for the first n (valid) tokens
//      d_logits = bf16(p * (d_p - sum_e p * d_p))
//  dx_kernel  (one warp per token)
//      dx[t] = bf16(dx_router[t] + bf16(sum_j d_x_sorted[pos(t,j)]))
//    the sum in fp32 over the token's rows in ascending sorted position
//    (the reference's CPU autograd gives exactly this on the fixtures).
//  aux_partial_kernel / aux_finish_kernel  (layers.py:163-170, 619-632)
//      aux = E * sum_e (count_e / n) * (sum_{t<n} p[t,e] / n),
//      expert_counts[e] = count_e (fp32), n = valid tokens;
//    fixed block partials summed in order: deterministic.
//  colsum kernels: the router bias gradient, bf16(sum_t d_logits[t, e]).
#include "common.cuh"
#include "internal.h"

namespace hmoe {
namespace {

constexpr int kTThreads = 256;
constexpr int kTWarps = kTThreads / 32;
constexpr int kMaxEQ = 4;  // E <= 128: four expert slots per lane

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// The token's softmax over its bf16 logits: lane holds experts lane + 32 q.
__device__ __forceinline__ void token_softmax(const uint16_t* __restrict__ lrow, int E, int lane,
                                              float (&p)[kMaxEQ]) {
  float l[kMaxEQ];
  float mx = -INFINITY;
#pragma unroll
  for (int q = 0; q < kMaxEQ; ++q) {
    const int e = lane + 32 * q;
    l[q] = e < E ? bf16_bits_to_f32(lrow[e]) : -INFINITY;
    mx = fmaxf(mx, l[q]);
  }
  mx = warp_max(mx);
  float s = 0.0f;
#pragma unroll
  for (int q = 0; q < kMaxEQ; ++q) {
    p[q] = lane + 32 * q < E ? expf(l[q] - mx) : 0.0f;
    s += p[q];
  }
  s = warp_sum(s);
#pragma unroll
  for (int q = 0; q < kMaxEQ; ++q) p[q] = p[q] / s;
}

__device__ __forceinline__ float pick(const float (&v)[kMaxEQ], int q) {
  return q == 0 ? v[0] : q == 1 ? v[1] : q == 2 ? v[2] : v[3];
}

__global__ void __launch_bounds__(kTThreads)
combine_router_bwd_kernel(const uint4* __restrict__ grad_y, const uint4* __restrict__ expert_out,
                          const int32_t* __restrict__ pos, const int32_t* __restrict__ topk_idx,
                          const float* __restrict__ topk_w, const uint16_t* __restrict__ logits,
                          int64_t T, int row_chunks, int k, int E, int norm,
                          const float* __restrict__ aux_grad,
                          const float* __restrict__ expert_counts, int64_t n_valid,
                          uint4* __restrict__ d_expert_out, uint16_t* __restrict__ d_logits,
                          int32_t* __restrict__ count_out) {
  if (count_out && blockIdx.x == 0 && threadIdx.x == 0) *count_out = static_cast<int32_t>(T);
  const int lane = threadIdx.x & 31;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * kTWarps + (threadIdx.x >> 5);
  if (t >= T) return;
  int p_j = -1, e_j = -1;
  float w_j = 0.0f;
  if (lane < k) {
    p_j = pos[t * k + lane];
    e_j = topk_idx[t * k + lane];
    w_j = topk_w[t * k + lane];
  }
  // ------------------------------------------------------ combine backward
  const uint4* g = grad_y + t * row_chunks;
  float d_w = 0.0f;  // lane j < k: d_w of assignment j
  for (int j = 0; j < k; ++j) {
    const int pj = __shfl_sync(0xffffffffu, p_j, j);
    const float wj = __shfl_sync(0xffffffffu, w_j, j);
    if (pj < 0) continue;
    const uint32_t w2 = cvt_bf16x2(wj, wj);
    const uint4* eo = expert_out + static_cast<int64_t>(pj) * row_chunks;
    uint4* deo = d_expert_out + static_cast<int64_t>(pj) * row_chunks;
    float dot = 0.0f;
    for (int c = lane; c < row_chunks; c += 32) {
      const uint4 gv = __ldg(g + c);
      const uint4 ev = __ldg(eo + c);
      deo[c] = make_uint4(mul_bf16x2(gv.x, w2), mul_bf16x2(gv.y, w2), mul_bf16x2(gv.z, w2),
                          mul_bf16x2(gv.w, w2));
      const uint32_t q[4] = {mul_bf16x2(gv.x, ev.x), mul_bf16x2(gv.y, ev.y),
                             mul_bf16x2(gv.z, ev.z), mul_bf16x2(gv.w, ev.w)};
#pragma unroll
      for (int i = 0; i < 4; ++i) dot += bf16_lo(q[i]) + bf16_hi(q[i]);
    }
    dot = warp_sum(dot);
    if (lane == j) d_w = round_bf16(dot);
  }
  // ------------------------------------------------------ router backward
  float p[kMaxEQ];
  token_softmax(logits + t * E, E, lane, p);
  // selected probabilities s_j (lane j), their sum S
  float s_j = 0.0f;
  for (int j = 0; j < k; ++j) {
    const int ej = __shfl_sync(0xffffffffu, e_j, j);
    const float v = (ej >= 0 && ej < E) ? __shfl_sync(0xffffffffu, pick(p, ej >> 5), ej & 31) : 0.0f;
    if (lane == j) s_j = v;
  }
  float d_s = d_w;
  if (norm) {
    const float S = fmaxf(warp_sum(lane < k ? s_j : 0.0f), 1e-12f);
    const float dS = -warp_sum(lane < k ? d_w * s_j : 0.0f) / (S * S);
    d_s = d_w / S + dS;
  }
  float dp[kMaxEQ];
#pragma unroll
  for (int q = 0; q < kMaxEQ; ++q) {
    dp[q] = 0.0f;
    if (aux_grad && t < n_valid) {
      const int e = lane + 32 * q;
      if (e < E) {
        const float n = static_cast<float>(n_valid);
        dp[q] = *aux_grad * static_cast<float>(E) * (expert_counts[e] / n) / n;
      }
    }
  }
  for (int j = 0; j < k; ++j) {
    const int ej = __shfl_sync(0xffffffffu, e_j, j);
    const float v = __shfl_sync(0xffffffffu, d_s, j);
    if (ej >= 0 && ej < E && lane == (ej & 31)) {
      const int q = ej >> 5;
      if (q == 0) dp[0] += v; else if (q == 1) dp[1] += v; else if (q == 2) dp[2] += v; else dp[3] += v;
    }
  }
  float pdp = 0.0f;
#pragma unroll
  for (int q = 0; q < kMaxEQ; ++q) pdp += p[q] * dp[q];
  pdp = warp_sum(pdp);
  uint16_t* dl = d_logits + t * E;
#pragma unroll
  for (int q = 0; q < kMaxEQ; ++q) {
    const int e = lane + 32 * q;
    if (e < E) dl[e] = static_cast<uint16_t>(f32_to_bf16_bits(p[q] * (dp[q] - pdp)));
  }
}

__global__ void __launch_bounds__(kTThreads)
dx_kernel(const uint4* __restrict__ d_x_sorted, const int32_t* __restrict__ pos,
          const uint4* __restrict__ dx_router, int64_t T, int row_chunks, int k,
          uint4* __restrict__ dx) {
  const int lane = threadIdx.x & 31;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * kTWarps + (threadIdx.x >> 5);
  if (t >= T) return;
  int p = lane < k ? pos[t * k + lane] : -1;
  // ascending sorted position: lane r ends up with the r-th smallest
  const unsigned live = __ballot_sync(0xffffffffu, lane < k && p >= 0);
  int rank = 0;
  for (int j = 0; j < k; ++j) {
    const int pj = __shfl_sync(0xffffffffu, p, j);
    if (((live >> j) & 1u) && pj < p) ++rank;
  }
  const int nlive = __popc(live);
  int sp = -1;
  for (int r = 0; r < nlive; ++r) {
    const unsigned m = __ballot_sync(0xffffffffu, ((live >> lane) & 1u) && rank == r);
    const int pr = __shfl_sync(0xffffffffu, p, __ffs(m) - 1);
    if (lane == r) sp = pr;
  }
  // every lane runs the same trip count so the shuffles see all 32 lanes
  for (int c0 = 0; c0 < row_chunks; c0 += 32) {
    const int c = c0 + lane;
    const bool live_c = c < row_chunks;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int r = 0; r < nlive; ++r) {
      const int pr = __shfl_sync(0xffffffffu, sp, r);
      if (!live_c) continue;
      const uint4 u = __ldg(d_x_sorted + static_cast<int64_t>(pr) * row_chunks + c);
      const uint32_t q[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc[2 * i] += bf16_lo(q[i]);
        acc[2 * i + 1] += bf16_hi(q[i]);
      }
    }
    if (!live_c) continue;
    const uint4 rv = dx_router[t * row_chunks + c];
    const uint32_t rq[4] = {rv.x, rv.y, rv.z, rv.w};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t e2 = cvt_bf16x2(acc[2 * i], acc[2 * i + 1]);  // the experts' sum, rounded
      o[i] = cvt_bf16x2(bf16_lo(rq[i]) + bf16_lo(e2), bf16_hi(rq[i]) + bf16_hi(e2));
    }
    dx[t * row_chunks + c] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// Per-block partial sums over tokens [0, n) of the softmax probabilities
// (partial_p[block][e]) and of the selections (partial_c[block][e]).
__global__ void __launch_bounds__(kTThreads)
aux_partial_kernel(const uint16_t* __restrict__ logits, const int32_t* __restrict__ topk_idx,
                   int64_t n, int E, int k, float* __restrict__ partial_p,
                   int* __restrict__ partial_c) {
  __shared__ float sp[kTWarps][128];
  __shared__ int sc[kTWarps][128];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  float acc[kMaxEQ] = {0.f, 0.f, 0.f, 0.f};
  int cnt[kMaxEQ] = {0, 0, 0, 0};
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * kTWarps + w; t < n;
       t += static_cast<int64_t>(gridDim.x) * kTWarps) {
    float p[kMaxEQ];
    token_softmax(logits + t * E, E, lane, p);
#pragma unroll
    for (int q = 0; q < kMaxEQ; ++q) acc[q] += p[q];
    const int e = lane < k ? topk_idx[t * k + lane] : -1;
    for (int j = 0; j < k; ++j) {
      const int ej = __shfl_sync(0xffffffffu, e, j);
      if (ej >= 0 && ej < E && lane == (ej & 31)) {
        const int q = ej >> 5;
        if (q == 0) ++cnt[0]; else if (q == 1) ++cnt[1]; else if (q == 2) ++cnt[2]; else ++cnt[3];
      }
    }
  }
#pragma unroll
  for (int q = 0; q < kMaxEQ; ++q) {
    sp[w][lane + 32 * q] = acc[q];
    sc[w][lane + 32 * q] = cnt[q];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += kTThreads) {
    float s = 0.0f;
    int c = 0;
    for (int i = 0; i < kTWarps; ++i) {
      s += sp[i][e];
      c += sc[i][e];
    }
    partial_p[static_cast<int64_t>(blockIdx.x) * E + e] = s;
    partial_c[static_cast<int64_t>(blockIdx.x) * E + e] = c;
  }
}

__global__ void __launch_bounds__(128)
aux_finish_kernel(const float* __restrict__ partial_p, const int* __restrict__ partial_c,
                  int nblocks, int64_t n, int E, float* __restrict__ aux_out,
                  float* __restrict__ counts_out) {
  __shared__ float terms[128];
  const int e = threadIdx.x;
  float s = 0.0f;
  int c = 0;
  if (e < E) {
    for (int b = 0; b < nblocks; ++b) {
      s += partial_p[static_cast<int64_t>(b) * E + e];
      c += partial_c[static_cast<int64_t>(b) * E + e];
    }
    counts_out[e] = static_cast<float>(c);
  }
  const float nf = static_cast<float>(n > 0 ? n : 1);
  terms[e] = e < E ? (static_cast<float>(c) / nf) * (s / nf) : 0.0f;
  __syncthreads();
  if (e == 0) {
    float a = 0.0f;
    for (int i = 0; i < E; ++i) a += terms[i];
    *aux_out = a * static_cast<float>(E);
  }
}

// Column sums of a [T, E] bf16 matrix: per-block fp32 partials, then one
// pass over the blocks in order, rounded to bf16.
__global__ void __launch_bounds__(kTThreads)
colsum_partial_kernel(const uint16_t* __restrict__ m, int64_t T, int E,
                      float* __restrict__ partial) {
  __shared__ float s[kTThreads];
  const int e = threadIdx.x % 128, slice = threadIdx.x / 128;  // 2 row slices of 128 columns
  float acc = 0.0f;
  if (e < E)
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * 2 + slice; t < T;
         t += static_cast<int64_t>(gridDim.x) * 2)
      acc += bf16_bits_to_f32(m[t * E + e]);
  s[threadIdx.x] = acc;
  __syncthreads();
  if (threadIdx.x < E) partial[static_cast<int64_t>(blockIdx.x) * E + threadIdx.x] =
      s[threadIdx.x] + s[threadIdx.x + 128];
}

__global__ void __launch_bounds__(128)
colsum_finish_kernel(const float* __restrict__ partial, int nblocks, int E,
                     uint16_t* __restrict__ out) {
  const int e = threadIdx.x;
  if (e >= E) return;
  float s = 0.0f;
  for (int b = 0; b < nblocks; ++b) s += partial[static_cast<int64_t>(b) * E + e];
  out[e] = static_cast<uint16_t>(f32_to_bf16_bits(s));
}

}  // namespace

int train_partial_blocks(int64_t T) {
  const int64_t b = cdiv64(T, kTWarps * 16);
  return static_cast<int>(b < 1 ? 1 : (b > 592 ? 592 : b));
}

cudaError_t launch_combine_router_bwd(const void* grad_y, const void* expert_out,
                                      const int32_t* pos, const int32_t* topk_idx,
                                      const float* topk_w, const void* logits, int64_t T, int d,
                                      int k, int E, int norm, const float* aux_grad,
                                      const float* expert_counts, int64_t n_valid,
                                      void* d_expert_out, void* d_logits, int32_t* count_out,
                                      cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  if (E > 32 * kMaxEQ || k > 32 || d % 8 != 0) return cudaErrorInvalidValue;
  const unsigned blocks = static_cast<unsigned>(cdiv64(T, kTWarps));
  combine_router_bwd_kernel<<<blocks, kTThreads, 0, stream>>>(
      static_cast<const uint4*>(grad_y), static_cast<const uint4*>(expert_out), pos, topk_idx,
      topk_w, static_cast<const uint16_t*>(logits), T, d / 8, k, E, norm, aux_grad, expert_counts,
      n_valid, static_cast<uint4*>(d_expert_out), static_cast<uint16_t*>(d_logits), count_out);
  return cudaGetLastError();
}

cudaError_t launch_dx(const void* d_x_sorted, const int32_t* pos, const void* dx_router, int64_t T,
                      int d, int k, void* dx, cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  if (k > 32 || d % 8 != 0) return cudaErrorInvalidValue;
  const unsigned blocks = static_cast<unsigned>(cdiv64(T, kTWarps));
  dx_kernel<<<blocks, kTThreads, 0, stream>>>(static_cast<const uint4*>(d_x_sorted), pos,
                                              static_cast<const uint4*>(dx_router), T, d / 8, k,
                                              static_cast<uint4*>(dx));
  return cudaGetLastError();
}

cudaError_t launch_aux_stats(const void* logits, const int32_t* topk_idx, int64_t n, int E, int k,
                             float* partial_p, int* partial_c, int nblocks, float* aux_out,
                             float* counts_out, cudaStream_t stream) {
  if (E > 128) return cudaErrorInvalidValue;
  aux_partial_kernel<<<nblocks, kTThreads, 0, stream>>>(static_cast<const uint16_t*>(logits),
                                                        topk_idx, n, E, k, partial_p, partial_c);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  aux_finish_kernel<<<1, 128, 0, stream>>>(partial_p, partial_c, nblocks, n, E, aux_out,
                                           counts_out);
  return cudaGetLastError();
}

cudaError_t launch_colsum_bf16(const void* m, int64_t T, int E, float* partial, int nblocks,
                               void* out, cudaStream_t stream) {
  if (E > 128) return cudaErrorInvalidValue;
  colsum_partial_kernel<<<nblocks, kTThreads, 0, stream>>>(static_cast<const uint16_t*>(m), T, E,
                                                           partial);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  colsum_finish_kernel<<<1, 128, 0, stream>>>(partial, nblocks, E, static_cast<uint16_t*>(out));
  return cudaGetLastError();
}

}  // namespace hmoe
