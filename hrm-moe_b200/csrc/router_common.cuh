// Per-token routing shared by the router kernels: warp-shuffle top-k with
// lower-index ties, fp32 softmax, renormalisation and the output writes
// (models/layers.py:606-610).
#pragma once

#include <limits.h>

#include "common.cuh"

namespace hmoe {

// Lanes hold NV logits each (expert = lane + 32*q, -inf/INT_MAX when absent).
// Selects k (<= 32) experts in descending value, equal values by ascending
// index; lane r < k returns the r-th pick in (my_v, my_i).  All lanes return
// the maximum in `mx`.
template <int NV>
__device__ __forceinline__ void warp_topk(float (&v)[NV], int (&id)[NV], int k, int lane,
                                          float& my_v, int& my_i, float& mx) {
  my_v = 0.0f;
  my_i = 0;
  mx = 0.0f;
  for (int r = 0; r < k; ++r) {
    float bv = v[0];
    int bi = id[0];
#pragma unroll
    for (int q = 1; q < NV; ++q)
      if (v[q] > bv || (v[q] == bv && id[q] < bi)) { bv = v[q]; bi = id[q]; }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (r == 0) mx = bv;
    if (lane == r) { my_v = bv; my_i = bi; }
#pragma unroll
    for (int q = 0; q < NV; ++q)
      if (id[q] == bi) { v[q] = -INFINITY; id[q] = INT_MAX; }
  }
}

// Softmax weights of the picks held by lanes < k, renormalised (norm) and
// rounded to the layer dtype; `all` are the token's logits (lane + 32*q).
template <int NV, bool BF16>
__device__ __forceinline__ float warp_route_weight(const float (&all)[NV], int E, int k, int norm,
                                                   int lane, float my_v, float mx) {
  float s = 0.0f;
#pragma unroll
  for (int q = 0; q < NV; ++q)
    if (lane + 32 * q < E) s += expf(all[q] - mx);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  float p = lane < k ? expf(my_v - mx) / s : 0.0f;
  if (norm) {
    float ps = p;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
    p = p / fmaxf(ps, 1e-12f);
  }
  return BF16 ? round_bf16(p) : p;
}

template <bool BF16>
__device__ __forceinline__ void write_route(int64_t t, int k, int lane, int my_i, float p,
                                            int32_t* topk_idx, float* topk_w_f32,
                                            void* topk_w_dtype) {
  if (lane < k) {
    const int64_t o = t * k + lane;
    topk_idx[o] = my_i;
    if (topk_w_f32) topk_w_f32[o] = p;
    if (topk_w_dtype) {
      if (BF16)
        static_cast<uint16_t*>(topk_w_dtype)[o] = static_cast<uint16_t>(f32_to_bf16_bits(p));
      else
        static_cast<float*>(topk_w_dtype)[o] = p;
    }
  }
}

}  // namespace hmoe
