// Router: logits = x @ w_router^T (+ bias), fp32 softmax, top-k, renormalise.
//
// Mirrors models/layers.py:604-610 of HRM-MoE:
//   router_logits   = self.gate(hidden_states)          # F.linear, hidden dtype
//   routing_probs   = softmax(router_logits, fp32)
//   weights, idx    = topk(routing_probs, k)
//   weights        /= clamp(sum(weights), 1e-12)        # if norm_topk_prob
//   weights         = weights.to(hidden dtype)
//
// One CTA handles 64 tokens.  The logits GEMM runs on the CUDA cores in
// fp32: thread (ty, tx) owns 4 tokens x EPT experts and accumulates every
// output in the fixed order kLogitBlock defines (one fmaf per k ascending
// within each 64-wide block from +0, block sums added in order from +0) --
// the order the CPU oracle restates, so the logits are bit-identical to it.
// The sum (plus bias) is rounded to the layer dtype, like F.linear's output.
//
// Selection runs one warp per token over the rounded logits kept in shared
// memory: k rounds of a warp-shuffle argmax where equal values go to the
// lower expert index.  Softmax is monotone, so the k largest logits are the
// k largest probabilities.
#include <float.h>
#include <limits.h>

#include "common.cuh"
#include "internal.h"

namespace hmoe {
namespace {

constexpr int kRTok = 64;       // tokens per CTA
constexpr int kRThreads = 256;
constexpr int kRKc = 32;        // k-slab staged in shared memory

template <int EPAD, bool BF16>
__global__ void __launch_bounds__(kRThreads)
router_topk_kernel(const void* __restrict__ xv, const void* __restrict__ wv,
                   const void* __restrict__ biasv, int64_t T, int d, int E, int k, int norm,
                   int32_t* __restrict__ topk_idx, float* __restrict__ topk_w_f32,
                   void* __restrict__ topk_w_dtype, void* __restrict__ logits_out) {
  constexpr int EPT = EPAD / 16;   // experts per thread
  constexpr int NG = EPT / 4;      // groups of 4: expert = g*64 + tx*4 + j
  constexpr int LGS = EPAD + 1;    // padded logits row
  constexpr int GEMM_FLOATS = kRKc * (kRTok + EPAD);
  constexpr int LG_FLOATS = kRTok * LGS;
  constexpr int SMEM_FLOATS = GEMM_FLOATS > LG_FLOATS ? GEMM_FLOATS : LG_FLOATS;
  __shared__ __align__(16) float smem[SMEM_FLOATS];
  float* xs = smem;                     // [kRKc][64]
  float* ws = smem + kRKc * kRTok;      // [kRKc][EPAD]
  float* lg = smem;                     // [64][LGS], after the GEMM

  const int tid = threadIdx.x;
  const int ty = tid >> 4;
  const int tx = tid & 15;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kRTok;

  float acc[4][EPT], part[4][EPT];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < EPT; ++j) { acc[i][j] = 0.0f; part[i][j] = 0.0f; }

  for (int k0 = 0; k0 < d; k0 += kRKc) {
    const int kc = min(kRKc, d - k0);
    // ---- stage the x slab [64 tokens x kRKc] transposed to [k][token]
    if (BF16) {
      const int tok = tid & 63;
      const int q = tid >> 6;  // 8-element chunk
      const int64_t t = t0 + tok;
      uint4 u = make_uint4(0, 0, 0, 0);
      if (t < T && k0 + q * 8 < d)
        u = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(xv) + t * d + k0 + q * 8);
      const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        xs[(q * 8 + 2 * i) * kRTok + tok] = bf16_lo(w4[i]);
        xs[(q * 8 + 2 * i + 1) * kRTok + tok] = bf16_hi(w4[i]);
      }
    } else {
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int idx = tid + r * kRThreads;
        const int tok = idx & 63;
        const int q = idx >> 6;  // 4-element chunk, 0..7
        const int64_t t = t0 + tok;
        float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
        if (t < T && k0 + q * 4 < d)
          f = *reinterpret_cast<const float4*>(static_cast<const float*>(xv) + t * d + k0 + q * 4);
        xs[(q * 4 + 0) * kRTok + tok] = f.x;
        xs[(q * 4 + 1) * kRTok + tok] = f.y;
        xs[(q * 4 + 2) * kRTok + tok] = f.z;
        xs[(q * 4 + 3) * kRTok + tok] = f.w;
      }
    }
    // ---- stage the router-weight slab [EPAD experts x kRKc] as [k][expert]
    if (BF16) {
#pragma unroll
      for (int r = 0; r < EPAD / 64; ++r) {
        const int idx = tid + r * kRThreads;
        const int e = idx % EPAD;
        const int q = idx / EPAD;  // 0..3
        uint4 u = make_uint4(0, 0, 0, 0);
        if (e < E && k0 + q * 8 < d)
          u = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(wv) +
                                              static_cast<int64_t>(e) * d + k0 + q * 8);
        const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          ws[(q * 8 + 2 * i) * EPAD + e] = bf16_lo(w4[i]);
          ws[(q * 8 + 2 * i + 1) * EPAD + e] = bf16_hi(w4[i]);
        }
      }
    } else {
#pragma unroll
      for (int r = 0; r < EPAD / 32; ++r) {
        const int idx = tid + r * kRThreads;
        const int e = idx % EPAD;
        const int q = idx / EPAD;  // 0..7
        float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
        if (e < E && k0 + q * 4 < d)
          f = *reinterpret_cast<const float4*>(static_cast<const float*>(wv) +
                                               static_cast<int64_t>(e) * d + k0 + q * 4);
        ws[(q * 4 + 0) * EPAD + e] = f.x;
        ws[(q * 4 + 1) * EPAD + e] = f.y;
        ws[(q * 4 + 2) * EPAD + e] = f.z;
        ws[(q * 4 + 3) * EPAD + e] = f.w;
      }
    }
    __syncthreads();
    // ---- one fma per k, ascending (the order the oracle restates)
    for (int kk = 0; kk < kc; ++kk) {
      const float4 xq = *reinterpret_cast<const float4*>(&xs[kk * kRTok + ty * 4]);
      const float xr[4] = {xq.x, xq.y, xq.z, xq.w};
      float wr[EPT];
#pragma unroll
      for (int g = 0; g < NG; ++g) {
        const float4 wq = *reinterpret_cast<const float4*>(&ws[kk * EPAD + g * 64 + tx * 4]);
        wr[g * 4 + 0] = wq.x;
        wr[g * 4 + 1] = wq.y;
        wr[g * 4 + 2] = wq.z;
        wr[g * 4 + 3] = wq.w;
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < EPT; ++j) part[i][j] = fmaf(xr[i], wr[j], part[i][j]);
    }
    // end of a 64-wide block of k: add its sum into the total
    if ((k0 + kRKc) % kLogitBlock == 0 || k0 + kRKc >= d) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < EPT; ++j) { acc[i][j] = acc[i][j] + part[i][j]; part[i][j] = 0.0f; }
    }
    __syncthreads();
  }

  // ---- logits: + bias, round to the layer dtype, park in shared memory
#pragma unroll
  for (int g = 0; g < NG; ++g)
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int e = g * 64 + tx * 4 + jj;
      if (e >= E) continue;
      float b = 0.0f;
      const bool has_bias = biasv != nullptr;
      if (has_bias)
        b = BF16 ? bf16_bits_to_f32(static_cast<const uint16_t*>(biasv)[e])
                 : static_cast<const float*>(biasv)[e];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float v = acc[i][g * 4 + jj];
        if (has_bias) v = v + b;
        if (BF16) v = round_bf16(v);
        lg[(ty * 4 + i) * LGS + e] = v;
      }
    }
  __syncthreads();

  if (logits_out) {
    for (int i = tid; i < kRTok * E; i += kRThreads) {
      const int tl = i / E, e = i % E;
      const int64_t t = t0 + tl;
      if (t < T) {
        const float v = lg[tl * LGS + e];
        if (BF16)
          static_cast<uint16_t*>(logits_out)[t * E + e] = static_cast<uint16_t>(f32_to_bf16_bits(v));
        else
          static_cast<float*>(logits_out)[t * E + e] = v;
      }
    }
  }

  // ---- top-k per token, one warp per token
  constexpr int NV = EPAD / 32;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  for (int tl = warp; tl < kRTok; tl += kRThreads / 32) {
    const int64_t t = t0 + tl;
    if (t >= T) break;
    float v[NV];
    int id[NV];
#pragma unroll
    for (int q = 0; q < NV; ++q) {
      const int e = lane + 32 * q;
      v[q] = e < E ? lg[tl * LGS + e] : -INFINITY;
      id[q] = e < E ? e : INT_MAX;
    }
    float mx = 0.0f, my_v = 0.0f;
    int my_i = 0;
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
    // softmax denominator over all experts (fp32)
    float s = 0.0f;
#pragma unroll
    for (int q = 0; q < NV; ++q) {
      const int e = lane + 32 * q;
      if (e < E) s += expf(lg[tl * LGS + e] - mx);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    float p = lane < k ? expf(my_v - mx) / s : 0.0f;
    if (norm) {
      float ps = p;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
      p = p / fmaxf(ps, 1e-12f);
    }
    if (BF16) p = round_bf16(p);
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
}

template <int EPAD, bool BF16>
cudaError_t launch_router_t(const void* x, const void* w, const void* b, int64_t T, int d, int E,
                            int k, int norm, int32_t* idx, float* wf, void* wd, void* lo,
                            cudaStream_t s) {
  const int64_t blocks = cdiv64(T, kRTok);
  router_topk_kernel<EPAD, BF16><<<static_cast<unsigned>(blocks), kRThreads, 0, s>>>(
      x, w, b, T, d, E, k, norm, idx, wf, wd, lo);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_router_topk(const void* x, const void* w_router, const void* bias, int64_t T,
                               int d, int E, int k, int dtype, int norm, int32_t* topk_idx,
                               float* topk_w_f32, void* topk_w_dtype, void* logits_out,
                               cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  const bool bf16 = dtype == kDtypeBF16;
  if (E <= 64)
    return bf16 ? launch_router_t<64, true>(x, w_router, bias, T, d, E, k, norm, topk_idx,
                                           topk_w_f32, topk_w_dtype, logits_out, stream)
                : launch_router_t<64, false>(x, w_router, bias, T, d, E, k, norm, topk_idx,
                                            topk_w_f32, topk_w_dtype, logits_out, stream);
  return bf16 ? launch_router_t<128, true>(x, w_router, bias, T, d, E, k, norm, topk_idx,
                                          topk_w_f32, topk_w_dtype, logits_out, stream)
              : launch_router_t<128, false>(x, w_router, bias, T, d, E, k, norm, topk_idx,
                                           topk_w_f32, topk_w_dtype, logits_out, stream);
}

}  // namespace hmoe
