// Router for bf16 layers on the tensor cores, certified against the
// exact-order definition, with a fix-up pass for the tokens it cannot certify.
//
// Mirrors models/layers.py:604-610 (gate F.linear -> fp32 softmax -> top-k ->
// renormalise -> cast).  The routing a token gets is defined by its logits
// accumulated in fp32 in the fixed order of kLogitBlock (the order the CPU
// oracle and the CUDA-core router use), rounded to bf16.
//
// router_tc_kernel: one CTA per 128 tokens.  TMA streams the token tile
// [128 x 64] and the router weight [E x 64] per k-step through a smem ring;
// one thread issues tcgen05.mma (M=128, N=64/128, K=16) into TMEM.  The
// epilogue parks the fp32 logits in smem and routes one token per thread.  Each
// rounded logit carries the set of bf16 values the exact-order sum could
// round to: itself, plus a neighbour when the tensor-core sum lies within
// `cert_rel * max|logit|` of a rounding midpoint.  A token's top-k is
// accepted only if every order decision it contains (each pick against the
// next, the last pick against every unpicked expert) holds for all values in
// those sets; otherwise the token is appended to a fix-up list.
//
// The fix-up kernels recompute the listed tokens' logits in the exact order
// on the CUDA cores and route them again, overwriting the output:
// router_fixup_split_kernel (small T: token groups x expert groups over many
// CTAs, started early by programmatic dependent launch),
// router_fixup_wsmem_kernel (larger T, E <= 64: the whole weight in shared
// memory) and router_fixup_kernel (otherwise).
// The result equals the CUDA-core router's for every token.
#include <limits.h>
#include <stdlib.h>

#include <mutex>

#include "common.cuh"
#include "internal.h"
#include "router_common.cuh"

namespace hmoe {
namespace {

constexpr int RBM = 128;       // tokens per CTA (MMA M)
constexpr int RBK = 64;        // bf16 per 128-byte swizzled row
constexpr int kRtThreads = 192;

template <int EPAD>
struct RCfg {
  static constexpr int kStages = EPAD == 64 ? 6 : 4;
  static constexpr int kABytes = RBM * RBK * 2;
  static constexpr int kBBytes = EPAD * RBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kRingBytes = kStages * kStageBytes;
  static constexpr int kLgStride = EPAD + 1;
  static constexpr int kLgBytes = 3 * RBM * kLgStride * 4;  // values, keys, largest keys
  static constexpr int kMainBytes = kRingBytes > kLgBytes ? kRingBytes : kLgBytes;
  static constexpr int kCtlBytes = 256;
  static constexpr size_t kSmem = 1024 + kMainBytes + kCtlBytes;
  static_assert(kStageBytes % 1024 == 0, "stages keep the 1 KiB swizzle alignment");
  static_assert(kStages <= 8, "RtCtl holds eight stage barriers of each kind");
  static_assert(kSmem <= 232448, "shared memory budget");
};

struct RtCtl {
  uint64_t full[8];
  uint64_t empty[8];
  uint64_t acc_full;
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

struct RtParams {
  const uint16_t* bias;  // [E] bf16 or null
  int64_t T;
  int d, E, k, norm;
  int32_t* topk_idx;
  float* topk_w_f32;
  void* topk_w_dtype;
  uint16_t* logits_out;
  float* sums_out;        // diagnostic: the fp32 tensor-core sums (before the bias)
  int* fix_count;
  int32_t* fix_list;
  unsigned* group_done;   // split fix-up: finished expert groups per token group
  uint16_t* fix_logits;   // split fix-up: rounded logits per fix slot
  int* err;
  unsigned long long wait_limit_ns;
  float cert_rel;
};

// Orderable 16-bit image of a bf16 bit pattern: unsigned order = value
// order (negative values flipped), so key = (ob << 16) | (0xFFFF - e) sorts
// by value descending and, on equal values, by expert index ascending.
__device__ __forceinline__ uint32_t ob16(uint32_t b) {
  return (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
}

// Keys of the smallest and largest bf16 value the exact-order sum of this
// logit could round to (tensor-core sum v, margin delta).
__device__ __forceinline__ void key_range(float v, float delta, uint32_t e, uint32_t& kmin,
                                          uint32_t& kmax, uint32_t& key) {
  const uint32_t b = f32_to_bf16_bits(v);
  const uint32_t ob = ob16(b);
  const uint32_t lo16 = 0xFFFFu - e;
  key = (ob << 16) | lo16;
  uint32_t oblo = ob, obhi = ob;
  if (isfinite(v) && (b & 0x7F80u) != 0x7F80u) {
    const float a = fabsf(v);
    if (a <= delta) {
      // the sign itself is not certain: anything within +-delta (rounded out)
      const uint32_t m = (__float_as_uint(delta) >> 16) + 1;
      oblo = ob16(m | 0x8000u);
      obhi = ob16(m);
    } else {
      const uint32_t h = b & 0x7FFFu;  // magnitude as consecutive integers
      const bool up = a >= __uint_as_float((h << 16) | 0x8000u) - delta;
      const bool dn = h > 0 && a <= __uint_as_float(((h - 1) << 16) | 0x8000u) + delta;
      const bool neg = (b & 0x8000u) != 0;
      obhi = ob + ((neg ? dn : up) ? 1u : 0u);
      oblo = ob - ((neg ? up : dn) ? 1u : 0u);
    }
  }
  kmin = (oblo << 16) | lo16;
  kmax = (obhi << 16) | lo16;
}

// Route one token from its fp32 tensor-core logits.  vrow[0..E) holds the
// sums (biased in place), krow/xrow are scratch rows of the same thread.
// Picks the k largest rounded logits (lower index on ties); the result is
// certified when each pick's smallest possible key beats the next pick's
// largest, and the last pick's beats every unpicked expert's largest.
template <int KMAX>
__device__ __forceinline__ void route_row_certified(float* vrow, uint32_t* krow, uint32_t* xrow,
                                                    const RtParams& p, int64_t t) {
  const int E = p.E, k = p.k;
  if (p.sums_out)
    for (int e = 0; e < E; ++e) p.sums_out[t * E + e] = vrow[e];
  float mag = 0.0f;
  for (int e = 0; e < E; ++e) {
    float v = vrow[e];
    if (p.bias) v = v + bf16_bits_to_f32(p.bias[e]);
    vrow[e] = v;
    if (isfinite(v)) mag = fmaxf(mag, fabsf(v));
  }
  const float delta = p.cert_rel * mag;
  for (int e = 0; e < E; ++e) {
    uint32_t kmin, kmax, key;
    key_range(vrow[e], delta, static_cast<uint32_t>(e), kmin, kmax, key);
    krow[e] = key;
    xrow[e] = kmax;
  }
  uint32_t pk[KMAX];
  bool bad = false;
  uint32_t prev_min = 0;
#pragma unroll
  for (int j = 0; j < KMAX; ++j) {
    pk[j] = 0;
    if (j < k) {
      uint32_t best = 0;
      for (int e = 0; e < E; ++e) best = max(best, krow[e]);
      pk[j] = best;
      const int e = 0xFFFF - static_cast<int>(best & 0xFFFFu);
      krow[e] = 0;  // picked
      uint32_t kmin, kmax, key;
      key_range(vrow[e], delta, static_cast<uint32_t>(e), kmin, kmax, key);
      if (j > 0 && !(prev_min > kmax)) bad = true;
      prev_min = kmin;
    }
  }
  uint32_t rest = 0;  // largest key an unpicked expert could take
  for (int e = 0; e < E; ++e)
    if (krow[e] != 0) rest = max(rest, xrow[e]);
  if (!(prev_min > rest)) bad = true;
  // softmax over the rounded logits, weights of the picks
  const int e0 = 0xFFFF - static_cast<int>(pk[0] & 0xFFFFu);
  const float mx = round_bf16(vrow[e0]);
  float s = 0.0f;
  for (int e = 0; e < E; ++e) s += expf(round_bf16(vrow[e]) - mx);
  float pw[KMAX], ps = 0.0f;
#pragma unroll
  for (int j = 0; j < KMAX; ++j) {
    pw[j] = 0.0f;
    if (j < k) {
      const int e = 0xFFFF - static_cast<int>(pk[j] & 0xFFFFu);
      pw[j] = expf(round_bf16(vrow[e]) - mx) / s;
      ps += pw[j];
    }
  }
#pragma unroll
  for (int j = 0; j < KMAX; ++j) {
    if (j < k) {
      float w = p.norm ? pw[j] / fmaxf(ps, 1e-12f) : pw[j];
      w = round_bf16(w);
      const int64_t o = t * k + j;
      p.topk_idx[o] = 0xFFFF - static_cast<int>(pk[j] & 0xFFFFu);
      if (p.topk_w_f32) p.topk_w_f32[o] = w;
      if (p.topk_w_dtype)
        static_cast<uint16_t*>(p.topk_w_dtype)[o] = static_cast<uint16_t>(f32_to_bf16_bits(w));
    }
  }
  if (p.logits_out)
    for (int e = 0; e < E; ++e) p.logits_out[t * E + e] = static_cast<uint16_t>(f32_to_bf16_bits(vrow[e]));
  if (bad) {
    const int slot = atomicAdd(p.fix_count, 1);
    p.fix_list[slot] = static_cast<int32_t>(t);
  }
}

template <int EPAD, int KMAX>
__global__ void __launch_bounds__(kRtThreads, 1)
router_tc_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                 const RtParams p) {
  using C = RCfg<EPAD>;
  constexpr int NV = EPAD / 32;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  RtCtl& ctl = *reinterpret_cast<RtCtl*>(smem + C::kMainBytes);
  float* lg = reinterpret_cast<float*>(smem);
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * RBM;
  const int nkb = cdiv(p.d, RBK);
  const unsigned long long lim = p.wait_limit_ns;

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(smem_u32(&ctl.full[s]), 1);
      mbar_init(smem_u32(&ctl.empty[s]), 1);
    }
    mbar_init(smem_u32(&ctl.acc_full), 1);
    mbar_init(smem_u32(&ctl.drain), 1);
    ctl.abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW);
  } else if (warp == 1) {
    tmem_alloc(smem_u32(&ctl.tmem_base), EPAD);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl.tmem_base;
  volatile int* abort = &ctl.abort;
  int never = 0;
  bool acc_ok = true;
  // the fix-up grid may start now on the SMs this grid leaves free (it
  // waits for this grid's completion before it reads the fix list)
  grid_launch_dependents();
  // this CTA's 128 tokens own 32 counters of the split fix-up
  if (p.group_done && threadIdx.x < RBM / 4) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * (RBM / 4) + threadIdx.x;
    if (i < ((cdiv64(p.T, 4) + 3) & ~static_cast<int64_t>(3))) p.group_done[i] = 0u;
  }

  if (warp == 0) {
    if (lane == 0) {
      uint32_t phase = 0, pending = 0, pend_phase = 0;
      int stage = 0;
      for (int kb = 0; kb < nkb; ++kb) {
        if (!mbar_wait_bounded(smem_u32(&ctl.empty[stage]), phase ^ 1u, abort, p.err, lim)) break;
        const uint32_t fb = smem_u32(&ctl.full[stage]);
        const uint32_t sa = sbase + stage * C::kStageBytes;
        mbar_arrive_expect_tx(fb, C::kStageBytes);
        tma_load_2d(sa, &tmX, kb * RBK, static_cast<int>(t0), fb);
        tma_load_2d(sa + C::kABytes, &tmW, kb * RBK, 0, fb);
        pending |= 1u << stage;
        pend_phase = (pend_phase & ~(1u << stage)) | (phase << stage);
        if (++stage == C::kStages) { stage = 0; phase ^= 1u; }
      }
      for (int s = 0; s < C::kStages; ++s)
        if ((pending >> s) & 1u)
          mbar_wait_bounded(smem_u32(&ctl.full[s]), (pend_phase >> s) & 1u, &never, p.err, lim);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(RBM, EPAD);
      uint32_t phase = 0;
      int stage = 0;
      bool ok = true;
      for (int kb = 0; kb < nkb; ++kb) {
        if (!mbar_wait_bounded(smem_u32(&ctl.full[stage]), phase, abort, p.err, lim)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sa = sbase + stage * C::kStageBytes;
#pragma unroll
        for (int kk = 0; kk < RBK / 16; ++kk)
          tc_mma_bf16(tmem, smem_desc_sw128(sa + kk * 32), smem_desc_sw128(sa + C::kABytes + kk * 32),
                      idesc, (kb | kk) != 0 ? 1u : 0u);
        tc_commit(smem_u32(&ctl.empty[stage]));
        if (++stage == C::kStages) { stage = 0; phase ^= 1u; }
      }
      if (ok) tc_commit(smem_u32(&ctl.acc_full));
      tc_commit(smem_u32(&ctl.drain));
      mbar_wait_bounded(smem_u32(&ctl.drain), 0, &never, p.err, lim);
    }
  } else {
    // -------------- epilogue: one thread per token, its row of logits in smem
    const int quad = warp & 3;
    acc_ok = mbar_wait_bounded(smem_u32(&ctl.acc_full), 0, abort, p.err, lim);
    tc_fence_after();
    const int row = quad * 32 + lane;
    float* lrow = lg + row * C::kLgStride;
    if (acc_ok) {
#pragma unroll 1
      for (int c = 0; c < EPAD / 32; ++c) {
        uint32_t ra[32];
        tmem_ld_32cols(tmem + (static_cast<uint32_t>(quad * 32) << 16) + c * 32, ra);
        tc_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) lrow[c * 32 + i] = __uint_as_float(ra[i]);
      }
    }
    const int64_t t = t0 + row;
    uint32_t* krow = reinterpret_cast<uint32_t*>(lg + RBM * C::kLgStride) + row * C::kLgStride;
    uint32_t* xrow = reinterpret_cast<uint32_t*>(lg + 2 * RBM * C::kLgStride) + row * C::kLgStride;
    if (acc_ok && !*abort && t < p.T)
      route_row_certified<KMAX>(lrow, krow, xrow, p, t);
    tc_fence_before();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, EPAD);
  }
}

// Fix-up: exact-order logits for the listed tokens, then the same routing
// as every router.  The order (kLogitBlock) lets the blocks of k run in
// parallel: a CTA takes kFixG listed tokens; thread (expert e, block lane
// bg) runs the one-fma-per-k chains of blocks bg, bg + nbg, ... for all
// kFixG tokens at once, the block sums are then added in block order, and
// one warp per token routes it.
// One warp routes one token from its exact-order logits lrow[0..E) (bias
// included, not yet rounded): the same selection and weights as every router.
template <int NV>
__device__ __forceinline__ void fixup_route_token(const float* lrow, int64_t t, int E, int k,
                                                  int norm, int lane, int32_t* topk_idx,
                                                  float* topk_w_f32, void* topk_w_dtype,
                                                  uint16_t* logits_out) {
  float r[NV], sel[NV];
  int id[NV];
#pragma unroll
  for (int q = 0; q < NV; ++q) {
    const int ee = lane + 32 * q;
    r[q] = ee < E ? round_bf16(lrow[ee]) : -INFINITY;
    sel[q] = r[q];
    id[q] = ee < E ? ee : INT_MAX;
    if (logits_out && ee < E) logits_out[t * E + ee] = static_cast<uint16_t>(f32_to_bf16_bits(r[q]));
  }
  float my_v, mx;
  int my_i;
  warp_topk<NV>(sel, id, k, lane, my_v, my_i, mx);
  const float wgt = warp_route_weight<NV, true>(r, E, k, norm, lane, my_v, mx);
  write_route<true>(t, k, lane, my_i, wgt, topk_idx, topk_w_f32, topk_w_dtype);
}

constexpr int kFixThreads = 512;  // 64 experts x 8 block lanes (E <= 64), 128 x 4 (E <= 128)
constexpr int kFixG = 4;          // tokens per CTA pass

template <int NV>
__global__ void __launch_bounds__(kFixThreads)
router_fixup_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w,
                    const uint16_t* __restrict__ bias, int64_t T, int d, int E, int k, int norm,
                    const int* __restrict__ fix_count, const int32_t* __restrict__ fix_list,
                    int32_t* __restrict__ topk_idx, float* __restrict__ topk_w_f32,
                    void* __restrict__ topk_w_dtype, uint16_t* __restrict__ logits_out) {
  constexpr int EP = NV * 32;
  constexpr int NBG = kFixThreads / EP;       // block lanes per expert (8 / 4)
  extern __shared__ float fsm[];
  const int nb = cdiv(d, kLogitBlock);
  float* xs = fsm;                                        // [kFixG][d]
  float* part = fsm + kFixG * d;                          // [kFixG][EP][nb]
  float* lgt = part + kFixG * EP * nb;                    // [kFixG][EP]
  const int tid = threadIdx.x, lane = tid & 31, wib = tid >> 5;
  const int e = tid % EP, bg = tid / EP;
  const int n = *fix_count;
  for (int base = blockIdx.x * kFixG; base < n; base += gridDim.x * kFixG) {
    int64_t tok[kFixG];
#pragma unroll
    for (int g = 0; g < kFixG; ++g) {
      const int64_t tt = base + g < n ? fix_list[base + g] : -1;
      tok[g] = (tt >= 0 && tt < T) ? tt : -1;
    }
    for (int i = tid; i < kFixG * (d / 8); i += kFixThreads) {
      const int g = i / (d / 8), c = i % (d / 8);
      uint4 u = make_uint4(0, 0, 0, 0);
      if (tok[g] >= 0) u = __ldg(reinterpret_cast<const uint4*>(x + tok[g] * d) + c);
      float* xr = xs + g * d + c * 8;
      xr[0] = bf16_lo(u.x); xr[1] = bf16_hi(u.x); xr[2] = bf16_lo(u.y); xr[3] = bf16_hi(u.y);
      xr[4] = bf16_lo(u.z); xr[5] = bf16_hi(u.z); xr[6] = bf16_lo(u.w); xr[7] = bf16_hi(u.w);
    }
    __syncthreads();
    const uint16_t* wr = w + static_cast<int64_t>(min(e, E - 1)) * d;
    // A block's weights (64 k, 8 vectors) are loaded before its FMAs; the
    // token values come from shared memory four at a time.
    constexpr int kVec = kLogitBlock / 8;
    for (int b = bg; b < nb; b += NBG) {
      const int k0 = b * kLogitBlock, nvec = min(kLogitBlock, d - k0) / 8;
      uint4 wb[kVec];
#pragma unroll
      for (int c = 0; c < kVec; ++c)
        wb[c] = c < nvec ? __ldg(reinterpret_cast<const uint4*>(wr + k0) + c) : make_uint4(0, 0, 0, 0);
      float acc[kFixG];
#pragma unroll
      for (int g = 0; g < kFixG; ++g) acc[g] = 0.0f;
#pragma unroll
      for (int c = 0; c < kVec; ++c) {
        if (c < nvec) {
          const uint4 u = wb[c];
          const float wv[8] = {bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y),
                               bf16_lo(u.z), bf16_hi(u.z), bf16_lo(u.w), bf16_hi(u.w)};
#pragma unroll
          for (int g = 0; g < kFixG; ++g) {
            const float4* xv = reinterpret_cast<const float4*>(xs + g * d + k0 + c * 8);
            const float4 xa = xv[0], xb = xv[1];
            const float xr[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[g] = fmaf(xr[j], wv[j], acc[g]);
          }
        }
      }
#pragma unroll
      for (int g = 0; g < kFixG; ++g) part[(g * EP + e) * nb + b] = acc[g];
    }
    __syncthreads();
    for (int i = tid; i < kFixG * EP; i += kFixThreads) {
      const int g = i / EP, ee = i % EP;
      float tot = 0.0f;
      for (int b = 0; b < nb; ++b) tot = tot + part[(g * EP + ee) * nb + b];
      if (bias && ee < E) tot = tot + bf16_bits_to_f32(bias[ee]);
      lgt[g * EP + ee] = tot;
    }
    __syncthreads();
    if (wib < kFixG && tok[wib] >= 0)
      fixup_route_token<NV>(lgt + wib * EP, tok[wib], E, k, norm, lane, topk_idx, topk_w_f32,
                            topk_w_dtype, logits_out);
    __syncthreads();
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// Fix-up for E <= 64 with the whole router weight in shared memory (used
// where the split fix-up below would need more than one round): TMA
// brings W in [64 expert x 64 k] boxes (128-byte swizzle, the router's own
// map), so the weights are read from HBM/L2 once per CTA in large copies
// instead of one 16-byte load per thread and step.  Thread (expert e, token
// g) then runs every 64-k block of its logit in the exact order (one fma per
// k from +0, block sums added in ascending order from +0, then the bias), so
// the result is bit-identical to router_fixup_kernel.  Its 16-byte weight
// reads sit at e*128 + ((c ^ (e & 7)) * 16): four wavefronts per warp, the
// minimum for 512 bytes.
constexpr int kFixSmG = 4;  // tokens per CTA pass

__global__ void __launch_bounds__(64 * kFixSmG)
router_fixup_wsmem_kernel(const __grid_constant__ CUtensorMap tmW, const uint16_t* __restrict__ x,
                          const uint16_t* __restrict__ bias, int64_t T, int d, int E, int k, int norm,
                          const int* __restrict__ fix_count, const int32_t* __restrict__ fix_list,
                          int32_t* __restrict__ topk_idx, float* __restrict__ topk_w_f32,
                          void* __restrict__ topk_w_dtype, uint16_t* __restrict__ logits_out,
                          int* err, unsigned long long wait_limit_ns) {
  extern __shared__ uint8_t fraw[];
  uint8_t* wsm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(fraw) + 1023) &
                                            ~static_cast<uintptr_t>(1023));
  const int nb = cdiv(d, kLogitBlock);
  float* xs = reinterpret_cast<float*>(wsm + static_cast<size_t>(nb) * 8192);  // [G][d]
  float* lgt = xs + kFixSmG * d;                                                 // [G][64]
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  const int tid = threadIdx.x, lane = tid & 31, wib = tid >> 5;
  const int n = *fix_count;
  if (static_cast<int64_t>(blockIdx.x) * kFixSmG >= n) return;  // nothing listed for this CTA
  if (tid == 0) {
    abort_flag = 0;
    mbar_init(smem_u32(&bar), 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(smem_u32(&bar), static_cast<uint32_t>(nb) * 8192u);
    for (int b = 0; b < nb; ++b) tma_load_2d(smem_u32(wsm + b * 8192), &tmW, b * kLogitBlock, 0, smem_u32(&bar));
  }
  __syncthreads();
  bool have_w = false;
  const int e = tid & 63, g = tid >> 6;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * kFixSmG; base < n;
       base += static_cast<int64_t>(gridDim.x) * kFixSmG) {
    int64_t tok[kFixSmG];
#pragma unroll
    for (int j = 0; j < kFixSmG; ++j) {
      const int64_t tt = base + j < n ? fix_list[base + j] : -1;
      tok[j] = (tt >= 0 && tt < T) ? tt : -1;
    }
    // token rows -> fp32 in shared memory; each thread's loads are all issued
    // before its stores
    constexpr int kXLoads = 8;
    const int nx = kFixSmG * (d / 8);
    for (int i0 = tid; i0 < nx; i0 += blockDim.x * kXLoads) {
      uint4 u[kXLoads];
#pragma unroll
      for (int q = 0; q < kXLoads; ++q) {
        const int i = i0 + q * blockDim.x;
        u[q] = make_uint4(0, 0, 0, 0);
        if (i < nx) {
          const int j = i / (d / 8), c = i % (d / 8);
          if (tok[j] >= 0) u[q] = __ldg(reinterpret_cast<const uint4*>(x + tok[j] * d) + c);
        }
      }
#pragma unroll
      for (int q = 0; q < kXLoads; ++q) {
        const int i = i0 + q * blockDim.x;
        if (i < nx) {
          const int j = i / (d / 8), c = i % (d / 8);
          float* xr = xs + j * d + c * 8;
          xr[0] = bf16_lo(u[q].x); xr[1] = bf16_hi(u[q].x); xr[2] = bf16_lo(u[q].y);
          xr[3] = bf16_hi(u[q].y); xr[4] = bf16_lo(u[q].z); xr[5] = bf16_hi(u[q].z);
          xr[6] = bf16_lo(u[q].w); xr[7] = bf16_hi(u[q].w);
        }
      }
    }
    if (!have_w) {  // every thread sees the weights land (bounded)
      have_w = mbar_wait_bounded(smem_u32(&bar), 0, &abort_flag, err, wait_limit_ns);
      if (!have_w) return;  // the copies are gone or the error is recorded
    }
    __syncthreads();
    // Four blocks' chains at a time (independent accumulators hide the fma
    // latency); their sums are added to the total in ascending block order.
    constexpr int kIl = 4;
    float tot = 0.0f;
    for (int b0 = 0; b0 < nb; b0 += kIl) {
      float acc[kIl];
      int nvec[kIl];
#pragma unroll
      for (int q = 0; q < kIl; ++q) {
        acc[q] = 0.0f;
        nvec[q] = b0 + q < nb ? min(kLogitBlock, d - (b0 + q) * kLogitBlock) / 8 : 0;
      }
#pragma unroll
      for (int c = 0; c < kLogitBlock / 8; ++c) {
#pragma unroll
        for (int q = 0; q < kIl; ++q) {
          if (c < nvec[q]) {
            const uint8_t* box = wsm + (b0 + q) * 8192 + e * 128;
            const float* xb = xs + g * d + (b0 + q) * kLogitBlock;
            const uint4 u = *reinterpret_cast<const uint4*>(box + ((c ^ (e & 7)) << 4));
            const float4 xa = reinterpret_cast<const float4*>(xb + c * 8)[0];
            const float4 xc = reinterpret_cast<const float4*>(xb + c * 8)[1];
            float a = acc[q];
            a = fmaf(xa.x, bf16_lo(u.x), a);
            a = fmaf(xa.y, bf16_hi(u.x), a);
            a = fmaf(xa.z, bf16_lo(u.y), a);
            a = fmaf(xa.w, bf16_hi(u.y), a);
            a = fmaf(xc.x, bf16_lo(u.z), a);
            a = fmaf(xc.y, bf16_hi(u.z), a);
            a = fmaf(xc.z, bf16_lo(u.w), a);
            a = fmaf(xc.w, bf16_hi(u.w), a);
            acc[q] = a;
          }
        }
      }
#pragma unroll
      for (int q = 0; q < kIl; ++q)
        if (b0 + q < nb) tot = tot + acc[q];
    }
    if (bias && e < E) tot = tot + bf16_bits_to_f32(bias[e]);
    lgt[g * 64 + e] = tot;
    __syncthreads();
    if (wib < kFixSmG && tok[wib] >= 0)
      fixup_route_token<2>(lgt + wib * 64, tok[wib], E, k, norm, lane, topk_idx, topk_w_f32,
                           topk_w_dtype, logits_out);
    __syncthreads();
  }
  if (!have_w) mbar_wait_bounded(smem_u32(&bar), 0, &abort_flag, err, wait_limit_ns);
}

// Fix-up split over CTAs (d <= 2048, any E <= 128).
//
// The fix list is cut into groups of kSplitG tokens and the experts into
// groups of kSplitE; a work item is one (token group, expert group) and a CTA
// keeps one expert group for all its items, so it loads that slice of the
// weight (kSplitE rows) into shared memory once.  The kernel is launched as a
// programmatic dependent of router_tc_kernel: the slice is loaded before
// grid_dependency_wait(), while the tensor-core pass still runs, and the fix
// list only after it.
//
// Warp w takes expert e = group * kSplitE + w; lane (token g, eighth h) runs
// the blocks [h * nbh, (h + 1) * nbh) of that expert's logit for token g: one
// fma per k from +0 in ascending k within a block.  The block sums are added
// in ascending block order from +0, handed from eighth to eighth with
// shuffles, then the bias: the exact-order logit, bit-identical to
// router_fixup_kernel and to the CUDA-core router (padding past d adds +0
// products, which leave a block sum unchanged).  The rounded logits go to
// scratch; the last CTA to finish a token group (a counter per group) routes
// its tokens, one warp each.
constexpr int kSplitG = 4;                    // tokens per work item
constexpr int kSplitE = 8;                    // experts per work item (one warp each)
constexpr int kSplitH = 8;                    // lanes per (expert, token)
constexpr int kSplitMaxNbh = 4;               // blocks per lane: d <= 2048
constexpr int kSplitWRow = kLogitBlock + 8;   // bf16 per weight block in smem (16 B padding)
constexpr int kSplitXRow = kLogitBlock + 4;   // floats per token block in smem (16 B padding)
constexpr int kSplitLogitStride = 128;        // rounded logits per fix slot in scratch
constexpr int kSplitThreads = 32 * kSplitE;

size_t split_smem_bytes(int d) {
  const size_t nb = static_cast<size_t>(cdiv(d, kLogitBlock));
  return nb * (kSplitE * kSplitWRow * 2 + kSplitG * kSplitXRow * 4) +
         kSplitG * kSplitLogitStride * 4;
}

template <int NV>
__global__ void __launch_bounds__(kSplitThreads)
router_fixup_split_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w,
                          const uint16_t* __restrict__ bias, int64_t T, int d, int E, int k,
                          int norm, const int* fix_count, const int32_t* fix_list,
                          unsigned* group_done, uint16_t* fix_logits, int32_t* topk_idx,
                          float* topk_w_f32, void* topk_w_dtype, uint16_t* logits_out) {
  // fix_count, fix_list and group_done are written by the grid this one
  // depends on (or by other CTAs): they are read (volatile) only after
  // grid_dependency_wait(), never as read-only data that could be loaded
  // earlier.
  extern __shared__ float4 sraw4[];
  const int nb = cdiv(d, kLogitBlock);
  const int nbh = cdiv(nb, kSplitH);
  const int n_eg = cdiv(E, kSplitE);
  const int eg = static_cast<int>(blockIdx.x) % n_eg;
  const int lanes_tg = static_cast<int>(gridDim.x) / n_eg;  // the grid is a multiple of n_eg
  uint16_t* ws = reinterpret_cast<uint16_t*>(sraw4);                   // [kSplitE][nb][72]
  float* xs = reinterpret_cast<float*>(ws + kSplitE * nb * kSplitWRow);  // [kSplitG][nb][68]
  float* lg = xs + kSplitG * nb * kSplitXRow;                          // [kSplitG][128]
  __shared__ int64_t s_tok[kSplitG];
  __shared__ int s_last;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane / kSplitH, h = lane % kSplitH;
  const int e = eg * kSplitE + warp;
  // this CTA's weight slice (zeros past E and d); it does not depend on the
  // grid before this one
  // (warp w loads the row of its own expert e)
  for (int r = lane; r < nb * (kLogitBlock / 8); r += 32) {
    const int b = r >> 3, c = r & 7;
    uint4 u = make_uint4(0, 0, 0, 0);
    if (e < E && r * 8 < d) u = __ldg(reinterpret_cast<const uint4*>(w + static_cast<int64_t>(e) * d) + r);
    *reinterpret_cast<uint4*>(ws + (warp * nb + b) * kSplitWRow + c * 8) = u;
  }
  grid_dependency_wait();  // the tensor-core pass and its fix list are complete
  const int n = *reinterpret_cast<const volatile int*>(fix_count);
  const int ngroups = cdiv(n, kSplitG);
  for (int tg = static_cast<int>(blockIdx.x) / n_eg; tg < ngroups; tg += lanes_tg) {
    __syncthreads();  // the previous item is finished with xs, lg and s_tok
    if (tid < kSplitG) {
      const int slot = tg * kSplitG + tid;
      const int64_t t = slot < n ? reinterpret_cast<const volatile int32_t*>(fix_list)[slot] : -1;
      s_tok[tid] = (t >= 0 && t < T) ? t : -1;
    }
    __syncthreads();
    // the group's token rows -> fp32 (zeros past d and for empty slots)
    // (warp w < kSplitG loads the row of token w)
    if (warp < kSplitG) {
      const int64_t t = s_tok[warp];
      for (int r = lane; r < nb * (kLogitBlock / 8); r += 32) {
        const int b = r >> 3, c = r & 7;
        uint4 u = make_uint4(0, 0, 0, 0);
        if (t >= 0 && r * 8 < d) u = __ldg(reinterpret_cast<const uint4*>(x + t * d) + r);
        float* xr = xs + (warp * nb + b) * kSplitXRow + c * 8;
        reinterpret_cast<float4*>(xr)[0] = make_float4(bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y));
        reinterpret_cast<float4*>(xr)[1] = make_float4(bf16_lo(u.z), bf16_hi(u.z), bf16_lo(u.w), bf16_hi(u.w));
      }
    }
    __syncthreads();
    float acc[kSplitMaxNbh];
#pragma unroll
    for (int j = 0; j < kSplitMaxNbh; ++j) acc[j] = 0.0f;
    const int b0 = h * nbh;
#pragma unroll
    for (int c = 0; c < kLogitBlock / 8; ++c) {
#pragma unroll
      for (int j = 0; j < kSplitMaxNbh; ++j) {
        const int b = b0 + j;
        if (j < nbh && b < nb) {
          const uint4 u = *reinterpret_cast<const uint4*>(ws + (warp * nb + b) * kSplitWRow + c * 8);
          const float* xb = xs + (g * nb + b) * kSplitXRow + c * 8;
          const float4 xa = reinterpret_cast<const float4*>(xb)[0];
          const float4 xc = reinterpret_cast<const float4*>(xb)[1];
          float a = acc[j];
          a = fmaf(xa.x, bf16_lo(u.x), a);
          a = fmaf(xa.y, bf16_hi(u.x), a);
          a = fmaf(xa.z, bf16_lo(u.y), a);
          a = fmaf(xa.w, bf16_hi(u.y), a);
          a = fmaf(xc.x, bf16_lo(u.z), a);
          a = fmaf(xc.y, bf16_hi(u.z), a);
          a = fmaf(xc.z, bf16_lo(u.w), a);
          a = fmaf(xc.w, bf16_hi(u.w), a);
          acc[j] = a;
        }
      }
    }
    // ascending block order: eighth h continues the running sum of h - 1
    // (the eighths of one (expert, token) are adjacent lanes)
    float run = 0.0f;
#pragma unroll
    for (int q = 0; q < kSplitH; ++q) {
      const float prev = __shfl_up_sync(0xffffffffu, run, 1);
      if (h == q) {
        float t = q == 0 ? 0.0f : prev;
#pragma unroll
        for (int j = 0; j < kSplitMaxNbh; ++j)
          if (j < nbh && b0 + j < nb) t = t + acc[j];
        run = t;
      }
    }
    if (h == kSplitH - 1 && e < E) {
      float tot = run;
      if (bias) tot = tot + bf16_bits_to_f32(bias[e]);
      fix_logits[static_cast<int64_t>(tg * kSplitG + g) * kSplitLogitStride + e] =
          static_cast<uint16_t>(f32_to_bf16_bits(tot));
      __threadfence();
    }
    __syncthreads();
    if (tid == 0) {
      const unsigned prev = atomicAdd(group_done + tg, 1u);
      s_last = prev == static_cast<unsigned>(n_eg - 1);
    }
    __syncthreads();
    if (s_last) {  // every expert group of this token group is written: route it
      __threadfence();
      if (warp < kSplitG) {
        const int64_t slot = static_cast<int64_t>(tg) * kSplitG + warp;
        const volatile uint16_t* src = fix_logits + slot * kSplitLogitStride;
        for (int ee = lane; ee < NV * 32; ee += 32)
          lg[warp * kSplitLogitStride + ee] = ee < E ? bf16_bits_to_f32(src[ee]) : 0.0f;
        __syncwarp();
        if (s_tok[warp] >= 0)
          fixup_route_token<NV>(lg + warp * kSplitLogitStride, s_tok[warp], E, k, norm, lane,
                                topk_idx, topk_w_f32, topk_w_dtype, logits_out);
      }
    }
  }
}

bool map_rows(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {RBK, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// ----------------------------------------------------------------------------
// router_rows_kernel: the tensor-core pass with 64 tokens per CTA.
//
// x [T, d] is read as the row-major matrix [2T, d/2] (the same bytes): row
// 2t is the first half of token t's hidden state, row 2t+1 the second.  One
// 128-row MMA tile is then 64 tokens, and its B operand stacks the two
// halves of the router weight, [W[:, :d/2]; W[:, d/2:]] (2E rows), so that
// accumulator row 2t, columns [0, E) hold the first half's sums and row
// 2t+1, columns [E, 2E) the second half's; logit = first + second.  (The
// other two quarters of the product are not used: the tensor cores have
// time to spare, HBM does not.)  Twice as many CTAs as 128-token tiles, two
// per SM for E <= 64, so one CTA's epilogue overlaps another's stream.
//
// A configuration serves every E up to its EMAX (64 or 128): weight rows
// E..EMAX-1 of each half are past the end of W, so TMA fills them with zeros
// and those experts are never picked.
//
// Epilogue: 8 warps.  The four warps that own the accumulator's TMEM lane
// quadrants park each row's useful half in shared memory and meet the other
// four at a hardware named barrier (no spinning).  Then every token is routed
// by 4 lanes, each holding E/4 logits (experts s, s+4, ...): the same
// certified selection as route_row_certified (order-preserving keys, the
// set of bf16 values an exact-order sum could round to, each pick against
// the next, the last against every unpicked expert) with group shuffles,
// the softmax over the rounded logits, and the same outputs; uncertified
// tokens go to the fix list.
constexpr int RRT = 64;          // tokens per CTA
constexpr int kRrEpiWarps = 8;   // warps 2..9; 4 lanes per token
constexpr int kRrThreads = 64 + 32 * kRrEpiWarps;

template <int E>  // the largest expert count of the configuration (64 or 128)
struct RrCfg {
  static constexpr int kN = 2 * E;                    // MMA N (and TMEM columns)
  static constexpr int kABytes = 128 * RBK * 2;        // 16 KiB: 64 tokens x 2 halves
  static constexpr int kBBytes = kN * RBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = E <= 64 ? 3 : 4;       // E <= 64: two CTAs per SM
  static constexpr int kRingBytes = kStages * kStageBytes;
  // floats per token row: E + 4 puts the 32 lanes of a routing warp (8
  // tokens x 4 lanes, lane s reading expert s + 4i) in 32 different banks
  static constexpr int kLgStride = E + 4;
  static constexpr int kLgBytes = 2 * RRT * kLgStride * 4;  // the two halves' sums
  static constexpr int kMainBytes = kRingBytes > kLgBytes ? kRingBytes : kLgBytes;
  static constexpr int kCtlBytes = 256;
  static constexpr size_t kSmem = 1024 + kMainBytes + kCtlBytes;
  static_assert(kStageBytes % 1024 == 0, "stages keep the 1 KiB swizzle alignment");
  static_assert(kStages <= 8, "RtCtl holds eight stage barriers of each kind");
  static_assert(kSmem <= 232448, "shared memory budget");
};

// Reductions over the 4 lanes of one token.  `gm` names exactly those four
// lanes: a warp's other tokens may be past T and not take part.
__device__ __forceinline__ uint32_t shfl4_max(uint32_t v, unsigned gm) {
  v = max(v, __shfl_xor_sync(gm, v, 1));
  return max(v, __shfl_xor_sync(gm, v, 2));
}
__device__ __forceinline__ float shfl4_maxf(float v, unsigned gm) {
  v = fmaxf(v, __shfl_xor_sync(gm, v, 1));
  return fmaxf(v, __shfl_xor_sync(gm, v, 2));
}
__device__ __forceinline__ float shfl4_sum(float v, unsigned gm) {
  v += __shfl_xor_sync(gm, v, 1);
  return v + __shfl_xor_sync(gm, v, 2);
}
// bf16 value (as fp32) of an order-preserving key
__device__ __forceinline__ float key_value(uint32_t key) {
  const uint32_t ob = key >> 16;
  const uint32_t b = (ob & 0x8000u) ? (ob & 0x7FFFu) : (~ob & 0xFFFFu);
  return bf16_bits_to_f32(b);
}

__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Route token t on the 4 lanes (s = 0..3, mask gm) of its group.  The
// logits are a0[e] (+ a1[e] when a1 is set: the two halves' sums), plus the
// bias.  Lane s holds experts s, s+4, ...  delta_rel > 0: certified selection
// against the bf16 values each logit could round to within delta_rel *
// max|logit|, returning true when some order decision is not certain
// (the caller lists the token for the fix-up); delta_rel = 0: the logits are
// exact and every decision holds.  Writes topk_idx, the weights and (when
// asked) the rounded logits; with `sums` also the unbiased sums.
template <int E, int KMAX>
__device__ __forceinline__ bool route4(const float* a0, const float* a1, const RtParams& p,
                                       float delta_rel, int64_t t, int s, unsigned gm,
                                       bool sums) {
  constexpr int NE = E / 4;
  const int En = p.E;
  float v[NE];
  float mag = 0.0f;
#pragma unroll
  for (int i = 0; i < NE; ++i) {
    const int e = s + 4 * i;
    float x = -INFINITY;  // experts past E: never picked (key 0 below)
    if (e < En) {
      x = a1 ? a0[e] + a1[e] : a0[e];
      if (sums && p.sums_out) p.sums_out[t * En + e] = x;
      if (p.bias) x = x + bf16_bits_to_f32(p.bias[e]);
      if (isfinite(x)) mag = fmaxf(mag, fabsf(x));
      if (p.logits_out) p.logits_out[t * En + e] = static_cast<uint16_t>(f32_to_bf16_bits(x));
    }
    v[i] = x;
  }
  mag = shfl4_maxf(mag, gm);
  const float delta = delta_rel * mag;
  // softmax over the rounded logits
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < NE; ++i) mx = fmaxf(mx, round_bf16(v[i]));
  mx = shfl4_maxf(mx, gm);
  float ssum = 0.0f;
#pragma unroll
  for (int i = 0; i < NE; ++i) ssum += expf(round_bf16(v[i]) - mx);
  ssum = shfl4_sum(ssum, gm);
  uint32_t key[NE], kmn[NE], kmx[NE];
#pragma unroll
  for (int i = 0; i < NE; ++i) {
    key_range(v[i], delta, static_cast<uint32_t>(s + 4 * i), kmn[i], kmx[i], key[i]);
    if (s + 4 * i >= En) key[i] = kmn[i] = kmx[i] = 0u;
  }
  uint32_t pk[KMAX];
  bool bad = false;
  uint32_t prev_min = 0;
#pragma unroll
  for (int r = 0; r < KMAX; ++r) {
    pk[r] = 0;
    if (r < p.k) {
      uint32_t best = 0;
#pragma unroll
      for (int i = 0; i < NE; ++i) best = max(best, key[i]);
      best = shfl4_max(best, gm);
      uint32_t bmin = 0, bmax = 0;
#pragma unroll
      for (int i = 0; i < NE; ++i)
        if (key[i] == best) { bmin = kmn[i]; bmax = kmx[i]; key[i] = 0; }
      // only the owner lane found it: the others hold zeros
      bmin = shfl4_max(bmin, gm);
      bmax = shfl4_max(bmax, gm);
      if (r > 0 && !(prev_min > bmax)) bad = true;
      prev_min = bmin;
      pk[r] = best;
    }
  }
  uint32_t rest = 0;  // largest key an unpicked expert could take
#pragma unroll
  for (int i = 0; i < NE; ++i)
    if (key[i] != 0) rest = max(rest, kmx[i]);
  rest = shfl4_max(rest, gm);
  if (!(prev_min > rest)) bad = true;
  float pw[KMAX], ps = 0.0f;
#pragma unroll
  for (int r = 0; r < KMAX; ++r) {
    pw[r] = 0.0f;
    if (r < p.k) {
      pw[r] = expf(key_value(pk[r]) - mx) / ssum;
      ps += pw[r];
    }
  }
#pragma unroll
  for (int r = 0; r < KMAX; ++r) {
    if (r < p.k && (r & 3) == s) {
      float w = p.norm ? pw[r] / fmaxf(ps, 1e-12f) : pw[r];
      w = round_bf16(w);
      const int64_t o = t * p.k + r;
      p.topk_idx[o] = 0xFFFF - static_cast<int>(pk[r] & 0xFFFFu);
      if (p.topk_w_f32) p.topk_w_f32[o] = w;
      if (p.topk_w_dtype)
        static_cast<uint16_t*>(p.topk_w_dtype)[o] = static_cast<uint16_t>(f32_to_bf16_bits(w));
    }
  }
  return bad;
}

template <int E, int KMAX>  // E: the configuration's expert maximum (p.E <= E)
__global__ void __launch_bounds__(kRrThreads, E <= 64 ? 2 : 1)
router_rows_kernel(const __grid_constant__ CUtensorMap tmX2, const __grid_constant__ CUtensorMap tmW,
                   const RtParams p) {
  using C = RrCfg<E>;
  constexpr int NE = E / 4;  // logits per lane
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  RtCtl& ctl = *reinterpret_cast<RtCtl*>(smem + C::kMainBytes);
  float* lg0 = reinterpret_cast<float*>(smem);          // [64][E+1] first halves
  float* lg1 = lg0 + RRT * C::kLgStride;                // [64][E+1] second halves
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * RRT;
  const int half = p.d / 2;
  const int nkb = cdiv(half, RBK);
  const unsigned long long lim = p.wait_limit_ns;

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(smem_u32(&ctl.full[s]), 1);
      mbar_init(smem_u32(&ctl.empty[s]), 1);
    }
    mbar_init(smem_u32(&ctl.acc_full), 1);
    mbar_init(smem_u32(&ctl.drain), 1);
    ctl.abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmX2);
    tma_prefetch_desc(&tmW);
  } else if (warp == 1) {
    tmem_alloc(smem_u32(&ctl.tmem_base), C::kN);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl.tmem_base;
  volatile int* abort = &ctl.abort;
  int never = 0;
  grid_launch_dependents();
  // this CTA's 64 tokens own 16 counters of the split fix-up
  if (p.group_done && threadIdx.x < RRT / 4) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * (RRT / 4) + threadIdx.x;
    if (i < ((cdiv64(p.T, 4) + 3) & ~static_cast<int64_t>(3))) p.group_done[i] = 0u;
  }

  if (warp == 0) {
    if (lane == 0) {
      uint32_t phase = 0, pending = 0, pend_phase = 0;
      int stage = 0;
      for (int kb = 0; kb < nkb; ++kb) {
        if (!mbar_wait_bounded(smem_u32(&ctl.empty[stage]), phase ^ 1u, abort, p.err, lim)) break;
        const uint32_t fb = smem_u32(&ctl.full[stage]);
        const uint32_t sa = sbase + stage * C::kStageBytes;
        mbar_arrive_expect_tx(fb, C::kStageBytes);
        tma_load_2d(sa, &tmX2, kb * RBK, static_cast<int>(2 * t0), fb);
        tma_load_2d(sa + C::kABytes, &tmW, kb * RBK, 0, fb);
        tma_load_2d(sa + C::kABytes + E * 128, &tmW, half + kb * RBK, 0, fb);
        pending |= 1u << stage;
        pend_phase = (pend_phase & ~(1u << stage)) | (phase << stage);
        if (++stage == C::kStages) { stage = 0; phase ^= 1u; }
      }
      for (int s = 0; s < C::kStages; ++s)
        if ((pending >> s) & 1u)
          mbar_wait_bounded(smem_u32(&ctl.full[s]), (pend_phase >> s) & 1u, &never, p.err, lim);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(128, C::kN);
      uint32_t phase = 0;
      int stage = 0;
      bool ok = true;
      for (int kb = 0; kb < nkb; ++kb) {
        if (!mbar_wait_bounded(smem_u32(&ctl.full[stage]), phase, abort, p.err, lim)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sa = sbase + stage * C::kStageBytes;
#pragma unroll
        for (int kk = 0; kk < RBK / 16; ++kk)
          tc_mma_bf16(tmem, smem_desc_sw128(sa + kk * 32), smem_desc_sw128(sa + C::kABytes + kk * 32),
                      idesc, (kb | kk) != 0 ? 1u : 0u);
        tc_commit(smem_u32(&ctl.empty[stage]));
        if (++stage == C::kStages) { stage = 0; phase ^= 1u; }
      }
      if (ok) tc_commit(smem_u32(&ctl.acc_full));
      tc_commit(smem_u32(&ctl.drain));
      mbar_wait_bounded(smem_u32(&ctl.drain), 0, &never, p.err, lim);
    }
  } else {
    const int ew = warp - 2;
    constexpr int kEpi = 32 * kRrEpiWarps;
    // One warp waits (bounded) for the accumulator; the other seven block at
    // a hardware named barrier meanwhile instead of spinning next to the
    // producer and MMA warps.
    if (ew == 0) {
      const bool ok = mbar_wait_bounded(smem_u32(&ctl.acc_full), 0, abort, p.err, lim);
      if (!ok && lane == 0) *abort = 1;
    }
    named_barrier_sync(1, kEpi);
    tc_fence_after();
    if (ew < 4 && !*abort) {
      // ---- TMEM readers: row r = 32 quad + lane is token r / 2, half r & 1
      const int quad = warp & 3;
      const int r = quad * 32 + lane;
      float* dst = ((r & 1) ? lg1 : lg0) + (r >> 1) * C::kLgStride;
      const uint32_t col0 = (r & 1) ? E : 0;  // this half's useful columns
#pragma unroll 1
      for (int c = 0; c < E / 32; ++c) {
        uint32_t ra[32], rb[32];
        tmem_ld_32cols(tmem + (static_cast<uint32_t>(quad * 32) << 16) + c * 32, ra);
        tmem_ld_32cols(tmem + (static_cast<uint32_t>(quad * 32) << 16) + E + c * 32, rb);
        tc_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) dst[c * 32 + i] = __uint_as_float(col0 ? rb[i] : ra[i]);
      }
    }
    tc_fence_before();
    named_barrier_sync(1, kEpi);
    // ---- routing: token j on lanes 4 (j % 8) .. +3 of warp j / 8
    const bool live = !*abort;
    {
      const int j = ew * 8 + (lane >> 2), s = lane & 3;
      const unsigned gm = 0xFu << (lane & 28);  // this token's four lanes
      const int64_t t = t0 + j;
      if (live && t < p.T) {  // uniform over the 4 lanes of a token
        const bool bad = route4<E, KMAX>(lg0 + j * C::kLgStride, lg1 + j * C::kLgStride, p,
                                         p.cert_rel, t, s, gm, true);
        if (bad && s == 0) p.fix_list[atomicAdd(p.fix_count, 1)] = static_cast<int32_t>(t);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kN);
  }
}

// x [T, d] as [2T, d/2] rows with [128 x 64] boxes (the row-split operand).
bool map_half_rows(CUtensorMap* m, const void* base, uint64_t T, uint64_t d) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[2] = {d / 2, 2 * T};
  const cuuint64_t strides[1] = {d};  // (d / 2) bf16
  const cuuint32_t box[2] = {RBK, 128};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The row-split pass needs 16-byte aligned halves of each row.
inline bool rows_pass_fits(int d) { return d % 16 == 0; }

// HMOE_ROUTER_WHOLE_ROWS=1 (read once per process) keeps the 128-token
// whole-row kernel for every d, so tests can compare the two passes.
bool router_whole_rows_forced() {
  static const bool forced = [] {
    const char* v = getenv("HMOE_ROUTER_WHOLE_ROWS");
    return v && atoi(v) != 0;
  }();
  return forced;
}

template <int E, int KMAX>
cudaError_t launch_rows_tc(const void* x, const void* w, const RtParams& p, cudaStream_t st) {
  using C = RrCfg<E>;
  static int done[64] = {0};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!done[dev]) {
      e = cudaFuncSetAttribute(router_rows_kernel<E, KMAX>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(C::kSmem));
      if (e != cudaSuccess) return e;
      e = cudaFuncSetAttribute(router_rows_kernel<E, KMAX>,
                               cudaFuncAttributePreferredSharedMemoryCarveout, 100);
      if (e != cudaSuccess) return e;
      done[dev] = 1;
    }
  }
  CUtensorMap mx, mw;
  if (!map_half_rows(&mx, x, static_cast<uint64_t>(p.T), static_cast<uint64_t>(p.d)) ||
      !map_rows(&mw, w, static_cast<uint64_t>(p.E), static_cast<uint64_t>(p.d), E))
    return cudaErrorInvalidValue;
  router_rows_kernel<E, KMAX><<<static_cast<unsigned>(cdiv64(p.T, RRT)), kRrThreads, C::kSmem, st>>>(
      mx, mw, p);
  return cudaGetLastError();
}

template <int EPAD, int KMAX>
cudaError_t launch_tc(const void* x, const void* w, const RtParams& p, cudaStream_t st) {
  using C = RCfg<EPAD>;
  constexpr int NV = EPAD / 32;
  static int done[64] = {0};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  const size_t fix_smem =
      sizeof(float) * (static_cast<size_t>(kFixG) * p.d +
                       static_cast<size_t>(kFixG) * EPAD * cdiv(p.d, kLogitBlock) +
                       static_cast<size_t>(kFixG) * EPAD);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!done[dev]) {
      e = cudaFuncSetAttribute(router_tc_kernel<EPAD, KMAX>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(C::kSmem));
      if (e != cudaSuccess) return e;
      e = cudaFuncSetAttribute(router_fixup_kernel<NV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               232448);
      if (e != cudaSuccess) return e;
      e = cudaFuncSetAttribute(router_fixup_wsmem_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               232448 - 64);
      if (e != cudaSuccess) return e;
      e = cudaFuncSetAttribute(router_fixup_split_kernel<NV>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(split_smem_bytes(kLogitBlock * kSplitH * kSplitMaxNbh)));
      if (e != cudaSuccess) return e;
      done[dev] = 1;
    }
  }
  if (fix_smem > 232448) return cudaErrorInvalidValue;
  CUtensorMap mx, mw;
  if (!map_rows(&mx, x, static_cast<uint64_t>(p.T), static_cast<uint64_t>(p.d), RBM) ||
      !map_rows(&mw, w, static_cast<uint64_t>(p.E), static_cast<uint64_t>(p.d), EPAD))
    return cudaErrorInvalidValue;
  // the tensor-core pass: 64-token CTAs over the two halves of each row when
  // d splits into 16-byte aligned halves (router_rows_kernel), else 128-token
  // CTAs over whole rows
  if (rows_pass_fits(p.d) && !router_whole_rows_forced())
    e = launch_rows_tc<EPAD, KMAX>(x, w, p, st);
  else
    router_tc_kernel<EPAD, KMAX><<<static_cast<unsigned>(cdiv64(p.T, RBM)), kRtThreads, C::kSmem,
                                   st>>>(mx, mw, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int nb = cdiv(p.d, kLogitBlock);
  // The split fix-up's grid: a multiple of the expert groups, one token group
  // lane per 128 tokens (a few percent of the tokens go to the fix-up, four
  // per group), at most four CTAs per SM.  Where that cap would leave the
  // usual load more than one round per lane, the single-pass kernel with the
  // whole weight in shared memory is faster.
  const int n_eg = cdiv(p.E, kSplitE);
  const int sms = num_sms_for_current_device();
  // expected fix list: under 1% of the tokens at the margin in use, four per group
  const int64_t want = cdiv64(p.T, 512);
  const int cap = (4 * sms) / n_eg > 1 ? (4 * sms) / n_eg : 1;
  const size_t wsm_smem = 1024 + static_cast<size_t>(nb) * 8192 +
                          sizeof(float) * (static_cast<size_t>(kFixSmG) * p.d + kFixSmG * 64);
  const bool wsmem_ok = EPAD == 64 && wsm_smem <= 232448 - 64;
  if (nb <= kSplitH * kSplitMaxNbh && (want <= cap || !wsmem_ok)) {
    // programmatic dependent launch: the CTAs start (and load their weight
    // slice) while the tensor-core pass is still running; the loop covers
    // any fix count
    const int lanes = static_cast<int>(want < 1 ? 1 : (want > cap ? cap : want));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(lanes * n_eg));
    cfg.blockDim = dim3(kSplitThreads);
    cfg.dynamicSmemBytes = split_smem_bytes(p.d);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, router_fixup_split_kernel<NV>, static_cast<const uint16_t*>(x),
                           static_cast<const uint16_t*>(w), p.bias, p.T, p.d, p.E, p.k, p.norm,
                           static_cast<const int*>(p.fix_count),
                           static_cast<const int32_t*>(p.fix_list), p.group_done, p.fix_logits,
                           p.topk_idx, p.topk_w_f32, p.topk_w_dtype, p.logits_out);
    if (e != cudaSuccess) return e;
  } else if (wsmem_ok) {
    router_fixup_wsmem_kernel<<<sms, 64 * kFixSmG, wsm_smem, st>>>(
        mw, static_cast<const uint16_t*>(x), p.bias, p.T, p.d, p.E, p.k, p.norm, p.fix_count,
        p.fix_list, p.topk_idx, p.topk_w_f32, p.topk_w_dtype, p.logits_out, p.err,
        p.wait_limit_ns);
  } else {
    router_fixup_kernel<NV><<<num_sms_for_current_device() * 2, kFixThreads, fix_smem, st>>>(
        static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(w), p.bias, p.T, p.d, p.E,
        p.k, p.norm, p.fix_count, p.fix_list, p.topk_idx, p.topk_w_f32, p.topk_w_dtype,
        p.logits_out);
  }
  return cudaGetLastError();
}

}  // namespace

// Certification margin, relative to a token's largest |logit|.  The
// environment variable HMOE_ROUTER_CERT_REL (read once) overrides it; the
// tests set it to 1 so that no token is certified and every one takes the
// exact-order fix-up pass.  A larger margin only sends more tokens there.
static float router_cert_rel() {
  static const float rel = [] {
    const char* v = getenv("HMOE_ROUTER_CERT_REL");
    const float f = v ? static_cast<float>(atof(v)) : 0.0f;
    return f > kRouterCertRel ? f : kRouterCertRel;
  }();
  return rel;
}

// Scratch: 64 ints of header (the fix count first, zeroed per call), the
// per-token-group counters of the split fix-up (zeroed by router_tc_kernel),
// the fix list, then the rounded logits of every fix slot.
static int64_t align4(int64_t v) { return (v + 3) & ~static_cast<int64_t>(3); }
static int64_t fix_groups(int64_t T) { return align4(cdiv64(T, kSplitG)); }

size_t router_tc_scratch_bytes(int64_t T) {
  return sizeof(int) * (64 + fix_groups(T) + align4(T)) +
         sizeof(uint16_t) * static_cast<size_t>(fix_groups(T)) * kSplitG * kSplitLogitStride;
}

cudaError_t launch_router_topk_tc(const void* x, const void* w_router, const void* bias,
                                  int64_t T, int d, int E, int k, int norm, int32_t* topk_idx,
                                  float* topk_w_f32, void* topk_w_dtype, void* logits_out,
                                  void* scratch, int* err, cudaStream_t stream, float* sums_out) {
  if (T == 0) return cudaSuccess;
  int* fix_count = static_cast<int*>(scratch);
  cudaError_t e = cudaMemsetAsync(fix_count, 0, sizeof(int), stream);
  if (e != cudaSuccess) return e;
  RtParams p;
  p.bias = static_cast<const uint16_t*>(bias);
  p.T = T;
  p.d = d;
  p.E = E;
  p.k = k;
  p.norm = norm;
  p.topk_idx = topk_idx;
  p.topk_w_f32 = topk_w_f32;
  p.topk_w_dtype = topk_w_dtype;
  p.logits_out = static_cast<uint16_t*>(logits_out);
  p.sums_out = sums_out;
  p.fix_count = fix_count;
  p.group_done = reinterpret_cast<unsigned*>(fix_count + 64);
  p.fix_list = fix_count + 64 + fix_groups(T);
  p.fix_logits = reinterpret_cast<uint16_t*>(p.fix_list + align4(T));
  p.err = err;
  p.wait_limit_ns = kWaitLimitNs;
  p.cert_rel = router_cert_rel();
  if (k <= 8)
    return E <= 64 ? launch_tc<64, 8>(x, w_router, p, stream)
                   : launch_tc<128, 8>(x, w_router, p, stream);
  return E <= 64 ? launch_tc<64, 32>(x, w_router, p, stream)
                 : launch_tc<128, 32>(x, w_router, p, stream);
}

}  // namespace hmoe
