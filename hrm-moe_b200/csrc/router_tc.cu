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

// Position of expert e in a token's logits row: 4 floats of padding after
// every 32, so that the lanes routing a warp's tokens (4 or 8 per token,
// each reading its own run of experts as 16-byte vectors) meet 32 different
// banks.  Rows are LgRow<E>::kStride floats apart (E + E/8).
__host__ __device__ constexpr int lg_idx(int e) { return e + 4 * (e >> 5); }
template <int E>
struct LgRow {
  static constexpr int kStride = E + E / 8;
};


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
  int reset_err;          // pair pass: CTA 0 clears *err once its dependency wait returns
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
  static constexpr int kLgStride = LgRow<E>::kStride;  // floats per token row (lg_idx)
  static constexpr int kLgBytes = 2 * RRT * kLgStride * 4;  // the two halves' sums
  static constexpr int kMainBytes = kRingBytes > kLgBytes ? kRingBytes : kLgBytes;
  static constexpr int kCtlBytes = 256;
  static constexpr size_t kSmem = 1024 + kMainBytes + kCtlBytes;
  static_assert(kStageBytes % 1024 == 0, "stages keep the 1 KiB swizzle alignment");
  static_assert(kStages <= 8, "RtCtl holds eight stage barriers of each kind");
  static_assert(kSmem <= 232448, "shared memory budget");
};

// Reductions over the L lanes of one token (xor 1, 2, ...).  Every lane of
// the warp executes them together.
template <int L>
__device__ __forceinline__ uint32_t grp_max(uint32_t v) {
#pragma unroll
  for (int o = 1; o < L; o <<= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
template <int L>
__device__ __forceinline__ float grp_maxf(float v) {
#pragma unroll
  for (int o = 1; o < L; o <<= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
template <int L>
__device__ __forceinline__ float grp_sum(float v) {
#pragma unroll
  for (int o = 1; o < L; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Routing keys.  A logit's key orders experts by rounded value, then by
// ascending index, and carries the rounding range of the exact-order sum:
// bits [16, 32) the order-preserving image (ob16) of the rounded value,
// [3, 10) 127 - e, bit 2 "wide" (the exact sum may round more than one step
// away), bit 1 "may round one step up", bit 0 "one step down".  Any lane can
// then tell a pick's range from its key alone.
constexpr uint32_t kKeyDn = 1u, kKeyUp = 2u, kKeyWide = 4u;

__device__ __forceinline__ float ob_value(uint32_t ob) {
  return bf16_bits_to_f32((ob & 0x8000u) ? (ob & 0x7FFFu) : (~ob & 0xFFFFu));
}
// bf16 value (as fp32) of an order-preserving key
__device__ __forceinline__ float key_value(uint32_t key) { return ob_value(key >> 16); }
__device__ __forceinline__ int key_expert(uint32_t key) { return 127 - static_cast<int>((key >> 3) & 127u); }

// Key of logit v (tensor-core sum, bias included) of expert e, with margin
// delta: the exact-order sum lies in [v - delta, v + delta] (ends rounded
// outward), so its bf16 rounding lies between the roundings of the two ends.
// Where |v| >= 1024 delta, the gap to either bf16 neighbour is at least
// 2 delta, so that rounding is the value itself or one neighbour; smaller
// logits whose rounding is not certain are marked wide.  Branch-free: the
// routing runs it for every logit.
__device__ __forceinline__ uint32_t logit_key(float v, float delta, float wide_below, uint32_t e) {
  const uint32_t b = f32_to_bf16_bits(v);
  const uint32_t lh = cvt_bf16x2(__fsub_rd(v, delta), __fadd_ru(v, delta));
  const uint32_t dn = (lh & 0xFFFFu) != b ? 1u : 0u;
  const uint32_t up = (lh >> 16) != b ? 1u : 0u;
  const uint32_t fl = (dn | up) && fabsf(v) < wide_below ? kKeyWide : (dn | (up << 1));
  return (ob16(b) << 16) | ((127u - e) << 3) | fl;
}
// Smallest / largest key the exact-order sum of this logit could take.  A
// wide logit rounded to r came from a sum between r's neighbours, so its
// exact sum lies within delta of that interval.  WIDE = false: the caller
// knows that no key of the token is wide.
template <bool WIDE = true>
__device__ __forceinline__ uint32_t key_min(uint32_t key, float delta) {
  if (WIDE && (key & kKeyWide)) {
    const uint32_t ob = key >> 16;
    const float lo = __fsub_rd(ob_value(ob > 0u ? ob - 1u : ob), delta);
    return (ob16(f32_to_bf16_bits(lo)) << 16) | (key & 0xFFFFu);
  }
  return key - ((key & kKeyDn) << 16);
}
template <bool WIDE = true>
__device__ __forceinline__ uint32_t key_max(uint32_t key, float delta) {
  if (WIDE && (key & kKeyWide)) {
    const uint32_t ob = key >> 16;
    const float hi = __fadd_ru(ob_value(ob < 0xFFFFu ? ob + 1u : ob), delta);
    return (ob16(f32_to_bf16_bits(hi)) << 16) | (key & 0xFFFFu);
  }
  return key + ((key & kKeyUp) << 15);
}

// Certification of a selection: each pick's smallest key beats the next
// pick's largest, and the last pick's beats every unpicked expert's largest
// (rest: the lane's unpicked keys, 0 for picked or absent ones).  Returns
// true when some decision is not certain; lmin = the smallest pick key.
template <bool WIDE, int L, int KMAX, int NE>
__device__ __forceinline__ bool certify(const uint32_t (&pk)[KMAX], const uint32_t (&rest)[NE],
                                        int k, float delta, uint32_t& lmin) {
  bool bad = false;
  uint32_t last_min = 0;
  lmin = 0xFFFFFFFFu;
#pragma unroll
  for (int r = 0; r < KMAX; ++r) {
    if (r < k) {
      const uint32_t mn = key_min<WIDE>(pk[r], delta);
      lmin = min(lmin, mn);
      last_min = mn;
      if (r + 1 < k) bad |= !(mn > key_max<WIDE>(pk[r + 1], delta));
    }
  }
  uint32_t rmax = 0;
#pragma unroll
  for (int i = 0; i < NE; ++i) rmax = max(rmax, key_max<WIDE>(rest[i], delta));
  rmax = grp_max<L>(rmax);
  return bad || !(last_min > rmax);
}

__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// What route_tok found out about a token whose order decisions were not all
// certain: the margin in use and the smallest key any pick could take.
struct RouteCert {
  float delta;
  uint32_t lmin;
};

// Bitonic sort of N keys into descending order (registers, unrolled).
template <int N>
__device__ __forceinline__ void sort_desc(uint32_t (&a)[N]) {
#pragma unroll
  for (int size = 2; size <= N; size <<= 1) {
#pragma unroll
    for (int stride = size / 2; stride > 0; stride >>= 1) {
#pragma unroll
      for (int i = 0; i < N; ++i) {
        const int j = i ^ stride;
        if (j > i) {
          const uint32_t x = a[i], y = a[j];
          const bool desc = (i & size) == 0 || size == N;
          a[i] = desc ? max(x, y) : min(x, y);
          a[j] = desc ? min(x, y) : max(x, y);
        }
      }
    }
  }
}
// a: this lane's N largest keys, descending.  After the call every lane of
// the L-lane group holds the group's N largest keys, descending: at each
// level a lane and its partner keep the larger half of their two lists
// (max of a[i] and the partner's a[N-1-i] is a bitonic sequence holding
// them), then sort it with a bitonic merge.
template <int N, int L>
__device__ __forceinline__ void group_top(uint32_t (&a)[N]) {
#pragma unroll
  for (int o = 1; o < L; o <<= 1) {
    uint32_t b[N];
#pragma unroll
    for (int i = 0; i < N; ++i) b[i] = __shfl_xor_sync(0xffffffffu, a[i], o);
#pragma unroll
    for (int i = 0; i < N; ++i) a[i] = max(a[i], b[N - 1 - i]);
#pragma unroll
    for (int stride = N / 2; stride > 0; stride >>= 1) {
#pragma unroll
      for (int i = 0; i < N; ++i) {
        const int j = i ^ stride;
        if (j > i) {
          const uint32_t x = a[i], y = a[j];
          a[i] = max(x, y);
          a[j] = min(x, y);
        }
      }
    }
  }
}

// Route token t on the L lanes (s = 0..L-1) of its group; lane s holds
// experts [s E/L, (s+1) E/L).  The logits are a0[lg_idx(e)] (+ a1[...] when
// a1 is set: the two halves' sums), plus the bias.  Every lane of the warp
// calls it together (the group reductions are full-warp shuffles); lanes
// whose token is past the end pass live = false and write nothing.
// delta_rel > 0: certified selection against the bf16 values each logit
// could round to within delta_rel * max|logit|, returning true when some
// order decision is not certain (each pick against the next, the last pick
// against every unpicked expert); delta_rel = 0: the logits are exact and
// every decision holds.  The k picks are found on plain keys (one group
// maximum each); the ranges ride in the keys, so the certification needs no
// further exchange.  Writes topk_idx, the weights and (when asked) the
// rounded logits; with `sums` also the unbiased sums; with `cert` the margin
// and the smallest pick key.
template <int E, int KMAX, int L, bool KFIX = false>
__device__ __forceinline__ bool route_tok(const float* a0, const float* a1, const RtParams& p,
                                          float delta_rel, int64_t t, int s, bool live, bool sums,
                                          RouteCert* cert = nullptr) {
  constexpr int NE = E / L;
  static_assert(NE % 4 == 0 && KMAX % L == 0, "lane shares");
  const int En = p.E;
  const int k = KFIX ? KMAX : p.k;  // KFIX: the caller knows k == KMAX
  const int e0 = NE * s;
  const bool full = e0 + NE <= En;  // every expert of this lane exists
  float v[NE];
#pragma unroll
  for (int q = 0; q < NE / 4; ++q) {
    float4 u = *reinterpret_cast<const float4*>(a0 + lg_idx(e0 + 4 * q));
    if (a1) {
      const float4 u1 = *reinterpret_cast<const float4*>(a1 + lg_idx(e0 + 4 * q));
      u.x = u.x + u1.x;
      u.y = u.y + u1.y;
      u.z = u.z + u1.z;
      u.w = u.w + u1.w;
    }
    v[4 * q] = u.x;
    v[4 * q + 1] = u.y;
    v[4 * q + 2] = u.z;
    v[4 * q + 3] = u.w;
  }
  if (sums && p.sums_out && live) {
#pragma unroll
    for (int i = 0; i < NE; ++i)
      if (e0 + i < En) p.sums_out[t * En + e0 + i] = v[i];
  }
  if (p.bias) {
#pragma unroll
    for (int i = 0; i < NE; ++i) v[i] = v[i] + bf16_bits_to_f32(p.bias[e0 + i < En ? e0 + i : 0]);
  }
  if (!full) {  // experts past E: never picked (key 0 below)
#pragma unroll
    for (int i = 0; i < NE; ++i) v[i] = e0 + i < En ? v[i] : -INFINITY;
  }
  if (p.logits_out && live) {
#pragma unroll
    for (int i = 0; i < NE; ++i)
      if (e0 + i < En) p.logits_out[t * En + e0 + i] = static_cast<uint16_t>(f32_to_bf16_bits(v[i]));
  }
  float mag = 0.0f;
#pragma unroll
  for (int i = 0; i < NE; ++i) mag = fmaxf(mag, isfinite(v[i]) ? fabsf(v[i]) : 0.0f);
  mag = grp_maxf<L>(mag);
  const float delta = delta_rel * mag;
  const float wide_below = 1024.0f * delta;
  uint32_t key[NE], wide = 0;
#pragma unroll
  for (int i = 0; i < NE; ++i) {
    key[i] = logit_key(v[i], delta, wide_below, static_cast<uint32_t>(e0 + i));
    if (!full) key[i] = e0 + i < En ? key[i] : 0u;
    wide |= key[i];
  }
  // the KMAX largest keys of the token on every lane of its group: each
  // lane sorts its own (zeros pad a short list), then the group merges
  constexpr int NS = NE > KMAX ? NE : KMAX;
  uint32_t srt[NS];
#pragma unroll
  for (int i = 0; i < NS; ++i) srt[i] = i < NE ? key[i] : 0u;
  sort_desc<NS>(srt);
  uint32_t pk[KMAX];
#pragma unroll
  for (int r = 0; r < KMAX; ++r) pk[r] = srt[r];
  group_top<KMAX, L>(pk);
  // unpicked keys: the lane's keys below the k-th pick (keys are distinct)
  uint32_t kth = pk[0];
#pragma unroll
  for (int r = 1; r < KMAX; ++r) kth = r < k ? pk[r] : kth;
#pragma unroll
  for (int i = 0; i < NE; ++i) key[i] = key[i] < kth ? key[i] : 0u;
  // softmax over the rounded logits; the largest is the first pick's value
  const float mx = key_value(pk[0]);
  float ssum = 0.0f;
#pragma unroll
  for (int i = 0; i < NE; ++i) ssum += __expf(round_bf16(v[i]) - mx);
  ssum = grp_sum<L>(ssum);
  // certification; the exact form for wide ranges only where the warp has one
  uint32_t lmin;
  const bool bad = __any_sync(0xffffffffu, (wide & kKeyWide) != 0u)
                       ? certify<true, L>(pk, key, k, delta, lmin)
                       : certify<false, L>(pk, key, k, delta, lmin);
  if (cert) {
    cert->delta = delta;
    cert->lmin = lmin;
  }
  // weights: lane s takes picks s, s+L, ...; every lane then adds the k
  // probabilities in pick order
  uint32_t mk[KMAX / L];
  float pw[KMAX / L];
#pragma unroll
  for (int j = 0; j < KMAX / L; ++j) {
    mk[j] = pk[L * j];
#pragma unroll
    for (int i = 1; i < L; ++i) mk[j] = s == i ? pk[L * j + i] : mk[j];
    pw[j] = L * j + s < k ? expf(key_value(mk[j]) - mx) / ssum : 0.0f;
  }
  float ps = 0.0f;
#pragma unroll
  for (int r = 0; r < KMAX; ++r)
    if (r < k) ps += __shfl_sync(0xffffffffu, pw[r / L], (threadIdx.x & (32 - L)) | (r % L));
#pragma unroll
  for (int j = 0; j < KMAX / L; ++j) {
    const int r = L * j + s;
    float w = p.norm ? pw[j] / fmaxf(ps, 1e-12f) : pw[j];
    w = round_bf16(w);
    if (live && r < k) {
      const int64_t o = t * k + r;
      p.topk_idx[o] = key_expert(mk[j]);
      if (p.topk_w_f32) p.topk_w_f32[o] = w;
      if (p.topk_w_dtype)
        static_cast<uint16_t*>(p.topk_w_dtype)[o] = static_cast<uint16_t>(f32_to_bf16_bits(w));
    }
  }
  return bad;
}

// Lane s's experts (bit i: expert s E/L + i) of a token that route_tok could
// not certify whose rounding is not certain and whose largest key reaches
// the smallest key any pick could take.  An expert below that bound stays
// below every pick, in exact values and in its own rounding alike, so exact
// values for these experts alone make the routing exact.
template <int E, int L>
__device__ __forceinline__ uint32_t fix_mask_tok(const float* row, const RtParams& p,
                                                 const RouteCert& c, int s) {
  constexpr int NE = E / L;
  uint32_t m = 0;
#pragma unroll
  for (int i = 0; i < NE; ++i) {
    const int e = NE * s + i;
    if (e < p.E) {
      float x = row[lg_idx(e)];
      if (p.bias) x = x + bf16_bits_to_f32(p.bias[e]);
      const uint32_t key = logit_key(x, c.delta, 1024.0f * c.delta, static_cast<uint32_t>(e));
      if ((key & 7u) != 0u && key_max(key, c.delta) >= c.lmin) m |= 1u << i;
    }
  }
  return m;
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
  float* lg0 = reinterpret_cast<float*>(smem);          // [64][kLgStride] first halves
  float* lg1 = lg0 + RRT * C::kLgStride;                // [64][kLgStride] second halves
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
        for (int i = 0; i < 32; ++i) dst[lg_idx(c * 32 + i)] = __uint_as_float(col0 ? rb[i] : ra[i]);
      }
    }
    tc_fence_before();
    named_barrier_sync(1, kEpi);
    // ---- routing: token j on lanes 4 (j % 8) .. +3 of warp j / 8
    const bool live = !*abort;
    if (live) {  // uniform over the CTA
      const int j = ew * 8 + (lane >> 2), s = lane & 3;
      const int64_t t = t0 + j;
      const bool bad = route_tok<E, KMAX, 4>(lg0 + j * C::kLgStride, lg1 + j * C::kLgStride, p,
                                             p.cert_rel, t, s, t < p.T, true);
      if (bad && s == 0 && t < p.T) p.fix_list[atomicAdd(p.fix_count, 1)] = static_cast<int32_t>(t);
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

// ----------------------------------------------------------------------------
// router_pair_kernel: the tensor-core pass for E <= 128 on CTA pairs,
// persistent over 128-token tiles, with the fix-up done in the kernel itself;
// for E <= 64 the router weight is resident in shared memory.
//
// The operands are router_rows_kernel's (x read as [2T, d/2]: rows 2t and
// 2t+1 are the two halves of token t), but the two CTAs of a cluster share
// one 256-row MMA (tcgen05.mma.cta_group::2, M=256, N=128).  Each CTA stages
// its own 64 tokens (128 rows) per tile and holds one half of the stacked
// weight for the whole kernel: the even CTA W[:, :d/2], the odd CTA
// W[:, d/2:], 64 rows each (zeros past E).  The weight therefore crosses L2
// once per CTA instead of once per k-step and tile, and the TMA ring holds
// token rows only (up to 8 stages of 16 KiB).  Accumulator row 2j of a CTA
// holds token j's first-half sums in columns [0, 64), row 2j+1 its
// second-half sums in columns [64, 128).  The weight's k-blocks are loaded
// with the first tile's token blocks, on the same stage barriers.  For
// 64 < E <= 128 (EMAX = 128: N = 256, 128 weight rows per CTA) a weight half
// does not fit next to a ring, so each stage carries the k-block of both
// the tokens and this CTA's weight half: the pair still reads each weight
// byte once per tile, not twice as the single-CTA row-split pass does.
//
// Roles: warp 0 TMA, warp 1 MMA (the even CTA issues for both), warps 2-5
// read the accumulator (one TMEM lane quadrant each), add each token's two
// halves (lanes 2j and 2j+1 each take 8 of every 16 experts and trade the
// other half of their sums with shuffles) and park the logits in shared
// memory, which frees the accumulator; warps 6-21 route each token on 8
// lanes (route_tok).  Two accumulators and the logits buffer let one tile's
// routing run under the next tile's stream.
//
// Uncertified tokens are fixed where they are found.  Their decision-
// relevant uncertain logits (fix_mask_tok) go to the tile's fix list, and the
// routing warps share the list out: a warp computes one exact-order logit at
// a time from x and W in global memory (lane = 64-k block, block sums folded
// in order).  A token with more than kRpFixPerToken such logits is
// recomputed whole by its own warp (lane = expert, blocks in order).  A token
// whose exact logits all round as its tensor-core sums did keeps the first
// pass's results; the others are routed once more from exact values, with no
// margin.  The result equals the exact-order routing, as the fix-up kernels'
// does, without a second launch.
constexpr int kRpTok = 64;                 // tokens per CTA and tile (128 per pair)
constexpr int kRpReaders = 4;              // warps 2..5
constexpr int kRpRouters = 16;             // warps 6..21
constexpr int kRpLanes = 8;                // routing lanes per token
constexpr int kRpThreads = 32 * (2 + kRpReaders + kRpRouters);
constexpr int kRpMaxStages = 8;
constexpr int kRpABytes = 128 * RBK * 2;   // 16 KiB: 64 tokens x 2 halves
constexpr int kRpFixPerToken = 4;         // listed exact logits per token; more: the whole token
constexpr int kRpFixCap = kRpTok * kRpFixPerToken;  // (token, expert) fixes per tile
constexpr int kRpCtlBytes = 768;
constexpr long kRpSmemMax = 232448;

template <int EMAX>  // the configuration's expert maximum: 64 or 128
struct RpCfg {
  static constexpr bool kResident = EMAX == 64;       // the weight half stays in shared memory
  static constexpr int kBBlock = EMAX * RBK * 2;      // one k-block of a weight half
  static constexpr int kN = 2 * EMAX;                 // MMA N: EMAX experts x 2 halves
  static constexpr int kTmemCols = 2 * kN;            // two accumulators
  static constexpr int kStage = kResident ? kRpABytes : kRpABytes + kBBlock;
  static constexpr int kLgStride = LgRow<EMAX>::kStride;  // floats per token row (lg_idx)
  static constexpr int kLgBytes = kRpTok * kLgStride * 4;
  // ring stages that fit next to the logits, the control block and (when
  // resident) a weight half of nkb k-blocks
  static int stages(int nkb) {
    const long s = (kRpSmemMax - 1024 - kRpCtlBytes - kLgBytes -
                    (kResident ? static_cast<long>(nkb) * kBBlock : 0)) / kStage;
    return s > kRpMaxStages ? kRpMaxStages : static_cast<int>(s);
  }
  static size_t smem(int nkb, int stages) {
    return 1024 + (kResident ? static_cast<size_t>(nkb) * kBBlock : 0) +
           static_cast<size_t>(stages) * kStage + kLgBytes + kRpCtlBytes;
  }
};

struct RpCtl {
  uint64_t full[kRpMaxStages];   // even CTA: both CTAs' blocks of a stage landed
  uint64_t empty[kRpMaxStages];  // each CTA: the pair's MMAs released the stage
  uint64_t acc_full[2];          // each CTA: its accumulator rows are complete
  uint64_t acc_empty[2];         // even CTA: both CTAs' readers drained it
  uint64_t lg_full;              // the readers parked a tile's logits
  uint64_t lg_empty;             // the routing warps are done with them
  uint64_t drain;                // even CTA: every MMA issued has completed
  uint64_t reroute[2];           // tokens of a tile (bit jt) to route again, by tile parity
  uint32_t tmem_base;
  int abort;
  int fix_n;                     // entries in fix_list for the current tile
  uint16_t fix_list[kRpFixCap];  // (token jt << 8) | expert: exact logits to compute
};
static_assert(sizeof(RpCtl) <= kRpCtlBytes, "control block");

// One exact-order logit (without the bias) of token t, expert e, on a whole
// warp: lane b runs 64-k block b (one fma per k, ascending, from +0), and
// the block sums are added in ascending block order from +0 on every lane.
__device__ __forceinline__ float warp_exact_logit(const uint16_t* __restrict__ x,
                                                  const uint16_t* __restrict__ w, int64_t t, int e,
                                                  int d, int lane) {
  const int nb = cdiv(d, kLogitBlock);
  const uint16_t* xr = x + t * d;
  const uint16_t* wr = w + static_cast<int64_t>(e) * d;
  float tot = 0.0f;
  for (int b0 = 0; b0 < nb; b0 += 32) {
    const int b = b0 + lane;
    float part = 0.0f;
    if (b < nb) {
      const int k0 = b * kLogitBlock;
      const int nv = min(kLogitBlock, d - k0) / 8;
      // half a block's loads at a time, issued before its fmas
#pragma unroll
      for (int c0 = 0; c0 < kLogitBlock / 8; c0 += 4) {
        uint4 xv[4], wv[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const bool in = c0 + c < nv;
          xv[c] = in ? __ldg(reinterpret_cast<const uint4*>(xr + k0) + c0 + c) : make_uint4(0, 0, 0, 0);
          wv[c] = in ? __ldg(reinterpret_cast<const uint4*>(wr + k0) + c0 + c) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          if (c0 + c < nv) {
            part = fmaf(bf16_lo(xv[c].x), bf16_lo(wv[c].x), part);
            part = fmaf(bf16_hi(xv[c].x), bf16_hi(wv[c].x), part);
            part = fmaf(bf16_lo(xv[c].y), bf16_lo(wv[c].y), part);
            part = fmaf(bf16_hi(xv[c].y), bf16_hi(wv[c].y), part);
            part = fmaf(bf16_lo(xv[c].z), bf16_lo(wv[c].z), part);
            part = fmaf(bf16_hi(xv[c].z), bf16_hi(wv[c].z), part);
            part = fmaf(bf16_lo(xv[c].w), bf16_lo(wv[c].w), part);
            part = fmaf(bf16_hi(xv[c].w), bf16_hi(wv[c].w), part);
          }
        }
      }
    }
    // ascending block order: eight blocks' sums are fetched, then added
    const int nq = min(32, nb - b0);
    for (int q0 = 0; q0 < nq; q0 += 8) {
      float bs[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) bs[q] = __shfl_sync(0xffffffffu, part, (q0 + q) & 31);
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (q0 + q < nq) tot = tot + bs[q];
    }
  }
  return tot;
}

// Exact-order logits (without the bias) of token t on a whole warp, for
// experts [eb, eb + 64): lane l computes experts eb + l and eb + l + 32,
// block after block in ascending order, and stores them in row[lg_idx(e)].
__device__ __forceinline__ void warp_exact_token(const uint16_t* __restrict__ x,
                                                 const uint16_t* __restrict__ w, int64_t t, int d,
                                                 int E, int lane, float* row, int eb) {
  const int nb = cdiv(d, kLogitBlock);
  const uint16_t* xr = x + t * d;
  const int e0 = eb + lane, e1 = eb + lane + 32;
  const uint16_t* w0 = w + static_cast<int64_t>(min(e0, E - 1)) * d;
  const uint16_t* w1 = w + static_cast<int64_t>(min(e1, E - 1)) * d;
  float acc0 = 0.0f, acc1 = 0.0f;
  for (int b = 0; b < nb; ++b) {
    const int k0 = b * kLogitBlock;
    const int nv = min(kLogitBlock, d - k0) / 8;
    float p0 = 0.0f, p1 = 0.0f;
    // a half block's loads are issued before its fmas
#pragma unroll
    for (int c0 = 0; c0 < kLogitBlock / 8; c0 += 4) {
      uint4 xv[4], u0[4], u1[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const bool in = c0 + c < nv;
        xv[c] = in ? __ldg(reinterpret_cast<const uint4*>(xr + k0) + c0 + c) : make_uint4(0, 0, 0, 0);
        u0[c] = in ? __ldg(reinterpret_cast<const uint4*>(w0 + k0) + c0 + c) : make_uint4(0, 0, 0, 0);
        u1[c] = in ? __ldg(reinterpret_cast<const uint4*>(w1 + k0) + c0 + c) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        if (c0 + c < nv) {
          const float xs[8] = {bf16_lo(xv[c].x), bf16_hi(xv[c].x), bf16_lo(xv[c].y), bf16_hi(xv[c].y),
                               bf16_lo(xv[c].z), bf16_hi(xv[c].z), bf16_lo(xv[c].w), bf16_hi(xv[c].w)};
          const float ws0[8] = {bf16_lo(u0[c].x), bf16_hi(u0[c].x), bf16_lo(u0[c].y), bf16_hi(u0[c].y),
                                bf16_lo(u0[c].z), bf16_hi(u0[c].z), bf16_lo(u0[c].w), bf16_hi(u0[c].w)};
          const float ws1[8] = {bf16_lo(u1[c].x), bf16_hi(u1[c].x), bf16_lo(u1[c].y), bf16_hi(u1[c].y),
                                bf16_lo(u1[c].z), bf16_hi(u1[c].z), bf16_lo(u1[c].w), bf16_hi(u1[c].w)};
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            p0 = fmaf(xs[j], ws0[j], p0);
            p1 = fmaf(xs[j], ws1[j], p1);
          }
        }
      }
    }
    acc0 = acc0 + p0;
    acc1 = acc1 + p1;
  }
  if (e0 < E) row[lg_idx(e0)] = acc0;
  if (e1 < E) row[lg_idx(e1)] = acc1;
}

template <int EMAX, int KMAX, bool KFIX>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kRpThreads, 1)
router_pair_kernel(const __grid_constant__ CUtensorMap tmX2, const __grid_constant__ CUtensorMap tmW,
                   const RtParams p, const uint16_t* __restrict__ xg,
                   const uint16_t* __restrict__ wg, int stages) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  using C = RpCfg<EMAX>;
  const int half = p.d / 2;
  const int nkb = cdiv(half, RBK);
  const int bres = C::kResident ? nkb * C::kBBlock : 0;
  const uint32_t sB = smem_u32(smem);                       // resident weight half: nkb blocks
  const uint32_t sRing = sB + bres;                         // stages: token block (+ weight block)
  float* lg = reinterpret_cast<float*>(smem + bres + stages * C::kStage);
  RpCtl& ctl = *reinterpret_cast<RpCtl*>(reinterpret_cast<uint8_t*>(lg) + C::kLgBytes);
  constexpr int kLgS = C::kLgStride;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int64_t pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int64_t ntiles = cdiv64(p.T, 2 * kRpTok);
  const unsigned long long lim = p.wait_limit_ns;

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(smem_u32(&ctl.full[s]), 1);   // the even CTA's arm
      mbar_init(smem_u32(&ctl.empty[s]), 1);  // one commit per stage use
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&ctl.acc_full[a]), 1);
      mbar_init(smem_u32(&ctl.acc_empty[a]), 2 * kRpReaders);  // both CTAs' readers
    }
    mbar_init(smem_u32(&ctl.lg_full), kRpReaders);
    mbar_init(smem_u32(&ctl.lg_empty), kRpRouters);
    mbar_init(smem_u32(&ctl.drain), 1);
    ctl.abort = 0;
    ctl.fix_n = 0;
    ctl.reroute[0] = ctl.reroute[1] = 0ull;
    fence_mbar_init();
    tma_prefetch_desc(&tmX2);
    tma_prefetch_desc(&tmW);
  } else if (warp == 1) {
    tmem_alloc_pair(smem_u32(&ctl.tmem_base), C::kTmemCols);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // barrier inits visible to the peer CTA before any remote signal
  tc_fence_after();
  grid_dependency_wait();  // launched early (launch_pdl): no global access before this
  grid_launch_dependents();
  // The call's error word starts clear.  The pass records an error only
  // after a wait of kWaitLimitNs, and every later kernel of the call waits
  // for this grid, so nothing is overwritten.
  if (p.reset_err && blockIdx.x == 0 && threadIdx.x == 0) *p.err = 0;
  const uint32_t tmem = ctl.tmem_base;
  volatile int* abort = &ctl.abort;
  int never = 0;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true, first = true;
      for (int64_t tile = pair; ok && tile < ntiles; tile += npairs) {
        const int row0 = static_cast<int>(2 * (tile * 2 * kRpTok + rank * kRpTok));
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait_bounded(smem_u32(&ctl.empty[stage]), phase ^ 1u, abort, p.err, lim)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(&ctl.full[stage]);
          const uint32_t fb_leader = map_to_rank(fb, 0);
          const uint32_t sa = sRing + stage * C::kStage;
          const bool wb = !C::kResident || first;  // this stage carries a weight block
          if (leader) mbar_arrive_expect_tx(fb, 2 * (kRpABytes + (wb ? C::kBBlock : 0)));
          tma_load_2d_pair(sa, &tmX2, kb * RBK, row0, fb_leader);
          if (wb)
            tma_load_2d_pair(C::kResident ? sB + kb * C::kBBlock : sa + kRpABytes, &tmW,
                             (rank ? half : 0) + kb * RBK, 0, fb_leader);
          if (++stage == stages) { stage = 0; phase ^= 1u; }
        }
        first = false;
      }
      // every stage this CTA filled is released by the pair's MMAs before
      // the CTA leaves (no copy still landing, no commit on its way)
      for (int i = 0; i < stages; ++i) {
        if (!mbar_wait_bounded(smem_u32(&ctl.empty[stage]), phase ^ 1u, &never, p.err, lim)) break;
        if (++stage == stages) { stage = 0; phase ^= 1u; }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (leader && lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(256, C::kN);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int64_t tile = pair; ok && tile < ntiles; tile += npairs) {
        if (!mbar_wait_bounded(smem_u32(&ctl.acc_empty[acc]), acc_phase ^ 1u, abort, p.err, lim))
          break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + static_cast<uint32_t>(acc * C::kN);
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait_bounded(smem_u32(&ctl.full[stage]), phase, abort, p.err, lim)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = sRing + stage * C::kStage;
          const uint32_t sb = C::kResident ? sB + kb * C::kBBlock : sa + kRpABytes;
#pragma unroll
          for (int kk = 0; kk < RBK / 16; ++kk)
            tc_mma_bf16_pair(d_tmem, smem_desc_sw128(sa + kk * 32), smem_desc_sw128(sb + kk * 32),
                             idesc, (kb | kk) != 0 ? 1u : 0u);
          tc_commit_pair_both(smem_u32(&ctl.empty[stage]));
          if (++stage == stages) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        tc_commit_pair_both(smem_u32(&ctl.acc_full[acc]));
        if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
      }
      tc_commit_pair(smem_u32(&ctl.drain));
      mbar_wait_bounded(smem_u32(&ctl.drain), 0, &never, p.err, lim);
      for (int i = 0; i < 2; ++i) {
        if (!mbar_wait_bounded(smem_u32(&ctl.acc_empty[acc]), acc_phase ^ 1u, &never, p.err, lim))
          break;
        if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
      }
    }
  } else if (warp < 2 + kRpReaders) {
    // ------------------------------------------------- accumulator readers
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // accumulator row: token r / 2, half r & 1
    const int h = r & 1;
    float* dst = lg + (r >> 1) * kLgS;
    int acc = 0;
    uint32_t acc_phase = 0, lg_phase = 0;
    for (int64_t tile = pair; tile < ntiles; tile += npairs) {
      if (!mbar_wait_bounded(smem_u32(&ctl.acc_full[acc]), acc_phase, abort, p.err, lim)) break;
      if (!mbar_wait_bounded(smem_u32(&ctl.lg_empty), lg_phase ^ 1u, abort, p.err, lim)) break;
      tc_fence_after();
      const uint32_t trow = tmem + (static_cast<uint32_t>(quad * 32) << 16) +
                            static_cast<uint32_t>(acc * C::kN);
#pragma unroll 1
      for (int c = 0; c < EMAX / 16; ++c) {
        // experts 16c..16c+15: lane 2j holds their first-half sums, lane
        // 2j+1 their second-half sums; lane 2j keeps experts 16c..+7, lane
        // 2j+1 16c+8..+15, each receiving the partner's half of them:
        // logit = first + second
        uint32_t ra[16], rb[16];
        tmem_ld_16cols(trow + c * 16, ra);
        tmem_ld_16cols(trow + EMAX + c * 16, rb);
        tc_wait_ld();
        float o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float send = __uint_as_float(h ? rb[i] : ra[8 + i]);
          const float recv = __shfl_xor_sync(0xffffffffu, send, 1);
          o[i] = h ? recv + __uint_as_float(rb[8 + i]) : __uint_as_float(ra[i]) + recv;
        }
        float* q = dst + lg_idx(16 * c + 8 * h);
        reinterpret_cast<float4*>(q)[0] = make_float4(o[0], o[1], o[2], o[3]);
        reinterpret_cast<float4*>(q)[1] = make_float4(o[4], o[5], o[6], o[7]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive_cluster(map_to_rank(smem_u32(&ctl.acc_empty[acc]), 0));
        mbar_arrive(smem_u32(&ctl.lg_full));
      }
      if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
      lg_phase ^= 1u;
    }
  } else {
    // ------------------------------------------------------------- routing
    constexpr int L = kRpLanes;
    constexpr int TPW = 32 / L;  // tokens per routing warp
    const int rw = warp - 2 - kRpReaders;
    const int jt = rw * TPW + lane / L, s = lane % L;  // token jt of the tile on L lanes
    float* row = lg + jt * kLgS;
    constexpr int kRouteThreads = 32 * kRpRouters;
    uint32_t lg_phase = 0;
    // Every routing warp goes through every tile and both named barriers,
    // also after a wait gave up (it then does no work), so that none waits
    // at a barrier for a warp that left.
    for (int64_t tile = pair; tile < ntiles; tile += npairs) {
      const bool ok = mbar_wait_bounded(smem_u32(&ctl.lg_full), lg_phase, abort, p.err, lim);
      const int64_t tile0 = tile * 2 * kRpTok + rank * kRpTok;
      const int64_t t = tile0 + jt;
      RouteCert cert{0.0f, 0u};
      bool bad = false;
      if (ok) bad = route_tok<EMAX, KMAX, L, KFIX>(row, nullptr, p, p.cert_rel, t, s, t < p.T, true,
                                                 &cert) &&
                    t < p.T;
      // Tokens whose order decisions are not certain need exact-order
      // logits for their relevant uncertain experts.  Those (token, expert)
      // pairs go to the tile's fix list, which all routing warps then share
      // out; a token with more of them than fix_logits_max is recomputed
      // whole by its own warp.  Where every exact logit rounds as its
      // tensor-core sum did, the keys, the selection and the weights of the
      // first pass stand; the other tokens are routed once more.
      unsigned todo = __ballot_sync(0xffffffffu, bad && s == 0);
      while (todo) {
        const int src = __ffs(todo) - 1;
        todo &= todo - 1;
        const int jsrc = rw * TPW + src / L;
        float* trow = lg + jsrc * kLgS;
        uint32_t um = 0;
        if (lane / L == src / L) um = fix_mask_tok<EMAX, L>(trow, p, cert, s);
        uint32_t m[L];
        int nu = 0;
#pragma unroll
        for (int q = 0; q < L; ++q) {
          m[q] = __shfl_sync(0xffffffffu, um, src + q);
          nu += __popc(m[q]);
        }
        if (nu <= kRpFixPerToken) {
          if (lane == 0) {
            int slot = atomicAdd(&ctl.fix_n, nu);
#pragma unroll
            for (int q = 0; q < L; ++q) {
              uint32_t mm = m[q];
              while (mm) {
                const int i = __ffs(mm) - 1;
                mm &= mm - 1;
                ctl.fix_list[slot++] = static_cast<uint16_t>((jsrc << 8) | ((EMAX / L) * q + i));
              }
            }
          }
        } else {
          for (int eb = 0; eb < EMAX; eb += 64)
            warp_exact_token(xg, wg, tile0 + jsrc, p.d, p.E, lane, trow, eb);
          if (lane == 0) atomicOr(reinterpret_cast<unsigned long long*>(&ctl.reroute[lg_phase]),
                                  1ull << jsrc);
        }
      }
      named_barrier_sync(1, kRouteThreads);  // the tile's fix list is complete
      const int nfix = ctl.fix_n;
      for (int i = rw; i < nfix; i += kRpRouters) {
        const int jf = ctl.fix_list[i] >> 8, e = ctl.fix_list[i] & 0xFF;
        const float v = warp_exact_logit(xg, wg, tile0 + jf, e, p.d, lane);
        float* frow = lg + jf * kLgS;
        const float bias = p.bias ? bf16_bits_to_f32(p.bias[e]) : 0.0f;
        const bool changed = round_bf16(v + bias) != round_bf16(frow[lg_idx(e)] + bias);
        __syncwarp();
        if (lane == 0) {
          frow[lg_idx(e)] = v;
          if (changed)
            atomicOr(reinterpret_cast<unsigned long long*>(&ctl.reroute[lg_phase]), 1ull << jf);
        }
      }
      named_barrier_sync(1, kRouteThreads);  // exact logits written, tokens to re-route marked
      const uint64_t rr = ctl.reroute[lg_phase];
      const bool mine = ((rr >> jt) & 1ull) != 0ull;
      if (__any_sync(0xffffffffu, mine))
        route_tok<EMAX, KMAX, L, KFIX>(row, nullptr, p, 0.0f, t, s, mine && t < p.T, false);
      if (rw == 0 && lane == 0) {
        // the next tile's list starts empty; the other parity's mask was
        // last read before this tile's logits arrived
        ctl.fix_n = 0;
        ctl.reroute[lg_phase ^ 1u] = 0ull;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&ctl.lg_empty));
      lg_phase ^= 1u;
    }
  }

  // --------------------------------------------------------------- teardown
  __syncwarp();  // single-lane roles rejoin their warps before the CTA barrier
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // neither CTA leaves while the pair's MMAs or the peer use it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, C::kTmemCols);
  }
}

// HMOE_ROUTER_PAIR=0 (read once per process) turns the pair pass off, so
// tests can run the other passes and fix-up kernels for E <= 64.
bool router_pair_enabled() {
  static const bool on = [] {
    const char* v = getenv("HMOE_ROUTER_PAIR");
    return !(v && atoi(v) == 0);
  }();
  return on;
}

bool pair_pass_fits(int64_t T, int d, int E) {
  if (E > 128 || d % 16 != 0 || !router_pair_enabled() || router_whole_rows_forced()) return false;
  const int nkb = cdiv(d / 2, RBK);
  const int st = E <= 64 ? RpCfg<64>::stages(nkb) : RpCfg<128>::stages(nkb);
  return st >= 3 && 2 * T < (static_cast<int64_t>(1) << 31);
}

template <int EMAX, int KMAX, bool KFIX>
cudaError_t launch_pair_tc(const void* x, const void* w, const RtParams& p, cudaStream_t st) {
  static int done[64] = {0};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!done[dev]) {
      e = cudaFuncSetAttribute(router_pair_kernel<EMAX, KMAX, KFIX>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(kRpSmemMax));
      if (e != cudaSuccess) return e;
      done[dev] = 1;
    }
  }
  const int nkb = cdiv(p.d / 2, RBK);
  using C = RpCfg<EMAX>;
  const int stages = C::stages(nkb);
  CUtensorMap mx, mw;
  if (!map_half_rows(&mx, x, static_cast<uint64_t>(p.T), static_cast<uint64_t>(p.d)) ||
      !map_rows(&mw, w, static_cast<uint64_t>(p.E), static_cast<uint64_t>(p.d), EMAX))
    return cudaErrorInvalidValue;
  const int64_t ntiles = cdiv64(p.T, 2 * kRpTok);
  const int sms = num_sms_for_current_device();
  const int64_t pairs = ntiles < sms / 2 ? ntiles : sms / 2;
  return launch_pdl(kPdlRouter, router_pair_kernel<EMAX, KMAX, KFIX>,
                    dim3(static_cast<unsigned>(2 * (pairs < 1 ? 1 : pairs))), dim3(kRpThreads),
                    C::smem(nkb, stages), st, mx, mw, p, static_cast<const uint16_t*>(x),
                    static_cast<const uint16_t*>(w), stages);
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
                                  void* scratch, int* err, cudaStream_t stream, float* sums_out,
                                  bool reset_err) {
  // the pair pass fixes its uncertified tokens itself (no fix list) and can
  // clear the error word itself; the other passes get both cleared here
  const bool pair = T > 0 && pair_pass_fits(T, d, E);
  if (reset_err && !pair) {
    cudaError_t e = cudaMemsetAsync(err, 0, sizeof(int), stream);
    if (e != cudaSuccess) return e;
  }
  if (T == 0) return cudaSuccess;
  int* fix_count = static_cast<int*>(scratch);
  if (!pair) {
    cudaError_t e = cudaMemsetAsync(fix_count, 0, sizeof(int), stream);
    if (e != cudaSuccess) return e;
  }
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
  p.reset_err = pair && reset_err ? 1 : 0;
  p.wait_limit_ns = kWaitLimitNs;
  p.cert_rel = router_cert_rel();
  if (pair)
    return E <= 64 ? (k == 8  ? launch_pair_tc<64, 8, true>(x, w_router, p, stream)
                      : k < 8 ? launch_pair_tc<64, 8, false>(x, w_router, p, stream)
                              : launch_pair_tc<64, 32, false>(x, w_router, p, stream))
                   : (k == 8  ? launch_pair_tc<128, 8, true>(x, w_router, p, stream)
                      : k < 8 ? launch_pair_tc<128, 8, false>(x, w_router, p, stream)
                              : launch_pair_tc<128, 32, false>(x, w_router, p, stream));
  if (k <= 8)
    return E <= 64 ? launch_tc<64, 8>(x, w_router, p, stream)
                   : launch_tc<128, 8>(x, w_router, p, stream);
  return E <= 64 ? launch_tc<64, 32>(x, w_router, p, stream)
                 : launch_tc<128, 32>(x, w_router, p, stream);
}

}  // namespace hmoe
