/*
 * TEST ORACLE -- not product code.  Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg load this library, and only as the checker.
 *
 * Router logits of the reference MoE layer, restated in C:
 *   logits = F.linear(hidden_states, gate.weight[, bias])      models/layers.py:605
 * computed in fp32 with a FIXED accumulation order: for each (token, expert)
 * k is cut into blocks of 64; within a block the products x[t,k] * w[e,k]
 * are accumulated by one fused multiply-add per k in ascending order from
 * +0.0f, and the block sums are added (fp32 add) in ascending block order
 * from +0.0f.  The bias (if any) is then added in fp32 and the result is
 * rounded once to the hidden dtype (bf16 round-to-nearest-even, or fp32).
 *
 * The GPU's exact-order router kernels accumulate in exactly this order, so
 * their logits are bit-identical to these (fmaf is correctly rounded on both
 * sides).  The
 * reference's own logits come from a BLAS GEMM whose order is unspecified;
 * they agree with these except where the exact sum sits within the fp32
 * accumulation error of a bf16 rounding midpoint.
 *
 * Build: oracle/Makefile (gcc -O3 -fopenmp; no -ffast-math, which would let
 * the compiler reorder the sums).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static float round_bf16(float v) {
  uint32_t u;
  memcpy(&u, &v, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) return v; /* NaN */
  u = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
  memcpy(&v, &u, 4);
  return v;
}

/* Per 64-wide block of k: part[e] = fma(x[k], wT[k][e], part[e]) over the
 * block's k ascending from +0; acc[e] = acc[e] + part[e] block after block,
 * from +0.  Vectorised across e. */
#define LOGIT_BLOCK 64
__attribute__((target_clones("arch=x86-64-v3", "default")))
static void logits_block(const float* x, const float* wT, const float* bias,
                         float* out, int64_t t0, int64_t t1, int d, int E,
                         int to_bf16) {
  float acc[512], part[512];
  for (int64_t t = t0; t < t1; ++t) {
    const float* xr = x + t * (int64_t)d;
    for (int e = 0; e < E; ++e) acc[e] = 0.0f;
    for (int k0 = 0; k0 < d; k0 += LOGIT_BLOCK) {
      const int k1 = k0 + LOGIT_BLOCK < d ? k0 + LOGIT_BLOCK : d;
      for (int e = 0; e < E; ++e) part[e] = 0.0f;
      for (int k = k0; k < k1; ++k) {
        const float xv = xr[k];
        const float* wr = wT + (int64_t)k * E;
        for (int e = 0; e < E; ++e) part[e] = fmaf(xv, wr[e], part[e]);
      }
      for (int e = 0; e < E; ++e) acc[e] = acc[e] + part[e];
    }
    float* o = out + t * (int64_t)E;
    for (int e = 0; e < E; ++e) {
      float v = acc[e];
      if (bias) v = v + bias[e];
      o[e] = to_bf16 ? round_bf16(v) : v;
    }
  }
}

/*
 * x      [T, d] fp32 (bf16-exact values for a bf16 layer)
 * w      [E, d] fp32
 * bias   [E] fp32 or NULL
 * out    [T, E] fp32 (holding bf16-exact values when to_bf16 != 0)
 * Returns 0, or -1 when E > 512 or an allocation fails.
 */
int oracle_router_logits(const float* x, const float* w, const float* bias,
                         float* out, int64_t T, int d, int E, int to_bf16,
                         int nthreads) {
  if (E <= 0 || E > 512 || d <= 0 || T < 0) return -1;
  float* wT = (float*)malloc(sizeof(float) * (size_t)d * (size_t)E);
  if (!wT) return -1;
  for (int e = 0; e < E; ++e)
    for (int k = 0; k < d; ++k) wT[(int64_t)k * E + e] = w[(int64_t)e * d + k];
  const int64_t chunk = 16;
  const int64_t nchunks = (T + chunk - 1) / chunk;
#pragma omp parallel for schedule(dynamic, 4) num_threads(nthreads > 0 ? nthreads : 1)
  for (int64_t c = 0; c < nchunks; ++c) {
    const int64_t t0 = c * chunk;
    const int64_t t1 = t0 + chunk < T ? t0 + chunk : T;
    logits_block(x, wT, bias, out, t0, t1, d, E, to_bf16);
  }
  free(wT);
  return 0;
}
