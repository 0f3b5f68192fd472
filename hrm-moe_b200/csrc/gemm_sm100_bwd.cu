// Backward grouped GEMMs on the sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// Replaces the backward of models/moe_triton_grouped_gemm.py
// (_TritonGroupedLinear.backward, :427-456) for y = x @ W[g]^T, W: [G, N, K]:
//   dgrad  grad_x[r, :]  = grad_y[r, :] @ W[g]          (_m_grouped_gemm_bn_kernel, :187-260)
//   wgrad  grad_W[g]     = grad_y[g]^T @ x[g]            (_k_grouped_gemm_kernel, :277-347)
// with fp32 accumulation and one rounding to bf16, plus a dgrad whose
// epilogue is the backward of SiLU(gate) * up (models/layers.py:327-329), so
// the down projection's grad_input never reaches HBM as such:
//   swiglu dgrad  dh = bf16(grad_y @ W_down[g]);  with g, u from the saved
//                 gate_up rows and sg = bf16(silu(g)):
//                 d_up = bf16(dh * sg), d_sg = bf16(dh * u),
//                 d_gate = bf16(d_sg * s * (1 + g * (1 - s))), s = sigmoid(g)
//                 written as one [rows, 2I] gradient (gate half, then up half).
//
// Operand layouts.  The forward kernels read both operands K-major (the
// contraction dimension contiguous).  Here one or both are MN-major:
//   dgrad: A = grad rows [M, Kc] (K-major, as in the forward), B = W[g] stored
//          [Kc][Nout] (Nout contiguous: MN-major), loaded through a 3-D tensor
//          map {Nout, Kc, G} so a box never reads into the next group's weight.
//   wgrad: the contraction runs over the group's rows: A = grad rows [M, Mw]
//          and B = input rows [M, Nw], both MN-major.  A group's last k-block
//          of 64 rows runs into the next group's rows; the MMA warp zeroes
//          those rows of the staged A and B boxes before it issues, so they
//          add nothing (not even for non-finite neighbours).
// An MN-major operand is staged as TMA boxes of [64 k-rows][64 elements]
// (128-byte rows, 128-byte swizzle); its smem descriptor has the 8-row
// groups 1024 B apart (stride offset) and consecutive 64-element boxes 8 KiB
// apart (leading offset), and each MMA (K = 16) advances 2048 B.
//
// One persistent CTA per SM: warp 0 TMA producer (4-stage ring of 48 KiB:
// A 16 KiB + B 32 KiB), warp 1 allocates 512 TMEM columns and issues
// tcgen05.mma (M = 128, N = 256, K = 16) into two 256-column accumulators,
// 4 (8 for the SwiGLU backward) epilogue warps read TMEM quadrants, round
// and store (TMA-store staging boxes, or direct stores where a quadrant
// crosses a group end).  Every mbarrier wait is bounded; on a timeout the
// kernel records kDevTimeout, the roles leave their loops, drain with bounded
// waits and free TMEM.  No TMA multicast anywhere.
#include <cuda.h>
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace hmoe {
namespace {

constexpr int QM = 128;            // MMA M: output rows per tile
constexpr int QN = 256;            // MMA N: output columns per tile
constexpr int QK = 64;             // k per stage (one 128-byte swizzled row of bf16)
constexpr int kQStages = 4;
constexpr int kQABytes = QM * QK * 2;           // 16 KiB
constexpr int kQBBytes = QN * QK * 2;           // 32 KiB
constexpr int kQStageBytes = kQABytes + kQBBytes;
constexpr int kQBox = 64 * 64 * 2;              // one [64][64] bf16 box, 8 KiB
constexpr int kQAcc = 2;
constexpr int kQTmemCols = QN * kQAcc;          // all 512 columns
constexpr int kQMaxGroups = 1024;
constexpr int kQEpiChunk = 32 * 32 * 2;
// plain epilogue: 2 staging boxes for each of 4 warps; SwiGLU backward: one
// 2 KiB transpose buffer for each of 8 warps
constexpr int kQEpiBytes = 4 * 2 * kQEpiChunk;

enum BwdMode : int { kModeDgrad = 0, kModeDgradSwiglu = 1, kModeWgrad = 2 };

template <int MODE>
__host__ __device__ constexpr int bwd_epi_warps() { return MODE == kModeDgradSwiglu ? 8 : 4; }
template <int MODE>
__host__ __device__ constexpr int bwd_threads() { return 64 + 32 * bwd_epi_warps<MODE>(); }

struct BwdCtl {
  uint64_t full[kQStages];
  uint64_t empty[kQStages];
  uint64_t acc_full[kQAcc];
  uint64_t acc_empty[kQAcc];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int num_m_tiles;   // dgrad: 128-row blocks over all groups
  int pad_;
  int group_rows[kQMaxGroups + 1];   // exclusive prefix of rows
  int tile_prefix[kQMaxGroups + 1];  // dgrad: exclusive prefix of 128-row blocks
};

constexpr size_t kQSmemBytes =
    1024 + static_cast<size_t>(kQStages) * kQStageBytes + kQEpiBytes + sizeof(BwdCtl);
static_assert(kQSmemBytes <= 232448, "shared memory budget of one sm_100 CTA");

struct BwdParams {
  const int32_t* counts;  // [G] rows per group
  int G;
  int64_t M;              // rows of the row-indexed operands
  int Kc;                 // dgrad: contraction length (columns of A)
  int Nout;               // output columns (dgrad: of the [M, Nout] result; wgrad: Nw)
  int Mw;                 // wgrad: output rows per group
  int n_tiles;            // column blocks of QN
  int m_tiles;            // wgrad: row blocks of QM per group
  int ksplit;             // wgrad: slices of each group's rows (1 = none)
  uint16_t* out;          // plain dgrad [M, Nout]; wgrad [G * Mw, Nout]
  float* out_f32;         // wgrad with ksplit > 1: fp32 partials [ksplit, G * Mw, Nout]
  // swiglu dgrad: saved gate_up rows [M, 2I] in, their gradient [M, 2I] out (I = Nout)
  const uint16_t* gate_up;
  uint16_t* d_gate_up;
  int* err;
  unsigned long long wait_limit_ns;
};

// Shared-memory descriptor of an MN-major operand staged as [64 k][64]
// boxes with the 128-byte swizzle: 8-row groups 1024 B apart (stride
// offset), consecutive 64-element boxes `box_stride` bytes apart (leading
// offset).
__device__ __forceinline__ uint64_t smem_desc_sw128_mn(uint32_t saddr, uint32_t box_stride) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((box_stride >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// kind::f16 instruction descriptor with the operand majors set: bit 15 = A
// MN-major, bit 16 = B MN-major.
__host__ __device__ constexpr uint32_t idesc_bf16_major(int m, int n, bool a_mn, bool b_mn) {
  return idesc_bf16_f32(m, n) | (a_mn ? (1u << 15) : 0u) | (b_mn ? (1u << 16) : 0u);
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int c0, int c1,
                                            int c2, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}

__device__ __forceinline__ uint4 ld_shared_v4q(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ void st_shared_v4q(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

// Tile t of the schedule.  dgrad: (128-row block over all groups, column
// block), column blocks innermost; wgrad: (group, row slice, row block,
// column block), where a group's rows are cut into ksplit slices of whole
// 64-row blocks (split-K: each slice's product is an fp32 partial).
struct QTile {
  int g;
  int split;    // wgrad: row slice
  int row0;     // dgrad: first output row; wgrad: first row of the slice
  int row_end;  // dgrad: the group's end row; wgrad: the slice's end row
  int m0;       // wgrad: first output row inside the group's block
  int n0;       // first output column
  int nkb;      // k-blocks of 64
};

template <int MODE>
__device__ __forceinline__ QTile decode_q(const BwdCtl& ctl, const BwdParams& p, int tile) {
  QTile t;
  if (MODE == kModeWgrad) {
    const int per_s = p.m_tiles * p.n_tiles;
    const int per_g = per_s * p.ksplit;
    t.g = tile / per_g;
    int r = tile - t.g * per_g;
    t.split = r / per_s;
    r -= t.split * per_s;
    const int mt = r / p.n_tiles;
    t.n0 = (r - mt * p.n_tiles) * QN;
    t.m0 = mt * QM;
    const int g0 = ctl.group_rows[t.g], g1 = ctl.group_rows[t.g + 1];
    const int slice = cdiv(cdiv(g1 - g0, p.ksplit), QK) * QK;
    t.row0 = min(g1, g0 + t.split * slice);
    t.row_end = min(g1, t.row0 + slice);
    t.nkb = cdiv(t.row_end - t.row0, QK);
  } else {
    const int mt = tile / p.n_tiles;
    t.n0 = (tile - mt * p.n_tiles) * QN;
    int lo = 0, hi = p.G;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (ctl.tile_prefix[mid] <= mt) lo = mid; else hi = mid;
    }
    t.g = lo;
    t.row0 = ctl.group_rows[lo] + (mt - ctl.tile_prefix[lo]) * QM;
    t.row_end = ctl.group_rows[lo + 1];
    t.m0 = 0;
    t.split = 0;
    t.nkb = cdiv(p.Kc, QK);
  }
  return t;
}

__device__ __forceinline__ float silu_fast(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

// SiLU(gate) * up backward for 32 columns of one row: dh (fp32 accumulator,
// rounded to bf16 here as the reference's grad_input tensor is), g and u the
// saved bf16 gate and up values -> d_gate, d_up (packed bf16x2).
__device__ __forceinline__ void swiglu_bwd_pack(const uint32_t (&acc)[32], const uint4 (&gw)[4],
                                                const uint4 (&uw)[4], uint4 (&dg)[4],
                                                uint4 (&du)[4]) {
  const uint32_t* g = reinterpret_cast<const uint32_t*>(gw);
  const uint32_t* u = reinterpret_cast<const uint32_t*>(uw);
  uint32_t* og = reinterpret_cast<uint32_t*>(dg);
  uint32_t* ou = reinterpret_cast<uint32_t*>(du);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint32_t dh = cvt_bf16x2(__uint_as_float(acc[2 * i]), __uint_as_float(acc[2 * i + 1]));
    const float g0 = bf16_lo(g[i]), g1 = bf16_hi(g[i]);
    const uint32_t sg = cvt_bf16x2(silu_fast(g0), silu_fast(g1));  // the forward's rounded silu
    ou[i] = mul_bf16x2(dh, sg);                                      // d_up
    const uint32_t dsg = mul_bf16x2(dh, u[i]);                       // d(silu(gate))
    const float s0 = __fdividef(1.0f, 1.0f + __expf(-g0));
    const float s1 = __fdividef(1.0f, 1.0f + __expf(-g1));
    og[i] = cvt_bf16x2(bf16_lo(dsg) * s0 * (1.0f + g0 * (1.0f - s0)),
                       bf16_hi(dsg) * s1 * (1.0f + g1 * (1.0f - s1)));
  }
}

template <int MODE>
__global__ void __launch_bounds__(bwd_threads<MODE>(), 1)
grouped_gemm_bwd_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmC, const BwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  BwdCtl& ctl = *reinterpret_cast<BwdCtl*>(smem + kQStages * kQStageBytes + kQEpiBytes);
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = p.G;
  constexpr int EPI = bwd_epi_warps<MODE>();
  constexpr bool kWgrad = MODE == kModeWgrad;

  // ---------------------------------------------------------------- setup
  if (warp == 0) {
    const int per = cdiv(G, 32);
    const int g0 = min(G, lane * per), g1 = min(G, g0 + per);
    int rows = 0, tiles = 0;
    for (int g = g0; g < g1; ++g) {
      const int c = max(0, p.counts[g]);
      rows += c;
      tiles += cdiv(c, QM);
    }
    int rin = rows, tin = tiles;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int ro = __shfl_up_sync(0xffffffffu, rin, off);
      const int to = __shfl_up_sync(0xffffffffu, tin, off);
      if (lane >= off) { rin += ro; tin += to; }
    }
    int rr = rin - rows, tr = tin - tiles;
    for (int g = g0; g < g1; ++g) {
      const int c = max(0, p.counts[g]);
      ctl.group_rows[g] = rr;
      ctl.tile_prefix[g] = tr;
      rr += c;
      tr += cdiv(c, QM);
    }
    if (lane == 31) {
      ctl.group_rows[G] = rin;
      ctl.tile_prefix[G] = tin;
      ctl.num_m_tiles = tin;
    }
    if (lane == 0) {
      for (int s = 0; s < kQStages; ++s) {
        mbar_init(smem_u32(&ctl.full[s]), 1);
        mbar_init(smem_u32(&ctl.empty[s]), 1);
      }
      for (int a = 0; a < kQAcc; ++a) {
        mbar_init(smem_u32(&ctl.acc_full[a]), 1);
        mbar_init(smem_u32(&ctl.acc_empty[a]), EPI);
      }
      mbar_init(smem_u32(&ctl.drain), 1);
      ctl.abort = 0;
      fence_mbar_init();
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      if (MODE != kModeDgradSwiglu) tma_prefetch_desc(&tmC);
    }
  } else if (warp == 1) {
    tmem_alloc(smem_u32(&ctl.tmem_base), kQTmemCols);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  const uint32_t tmem_base = ctl.tmem_base;
  const int num_tiles =
      kWgrad ? G * p.ksplit * p.m_tiles * p.n_tiles : ctl.num_m_tiles * p.n_tiles;
  volatile int* abort = &ctl.abort;
  int never = 0;
  const unsigned long long lim = p.wait_limit_ns;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        const QTile t = decode_q<MODE>(ctl, p, tile);
        for (int kb = 0; kb < t.nkb; ++kb) {
          if (!mbar_wait_bounded(smem_u32(&ctl.empty[stage]), phase ^ 1u, abort, p.err, lim)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(&ctl.full[stage]);
          const uint32_t sa = sbase + stage * kQStageBytes;
          const uint32_t sb = sa + kQABytes;
          mbar_arrive_expect_tx(fb, kQStageBytes);
          if (kWgrad) {
            const int r = t.row0 + kb * QK;
            tma_load_2d(sa, &tmA, t.m0, r, fb);
            tma_load_2d(sa + kQBox, &tmA, t.m0 + 64, r, fb);
#pragma unroll
            for (int i = 0; i < 4; ++i) tma_load_2d(sb + i * kQBox, &tmB, t.n0 + 64 * i, r, fb);
          } else {
            tma_load_2d(sa, &tmA, kb * QK, t.row0, fb);
#pragma unroll
            for (int i = 0; i < 4; ++i) tma_load_3d(sb + i * kQBox, &tmB, t.n0 + 64 * i, kb * QK, t.g, fb);
          }
          if (++stage == kQStages) { stage = 0; phase ^= 1u; }
        }
      }
      // every stage this CTA filled is released before it leaves
      for (int i = 0; i < kQStages; ++i) {
        if (!mbar_wait_bounded(smem_u32(&ctl.empty[stage]), phase ^ 1u, &never, p.err, lim)) break;
        if (++stage == kQStages) { stage = 0; phase ^= 1u; }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    // The whole warp walks the schedule (its lanes zero the rows past a
    // group's end in wgrad); lane 0 issues and commits.
    int stage = 0, acc = 0;
    uint32_t phase = 0, acc_phase = 0;
    constexpr uint32_t idesc = idesc_bf16_major(QM, QN, kWgrad, true);
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
      const QTile t = decode_q<MODE>(ctl, p, tile);
      if (t.nkb == 0) continue;  // an empty wgrad group: the epilogue writes zeros
      if (!mbar_wait_bounded(smem_u32(&ctl.acc_empty[acc]), acc_phase ^ 1u, abort, p.err, lim))
        break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * QN);
      for (int kb = 0; kb < t.nkb; ++kb) {
        if (!mbar_wait_bounded(smem_u32(&ctl.full[stage]), phase, abort, p.err, lim)) {
          ok = false;
          break;
        }
        const uint32_t sa = sbase + stage * kQStageBytes;
        const uint32_t sb = sa + kQABytes;
        if (kWgrad) {
          const int valid = t.row_end - (t.row0 + kb * QK);
          if (valid < QK) {
            // rows [valid, 64) of the 2 A boxes and 4 B boxes belong to the
            // next group: 128 zero bytes each
            const int nrow = QK - valid;
            const uint4 z = make_uint4(0u, 0u, 0u, 0u);
            for (int i = lane; i < 6 * nrow * 8; i += 32) {
              const int box = i / (nrow * 8);
              const int rem = i - box * nrow * 8;
              const int row = valid + (rem >> 3);
              st_shared_v4q(sa + box * kQBox + row * 128 + ((rem & 7) << 4), z);
            }
            fence_proxy_async_smem();
          }
          __syncwarp();
        }
        tc_fence_after();
        if (lane == 0) {
#pragma unroll
          for (int kk = 0; kk < QK / 16; ++kk) {
            const uint64_t ad = kWgrad ? smem_desc_sw128_mn(sa + kk * 2048, kQBox)
                                       : smem_desc_sw128(sa + kk * 32);
            const uint64_t bd = smem_desc_sw128_mn(sb + kk * 2048, kQBox);
            tc_mma_bf16(d_tmem, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          tc_commit(smem_u32(&ctl.empty[stage]));
        }
        __syncwarp();
        if (++stage == kQStages) { stage = 0; phase ^= 1u; }
      }
      if (!ok) break;
      if (lane == 0) tc_commit(smem_u32(&ctl.acc_full[acc]));
      __syncwarp();
      if (++acc == kQAcc) { acc = 0; acc_phase ^= 1u; }
    }
    if (lane == 0) {
      // every MMA issued has completed, and the epilogue released every
      // accumulator, before TMEM is freed
      tc_commit(smem_u32(&ctl.drain));
      mbar_wait_bounded(smem_u32(&ctl.drain), 0, &never, p.err, lim);
      for (int i = 0; i < kQAcc; ++i) {
        if (!mbar_wait_bounded(smem_u32(&ctl.acc_empty[acc]), acc_phase ^ 1u, &never, p.err, lim))
          break;
        if (++acc == kQAcc) { acc = 0; acc_phase ^= 1u; }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;
    const int quad = warp & 3;
    const int r_in_tile = quad * 32 + lane;
    constexpr int kStride = EPI / 4;   // warps per quadrant
    const int first = ew >> 2;         // this warp's first 32-column chunk
    const uint32_t stg = sbase + kQStages * kQStageBytes + (ew & 3) * 2 * kQEpiChunk;
    int acc = 0, buf = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const QTile t = decode_q<MODE>(ctl, p, tile);
      // output rows of this tile: dgrad rows [row0, min(row0 + 128, row_end));
      // wgrad rows g * Mw + [m0, min(m0 + 128, Mw))
      int nrows;
      int64_t orow0;
      if (kWgrad) {
        nrows = min(QM, p.Mw - t.m0);
        orow0 = static_cast<int64_t>(t.g) * p.Mw + t.m0;
      } else {
        nrows = min(QM, t.row_end - t.row0);
        orow0 = t.row0;
      }
      const bool row_ok = r_in_tile < nrows && (kWgrad || orow0 + r_in_tile < p.M);
      const bool quad_full = (quad + 1) * 32 <= nrows && (kWgrad || orow0 + (quad + 1) * 32 <= p.M);
      const int64_t grow = orow0 + r_in_tile;
      float* prow = nullptr;  // wgrad split-K: this row's fp32 partial
      if (kWgrad && p.out_f32)
        prow = p.out_f32 + (static_cast<int64_t>(t.split) * G * p.Mw + grow) * p.Nout;
      if (kWgrad && t.nkb == 0) {
        // a group (or slice) with no rows: its contribution is zero
        if (row_ok) {
          for (int c = first; c < QN / 32; c += kStride) {
            const int col0 = t.n0 + c * 32;
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4) {
              if (col0 + c4 * 8 + 8 > p.Nout) continue;
              if (prow) {
                *reinterpret_cast<uint4*>(prow + col0 + c4 * 8) = make_uint4(0u, 0u, 0u, 0u);
                *reinterpret_cast<uint4*>(prow + col0 + c4 * 8 + 4) = make_uint4(0u, 0u, 0u, 0u);
              } else {
                *reinterpret_cast<uint4*>(p.out + grow * p.Nout + col0 + c4 * 8) =
                    make_uint4(0u, 0u, 0u, 0u);
              }
            }
          }
        }
        continue;
      }
      if (MODE == kModeDgradSwiglu) {
        // SiLU(gate) * up backward.  Nout = I; the saved gate_up row holds
        // gate at [0, I) and up at [I, 2I).  A lane owns one accumulator row,
        // so reading and writing 64 B per lane and row would touch 32 lines
        // per instruction; instead the warp moves each 32-row x 32-column
        // block through a 2 KiB swizzled buffer: global loads and stores are
        // coalesced (8 rows x 64 B per instruction) and the buffer turns them
        // into one row per lane.  The gate/up values of a chunk are loaded
        // one chunk ahead (the first while the accumulator is being
        // computed).  A chunk may end past I (a multiple of 8, not of 32):
        // only its 8-column groups inside [0, I) are read and written.
        const int64_t I = p.Nout;
        const uint32_t tbuf = sbase + kQStages * kQStageBytes + ew * 2048;
        const int cr = lane >> 2, cc = lane & 3;  // coalesced: row 8 i + cr, 16 B column cc
        // rows of this quadrant that are inside the tile's group and inside M
        const int64_t qrow0 = orow0 + quad * 32;
        const int qrows = static_cast<int>(
            max(int64_t(0), min(min(int64_t(32), int64_t(nrows) - quad * 32), p.M - qrow0)));
        auto load_gu = [&](int c, uint4 (&g)[4], uint4 (&u)[4]) {
          const int col = t.n0 + c * 32 + cc * 8;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int r = 8 * i + cr;
            const bool in = r < qrows && col + 8 <= p.Nout;
            const uint16_t* src = p.gate_up + (qrow0 + (in ? r : 0)) * 2 * I + col;
            g[i] = in ? *reinterpret_cast<const uint4*>(src) : make_uint4(0u, 0u, 0u, 0u);
            u[i] = in ? *reinterpret_cast<const uint4*>(src + I) : make_uint4(0u, 0u, 0u, 0u);
          }
        };
        // coalesced layout <-> one row per lane, through the warp's buffer
        auto to_rows = [&](const uint4 (&q)[4], uint4 (&row)[4]) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int r = 8 * i + cr;
            st_shared_v4q(tbuf + r * 64 + ((cc ^ ((r >> 1) & 3)) << 4), q[i]);
          }
          __syncwarp();
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4)
            row[c4] = ld_shared_v4q(tbuf + lane * 64 + ((c4 ^ ((lane >> 1) & 3)) << 4));
          __syncwarp();
        };
        auto store_rows = [&](const uint4 (&row)[4], uint16_t* base_col) {
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4)
            st_shared_v4q(tbuf + lane * 64 + ((c4 ^ ((lane >> 1) & 3)) << 4), row[c4]);
          __syncwarp();
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int r = 8 * i + cr;
            const uint4 v = ld_shared_v4q(tbuf + r * 64 + ((cc ^ ((r >> 1) & 3)) << 4));
            if (r < qrows && base_col) *reinterpret_cast<uint4*>(base_col + (qrow0 + r) * 2 * I) = v;
          }
          __syncwarp();
        };
        uint4 gq[4], uq[4];
        load_gu(first, gq, uq);
        if (!mbar_wait_bounded(smem_u32(&ctl.acc_full[acc]), acc_phase, abort, p.err, lim)) break;
        tc_fence_after();
        const uint32_t trow = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                              static_cast<uint32_t>(acc * QN);
#pragma unroll 1
        for (int c = first; c < QN / 32; c += kStride) {
          uint4 gn[4], un[4];
          if (c + kStride < QN / 32) load_gu(c + kStride, gn, un);
          uint32_t ra[32];
          tmem_ld_32cols(trow + c * 32, ra);
          tc_wait_ld();
          const int col0 = t.n0 + c * 32;
          if (qrows > 0 && col0 < p.Nout) {
            uint4 gw[4], uw[4], dg[4], du[4];
            to_rows(gq, gw);
            to_rows(uq, uw);
            swiglu_bwd_pack(ra, gw, uw, dg, du);
            const int col = col0 + cc * 8;
            const bool col_in = col + 8 <= p.Nout;
            store_rows(dg, col_in ? p.d_gate_up + col : nullptr);
            store_rows(du, col_in ? p.d_gate_up + I + col : nullptr);
          }
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            gq[i] = gn[i];
            uq[i] = un[i];
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&ctl.acc_empty[acc]));
        if (++acc == kQAcc) { acc = 0; acc_phase ^= 1u; }
        continue;
      }
      if (!mbar_wait_bounded(smem_u32(&ctl.acc_full[acc]), acc_phase, abort, p.err, lim)) break;
      tc_fence_after();
      const uint32_t trow = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                            static_cast<uint32_t>(acc * QN);
#pragma unroll 1
      for (int c = first; c < QN / 32; c += kStride) {
        uint32_t ra[32];
        tmem_ld_32cols(trow + c * 32, ra);
        tc_wait_ld();
        const int col0 = t.n0 + c * 32;
        if (col0 >= p.Nout) continue;
        if (kWgrad && prow) {
          // split-K partial: the fp32 sums, unrounded
          if (row_ok) {
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4) {
              if (col0 + c4 * 8 + 8 > p.Nout) continue;
              *reinterpret_cast<uint4*>(prow + col0 + c4 * 8) =
                  make_uint4(ra[8 * c4], ra[8 * c4 + 1], ra[8 * c4 + 2], ra[8 * c4 + 3]);
              *reinterpret_cast<uint4*>(prow + col0 + c4 * 8 + 4) =
                  make_uint4(ra[8 * c4 + 4], ra[8 * c4 + 5], ra[8 * c4 + 6], ra[8 * c4 + 7]);
            }
          }
          continue;
        }
        uint32_t packed[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          packed[i] = cvt_bf16x2(__uint_as_float(ra[2 * i]), __uint_as_float(ra[2 * i + 1]));
        if (quad_full && col0 + 32 <= p.Nout) {
          if (lane == 0) bulk_wait_group_read<1>();
          __syncwarp();
          const uint32_t dst = stg + buf * kQEpiChunk + lane * 64;
          const uint32_t sw = (lane >> 1) & 3;
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4)
            st_shared_v4q(dst + ((c4 ^ sw) << 4), make_uint4(packed[4 * c4], packed[4 * c4 + 1],
                                                             packed[4 * c4 + 2], packed[4 * c4 + 3]));
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC, col0, static_cast<int>(orow0) + quad * 32, stg + buf * kQEpiChunk);
            bulk_commit_group();
          }
          buf ^= 1;
        } else if (row_ok) {
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4)
            if (col0 + c4 * 8 + 8 <= p.Nout)
              *reinterpret_cast<uint4*>(p.out + grow * p.Nout + col0 + c4 * 8) =
                  make_uint4(packed[4 * c4], packed[4 * c4 + 1], packed[4 * c4 + 2],
                             packed[4 * c4 + 3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&ctl.acc_empty[acc]));
      if (++acc == kQAcc) { acc = 0; acc_phase ^= 1u; }
    }
    if (lane == 0) bulk_wait_group_all();
    __syncwarp();
  }

  // --------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kQTmemCols);
  }
}

// Split-K wgrad: out[i] = bf16(sum over slices, in order, of partial[s][i]).
__global__ void __launch_bounds__(256)
splitk_reduce_kernel(const float4* __restrict__ partial, int64_t n4, int ksplit,
                     uint2* __restrict__ out) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float4 a = partial[i];
    for (int s2 = 1; s2 < ksplit; ++s2) {
      const float4 b = partial[static_cast<int64_t>(s2) * n4 + i];
      a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
    }
    out[i] = make_uint2(cvt_bf16x2(a.x, a.y), cvt_bf16x2(a.z, a.w));
  }
}

// ------------------------------------------------------------ host side ----
typedef CUresult (*EncodeTiledFnQ)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFnQ encode_fn_q() {
  static EncodeTiledFnQ fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFnQ>(ptr);
  });
  return fn;
}

// 2-D bf16 map over a row-major [rows, cols] matrix.
bool map2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows,
           uint32_t box_cols, CUtensorMapSwizzle swizzle) {
  EncodeTiledFnQ enc = encode_fn_q();
  if (!enc) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 3-D bf16 map over [G][rows][cols] with [64 rows][64 cols] boxes of one group.
bool map3d_groups(CUtensorMap* map, const void* base, uint64_t G, uint64_t rows, uint64_t cols) {
  EncodeTiledFnQ enc = encode_fn_q();
  if (!enc) return false;
  const cuuint64_t dims[3] = {cols, rows, G};
  const cuuint64_t strides[2] = {cols * 2, rows * cols * 2};
  const cuuint32_t box[3] = {64, 64, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int MODE>
cudaError_t ensure_bwd_attr() {
  static int done[64] = {0};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (!done[dev]) {
    e = cudaFuncSetAttribute(grouped_gemm_bwd_kernel<MODE>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kQSmemBytes));
    if (e != cudaSuccess) return e;
    done[dev] = 1;
  }
  return cudaSuccess;
}

template <int MODE>
cudaError_t launch_bwd(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc,
                       const BwdParams& p, int64_t max_tiles, int sm_limit, cudaStream_t stream) {
  cudaError_t e = ensure_bwd_attr<MODE>();
  if (e != cudaSuccess) return e;
  const int sms = sm_limit > 0 ? sm_limit : num_sms_for_current_device();
  int grid = static_cast<int>(max_tiles < sms ? max_tiles : sms);
  if (grid < 1) grid = 1;
  grouped_gemm_bwd_kernel<MODE><<<grid, bwd_threads<MODE>(), kQSmemBytes, stream>>>(ma, mb, mc, p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_grouped_dgrad(const GroupedDgradArgs& a, cudaStream_t stream) {
  if (a.M == 0 || a.G == 0) return cudaSuccess;
  if (a.G > kQMaxGroups || a.Kc % 8 != 0 || a.Nout % 8 != 0) return cudaErrorInvalidValue;
  CUtensorMap ma, mb, mc;
  const bool swiglu = a.gate_up != nullptr;
  if (!map2d(&ma, a.grad_out, static_cast<uint64_t>(a.M), static_cast<uint64_t>(a.Kc), QM, QK,
             CU_TENSOR_MAP_SWIZZLE_128B) ||
      !map3d_groups(&mb, a.weight, static_cast<uint64_t>(a.G), static_cast<uint64_t>(a.Kc),
                    static_cast<uint64_t>(a.Nout)))
    return cudaErrorInvalidValue;
  if (swiglu) {
    mc = mb;  // unused: the SwiGLU backward stores directly
  } else if (!map2d(&mc, a.out, static_cast<uint64_t>(a.M), static_cast<uint64_t>(a.Nout), 32, 32,
                    CU_TENSOR_MAP_SWIZZLE_64B)) {
    return cudaErrorInvalidValue;
  }
  BwdParams p = {};
  p.ksplit = 1;
  p.counts = a.counts;
  p.G = a.G;
  p.M = a.M;
  p.Kc = a.Kc;
  p.Nout = a.Nout;
  p.n_tiles = cdiv(a.Nout, QN);
  p.out = static_cast<uint16_t*>(a.out);
  p.gate_up = static_cast<const uint16_t*>(a.gate_up);
  p.d_gate_up = static_cast<uint16_t*>(a.d_gate_up);
  p.err = a.err;
  p.wait_limit_ns = kWaitLimitNs;
  const int64_t max_tiles = (cdiv64(a.M, QM) + a.G) * p.n_tiles;
  return swiglu ? launch_bwd<kModeDgradSwiglu>(ma, mb, mc, p, max_tiles, a.sm_limit, stream)
                : launch_bwd<kModeDgrad>(ma, mb, mc, p, max_tiles, a.sm_limit, stream);
}

cudaError_t launch_grouped_wgrad(const GroupedWgradArgs& a, cudaStream_t stream) {
  if (a.G == 0) return cudaSuccess;
  if (a.G > kQMaxGroups || a.Mw % 8 != 0 || a.Nw % 8 != 0) return cudaErrorInvalidValue;
  if (a.M == 0)  // no rows at all: every group's gradient is zero
    return cudaMemsetAsync(a.out, 0, sizeof(uint16_t) * static_cast<size_t>(a.G) * a.Mw * a.Nw,
                           stream);
  CUtensorMap ma, mb, mc;
  const uint64_t rows = static_cast<uint64_t>(a.M);
  if (!map2d(&ma, a.grad_out, rows, static_cast<uint64_t>(a.Mw), 64, 64, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !map2d(&mb, a.input, rows, static_cast<uint64_t>(a.Nw), 64, 64, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !map2d(&mc, a.out, static_cast<uint64_t>(a.G) * a.Mw, static_cast<uint64_t>(a.Nw), 32, 32,
             CU_TENSOR_MAP_SWIZZLE_64B))
    return cudaErrorInvalidValue;
  BwdParams p = {};
  p.counts = a.counts;
  p.G = a.G;
  p.M = a.M;
  p.Mw = a.Mw;
  p.Nout = a.Nw;
  p.m_tiles = cdiv(a.Mw, QM);
  p.n_tiles = cdiv(a.Nw, QN);
  p.ksplit = a.partial && a.ksplit > 1 ? a.ksplit : 1;
  p.out = static_cast<uint16_t*>(a.out);
  p.out_f32 = p.ksplit > 1 ? a.partial : nullptr;
  p.err = a.err;
  p.wait_limit_ns = kWaitLimitNs;
  const int64_t max_tiles = static_cast<int64_t>(a.G) * p.ksplit * p.m_tiles * p.n_tiles;
  cudaError_t e = launch_bwd<kModeWgrad>(ma, mb, mc, p, max_tiles, a.sm_limit, stream);
  if (e != cudaSuccess || p.ksplit == 1) return e;
  const int64_t n4 = static_cast<int64_t>(a.G) * a.Mw * a.Nw / 4;
  const int blocks = static_cast<int>(cdiv64(n4, 256) < 4 * 148 ? cdiv64(n4, 256) : 4 * 148);
  splitk_reduce_kernel<<<blocks, 256, 0, stream>>>(reinterpret_cast<const float4*>(a.partial), n4,
                                                    p.ksplit, reinterpret_cast<uint2*>(a.out));
  return cudaGetLastError();
}

}  // namespace hmoe

namespace hmoe {
int wgrad_ksplit(int64_t M, int Mw, int Nw, int G) {
  const int64_t tiles = static_cast<int64_t>(G) * cdiv(Mw, QM) * cdiv(Nw, QN);
  const int64_t sms = num_sms_for_current_device();
  if (tiles >= sms) return 1;
  int64_t ks = cdiv64(sms, tiles);
  const int64_t max_by_rows = cdiv64(M, 4 * QK);  // at least four 64-row blocks per slice
  if (ks > max_by_rows) ks = max_by_rows;
  return ks < 1 ? 1 : static_cast<int>(ks > 64 ? 64 : ks);
}
}  // namespace hmoe
