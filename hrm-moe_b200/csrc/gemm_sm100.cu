// Grouped expert GEMMs on the sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// Replaces the forward kernel of models/moe_triton_grouped_gemm.py
// (_m_grouped_gemm_bk_kernel, :113-184, launched from :358-417): for every
// group g (an expert) the rows [off_g, off_g + n_g) of A are multiplied by
// B[g]^T, with fp32 accumulation and a bf16 result:
//   plain:   out[r, :] = A[r, :] @ B[g]^T                      B[g]: [N, K]
//   swiglu:  out[r, :] = silu(A[r] @ Bg^T) * (A[r] @ Bu^T)     B[g]: [2N, K]
//            (Bg = rows 0..N-1, Bu = rows N..2N-1; models/layers.py:326-329)
//
// Design (one persistent CTA per SM, 192 threads):
//   warp 0      TMA producer: A tile [128 x 64] and two B boxes [128 x 64]
//               per k-step into a 4-stage ring (128-byte swizzle).
//   warp 1      allocates 512 TMEM columns; lane 0 issues tcgen05.mma
//               (M=128, N=256, K=16) into one of two 256-column fp32
//               accumulators and commits stage / accumulator barriers.
//   warps 2..5  epilogue: tcgen05.ld the accumulator (each warp its 32-lane
//               quadrant), apply the activation, convert to bf16, stage 32x32
//               chunks in shared memory and TMA-store them (rows past a group
//               end are stored directly, masked); then free the accumulator
//               so the next tile's MMAs overlap this tile's stores.
// Tiles are (group, 128-row block, column block); the table of group row
// offsets and tile prefixes is built in shared memory from the per-group
// counts on the device, so no host synchronisation is needed.  A group's
// last row block may run into the next group's rows: those rows are loaded
// (or zero-filled past the end of A) but never stored.
//
// Every mbarrier wait is bounded (kWaitLimitNs): on a timeout the kernel
// records kDevTimeout, the roles leave their loops, outstanding bulk copies
// and MMAs are waited for (again bounded) and TMEM is released.
//
// No TMA multicast is used anywhere (this kernel also runs in expert-
// parallel jobs on several GPUs).
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace hmoe {
namespace {

constexpr int BM = 128;                       // rows per tile (MMA M)
constexpr int BK = 64;                        // bf16 per swizzled 128-byte row
constexpr int BNH = 128;                      // rows per B box
constexpr int kStages = 4;
constexpr int kABytes = BM * BK * 2;          // 16 KB
constexpr int kBBoxBytes = BNH * BK * 2;      // 16 KB
constexpr int kStageBytes = kABytes + 2 * kBBoxBytes;  // 48 KB
constexpr int kAccCols = 256;                 // fp32 accumulator columns (MMA N)
constexpr int kNumAcc = 2;
constexpr int kTmemCols = kAccCols * kNumAcc; // 512 = all of TMEM
// Epilogue warps: the SwiGLU tile (exp + divide per output, direct stores)
// takes two warps per TMEM lane quadrant to hide its latency; the plain tile
// takes one per quadrant with two TMA staging boxes each.
constexpr int kPushWarps = 8;    // row senders of the fused expert-parallel dispatch
constexpr int kPushEpiWarps = 8;  // epilogue warps of that kernel
template <bool SWIGLU, bool SCATTER, bool PUSH = false>
__host__ __device__ constexpr int epi_warps() { return PUSH ? kPushEpiWarps : (SWIGLU ? 8 : 4); }
template <bool SWIGLU, bool SCATTER, bool PUSH>
__host__ __device__ constexpr int num_threads() {  // + producer, MMA issuer (+ senders)
  return 64 + 32 * epi_warps<SWIGLU, SCATTER, PUSH>() + (PUSH ? 32 * kPushWarps : 0);
}
constexpr int kMaxGroups = 1024;
constexpr int kEpiChunkBytes = 32 * 32 * 2;                  // 32 rows x 32 bf16 columns
constexpr int kEpiBytes = 4 * 2 * kEpiChunkBytes;            // plain tile: 2 boxes per warp

struct SmemCtl {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t acc_full[kNumAcc];
  uint64_t acc_empty[kNumAcc];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int num_m_tiles;
  int pad_;
  int group_rows[kMaxGroups + 1];   // exclusive prefix of rows
  int tile_prefix[kMaxGroups + 1];  // exclusive prefix of 128-row blocks
  int group_w[kMaxGroups];          // weight (expert) index of each group
  // fused dispatch: the send order is (local expert, owner) so that every
  // owner's first groups fill first; vstart is the prefix of rows over it
  int push_vstart[129];
  int push_vexp[128];
  int push_ebase[128];              // first sorted position of each expert here
};

constexpr size_t kSmemBytes =
    1024 + static_cast<size_t>(kStages) * kStageBytes + kEpiBytes + sizeof(SmemCtl);
static_assert(kSmemBytes <= 232448, "shared memory budget of one sm_100 CTA");

struct KParams {
  const int32_t* counts;
  const int32_t* group_weight;  // [G] weight index per group, or null (= g)
  int G;
  int64_t M;
  int N;                    // output columns
  int K;
  int n_tiles;              // column blocks
  int out_cols_per_tile;    // 128 (swiglu) or 256 (plain)
  int b_rows_per_group;     // rows of B per group (2N swiglu, N plain)
  int b_second_off;         // row offset of the second B box (N swiglu, 128 plain)
  uint16_t* out;
  int* err;
  unsigned long long wait_limit_ns;
  // expert-parallel return (SCATTER): see GroupedGemmArgs
  const int32_t* scatter_src;
  char* scatter_base[8];
  int scatter_world;
  int64_t scatter_cap;
  unsigned* done;
  uint32_t* flag[8];
  uint32_t epoch;
  // fused expert-parallel dispatch (PUSH): see GroupedGemmArgs
  const uint4* push_x;
  const int32_t* push_sorted_token;
  const int32_t* push_counts;
  const int32_t* push_send_base;
  uint4* push_rows[8];
  int32_t* push_src[8];
  uint32_t* push_arrived[8];
  const uint32_t* arrived;
  int64_t push_A;
  int64_t push_cap;
  int push_E, push_El, push_world, push_me, push_row_chunks;
};

__device__ __forceinline__ void decode_tile(const SmemCtl& ctl, int G, int n_tiles, int tile,
                                            int& g, int& row0, int& nrows, int& n) {
  const int mt = tile / n_tiles;
  n = tile - mt * n_tiles;
  int lo = 0, hi = G;  // tile_prefix[lo] <= mt < tile_prefix[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (ctl.tile_prefix[mid] <= mt) lo = mid; else hi = mid;
  }
  g = lo;
  row0 = ctl.group_rows[g] + (mt - ctl.tile_prefix[g]) * BM;
  nrows = min(BM, ctl.group_rows[g + 1] - row0);
}

// 32 accumulator columns of one row -> 16 packed bf16x2 words.  SwiGLU
// rounds where the reference does (models/layers.py:326-329: gate_up is a
// bf16 tensor, F.silu returns bf16, the product is rounded again) with packed
// instructions: one paired conversion rounds two gate (or up) values, SiLU
// runs in fp32 on the rounded gate (the fast exp and divide intrinsics: a few
// fp32 ulps, far below the bf16 step the result is rounded to) and is rounded
// by another paired conversion, and mul.rn.bf16x2 rounds the product once
// (the product of two bf16 values is exact in fp32).
template <bool SWIGLU>
__device__ __forceinline__ void epi_pack(const uint32_t (&a)[32], const uint32_t (&b)[32],
                                         uint32_t (&packed)[16]) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    if (SWIGLU) {
      const uint32_t g = cvt_bf16x2(__uint_as_float(a[2 * i]), __uint_as_float(a[2 * i + 1]));
      const uint32_t u = cvt_bf16x2(__uint_as_float(b[2 * i]), __uint_as_float(b[2 * i + 1]));
      const float g0 = bf16_lo(g), g1 = bf16_hi(g);
      const uint32_t sg = cvt_bf16x2(__fdividef(g0, 1.0f + __expf(-g0)),
                                     __fdividef(g1, 1.0f + __expf(-g1)));
      packed[i] = mul_bf16x2(sg, u);
    } else {
      packed[i] = cvt_bf16x2(__uint_as_float(a[2 * i]), __uint_as_float(a[2 * i + 1]));
    }
  }
}

// Direct row store (rows whose 32-row quadrant crosses a group end).
__device__ __forceinline__ void store_row_direct(const uint32_t (&packed)[16], uint16_t* orow,
                                                 int col0, int N) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    if (col0 + c * 8 + 8 <= N) {
      uint4 v = make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2], packed[4 * c + 3]);
      *reinterpret_cast<uint4*>(orow + col0 + c * 8) = v;
    }
  }
}

__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

// Sender warps: this rank's rows in send order, dealt out round-robin in
// chunks of kPushChunk rows, so that all senders advance one frontier through
// the owners' groups and each group completes as early as it can.  Each row
// is read from x once and stored into its owner's receive buffer with its
// origin; after each run of one expert's rows within a chunk the warp fences
// and adds the run to the owner's arrival counter.  Sends nothing once the
// call has failed (the owners' waits then run out and report it).
constexpr int kPushChunk = 16;

// Copy one row, 16 bytes per lane, every load of a 4 KiB span issued before
// its stores.
__device__ __forceinline__ void push_copy_row(const uint4* __restrict__ src, uint4* dst, int rc,
                                              int lane) {
  for (int c0 = 0; c0 < rc; c0 += 256) {
    uint4 buf[8];
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      const int c = c0 + lane + 32 * s;
      if (c < rc) buf[s] = __ldg(src + c);
    }
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      const int c = c0 + lane + 32 * s;
      if (c < rc) dst[c] = buf[s];
    }
  }
}

__device__ __forceinline__ void push_rows(const KParams& p, const SmemCtl& ctl, int pw, int npw,
                                          int lane) {
  if (*reinterpret_cast<volatile const int*>(p.err) != kDevOk) return;
  const int64_t A = p.push_A;
  const int rc = p.push_row_chunks;  // 16-byte pieces per row
  const int64_t nch = (A + kPushChunk - 1) / kPushChunk;
  for (int64_t ch = pw; ch < nch; ch += npw) {
    int64_t v = ch * kPushChunk;
    const int64_t vend = min(A, v + kPushChunk);
    int lo = 0, hi = p.push_E;  // the segment holding v: vstart[lo] <= v < vstart[hi]
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (ctl.push_vstart[mid] <= v) lo = mid; else hi = mid;
    }
    for (int i = lo; v < vend && i < p.push_E; ++i) {
      const int64_t seg_end = min(vend, static_cast<int64_t>(ctl.push_vstart[i + 1]));
      if (v >= seg_end) continue;
      const int e = ctl.push_vexp[i];
      const int o = e / p.push_El, el = e - o * p.push_El;
      const int64_t sb = p.push_send_base[e];
      if (sb < 0) return;  // the exchange failed
      const int64_t vs = ctl.push_vstart[i];
      const int eb = ctl.push_ebase[e];
      uint4* rows = p.push_rows[o];
      int32_t* srcs = p.push_src[o];
      // q = sb + (vv - vs) grows with vv: rows from vv = vs + push_cap - sb on
      // would land beyond the owner's receive buffer and are not stored.
      const int64_t store_end = min(seg_end, vs + (p.push_cap - sb));
      if (store_end < seg_end && lane == 0) record_error(p.err, kDevEpOverflow);
      for (int64_t vv = v; vv < store_end; ++vv) {
        const int64_t rel = vv - vs;
        const int64_t q = sb + rel;
        const int pos = eb + static_cast<int>(rel);
        const int t = p.push_sorted_token[pos];
        push_copy_row(p.push_x + static_cast<int64_t>(t) * rc, rows + q * rc, rc, lane);
        if (lane == 0)
          srcs[q] = static_cast<int32_t>((static_cast<uint32_t>(p.push_me) << kEpSrcShift) |
                                         static_cast<uint32_t>(pos));
      }
      __threadfence_system();
      __syncwarp();
      // Only the rows actually stored count as arrived: after an overflow the
      // owner's group never completes, so its bounded wait reports a timeout
      // instead of computing on rows that were never written.
      if (lane == 0 && store_end > v)
        red_release_sys_add(p.push_arrived[o] + el, static_cast<uint32_t>(store_end - v));
      v = seg_end;
    }
  }
}

template <bool SWIGLU, bool SCATTER, bool PUSH>
__global__ void __launch_bounds__(num_threads<SWIGLU, SCATTER, PUSH>(), 1)
grouped_gemm_sm100_kernel(const __grid_constant__ CUtensorMap tmA,
                          const __grid_constant__ CUtensorMap tmB,
                          const __grid_constant__ CUtensorMap tmC, const KParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  SmemCtl& ctl = *reinterpret_cast<SmemCtl*>(smem + kStages * kStageBytes + kEpiBytes);
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = p.G;

  // ---------------------------------------------------------------- setup
  if (warp == 0) {
    grid_dependency_wait();  // launched early (launch_pdl): the counts are written before this
    const int per = cdiv(G, 32);
    const int g0 = min(G, lane * per), g1 = min(G, g0 + per);
    int rows = 0, tiles = 0;
    for (int g = g0; g < g1; ++g) {
      const int c = max(0, p.counts[g]);
      rows += c;
      tiles += cdiv(c, BM);
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
      ctl.group_w[g] = p.group_weight ? p.group_weight[g] : g;
      rr += c;
      tr += cdiv(c, BM);
    }
    if (lane == 31) {
      ctl.group_rows[G] = rin;
      ctl.tile_prefix[G] = tin;
      ctl.num_m_tiles = tin;
    }
    if (PUSH && lane == 0) {
      int run = 0;
      for (int e = 0; e < p.push_E; ++e) {
        ctl.push_ebase[e] = run;
        run += max(0, p.push_counts[e]);
      }
      int vrun = 0;
      for (int i = 0; i < p.push_E; ++i) {
        const int e = (i % p.push_world) * p.push_El + i / p.push_world;
        ctl.push_vexp[i] = e;
        ctl.push_vstart[i] = vrun;
        vrun += max(0, p.push_counts[e]);
      }
      ctl.push_vstart[p.push_E] = vrun;
    }
    if (lane == 0) {
      for (int s = 0; s < kStages; ++s) {
        mbar_init(smem_u32(&ctl.full[s]), 1);
        mbar_init(smem_u32(&ctl.empty[s]), 1);
      }
      for (int a = 0; a < kNumAcc; ++a) {
        mbar_init(smem_u32(&ctl.acc_full[a]), 1);
        mbar_init(smem_u32(&ctl.acc_empty[a]), epi_warps<SWIGLU, SCATTER, PUSH>());
      }
      mbar_init(smem_u32(&ctl.drain), 1);
      ctl.abort = 0;
      fence_mbar_init();
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      tma_prefetch_desc(&tmC);
    }
  } else if (warp == 1) {
    tmem_alloc(smem_u32(&ctl.tmem_base), kTmemCols);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  grid_dependency_wait();
  grid_launch_dependents();

  const uint32_t tmem_base = ctl.tmem_base;
  const int num_tiles = ctl.num_m_tiles * p.n_tiles;
  const int nkb = cdiv(p.K, BK);
  volatile int* abort = &ctl.abort;
  int never = 0;  // an abort flag nobody raises, for the teardown waits
  const unsigned long long lim = p.wait_limit_ns;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, pending = 0, pend_phase = 0;
      bool ok = true;
      int ready = -1;  // groups [0, ready] have all their rows (fused dispatch)
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        int g, row0, nrows, n;
        decode_tile(ctl, G, p.n_tiles, tile, g, row0, nrows, n);
        const int rb0 = ctl.group_w[g] * p.b_rows_per_group + n * p.out_cols_per_tile;
        const int rb1 = rb0 + p.b_second_off;
        if (PUSH && g > ready) {
          // every source's rows of this group have landed (bounded wait)
          const uint32_t want = static_cast<uint32_t>(max(0, p.counts[g]));
          const unsigned long long t0 = global_timer_ns();
          while (static_cast<int32_t>(ld_acquire_sys(p.arrived + g) - want) < 0) {
            if (*abort) { ok = false; break; }
            if (global_timer_ns() - t0 > lim) {
              *abort = 1;
              record_error(p.err, kDevTimeout);
              ok = false;
              break;
            }
          }
          if (!ok) break;
          fence_proxy_async_global();  // the rows were written by plain stores
          ready = g;
        }
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait_bounded(smem_u32(&ctl.empty[stage]), phase ^ 1u, abort, p.err, lim)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(&ctl.full[stage]);
          const uint32_t sa = sbase + stage * kStageBytes;
          mbar_arrive_expect_tx(fb, kStageBytes);
          tma_load_2d(sa, &tmA, kb * BK, row0, fb);
          tma_load_2d(sa + kABytes, &tmB, kb * BK, rb0, fb);
          tma_load_2d(sa + kABytes + kBBoxBytes, &tmB, kb * BK, rb1, fb);
          pending |= 1u << stage;
          pend_phase = (pend_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
      }
      // no bulk copy may still be landing in shared memory when the CTA exits
      for (int s = 0; s < kStages; ++s)
        if ((pending >> s) & 1u)
          mbar_wait_bounded(smem_u32(&ctl.full[s]), (pend_phase >> s) & 1u, &never, p.err, lim);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      constexpr uint32_t idesc = idesc_bf16_f32(BM, kAccCols);
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        if (!mbar_wait_bounded(smem_u32(&ctl.acc_empty[acc]), acc_phase ^ 1u, abort, p.err, lim)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kAccCols);
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait_bounded(smem_u32(&ctl.full[stage]), phase, abort, p.err, lim)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = sbase + stage * kStageBytes;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = smem_desc_sw128(sa + kk * 32);
            const uint64_t bd = smem_desc_sw128(sa + kABytes + kk * 32);
            tc_mma_bf16(d_tmem, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          tc_commit(smem_u32(&ctl.empty[stage]));
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        tc_commit(smem_u32(&ctl.acc_full[acc]));
        if (++acc == kNumAcc) { acc = 0; acc_phase ^= 1u; }
      }
      // every MMA issued above has finished before TMEM is released
      tc_commit(smem_u32(&ctl.drain));
      mbar_wait_bounded(smem_u32(&ctl.drain), 0, &never, p.err, lim);
    }
  } else if (warp < 2 + epi_warps<SWIGLU, SCATTER, PUSH>()) {
    // ------------------------------------------------------------ epilogue
    // Each warp reads one 32-lane TMEM quadrant (= 32 rows); with two warps
    // per quadrant (SwiGLU) they take alternate 32-column chunks.  Each chunk
    // is packed into a 2 KiB staging box (two per warp for the plain tile,
    // one for the SwiGLU tile's eight warps) and one lane issues a TMA tensor
    // store of the 32x32 box, so global writes are whole lines and run
    // asynchronously.  A quadrant that crosses the end of its group (or of
    // A) stores its valid rows directly.
    constexpr int kStride = epi_warps<SWIGLU, SCATTER, PUSH>() / 4;
    const int quad = warp & 3;                 // TMEM lanes this warp may read
    const int first = (warp - 2) >> 2;         // first chunk of this warp
    const int r_in_tile = quad * 32 + lane;
    constexpr int kBoxes = SWIGLU ? 1 : 2;  // staging boxes per warp (16 KiB in all)
    const uint32_t stg = sbase + kStages * kStageBytes + (warp - 2) * kBoxes * kEpiChunkBytes;
    int acc = 0, buf = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      int g, row0, nrows, n;
      decode_tile(ctl, G, p.n_tiles, tile, g, row0, nrows, n);
      if (!mbar_wait_bounded(smem_u32(&ctl.acc_full[acc]), acc_phase, abort, p.err, lim)) break;
      tc_fence_after();
      const uint32_t trow = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                            static_cast<uint32_t>(acc * kAccCols);
      const int64_t grow = static_cast<int64_t>(row0) + r_in_tile;
      bool row_ok = r_in_tile < nrows && grow < p.M;
      const bool quad_full = (quad + 1) * 32 <= nrows &&
                             static_cast<int64_t>(row0) + (quad + 1) * 32 <= p.M;
      uint16_t* orow = p.out + grow * p.N;
      if (SCATTER && row_ok) {
        // the row goes back to the rank it came from, at the position that
        // rank's dispatch gave it (peer memory over NVLink)
        const uint32_t v = static_cast<uint32_t>(p.scatter_src[grow]);
        const int src = static_cast<int>(v >> kEpSrcShift);
        const int64_t pos = v & ((1u << kEpSrcShift) - 1u);
        if (src < p.scatter_world && pos < p.scatter_cap) {
          orow = reinterpret_cast<uint16_t*>(p.scatter_base[src]) + pos * p.N;
        } else {
          record_error(p.err, kDevEpOverflow);
          row_ok = false;
        }
      }
      if constexpr (SCATTER) {
        // Rows go to scattered destinations (often another GPU), so each
        // store instruction must write few, long pieces: 64 columns of the
        // warp's 32 rows are packed into a 4 KiB box (row r at r*128, its
        // 16-byte piece j at slot j ^ (r & 7), so both passes are free of
        // bank conflicts), then read back so that 8 lanes write one row's
        // 128 contiguous bytes: 4 rows per instruction.
        const uint32_t box = stg;  // 4 KiB of this warp's staging
        const unsigned long long my_row =
            row_ok ? reinterpret_cast<unsigned long long>(orow) : 0ull;
#pragma unroll 1
        for (int c2 = 0; c2 < kAccCols / 64; ++c2) {
          uint32_t pa[16], pb[16];
          {
            uint32_t ra[32], rb[32];
            tmem_ld_32cols(trow + c2 * 64, ra);
            tmem_ld_32cols(trow + c2 * 64 + 32, rb);
            tc_wait_ld();
            epi_pack<false>(ra, ra, pa);
            epi_pack<false>(rb, rb, pb);
          }
          const int col0 = n * p.out_cols_per_tile + c2 * 64;
          __syncwarp();  // the previous pass has read the box
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            st_shared_v4(box + lane * 128 + ((j ^ (lane & 7)) << 4),
                         make_uint4(pa[4 * j], pa[4 * j + 1], pa[4 * j + 2], pa[4 * j + 3]));
            st_shared_v4(box + lane * 128 + (((j + 4) ^ (lane & 7)) << 4),
                         make_uint4(pb[4 * j], pb[4 * j + 1], pb[4 * j + 2], pb[4 * j + 3]));
          }
          __syncwarp();
          const int j = lane & 7;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int r = i * 4 + (lane >> 3);
            const unsigned long long dst = __shfl_sync(0xffffffffu, my_row, r);
            const uint4 v = ld_shared_v4(box + r * 128 + ((j ^ (r & 7)) << 4));
            if (dst != 0ull && col0 + j * 8 + 8 <= p.N)
              *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(dst) + col0 + j * 8) = v;
          }
        }
      } else {
      constexpr int kChunks = SWIGLU ? BNH / 32 : kAccCols / 32;
#pragma unroll 1
      for (int c = first; c < kChunks; c += kStride) {
        uint32_t packed[16];
        {
          uint32_t ra[32];
          tmem_ld_32cols(trow + c * 32, ra);
          if (SWIGLU) {
            uint32_t ua[32];
            tmem_ld_32cols(trow + BNH + c * 32, ua);
            tc_wait_ld();
            epi_pack<true>(ra, ua, packed);
          } else {
            tc_wait_ld();
            epi_pack<false>(ra, ra, packed);
          }
        }
        const int col0 = n * p.out_cols_per_tile + c * 32;
        if (col0 >= p.N) continue;
        if (quad_full) {
          if (lane == 0) {  // the store that last used this box has read it
            if (kBoxes == 2) bulk_wait_group_read<1>();
            else bulk_wait_group_read<0>();
          }
          __syncwarp();
          // 64-byte swizzle (matches the store map): 16-byte piece c of row r
          // sits at r*64 + ((c ^ ((r >> 1) & 3)) * 16), so the 8 lanes of each
          // store phase hit 8 different bank groups
          const uint32_t dst = stg + buf * kEpiChunkBytes + lane * 64;
          const uint32_t sw = (lane >> 1) & 3;
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4)
            st_shared_v4(dst + ((c4 ^ sw) << 4), make_uint4(packed[4 * c4], packed[4 * c4 + 1],
                                                            packed[4 * c4 + 2], packed[4 * c4 + 3]));
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC, col0, row0 + quad * 32, stg + buf * kEpiChunkBytes);
            bulk_commit_group();
          }
          buf ^= kBoxes - 1;
        } else if (row_ok) {
          store_row_direct(packed, orow, col0, p.N);
        }
      }
      }  // !SCATTER
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&ctl.acc_empty[acc]));
      if (++acc == kNumAcc) { acc = 0; acc_phase ^= 1u; }
    }
    if (lane == 0) bulk_wait_group_all();  // stores complete before the CTA exits
    __syncwarp();
  } else if (PUSH) {
    // ------------------------------------------------------------- senders
    const int pw = blockIdx.x * kPushWarps + (warp - 2 - epi_warps<SWIGLU, SCATTER, PUSH>());
    push_rows(p, ctl, pw, gridDim.x * kPushWarps, lane);
  }

  // --------------------------------------------------------------- teardown
  if (SCATTER) __threadfence_system();  // this thread's peer stores, before the count
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  if (SCATTER && threadIdx.x == 0 && p.done) {
    const unsigned prev = atomicAdd(p.done, 1u);
    if (prev == gridDim.x - 1 && (!p.err || *reinterpret_cast<volatile int*>(p.err) == kDevOk)) {
      __threadfence_system();
      for (int r = 0; r < p.scatter_world; ++r) st_release_sys(p.flag[r], p.epoch);
    }
  }
}

// ------------------------------------------------------------ host side ----
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
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

// Row-major bf16 matrix [rows, cols] as a 2-D map with [box_rows, box_cols] boxes.
bool make_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows,
              uint32_t box_cols, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <bool SWIGLU, bool SCATTER, bool PUSH>
cudaError_t ensure_smem_attr() {
  // once per device: opt in to the large dynamic shared memory carve-out
  static int done[64] = {0};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (!done[dev]) {
    e = cudaFuncSetAttribute(grouped_gemm_sm100_kernel<SWIGLU, SCATTER, PUSH>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kSmemBytes));
    if (e != cudaSuccess) return e;
    done[dev] = 1;
  }
  return cudaSuccess;
}

}  // namespace

cudaError_t launch_grouped_gemm_sm100(const GroupedGemmArgs& a, cudaStream_t stream) {
  if (a.M == 0 || a.G == 0) return cudaSuccess;
  if (a.G > kMaxGroups || a.K % 8 != 0 || a.N % 8 != 0) return cudaErrorInvalidValue;
  const bool scatter = a.scatter_src != nullptr;
  if (scatter && (a.swiglu || a.scatter_world < 1 || a.scatter_world > 8))
    return cudaErrorInvalidValue;
  const int nw = a.swiglu ? 2 * a.N : a.N;          // rows of B per weight
  const int nweights = a.num_weights > 0 ? a.num_weights : a.G;
  CUtensorMap ma, mb, mc;
  if (!make_map(&ma, a.a, static_cast<uint64_t>(a.M), static_cast<uint64_t>(a.K), BM, BK,
                CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map(&mb, a.b, static_cast<uint64_t>(nweights) * nw, static_cast<uint64_t>(a.K), BNH, BK,
                CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  if (scatter) {
    mc = ma;  // the scatter epilogue stores rows directly; the store map is unused
  } else if (!make_map(&mc, a.out, static_cast<uint64_t>(a.M), static_cast<uint64_t>(a.N), 32, 32,
                       CU_TENSOR_MAP_SWIZZLE_64B)) {
    return cudaErrorInvalidValue;
  }
  KParams p;
  p.counts = a.counts;
  p.group_weight = a.group_weight;
  p.G = a.G;
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.out_cols_per_tile = a.swiglu ? BNH : kAccCols;
  p.n_tiles = cdiv(a.N, p.out_cols_per_tile);
  p.b_rows_per_group = nw;
  p.b_second_off = a.swiglu ? a.N : BNH;
  p.out = static_cast<uint16_t*>(a.out);
  p.err = a.err;
  p.wait_limit_ns = kWaitLimitNs;
  p.scatter_src = a.scatter_src;
  p.scatter_world = a.scatter_world;
  p.scatter_cap = a.scatter_cap;
  p.done = a.done;
  p.epoch = a.epoch;
  for (int i = 0; i < 8; ++i) {
    p.scatter_base[i] = a.scatter_base[i];
    p.flag[i] = a.flag[i];
  }
  const int sms = a.sm_limit > 0 ? a.sm_limit : num_sms_for_current_device();
  const int64_t max_tiles = (cdiv64(a.M, BM) + a.G) * p.n_tiles;
  const int grid = static_cast<int>(max_tiles < sms ? max_tiles : sms);
  // fused dispatch: keyed on the arrival counters (a rank with no tokens of
  // its own still waits for its peers' rows)
  const bool push = a.arrived != nullptr;
  if (push && (!a.swiglu || scatter || a.push_world < 1 || a.push_world > 8 || a.push_E > 128 ||
               a.push_E != a.push_world * a.push_El || (a.K * 2) % 16 != 0 ||
               (a.push_A > 0 && (!a.push_x || !a.push_sorted_token || !a.push_counts ||
                                 !a.push_send_base))))
    return cudaErrorInvalidValue;
  p.push_x = static_cast<const uint4*>(a.push_x);
  p.push_sorted_token = a.push_sorted_token;
  p.push_counts = a.push_counts;
  p.push_send_base = a.push_send_base;
  for (int i = 0; i < 8; ++i) {
    p.push_rows[i] = reinterpret_cast<uint4*>(a.push_rows[i]);
    p.push_src[i] = a.push_src[i];
    p.push_arrived[i] = a.push_arrived[i];
  }
  p.arrived = a.arrived;
  p.push_A = a.push_A;
  p.push_cap = a.push_cap;
  p.push_E = a.push_E;
  p.push_El = a.push_El;
  p.push_world = a.push_world;
  p.push_me = a.push_me;
  p.push_row_chunks = a.K * 2 / 16;
  cudaError_t e;
  if (a.swiglu && push) {
    // the producers wait for rows that other CTAs' senders store: every CTA
    // must be resident at once, which a cooperative launch guarantees
    if ((e = ensure_smem_attr<true, false, true>()) != cudaSuccess) return e;
    void* args[] = {&ma, &mb, &mc, &p};
    e = cudaLaunchCooperativeKernel(
        reinterpret_cast<const void*>(&grouped_gemm_sm100_kernel<true, false, true>), dim3(grid),
        dim3(num_threads<true, false, true>()), args, kSmemBytes, stream);
  } else if (a.swiglu) {
    if ((e = ensure_smem_attr<true, false, false>()) != cudaSuccess) return e;
    e = launch_pdl(kPdlGemm, grouped_gemm_sm100_kernel<true, false, false>, dim3(grid),
                   dim3(num_threads<true, false, false>()), kSmemBytes, stream, ma, mb, mc, p);
  } else if (scatter) {
    if ((e = ensure_smem_attr<false, true, false>()) != cudaSuccess) return e;
    e = launch_pdl(kPdlGemm, grouped_gemm_sm100_kernel<false, true, false>, dim3(grid),
                   dim3(num_threads<false, true, false>()), kSmemBytes, stream, ma, mb, mc, p);
  } else {
    if ((e = ensure_smem_attr<false, false, false>()) != cudaSuccess) return e;
    e = launch_pdl(kPdlGemm, grouped_gemm_sm100_kernel<false, false, false>, dim3(grid),
                   dim3(num_threads<false, false, false>()), kSmemBytes, stream, ma, mb, mc, p);
  }
  return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace hmoe
