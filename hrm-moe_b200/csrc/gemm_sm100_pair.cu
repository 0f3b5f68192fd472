// Grouped GEMM on CTA pairs (tcgen05.mma.cta_group::2), same results as
// grouped_gemm_sm100_kernel: the forward of models/moe_triton_grouped_gemm.py
// (_m_grouped_gemm_bk_kernel, :113-184), plain or with the SiLU(gate) * up
// epilogue of models/layers.py:326-329, for the local (non expert-parallel)
// bf16 GEMMs.
//
// Two CTAs of a cluster share one 256-row x 256-column tile.  Each stages
// only its own 128 rows of A and its own 128 rows of B (one of the two B
// boxes: gate or up, or columns 0-127 / 128-255), so a stage is 32 KiB and
// six stages fit where the single-CTA kernel holds four: half the B bytes per
// SM and half again as many k-blocks in flight.  The even CTA (the leader)
// issues the MMAs for both; each CTA's TMEM accumulates its own 128 rows x
// 256 columns, and each CTA runs the single-CTA kernel's epilogue on them.
//
// Barriers: both CTAs' TMA loads complete on the leader's stage barrier (the
// leader alone arms it with the stage's 64 KiB); the leader's commits arrive
// on the stage-empty and accumulator-full barriers of both CTAs; both CTAs'
// epilogue warps arrive on the leader's accumulator-empty barrier.  Every
// wait is bounded (kWaitLimitNs).  The TMEM allocation and the two cluster
// barriers, which have no time limit of their own, are reached
// unconditionally by every thread of both CTAs, and neither CTA leaves
// before the other is done with its shared memory and TMEM.  No multicast
// load is used (the TMA loads carry .cta_group::2 only).
#include <cuda.h>
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace hmoe {
namespace {

constexpr int PM = 128;                       // rows per CTA (256 per pair)
constexpr int PBK = 64;                       // bf16 per swizzled 128-byte row
constexpr int PBN = 128;                      // B rows per CTA (256 per pair)
constexpr int kPStages = 6;
constexpr int kPABytes = PM * PBK * 2;        // 16 KiB
constexpr int kPBBytes = PBN * PBK * 2;       // 16 KiB
constexpr int kPStageBytes = kPABytes + kPBBytes;
constexpr int kPAccCols = 256;
constexpr int kPNumAcc = 2;
constexpr int kPTmemCols = kPAccCols * kPNumAcc;
constexpr int kPMaxGroups = 1024;
constexpr int kPEpiChunkBytes = 32 * 32 * 2;
constexpr int kPEpiBytes = 4 * 2 * kPEpiChunkBytes;  // 16 KiB of staging boxes

template <bool SWIGLU>
__host__ __device__ constexpr int pair_epi_warps() { return SWIGLU ? 8 : 4; }
template <bool SWIGLU>
__host__ __device__ constexpr int pair_threads() { return 64 + 32 * pair_epi_warps<SWIGLU>(); }

struct PairCtl {
  uint64_t full[kPStages];      // leader: both CTAs' loads of a stage landed
  uint64_t empty[kPStages];     // each CTA: the pair's MMAs are done with a stage
  uint64_t acc_full[kPNumAcc];  // each CTA: its accumulator is complete
  uint64_t acc_empty[kPNumAcc]; // leader: both CTAs' epilogues drained it
  uint64_t drain;               // leader: every MMA issued has completed
  uint32_t tmem_base;
  int abort;
  int num_m_tiles;
  int pad_;
  int group_rows[kPMaxGroups + 1];
  int tile_prefix[kPMaxGroups + 1];  // prefix of 256-row blocks
  int group_w[kPMaxGroups];
};

constexpr size_t kPSmemBytes =
    1024 + static_cast<size_t>(kPStages) * kPStageBytes + kPEpiBytes + sizeof(PairCtl);
static_assert(kPSmemBytes <= 232448, "shared memory budget of one sm_100 CTA");

struct PParams {
  const int32_t* counts;
  const int32_t* group_weight;
  int G;
  int64_t M;
  int N;
  int K;
  int n_tiles;
  int out_cols_per_tile;
  int b_rows_per_group;
  int b_second_off;
  uint16_t* out;
  uint16_t* save_gu;  // SAVE: the rounded gate and up values, [M, 2N] (training forward)
  int* err;
  unsigned long long wait_limit_ns;
};

__device__ __forceinline__ void st_shared_v4p(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

// Tile (group, 256-row block, column block) of the pair's schedule.
__device__ __forceinline__ void decode_pair_tile(const PairCtl& ctl, int G, int n_tiles, int tile,
                                                 int& g, int& row0, int& grow_end, int& n) {
  const int mt = tile / n_tiles;
  n = tile - mt * n_tiles;
  int lo = 0, hi = G;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (ctl.tile_prefix[mid] <= mt) lo = mid; else hi = mid;
  }
  g = lo;
  row0 = ctl.group_rows[g] + (mt - ctl.tile_prefix[g]) * (2 * PM);
  grow_end = ctl.group_rows[g + 1];
}

// 32 accumulator columns of one row -> 16 packed bf16x2 words.  SwiGLU
// rounds where the reference does (models/layers.py:326-329: gate_up is a
// bf16 tensor, F.silu returns bf16, the product is rounded again) with packed
// instructions: one paired conversion rounds two gate (or up) values, SiLU
// runs in fp32 on the rounded gate and is rounded by another paired
// conversion, and mul.rn.bf16x2 rounds the product once (the product of two
// bf16 values is exact in fp32).  Same code as grouped_gemm_sm100_kernel's
// epilogue.
template <bool SWIGLU>
__device__ __forceinline__ void pair_pack(const uint32_t (&a)[32], const uint32_t (&b)[32],
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

// SAVE (SwiGLU only): the epilogue also stores the bf16 gate and up values
// it rounded, [rows, 2N] with gate at columns [0, N) and up at [N, 2N) -- the
// gate_up tensor the reference materialises (layers.py:326-328), which the
// backward of SiLU(gate) * up needs.
template <bool SWIGLU, bool SAVE = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(pair_threads<SWIGLU>(), 1)
grouped_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                         const __grid_constant__ CUtensorMap tmB,
                         const __grid_constant__ CUtensorMap tmC, const PParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  PairCtl& ctl = *reinterpret_cast<PairCtl*>(smem + kPStages * kPStageBytes + kPEpiBytes);
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = p.G;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  constexpr int EPI = pair_epi_warps<SWIGLU>();

  // ---------------------------------------------------------------- setup
  if (warp == 0) {
    grid_dependency_wait();  // launched early (launch_pdl): the counts are written before this
    const int per = cdiv(G, 32);
    const int g0 = min(G, lane * per), g1 = min(G, g0 + per);
    int rows = 0, tiles = 0;
    for (int g = g0; g < g1; ++g) {
      const int c = max(0, p.counts[g]);
      rows += c;
      tiles += cdiv(c, 2 * PM);
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
      tr += cdiv(c, 2 * PM);
    }
    if (lane == 31) {
      ctl.group_rows[G] = rin;
      ctl.tile_prefix[G] = tin;
      ctl.num_m_tiles = tin;
    }
    if (lane == 0) {
      for (int s = 0; s < kPStages; ++s) {
        mbar_init(smem_u32(&ctl.full[s]), 1);   // the leader's arm
        mbar_init(smem_u32(&ctl.empty[s]), 1);  // one commit per stage use
      }
      for (int a = 0; a < kPNumAcc; ++a) {
        mbar_init(smem_u32(&ctl.acc_full[a]), 1);
        mbar_init(smem_u32(&ctl.acc_empty[a]), 2 * EPI);  // both CTAs' epilogue warps
      }
      mbar_init(smem_u32(&ctl.drain), 1);
      ctl.abort = 0;
      fence_mbar_init();
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      tma_prefetch_desc(&tmC);
    }
  } else if (warp == 1) {
    tmem_alloc_pair(smem_u32(&ctl.tmem_base), kPTmemCols);  // both CTAs, same warp
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // barrier inits visible to the peer CTA before any remote signal
  tc_fence_after();
  grid_dependency_wait();
  grid_launch_dependents();

  const uint32_t tmem_base = ctl.tmem_base;
  const int num_tiles = ctl.num_m_tiles * p.n_tiles;
  const int nkb = cdiv(p.K, PBK);
  volatile int* abort = &ctl.abort;
  int never = 0;
  const unsigned long long lim = p.wait_limit_ns;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < num_tiles; tile += npairs) {
        int g, row0, grow_end, n;
        decode_pair_tile(ctl, G, p.n_tiles, tile, g, row0, grow_end, n);
        const int my_row0 = row0 + static_cast<int>(rank) * PM;
        const int rb = ctl.group_w[g] * p.b_rows_per_group + n * p.out_cols_per_tile +
                       (rank ? p.b_second_off : 0);
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait_bounded(smem_u32(&ctl.empty[stage]), phase ^ 1u, abort, p.err, lim)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(&ctl.full[stage]);
          const uint32_t fb_leader = map_to_rank(fb, 0);
          const uint32_t sa = sbase + stage * kPStageBytes;
          if (leader) mbar_arrive_expect_tx(fb, 2 * kPStageBytes);  // both CTAs' bytes
          tma_load_2d_pair(sa, &tmA, kb * PBK, my_row0, fb_leader);
          tma_load_2d_pair(sa + kPABytes, &tmB, kb * PBK, rb, fb_leader);
          if (++stage == kPStages) { stage = 0; phase ^= 1u; }
        }
      }
      // Tail: continue the stage sequence until every stage this CTA filled
      // has been released by the pair's MMAs, so no copy is still landing in
      // this CTA's shared memory and no commit is still on its way to its
      // barriers when the CTA leaves.  After one wait gave up the MMAs are
      // not progressing, and the rest is skipped.
      for (int i = 0; i < kPStages; ++i) {
        if (!mbar_wait_bounded(smem_u32(&ctl.empty[stage]), phase ^ 1u, &never, p.err, lim)) break;
        if (++stage == kPStages) { stage = 0; phase ^= 1u; }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (leader && lane == 0) {
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      constexpr uint32_t idesc = idesc_bf16_f32(2 * PM, kPAccCols);
      bool ok = true;
      for (int tile = pair; ok && tile < num_tiles; tile += npairs) {
        if (!mbar_wait_bounded(smem_u32(&ctl.acc_empty[acc]), acc_phase ^ 1u, abort, p.err, lim))
          break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kPAccCols);
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait_bounded(smem_u32(&ctl.full[stage]), phase, abort, p.err, lim)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = sbase + stage * kPStageBytes;
#pragma unroll
          for (int kk = 0; kk < PBK / 16; ++kk) {
            const uint64_t ad = smem_desc_sw128(sa + kk * 32);
            const uint64_t bd = smem_desc_sw128(sa + kPABytes + kk * 32);
            tc_mma_bf16_pair(d_tmem, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          tc_commit_pair_both(smem_u32(&ctl.empty[stage]));
          if (++stage == kPStages) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        tc_commit_pair_both(smem_u32(&ctl.acc_full[acc]));
        if (++acc == kPNumAcc) { acc = 0; acc_phase ^= 1u; }
      }
      // every MMA issued has completed before the pair tears down, and both
      // CTAs' epilogues have released every accumulator (their arrivals on
      // this CTA's barriers are done)
      tc_commit_pair(smem_u32(&ctl.drain));
      mbar_wait_bounded(smem_u32(&ctl.drain), 0, &never, p.err, lim);
      for (int i = 0; i < kPNumAcc; ++i) {
        if (!mbar_wait_bounded(smem_u32(&ctl.acc_empty[acc]), acc_phase ^ 1u, &never, p.err, lim))
          break;
        if (++acc == kPNumAcc) { acc = 0; acc_phase ^= 1u; }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    constexpr int kStride = EPI / 4;
    constexpr int kBoxes = SWIGLU ? 1 : 2;
    const int quad = warp & 3;
    const int first = (warp - 2) >> 2;
    const int r_in_tile = quad * 32 + lane;
    const uint32_t stg = sbase + kPStages * kPStageBytes + (warp - 2) * kBoxes * kPEpiChunkBytes;
    int acc = 0, buf = 0;
    uint32_t acc_phase = 0;
    for (int tile = pair; tile < num_tiles; tile += npairs) {
      int g, row0, grow_end, n;
      decode_pair_tile(ctl, G, p.n_tiles, tile, g, row0, grow_end, n);
      const int my_row0 = row0 + static_cast<int>(rank) * PM;
      const int nrows = min(PM, grow_end - my_row0);  // may be <= 0: nothing to store
      if (!mbar_wait_bounded(smem_u32(&ctl.acc_full[acc]), acc_phase, abort, p.err, lim)) break;
      tc_fence_after();
      const uint32_t trow = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                            static_cast<uint32_t>(acc * kPAccCols);
      const int64_t grow = static_cast<int64_t>(my_row0) + r_in_tile;
      const bool row_ok = r_in_tile < nrows && grow < p.M;
      const bool quad_full = (quad + 1) * 32 <= nrows &&
                             static_cast<int64_t>(my_row0) + (quad + 1) * 32 <= p.M;
      uint16_t* orow = p.out + grow * p.N;
      constexpr int kChunks = SWIGLU ? PBN / 32 : kPAccCols / 32;
#pragma unroll 1
      for (int c = first; c < kChunks; c += kStride) {
        uint32_t packed[16];
        {
          uint32_t ra[32];
          tmem_ld_32cols(trow + c * 32, ra);
          if (SWIGLU) {
            uint32_t ua[32];
            tmem_ld_32cols(trow + PBN + c * 32, ua);
            tc_wait_ld();
            pair_pack<true>(ra, ua, packed);
            if (SAVE && row_ok) {
              const int gcol = n * p.out_cols_per_tile + c * 32;
              uint16_t* srow = p.save_gu + grow * 2 * p.N;
#pragma unroll
              for (int c4 = 0; c4 < 4; ++c4) {
                if (gcol + c4 * 8 + 8 > p.N) continue;
                uint4 gv, uv;
                gv.x = cvt_bf16x2(__uint_as_float(ra[8 * c4 + 0]), __uint_as_float(ra[8 * c4 + 1]));
                gv.y = cvt_bf16x2(__uint_as_float(ra[8 * c4 + 2]), __uint_as_float(ra[8 * c4 + 3]));
                gv.z = cvt_bf16x2(__uint_as_float(ra[8 * c4 + 4]), __uint_as_float(ra[8 * c4 + 5]));
                gv.w = cvt_bf16x2(__uint_as_float(ra[8 * c4 + 6]), __uint_as_float(ra[8 * c4 + 7]));
                uv.x = cvt_bf16x2(__uint_as_float(ua[8 * c4 + 0]), __uint_as_float(ua[8 * c4 + 1]));
                uv.y = cvt_bf16x2(__uint_as_float(ua[8 * c4 + 2]), __uint_as_float(ua[8 * c4 + 3]));
                uv.z = cvt_bf16x2(__uint_as_float(ua[8 * c4 + 4]), __uint_as_float(ua[8 * c4 + 5]));
                uv.w = cvt_bf16x2(__uint_as_float(ua[8 * c4 + 6]), __uint_as_float(ua[8 * c4 + 7]));
                *reinterpret_cast<uint4*>(srow + gcol + c4 * 8) = gv;
                *reinterpret_cast<uint4*>(srow + p.N + gcol + c4 * 8) = uv;
              }
            }
          } else {
            tc_wait_ld();
            pair_pack<false>(ra, ra, packed);
          }
        }
        const int col0 = n * p.out_cols_per_tile + c * 32;
        if (col0 >= p.N) continue;
        if (quad_full) {
          if (lane == 0) {
            if (kBoxes == 2) bulk_wait_group_read<1>();
            else bulk_wait_group_read<0>();
          }
          __syncwarp();
          const uint32_t dst = stg + buf * kPEpiChunkBytes + lane * 64;
          const uint32_t sw = (lane >> 1) & 3;
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4)
            st_shared_v4p(dst + ((c4 ^ sw) << 4), make_uint4(packed[4 * c4], packed[4 * c4 + 1],
                                                             packed[4 * c4 + 2], packed[4 * c4 + 3]));
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC, col0, my_row0 + quad * 32, stg + buf * kPEpiChunkBytes);
            bulk_commit_group();
          }
          buf ^= kBoxes - 1;
        } else if (row_ok) {
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4)
            if (col0 + c4 * 8 + 8 <= p.N)
              *reinterpret_cast<uint4*>(orow + col0 + c4 * 8) =
                  make_uint4(packed[4 * c4], packed[4 * c4 + 1], packed[4 * c4 + 2],
                             packed[4 * c4 + 3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(map_to_rank(smem_u32(&ctl.acc_empty[acc]), 0));
      if (++acc == kPNumAcc) { acc = 0; acc_phase ^= 1u; }
    }
    if (lane == 0) bulk_wait_group_all();
    __syncwarp();
  }

  // --------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // neither CTA leaves while the pair's MMAs or the peer use it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kPTmemCols);
  }
}

// ------------------------------------------------------------ host side ----
typedef CUresult (*EncodeTiledFnP)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFnP encode_fn_p() {
  static EncodeTiledFnP fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFnP>(ptr);
  });
  return fn;
}

bool make_map_p(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows,
                uint32_t box_cols, CUtensorMapSwizzle swizzle) {
  EncodeTiledFnP enc = encode_fn_p();
  if (!enc) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool SWIGLU, bool SAVE = false>
cudaError_t ensure_pair_attr() {
  static int done[64] = {0};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (!done[dev]) {
    e = cudaFuncSetAttribute(grouped_gemm_pair_kernel<SWIGLU, SAVE>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kPSmemBytes));
    if (e != cudaSuccess) return e;
    done[dev] = 1;
  }
  return cudaSuccess;
}

}  // namespace

cudaError_t launch_grouped_gemm_pair(const GroupedGemmArgs& a, cudaStream_t stream) {
  if (a.M == 0 || a.G == 0) return cudaSuccess;
  if (a.G > kPMaxGroups || a.K % 8 != 0 || a.N % 8 != 0 || a.scatter_src || a.arrived)
    return cudaErrorInvalidValue;
  const int nw = a.swiglu ? 2 * a.N : a.N;
  const int nweights = a.num_weights > 0 ? a.num_weights : a.G;
  CUtensorMap ma, mb, mc;
  if (!make_map_p(&ma, a.a, static_cast<uint64_t>(a.M), static_cast<uint64_t>(a.K), PM, PBK,
                  CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map_p(&mb, a.b, static_cast<uint64_t>(nweights) * nw, static_cast<uint64_t>(a.K), PBN,
                  PBK, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map_p(&mc, a.out, static_cast<uint64_t>(a.M), static_cast<uint64_t>(a.N), 32, 32,
                  CU_TENSOR_MAP_SWIZZLE_64B))
    return cudaErrorInvalidValue;
  PParams p;
  p.counts = a.counts;
  p.group_weight = a.group_weight;
  p.G = a.G;
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.out_cols_per_tile = a.swiglu ? PBN : kPAccCols;
  p.n_tiles = cdiv(a.N, p.out_cols_per_tile);
  p.b_rows_per_group = nw;
  p.b_second_off = a.swiglu ? a.N : PBN;
  p.out = static_cast<uint16_t*>(a.out);
  p.save_gu = static_cast<uint16_t*>(a.save_gate_up);
  p.err = a.err;
  p.wait_limit_ns = kWaitLimitNs;
  const int sms = a.sm_limit > 0 ? a.sm_limit : num_sms_for_current_device();
  const int64_t max_tiles = (cdiv64(a.M, 2 * PM) + a.G) * p.n_tiles;
  int pairs = static_cast<int>(max_tiles < sms / 2 ? max_tiles : sms / 2);
  if (pairs < 1) pairs = 1;
  cudaError_t e;
  if (a.swiglu && a.save_gate_up) {
    if ((e = ensure_pair_attr<true, true>()) != cudaSuccess) return e;
    e = launch_pdl(kPdlGemm, grouped_gemm_pair_kernel<true, true>, dim3(2 * pairs),
                   dim3(pair_threads<true>()), kPSmemBytes, stream, ma, mb, mc, p);
  } else if (a.swiglu) {
    if ((e = ensure_pair_attr<true>()) != cudaSuccess) return e;
    e = launch_pdl(kPdlGemm, grouped_gemm_pair_kernel<true>, dim3(2 * pairs),
                   dim3(pair_threads<true>()), kPSmemBytes, stream, ma, mb, mc, p);
  } else {
    if ((e = ensure_pair_attr<false>()) != cudaSuccess) return e;
    e = launch_pdl(kPdlGemm, grouped_gemm_pair_kernel<false>, dim3(2 * pairs),
                   dim3(pair_threads<false>()), kPSmemBytes, stream, ma, mb, mc, p);
  }
  return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace hmoe
