// fp32 grouped expert GEMMs on the CUDA cores.
//
// The fp32 layer (the reference's CPU configuration, checked to 1e-4) needs
// full fp32 products, which the bf16/tf32 tensor-core paths cannot give, so
// this kernel runs FFMA.  Semantics are those of the tcgen05 kernel:
//   plain:   out[r] = A[r] @ B[g]^T
//   swiglu:  out[r] = silu(A[r] @ Bg^T) * (A[r] @ Bu^T)   (layers.py:326-329)
// Tile 64 rows x 64 columns, 256 threads, 4x4 outputs per thread, K staged
// 16 at a time; every output accumulates one fma per k in ascending order.
// The grid covers an upper bound of the tile count; CTAs past the real
// count (known only on the device) exit at once.
#include "common.cuh"
#include "internal.h"

namespace hmoe {
namespace {

constexpr int SM_ = 64;    // rows per tile
constexpr int SN = 64;     // columns per tile
constexpr int SK = 16;
constexpr int kSThreads = 256;
constexpr int kSMaxGroups = 1024;

template <bool SWIGLU>
__global__ void __launch_bounds__(kSThreads)
grouped_gemm_simt_kernel(const float* __restrict__ A, const float* __restrict__ B,
                         const int32_t* __restrict__ counts, const int32_t* __restrict__ gweight,
                         int G, int64_t M, int N, int K, int n_tiles, float* __restrict__ out) {
  __shared__ int group_rows[kSMaxGroups + 1];
  __shared__ int tile_prefix[kSMaxGroups + 1];
  __shared__ __align__(16) float As[SK][SM_];
  __shared__ __align__(16) float Bs[SK][SN];
  __shared__ __align__(16) float Us[SWIGLU ? SK : 1][SWIGLU ? SN : 4];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  if (warp == 0) {
    const int per = cdiv(G, 32);
    const int g0 = min(G, lane * per), g1 = min(G, g0 + per);
    int rows = 0, tiles = 0;
    for (int g = g0; g < g1; ++g) {
      const int c = max(0, counts[g]);
      rows += c;
      tiles += cdiv(c, SM_);
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
      const int c = max(0, counts[g]);
      group_rows[g] = rr;
      tile_prefix[g] = tr;
      rr += c;
      tr += cdiv(c, SM_);
    }
    if (lane == 31) { group_rows[G] = rin; tile_prefix[G] = tin; }
  }
  __syncthreads();
  const int tile = blockIdx.x;
  if (tile >= tile_prefix[G] * n_tiles) return;
  const int mt = tile / n_tiles, n = tile % n_tiles;
  int lo = 0, hi = G;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (tile_prefix[mid] <= mt) lo = mid; else hi = mid;
  }
  const int g = lo;
  const int row0 = group_rows[g] + (mt - tile_prefix[g]) * SM_;
  const int nrows = min(SM_, group_rows[g + 1] - row0);
  const int col0 = n * SN;
  const int nw = SWIGLU ? 2 * N : N;
  const float* Bg = B + static_cast<int64_t>(gweight ? gweight[g] : g) * nw * K;

  const int ty = tid >> 4, tx = tid & 15;
  float acc[4][4], accu[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) { acc[i][j] = 0.f; accu[i][j] = 0.f; }

  // staging: thread -> (row/col = tid / 4, k quad = tid % 4)
  const int sr = tid >> 2, sq = tid & 3;
  for (int k0 = 0; k0 < K; k0 += SK) {
    const int kc = min(SK, K - k0);
    {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      const int64_t r = static_cast<int64_t>(row0) + sr;
      if (sr < nrows && r < M && k0 + sq * 4 < K)
        v = *reinterpret_cast<const float4*>(A + r * K + k0 + sq * 4);
      As[sq * 4 + 0][sr] = v.x; As[sq * 4 + 1][sr] = v.y;
      As[sq * 4 + 2][sr] = v.z; As[sq * 4 + 3][sr] = v.w;
    }
    {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      const int c = col0 + sr;
      if (c < N && k0 + sq * 4 < K) v = *reinterpret_cast<const float4*>(Bg + static_cast<int64_t>(c) * K + k0 + sq * 4);
      Bs[sq * 4 + 0][sr] = v.x; Bs[sq * 4 + 1][sr] = v.y;
      Bs[sq * 4 + 2][sr] = v.z; Bs[sq * 4 + 3][sr] = v.w;
      if (SWIGLU) {
        float4 u = make_float4(0.f, 0.f, 0.f, 0.f);
        if (c < N && k0 + sq * 4 < K)
          u = *reinterpret_cast<const float4*>(Bg + static_cast<int64_t>(N + c) * K + k0 + sq * 4);
        Us[sq * 4 + 0][sr] = u.x; Us[sq * 4 + 1][sr] = u.y;
        Us[sq * 4 + 2][sr] = u.z; Us[sq * 4 + 3][sr] = u.w;
      }
    }
    __syncthreads();
    for (int kk = 0; kk < kc; ++kk) {
      const float4 a = *reinterpret_cast<const float4*>(&As[kk][ty * 4]);
      const float4 b = *reinterpret_cast<const float4*>(&Bs[kk][tx * 4]);
      const float ar[4] = {a.x, a.y, a.z, a.w}, br[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(ar[i], br[j], acc[i][j]);
      if (SWIGLU) {
        const float4 u = *reinterpret_cast<const float4*>(&Us[kk][tx * 4]);
        const float ur[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) accu[i][j] = fmaf(ar[i], ur[j], accu[i][j]);
      }
    }
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int rl = ty * 4 + i;
    const int64_t r = static_cast<int64_t>(row0) + rl;
    if (rl >= nrows || r >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = col0 + tx * 4 + j;
      if (c >= N) continue;
      float v = acc[i][j];
      if (SWIGLU) v = (v / (1.0f + expf(-v))) * accu[i][j];
      out[r * N + c] = v;
    }
  }
}

}  // namespace

cudaError_t launch_grouped_gemm_simt(const GroupedGemmArgs& a, cudaStream_t stream) {
  if (a.M == 0 || a.G == 0) return cudaSuccess;
  if (a.G > kSMaxGroups || a.K % 4 != 0) return cudaErrorInvalidValue;
  const int n_tiles = cdiv(a.N, SN);
  const int64_t grid = (cdiv64(a.M, SM_) + a.G) * n_tiles;
  if (grid > 0x7fffffff) return cudaErrorInvalidValue;
  const float* A = static_cast<const float*>(a.a);
  const float* B = static_cast<const float*>(a.b);
  float* out = static_cast<float*>(a.out);
  if (a.swiglu)
    grouped_gemm_simt_kernel<true><<<static_cast<unsigned>(grid), kSThreads, 0, stream>>>(
        A, B, a.counts, a.group_weight, a.G, a.M, a.N, a.K, n_tiles, out);
  else
    grouped_gemm_simt_kernel<false><<<static_cast<unsigned>(grid), kSThreads, 0, stream>>>(
        A, B, a.counts, a.group_weight, a.G, a.M, a.N, a.K, n_tiles, out);
  return cudaGetLastError();
}

}  // namespace hmoe
