// seqpar_scan.cu — the start-state step of the sequence-parallel prefill:
// S_out = M S_in + L for a batch of d x d fp32 matrices (one per sequence and
// value head), where (M, L) is the affine map of one time segment of the
// delta-rule recurrence (S_end = M S_start + L).  fp32 throughout: the scan
// composes up to N - 1 such maps, so the start states keep full precision.
//
// One CTA per 64 x 64 output tile of one matrix, 256 threads, each computing a
// 4 x 4 block; M and S_in stream through shared memory in 32-wide K slices.
#include <cuda_runtime.h>

#include "common.cuh"

namespace {

constexpr int kTile = 64, kKs = 32;

__global__ void __launch_bounds__(256) affine_kernel(const float* __restrict__ M,
                                                     const float* __restrict__ L,
                                                     const float* __restrict__ Sin,
                                                     float* __restrict__ Sout, int d) {
  __shared__ float sm[kKs][kTile + 4];   // M[row0 + r][k0 + kk], stored [kk][r]
  __shared__ float ss[kKs][kTile + 4];   // Sin[k0 + kk][col0 + c]
  const int tiles = d / kTile;
  const int mat = blockIdx.x / (tiles * tiles);
  const int t = blockIdx.x % (tiles * tiles);
  const int row0 = (t / tiles) * kTile, col0 = (t % tiles) * kTile;
  const size_t base = static_cast<size_t>(mat) * d * d;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;  // 16 x 16 threads, 4 x 4 each
  float acc[4][4] = {};
  for (int k0 = 0; k0 < d; k0 += kKs) {
    for (int i = threadIdx.x; i < kTile * kKs; i += 256) {
      const int r = i / kKs, kk = i % kKs;  // M: rows r, K contiguous
      sm[kk][r] = M[base + static_cast<size_t>(row0 + r) * d + k0 + kk];
      const int kr = i / kTile, c = i % kTile;  // S_in: K rows, columns contiguous
      ss[kr][c] = Sin[base + static_cast<size_t>(k0 + kr) * d + col0 + c];
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < kKs; ++kk) {
      const float4 a = *reinterpret_cast<const float4*>(&sm[kk][ty * 4]);
      const float4 b = *reinterpret_cast<const float4*>(&ss[kk][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const size_t off = base + static_cast<size_t>(row0 + ty * 4 + i) * d + col0 + tx * 4;
    const float4 l = *reinterpret_cast<const float4*>(L + off);
    *reinterpret_cast<float4*>(Sout + off) =
        make_float4(acc[i][0] + l.x, acc[i][1] + l.y, acc[i][2] + l.z, acc[i][3] + l.w);
  }
}

}  // namespace

extern "C" int gdn_state_affine(const float* M, const float* L, const float* S_in, float* S_out,
                                int32_t count, int32_t d, gdn_stream_t stream) {
  if (!M || !L || !S_in || !S_out) return GDN_ERR_NULL;
  if (count < 1 || d < kTile || d % kTile) return GDN_ERR_SHAPE;
  if (S_out == S_in) return GDN_ERR_SHAPE;  // S_in is read while S_out is written
  if (!gdn::aligned16(M) || !gdn::aligned16(L) || !gdn::aligned16(S_in) || !gdn::aligned16(S_out))
    return GDN_ERR_ALIGN;
  const int64_t grid = static_cast<int64_t>(count) * (d / kTile) * (d / kTile);
  if (grid > 0x7FFFFFFF) return GDN_ERR_SHAPE;
  affine_kernel<<<static_cast<unsigned>(grid), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      M, L, S_in, S_out, d);
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}
