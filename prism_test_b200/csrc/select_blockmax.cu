// Block-maximum top-1 / top-4 of a score matrix: the selection semantics of the
// reference's Triton kernels (eval_harness/kernels/einsum_topk.py:97-161, with the
// 4-wide merge of eval_harness/kernels/bitonic_merge_wrapper.py:5-52), for callers
// that need the reference kernel's selections (mode PRISM_MODE_BLOCKMAX).
//
// Per row, keys are cut into blocks of 128. Each block contributes its maximum
// score at the first column that reaches it. The blocks are then visited in
// order:
//   top-1: the running best is replaced when a block maximum is >= it (start
//          -inf), so the last of equal maxima wins;
//   top-4: four slots start at the lowest finite fp32 value with index 0; a block
//          maximum strictly above slot 3 replaces it, then compare-exchanges
//          (0,2), (1,3), (0,1), (2,3) swap a pair when the left value is smaller.
// The top-4 network is order dependent (equal values can overtake each other),
// so it is run sequentially over the blocks of a row, one row per lane.
//
// Layout: a CTA takes 32 rows. For each chunk of 64 blocks, all threads compute
// block maxima (one thread per (row, block), a 512-byte contiguous read) into
// shared memory, then warp 0 (lane = row) advances the selection over the chunk.
// A NaN score never becomes a block maximum here (torch would propagate it).
#include <cfloat>

#include "common.cuh"
#include "kernels.h"

namespace prism {
namespace {

constexpr int kBlock = 128;
constexpr int kRowsPerCta = 32;
constexpr int kThreads = 256;
constexpr int kChunk = 64;

template <int K>
__global__ void __launch_bounds__(kThreads) select_blockmax_kernel(const SelectArgs a) {
  __shared__ float bmax[kRowsPerCta][kChunk + 1];
  __shared__ int32_t barg[kRowsPerCta][kChunk + 1];
  const int tid = threadIdx.x;
  const int64_t row0 = int64_t(blockIdx.x) * kRowsPerCta;
  const int nrows = int(a.rows - row0 < kRowsPerCta ? a.rows - row0 : kRowsPerCta);
  const int nb = int(a.n / kBlock);

  float v[4];
  int32_t ix[4];
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    v[s] = K == 1 ? -INFINITY : -FLT_MAX;
    ix[s] = 0;
  }

  for (int c0 = 0; c0 < nb; c0 += kChunk) {
    const int cn = min(kChunk, nb - c0);
    for (int task = tid; task < nrows * cn; task += kThreads) {
      const int r = task / cn, t = task - r * cn;
      const float4* p =
          reinterpret_cast<const float4*>(a.scores + (row0 + r) * a.ld + int64_t(c0 + t) * kBlock);
      float m = p[0].x;
      int mi = 0;
#pragma unroll 4
      for (int e4 = 0; e4 < kBlock / 4; ++e4) {
        const float4 x = p[e4];
        if (x.x > m) { m = x.x; mi = 4 * e4; }
        if (x.y > m) { m = x.y; mi = 4 * e4 + 1; }
        if (x.z > m) { m = x.z; mi = 4 * e4 + 2; }
        if (x.w > m) { m = x.w; mi = 4 * e4 + 3; }
      }
      bmax[r][t] = m;
      barg[r][t] = (c0 + t) * kBlock + mi;
    }
    __syncthreads();
    if (tid < nrows) {
      for (int t = 0; t < cn; ++t) {
        const float x = bmax[tid][t];
        const int32_t xi = barg[tid][t];
        if (K == 1) {
          if (x >= v[0]) {
            v[0] = x;
            ix[0] = xi;
          }
        } else if (x > v[3]) {
          v[3] = x;
          ix[3] = xi;
          auto cx = [&](int p, int q) {
            if (v[p] < v[q]) {
              const float tv = v[p];
              v[p] = v[q];
              v[q] = tv;
              const int32_t ti = ix[p];
              ix[p] = ix[q];
              ix[q] = ti;
            }
          };
          cx(0, 2);
          cx(1, 3);
          cx(0, 1);
          cx(2, 3);
        }
      }
    }
    __syncthreads();
  }
  if (tid < nrows) {
    const int64_t row = row0 + tid;
#pragma unroll
    for (int s = 0; s < K; ++s) {
      a.out_idx[row * K + s] = int32_t(int64_t(ix[s]) + a.index_base);
      if (a.out_scores) a.out_scores[row * K + s] = v[s];
    }
  }
}

}  // namespace

cudaError_t launch_select_blockmax(const SelectArgs& a, cudaStream_t stream) {
  if (a.rows <= 0) return cudaSuccess;
  const unsigned grid = unsigned((a.rows + kRowsPerCta - 1) / kRowsPerCta);
  if (a.k == 1)
    select_blockmax_kernel<1><<<grid, kThreads, 0, stream>>>(a);
  else
    select_blockmax_kernel<4><<<grid, kThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace prism
