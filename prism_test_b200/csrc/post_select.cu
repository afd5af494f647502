// Device post-selection of the recall path: the union of every query's top-k
// middle indices, optionally cut to the recall_clip most frequently selected,
// each expanded into a span of neighbouring positions, clamped to the middle
// range, deduplicated and sorted — what ReAttentionMethod._global_unique and
// _expand_spans do with torch.unique on the host side
// (eval_harness/attention_methods/reattention.py:844-874, and the span variant of
// eval_harness/attention_methods/reattention_exact.py:571-585).
//
// Over the n_mid middle positions:
//   1. count how often each position was selected (atomics into a count array);
//   2. with recall_clip >= 0, keep the recall_clip most frequent positions: the
//      exact top-k selection runs on the counts (ties toward lower positions,
//      where torch.topk leaves the order unspecified); otherwise keep every
//      position selected at least once;
//   3. position x is in the result iff a kept position p has x - p in the span's
//      offset range [lo, hi) — after clamping, positions below 0 land on 0 and
//      above n_mid - 1 on n_mid - 1, which is the same as intersecting [p+lo,
//      p+hi) with [0, n_mid) — so one CTA builds the prefix count P of kept
//      positions and tests P[x - lo + 1] - P[x - hi + 1] > 0, then compacts the
//      covered positions in ascending order.
#include "common.cuh"
#include "kernels.h"

namespace prism {
namespace {

constexpr int kThreads = 1024;

__global__ void count_kernel(const int32_t* __restrict__ idx, int64_t n_idx, int64_t n_mid,
                             uint32_t* __restrict__ counts) {
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n_idx;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int32_t p = idx[i];
    if (p >= 0 && p < n_mid) atomicAdd(&counts[p], 1u);
  }
}

__global__ void counts_to_scores_kernel(const uint32_t* __restrict__ counts, int64_t n_mid,
                                        float* __restrict__ scores) {
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n_mid;
       i += int64_t(gridDim.x) * blockDim.x)
    scores[i] = float(counts[i]);
}

// mark[p] = 1 for the selected top positions that were picked at least once
__global__ void mark_kept_kernel(const int32_t* __restrict__ top_idx, const float* __restrict__ top_cnt,
                                 int k, uint32_t* __restrict__ mark) {
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < k; j += gridDim.x * blockDim.x)
    if (top_cnt[j] >= 1.0f) mark[top_idx[j]] = 1u;
}

__device__ __forceinline__ uint32_t block_scan_excl(uint32_t v, uint32_t* warp_tot, uint32_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_tot[warp] = x;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = warp_tot[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    warp_tot[lane] = w;
  }
  __syncthreads();
  const uint32_t r = (warp ? warp_tot[warp - 1] : 0u) + x - v;
  *total = warp_tot[31];
  __syncthreads();
  return r;
}

// One CTA: P = prefix count of kept positions (kept: mark[x] > 0), then the
// covered positions in ascending order.
__global__ void __launch_bounds__(kThreads) span_compact_kernel(const uint32_t* __restrict__ mark,
                                                                int64_t n_mid, int lo, int hi,
                                                                uint32_t* __restrict__ prefix,
                                                                int32_t* __restrict__ out_pos,
                                                                int32_t* __restrict__ out_count) {
  __shared__ uint32_t warp_tot[32];
  const int64_t seg = (n_mid + kThreads - 1) / kThreads;
  const int64_t x0 = int64_t(threadIdx.x) * seg;
  const int64_t x1 = x0 + seg < n_mid ? x0 + seg : n_mid;
  uint32_t c = 0;
  for (int64_t x = x0; x < x1; ++x) c += mark[x] ? 1u : 0u;
  uint32_t total;
  uint32_t run = block_scan_excl(c, warp_tot, &total);
  for (int64_t x = x0; x < x1; ++x) {
    prefix[x] = run;  // kept positions in [0, x)
    run += mark[x] ? 1u : 0u;
  }
  if (threadIdx.x == 0) prefix[n_mid] = total;
  __syncthreads();  // prefix is visible to the whole CTA
  auto covered = [&](int64_t x) {
    const int64_t a = x - hi + 1 > 0 ? x - hi + 1 : 0;
    const int64_t b = x - lo + 1 < n_mid ? x - lo + 1 : n_mid;
    return a < b && prefix[b] - prefix[a] > 0;
  };
  c = 0;
  for (int64_t x = x0; x < x1; ++x) c += covered(x) ? 1u : 0u;
  uint32_t ncov;
  uint32_t slot = block_scan_excl(c, warp_tot, &ncov);
  for (int64_t x = x0; x < x1; ++x)
    if (covered(x)) out_pos[slot++] = int32_t(x);
  if (threadIdx.x == 0) *out_count = int32_t(ncov);
}

}  // namespace

size_t post_select_workspace_bytes(int64_t n_mid, int32_t recall_clip) {
  auto up = [](size_t x) { return (x + 255) / 256 * 256; };
  size_t b = up(size_t(n_mid) * 4)          // counts
             + up(size_t(n_mid) * 4)        // mark
             + up(size_t(n_mid + 1) * 4);   // prefix
  if (recall_clip > 0) {
    const int64_t k = recall_clip < n_mid ? recall_clip : n_mid;
    b += up(size_t(n_mid) * 4)              // counts as scores
         + up(size_t(k) * 4) * 2            // top positions and their counts
         + up(select_workspace_bytes(1, n_mid));
  }
  return b;
}

cudaError_t launch_post_select(const int32_t* idx, int64_t n_idx, int64_t n_mid, int32_t recall_clip,
                               int lo, int hi, int32_t* out_pos, int32_t* out_count, void* workspace,
                               int num_sms, cudaStream_t stream) {
  auto up = [](size_t x) { return (x + 255) / 256 * 256; };
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint32_t* counts = reinterpret_cast<uint32_t*>(ws);
  ws += up(size_t(n_mid) * 4);
  uint32_t* mark = reinterpret_cast<uint32_t*>(ws);
  ws += up(size_t(n_mid) * 4);
  uint32_t* prefix = reinterpret_cast<uint32_t*>(ws);
  ws += up(size_t(n_mid + 1) * 4);

  cudaError_t e = cudaMemsetAsync(counts, 0, size_t(n_mid) * 4, stream);
  if (e != cudaSuccess) return e;
  const int grid = num_sms * 4;
  if (n_idx > 0) count_kernel<<<grid, 256, 0, stream>>>(idx, n_idx, n_mid, counts);
  const uint32_t* kept = counts;
  if (recall_clip > 0) {
    const int k = int(recall_clip < n_mid ? recall_clip : n_mid);
    float* scores = reinterpret_cast<float*>(ws);
    ws += up(size_t(n_mid) * 4);
    int32_t* top_idx = reinterpret_cast<int32_t*>(ws);
    ws += up(size_t(k) * 4);
    float* top_cnt = reinterpret_cast<float*>(ws);
    ws += up(size_t(k) * 4);
    counts_to_scores_kernel<<<grid, 256, 0, stream>>>(counts, n_mid, scores);
    SelectArgs s{};
    s.scores = scores;
    s.idx_in = nullptr;
    s.rows = 1;
    s.n = n_mid;
    s.ld = (n_mid + 3) / 4 * 4;
    s.k = k;
    s.index_base = 0;
    s.out_idx = top_idx;
    s.out_scores = top_cnt;
    s.status = nullptr;
    e = launch_select_topk(s, ws, stream);
    if (e != cudaSuccess) return e;
    e = cudaMemsetAsync(mark, 0, size_t(n_mid) * 4, stream);
    if (e != cudaSuccess) return e;
    mark_kept_kernel<<<(k + 255) / 256, 256, 0, stream>>>(top_idx, top_cnt, k, mark);
    kept = mark;
  }
  span_compact_kernel<<<1, kThreads, 0, stream>>>(kept, n_mid, lo, hi, prefix, out_pos, out_count);
  return cudaGetLastError();
}

}  // namespace prism
