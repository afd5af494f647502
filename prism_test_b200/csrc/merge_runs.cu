// Top-k of the union of N sorted runs: the device merge of the sequence-sharded
// path, where run r of a row is rank r's local top-k (fp32 score bits, global
// index), sorted by descending score and then ascending index — the order
// prism_einsum_topk returns. It reproduces torch.topk over the union
// (reattention.py:497) with the merge of eval_harness/kernels/bitonic_merge_wrapper.py:36-52
// generalised to N runs of any length, without sorting anything.
//
// Candidates are compared as (order-preserving key << 32) | ~index, a strict total
// order for distinct indices. A summary of every run — its entries at positions
// s-1, 2s-1, ... with s = max(1, k / 128) — bounds from below how many entries of
// the run are at or above any value v (s per summary entry >= v). The threshold T
// is the largest summary entry whose bound, summed over the runs, still reaches k:
// the global k-th candidate is then at or above T, and fewer than k + (N + 1) s
// candidates are (about k, whatever the split over the runs). Only the prefix of
// each run at or above T can reach the output. The prefixes are staged in shared memory and
// every staged candidate x of run r at position j is written at output position
//   j + sum over the other runs of (number of their candidates above x),
// which is a permutation of [0, total) (an equal candidate of an earlier run
// counts as above); positions below k are kept. A thread takes
// 16 consecutive candidates of one run: the first finds its place in every other
// run by binary search, the following ones advance those places monotonically.
// Results are permuted in shared memory and stored coalesced.
//
// One CTA of 1024 threads per row. When the prefixes exceed the staging capacity
// (heavy ties at T, or runs padded below k on every rank) the same ranking runs
// on the runs in global memory and stores the outputs directly (slower, same
// result).
#include "common.cuh"
#include "kernels.h"

namespace prism {
namespace {

constexpr int kThreads = 1024;
constexpr int kMaxRuns = 16;
constexpr int kStage = 10240;   // staged candidates per row
constexpr int kSumm = 128;      // summary entries per run
constexpr int kOutCap = 16384;  // output entries permuted in shared memory
constexpr int kSeg = 16;        // consecutive candidates per thread

struct MergeSmem {
  uint64_t cand[kStage];      // run prefixes, run r at [off[r], off[r] + len[r])
  uint64_t summ[kMaxRuns][kSumm];  // run r's entries at positions s-1, 2s-1, ...
  uint64_t out[kOutCap];      // output order (first k)
  uint32_t off[kMaxRuns + 1];
  uint32_t len[kMaxRuns];
  uint64_t thr;
};

__device__ __forceinline__ uint64_t packed_at(const int32_t* e) {
  const uint32_t key = float_to_okey(__int_as_float(e[0]));
  return (uint64_t(key) << 32) | uint64_t(~uint32_t(e[1]));
}

// Number of entries of the sorted-descending sequence at(0..n-1) above x (at or
// above x when incl): equal candidates of different runs are ordered by run.
template <typename At>
__device__ __forceinline__ uint32_t count_above(At at, uint32_t n, uint64_t x, bool incl) {
  uint32_t lo = 0, hi = n;
  while (lo < hi) {
    const uint32_t mid = (lo + hi) >> 1;
    const uint64_t v = at(mid);
    if (v > x || (incl && v == x)) lo = mid + 1;
    else hi = mid;
  }
  return lo;
}

// Output positions of the candidates of runs[0, nruns), each sorted descending
// with len[r] entries read through get(r, j); store(p, x) for p < k. Thread t
// takes segments of kSeg consecutive candidates of one run.
template <typename Get, typename Store>
__device__ void rank_segments(int nruns, const uint32_t* len, uint32_t total, int k, Get get,
                              Store store) {
  const uint32_t nseg_total = (total + kSeg - 1) / kSeg + uint32_t(nruns);
  for (uint32_t sgi = threadIdx.x; sgi < nseg_total; sgi += kThreads) {
    int r = 0;
    uint32_t base_seg = 0, j0 = 0;
    bool ok = false;
    for (; r < nruns; ++r) {
      const uint32_t ns = (len[r] + kSeg - 1) / kSeg;
      if (sgi < base_seg + ns) {
        j0 = (sgi - base_seg) * kSeg;
        ok = true;
        break;
      }
      base_seg += ns;
    }
    if (!ok) continue;
    const uint32_t j1 = min(len[r], j0 + kSeg);
    uint32_t at[kMaxRuns];
    const uint64_t x0 = get(r, j0);
    for (int q = 0; q < nruns; ++q)
      at[q] = q == r ? 0u : count_above([&](uint32_t j) { return get(q, j); }, len[q], x0, q < r);
    for (uint32_t j = j0; j < j1; ++j) {
      const uint64_t x = get(r, j);
      uint32_t p = j;
      for (int q = 0; q < nruns; ++q) {
        if (q == r) continue;
        uint32_t a = at[q];
        while (a < len[q]) {
          const uint64_t v = get(q, a);
          if (!(v > x || (q < r && v == x))) break;
          ++a;
        }
        at[q] = a;
        p += a;
      }
      if (p < uint32_t(k)) store(p, x);
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    merge_runs_kernel(const int32_t* __restrict__ runs, int nruns, int64_t rows, int64_t run_len,
                      int k, int32_t* __restrict__ out_idx, float* __restrict__ out_scores) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  MergeSmem& sm = *reinterpret_cast<MergeSmem*>(smem_raw);
  const int64_t row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  auto entry = [&](int r, int64_t j) { return runs + ((int64_t(r) * rows + row) * run_len + j) * 2; };

  // T from the run summaries; without a summary that reaches k, the largest of
  // the runs' last candidates (every run's prefix above it may then be long)
  const int64_t sstep = k / kSumm > 1 ? k / kSumm : 1;
  const int nsum = int(run_len / sstep < kSumm ? run_len / sstep : kSumm);
  if (tid == 0) sm.thr = 0;
  for (int e = tid; e < nruns * nsum; e += kThreads) {
    const int r = e / nsum, i = e - r * nsum;
    sm.summ[r][i] = packed_at(entry(r, (int64_t(i) + 1) * sstep - 1));
  }
  __syncthreads();
  for (int e = tid; e < nruns * nsum; e += kThreads) {
    const int r = e / nsum, i = e - r * nsum;
    const uint64_t v = sm.summ[r][i];
    int64_t c = 0;
    for (int q = 0; q < nruns; ++q)
      c += count_above([&](uint32_t j) { return sm.summ[q][j]; }, uint32_t(nsum), v, true);
    if (c * sstep >= int64_t(k)) atomicMax(reinterpret_cast<unsigned long long*>(&sm.thr), v);
  }
  __syncthreads();
  if (sm.thr == 0 && warp == 0) {
    uint64_t t = 0;
    if (lane < nruns) t = packed_at(entry(lane, run_len - 1));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const uint64_t u = __shfl_xor_sync(0xffffffffu, t, o);
      t = u > t ? u : t;
    }
    if (lane == 0) sm.thr = t;
  }
  __syncthreads();
  const uint64_t thr = sm.thr;
  // prefix of each run at or above T: warp r narrows the boundary 32-fold per step
  if (warp < nruns) {
    int64_t lo = 0, hi = run_len;  // entries [0, lo) are >= T, entries [hi, run_len) are < T
    while (lo < hi) {
      const int64_t step = (hi - lo + 31) / 32;
      const int64_t p = lo + int64_t(lane) * step;
      const bool ge = p < hi && packed_at(entry(warp, p)) >= thr;
      // entries >= T form a prefix, so the passing probes are lanes 0 .. c-1
      const int c = __popc(__ballot_sync(0xffffffffu, ge));
      if (c == 0) break;
      const int64_t nhi = lo + int64_t(c) * step;
      lo = lo + int64_t(c - 1) * step + 1;
      hi = nhi < hi ? nhi : hi;
    }
    if (lane == 0) sm.len[warp] = uint32_t(lo);
  }
  __syncthreads();
  if (tid == 0) {
    uint32_t acc = 0;
    for (int r = 0; r < nruns; ++r) {
      sm.off[r] = acc;
      acc += sm.len[r];
    }
    sm.off[nruns] = acc;
  }
  __syncthreads();
  const uint32_t total = sm.off[nruns];
  int32_t* oi = out_idx + row * k;
  float* os = out_scores ? out_scores + row * k : nullptr;
  if (total > uint32_t(kStage)) {
    // too many candidates to stage: rank them in place in global memory
    rank_segments(
        nruns, sm.len, total, k, [&](int r, uint32_t j) { return packed_at(entry(r, j)); },
        [&](uint32_t p, uint64_t x) {
          oi[p] = int32_t(~uint32_t(x));
          if (os) os[p] = okey_to_float(uint32_t(x >> 32));
        });
    return;
  }
  for (int r = 0; r < nruns; ++r) {
    const uint32_t o = sm.off[r], n = sm.len[r];
    for (uint32_t j = tid; j < n; j += kThreads) sm.cand[o + j] = packed_at(entry(r, j));
  }
  __syncthreads();
  rank_segments(
      nruns, sm.len, total, k, [&](int r, uint32_t j) { return sm.cand[sm.off[r] + j]; },
      [&](uint32_t p, uint64_t x) { sm.out[p] = x; });
  __syncthreads();
  for (int p = tid; p < k; p += kThreads) {
    const uint64_t x = sm.out[p];
    oi[p] = int32_t(~uint32_t(x));
    if (os) os[p] = okey_to_float(uint32_t(x >> 32));
  }
}

}  // namespace

cudaError_t launch_merge_runs(const int32_t* runs, int nruns, int64_t rows, int64_t run_len, int k,
                              int32_t* out_idx, float* out_scores, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  const size_t smem = sizeof(MergeSmem);
  cudaError_t e = cudaFuncSetAttribute(merge_runs_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  merge_runs_kernel<<<dim3(unsigned(rows)), kThreads, smem, stream>>>(runs, nruns, rows, run_len, k,
                                                                      out_idx, out_scores);
  return cudaGetLastError();
}

}  // namespace prism
